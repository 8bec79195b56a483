"""SAELens SAE objects through saeflow_b200.saelens.

sae_lens is not installed here, so the SAEs are stand-ins with the attributes the adapter
reads (SAELens v5 style: cfg.architecture string, activation_fn_str / activation_fn_kwargs;
v6 style: cfg.architecture() method, cfg.k). The expected values restate SAELens's
forward in plain torch fp32 (normalise, subtract b_dec if configured, encode, activate,
decode, un-normalise).
"""

import math
from types import SimpleNamespace

import pytest
import torch

from saeflow_b200 import saelens


def make(arch="jumprelu", norm="none", apply_b_dec=True, style="v6", d_in=64, d_sae=256, k=8,
         dtype=torch.float32, device="cpu", seed=0):
    g = torch.Generator().manual_seed(seed)
    W_dec = torch.randn(d_sae, d_in, generator=g)
    W_dec /= W_dec.norm(dim=1, keepdim=True)
    sae = SimpleNamespace(
        W_enc=W_dec.T.contiguous(), W_dec=W_dec, b_enc=torch.randn(d_sae, generator=g) * 0.1 - 0.3,
        b_dec=torch.randn(d_in, generator=g) * 0.1,
        threshold=(torch.rand(d_sae, generator=g) * 0.3) if arch == "jumprelu" else None)
    for name in ("W_enc", "W_dec", "b_enc", "b_dec", "threshold"):
        t = getattr(sae, name)
        if t is not None:
            setattr(sae, name, t.to(device=device, dtype=dtype))
    if style == "v6":
        cfg = SimpleNamespace(d_in=d_in, d_sae=d_sae, apply_b_dec_to_input=apply_b_dec,
                              normalize_activations=norm, architecture=lambda: arch)
        if arch == "topk":
            cfg.k = k
    else:
        cfg = SimpleNamespace(d_in=d_in, d_sae=d_sae, apply_b_dec_to_input=apply_b_dec,
                              normalize_activations=norm, architecture=arch if arch != "topk" else "standard",
                              activation_fn_str="topk" if arch == "topk" else "relu",
                              activation_fn_kwargs={"k": k} if arch == "topk" else {})
    sae.cfg = cfg
    return sae


def saelens_forward(sae, x, arch, norm, apply_b_dec, k=8):
    """SAELens's forward restated in torch fp32; also returns the pre-activations and cut."""
    xf = x.float()
    if norm == "constant_norm_rescale":
        s = math.sqrt(x.shape[1]) / xf.norm(dim=1, keepdim=True)
        xn = xf * s
    elif norm == "layer_norm":
        mu = xf.mean(dim=1, keepdim=True)
        std = (xf - mu).std(dim=1, keepdim=True)
        xn = (xf - mu) / (std + 1e-5)
    else:
        xn = xf
    pre = (xn - sae.b_dec.float() * apply_b_dec) @ sae.W_enc.float() + sae.b_enc.float()
    if arch == "standard":
        f, cut = torch.relu(pre), torch.zeros_like(pre)
    elif arch == "jumprelu":
        cut = sae.threshold.float().expand_as(pre)
        f = torch.relu(pre) * (pre > cut)
    else:
        top = pre.topk(k, dim=1)
        f = torch.zeros_like(pre).scatter_(1, top.indices, torch.relu(top.values))
        cut = None
    out = f @ sae.W_dec.float() + sae.b_dec.float()
    if norm == "constant_norm_rescale":
        out = out / s
    elif norm == "layer_norm":
        out = out * std + mu
    return out, f, pre, cut


# ----------------------------------------------------------------------------- CPU

@pytest.mark.parametrize("style", ["v5", "v6"])
@pytest.mark.parametrize("arch,activation", [("standard", "relu"), ("jumprelu", "jumprelu"), ("topk", "topk")])
def test_adapt_reads_architecture_and_k(style, arch, activation):
    v = saelens.adapt(make(arch, style=style, k=12))
    assert v.activation == activation
    assert v.k == (12 if arch == "topk" else None)
    assert (v.threshold is not None) == (arch == "jumprelu")


def test_adapt_b_dec_to_input_switch():
    sae = make(apply_b_dec=False)
    v = saelens.adapt(sae)
    assert torch.equal(v.b_dec, sae.b_dec) and not v.b_dec_in.any()
    assert saelens.adapt(make(apply_b_dec=True)).b_dec_in is not None


def test_adapt_rejects_what_the_kernels_do_not_implement():
    sae = make()
    sae.cfg.architecture = lambda: "gated"
    with pytest.raises(ValueError, match="gated"):
        saelens.adapt(sae)
    with pytest.raises(ValueError, match="normalize_activations"):
        saelens.adapt(make(norm="batch_norm"))
    bad = make("topk")
    del bad.cfg.k
    with pytest.raises(ValueError, match="k"):
        saelens.adapt(bad)


@pytest.mark.parametrize("norm", ["none", "expected_average_only_in", "constant_norm_rescale", "layer_norm"])
def test_normalisation_round_trip(norm):
    v = saelens.adapt(make(norm=norm))
    x = torch.randn(10, 64) * 3 + 1
    xn, state = saelens._norm_in(v, x)
    if norm == "constant_norm_rescale":
        torch.testing.assert_close(xn.norm(dim=1), torch.full((10,), 8.0))
    if norm == "layer_norm":
        torch.testing.assert_close(xn.mean(dim=1), torch.zeros(10), atol=1e-5, rtol=0)
    torch.testing.assert_close(saelens._norm_out(xn, state), x, atol=1e-4, rtol=1e-5)


# ----------------------------------------------------------------------------- GPU

@pytest.mark.gpu
@pytest.mark.parametrize("arch", ["standard", "jumprelu", "topk"])
@pytest.mark.parametrize("norm", ["none", "constant_norm_rescale", "layer_norm"])
@pytest.mark.parametrize("apply_b_dec", [True, False])
def test_forward_matches_saelens_math(arch, norm, apply_b_dec):
    sae = make(arch, norm=norm, apply_b_dec=apply_b_dec, device="cuda")
    x = torch.randn(300, 64, device="cuda") * 2
    want, f_want, pre, cut = saelens_forward(sae, x, arch, norm, apply_b_dec)
    got = saelens.forward(sae, x)
    if cut is not None:
        clean = ((pre - cut).abs() > 1e-4).all(dim=1)  # rows with no feature at the cut
    else:
        kth = pre.topk(9, dim=1).values
        clean = (kth[:, 7] - kth[:, 8]).abs() > 1e-4  # rows without a k-th / (k+1)-th tie
    assert clean.float().mean() > 0.5
    torch.testing.assert_close(got[clean], want[clean], atol=1e-4, rtol=1e-4)
    f = saelens.encode(sae, x)
    torch.testing.assert_close(f[clean], f_want[clean], atol=1e-4, rtol=1e-4)
    ip, ix, vs = saelens.encode_sparse(sae, x)
    dec = saelens.decode_sparse(sae, (ip, ix, vs), x)
    torch.testing.assert_close(dec[clean], want[clean], atol=1e-4, rtol=1e-4)


@pytest.mark.gpu
def test_bf16_saelens_sae_runs_the_tensor_core_path():
    """bf16: the kernels round (x - b_dec) to bf16 before the product (as saeflow does), so
    the expected values take the same rounded shift; rows with a feature within 1e-3 of its
    threshold are left out (the north-star rule)."""
    sae = make("jumprelu", dtype=torch.bfloat16, device="cuda", d_in=256, d_sae=1024)
    x = torch.randn(500, 256, device="cuda").to(torch.bfloat16)
    xs = (x.float() - sae.b_dec.float()).to(torch.bfloat16).float()
    pre = xs @ sae.W_enc.float() + sae.b_enc.float()
    cut = sae.threshold.float()
    f = torch.relu(pre) * (pre > cut)
    want = f.to(torch.bfloat16).float() @ sae.W_dec.float() + sae.b_dec.float()
    got = saelens.forward(sae, x)
    clean = ((pre - cut).abs() > 1e-3).all(dim=1)
    assert clean.float().mean() > 0.3
    torch.testing.assert_close(got.float()[clean], want[clean], atol=2e-2, rtol=1e-2)
