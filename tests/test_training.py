"""Backward of the sparse forward (saeflow_b200.training, csrc/backward.cu) against torch
autograd of the same computation on the same active set.

The expected gradients come from a dense fp32 restatement in torch: pre = (x - b_dec) @ W_enc
+ b_enc, f = pre on the features the kernels' forward kept active (its CSR pattern, values
> 0 for TopK), x_hat = f @ W_dec + b_dec, loss = sum(x_hat * r). Taking the active set
from the kernels' own forward makes the comparison about the backward arithmetic only.
"""

import pytest
import torch

import oracle
from saeflow_b200 import training
from saeflow_b200.kernels import csr_to_dense, device_error
from saeflow_b200.kernels.backward import csc_accumulate, csr_sddmm, csr_transpose, transpose

pytestmark = pytest.mark.gpu


def _sae(d_in, d_sae, activation, dtype, k=None):
    torch.manual_seed(0)
    sae = oracle.RefSAE(d_in, d_sae, activation, k=k)
    sae.b_enc.normal_(0, 0.1)
    sae.b_dec.normal_(0, 0.1)
    if activation == "relu":
        sae.b_enc.sub_(1.5)
    if activation == "jumprelu":
        sae.threshold.uniform_(0.5, 1.5)
    sae = sae.to(dtype).cuda()
    for name in ("W_enc", "b_enc", "W_dec", "b_dec"):
        getattr(sae, name).requires_grad_(True)
    return sae


def _reference_grads(sae, x, r, active):
    Ws = {n: getattr(sae, n).detach().float().clone().requires_grad_(True) for n in ("W_enc", "b_enc", "W_dec", "b_dec")}
    xr = x.detach().float().clone().requires_grad_(True)
    v = xr - Ws["b_dec"]
    # the kernels multiply (x - b_dec) rounded to W's dtype; the rounding passes gradient through
    xs = v.detach().to(sae.W_enc.dtype).float() + (v - v.detach())
    pre = xs @ Ws["W_enc"] + Ws["b_enc"]
    f = pre * active
    out = f @ Ws["W_dec"] + Ws["b_dec"]
    (out * r).sum().backward()
    return {"x": xr.grad, **{n: w.grad for n, w in Ws.items()}}


@pytest.mark.parametrize("activation", ["relu", "jumprelu", "topk"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(37, 64, 300), (300, 128, 1000)])
def test_backward_matches_autograd_on_the_active_set(activation, dtype, shape):
    M, d_in, d_sae = shape
    sae = _sae(d_in, d_sae, activation, dtype, k=12 if activation == "topk" else None)
    x = (torch.randn(M, d_in, device="cuda") * 1.5).to(dtype).requires_grad_(True)
    out = training.forward(sae, x)
    r = torch.randn(M, d_in, device="cuda")
    (out.float() * r).sum().backward()

    from saeflow_b200 import encode_sparse

    ip, ix, vs = encode_sparse(sae, x.detach())
    active = (csr_to_dense(ip, ix, vs.float(), d_sae) > 0).float()
    want = _reference_grads(sae, x, r, active)
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    got = {"x": x.grad, "W_enc": sae.W_enc.grad, "b_enc": sae.b_enc.grad, "W_dec": sae.W_dec.grad,
           "b_dec": sae.b_dec.grad}
    for name, w in want.items():
        g = got[name].float()
        assert g.shape == w.shape, name
        scale = w.abs().max().item() + 1e-6
        err = (g - w).abs().max().item() / scale
        assert err < tol, f"{name}: max error {err:.3g} of the gradient's scale"
    assert device_error() == 0


def test_transpose_sddmm_accumulate_against_torch():
    """The three kernels on a random CSR pattern (with empty rows and empty columns)."""
    g = torch.Generator(device="cuda").manual_seed(3)
    M, n_cols, D = 200, 700, 96
    dense = (torch.rand(M, n_cols, generator=g, device="cuda") < 0.03).float() * torch.randn(
        M, n_cols, generator=g, device="cuda")
    dense[:, 40] = torch.randn(M, generator=g, device="cuda")  # two columns above the hot threshold (256)
    dense[:, 41] = torch.randn(M, generator=g, device="cuda")
    dense = torch.cat([dense, dense]).contiguous()
    M = dense.shape[0]
    dense[5] = 0     # an empty row
    dense[:, 13] = 0  # an empty column
    csr = dense.to_sparse_csr()
    ip, ix, vs = csr.crow_indices(), csr.col_indices().to(torch.int32), csr.values()
    col_ptr, row_idx, perm, order = csr_transpose(ip, ix, n_cols)
    assert torch.equal(col_ptr[1:] - col_ptr[:-1], (dense != 0).sum(0))
    assert torch.equal(order[:n_cols].long().sort().values, torch.arange(n_cols, device="cuda"))  # a permutation
    assert sorted(order[:2].tolist()) == [40, 41] and int(order[n_cols]) == 2                   # hot ones first
    rows = torch.repeat_interleave(torch.arange(M, device="cuda"), ip[1:] - ip[:-1])
    assert torch.equal(row_idx.long(), rows[perm])        # each slot names its entry's row
    assert torch.equal(ix.long()[perm].sort().values, ix.long().sort().values)
    cols = torch.repeat_interleave(torch.arange(n_cols, device="cuda"), col_ptr[1:] - col_ptr[:-1])
    assert torch.equal(ix.long()[perm], cols)             # ... and sits in its own column
    G = torch.randn(M, D, generator=g, device="cuda")
    W = torch.randn(n_cols, D, generator=g, device="cuda")
    dots = csr_sddmm(ip, ix, vs, G, W)
    want = (G[rows] * W[ix.long()]).sum(1)
    torch.testing.assert_close(dots, want, atol=1e-4, rtol=1e-4)
    acc, sums = csc_accumulate(col_ptr, row_idx, perm, order, vs, G, col_sums=True)
    torch.testing.assert_close(acc, dense.T @ G, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(sums, dense.sum(0), atol=1e-5, rtol=1e-5)
    assert device_error() == 0


@pytest.mark.parametrize("src,dst", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                     (torch.float16, torch.float32)])
@pytest.mark.parametrize("shape", [(1, 1), (33, 70), (300, 4099)])
def test_transpose_kernel(src, dst, shape):
    x = torch.randn(*shape, device="cuda").to(src)
    got = transpose(x, dst)
    assert got.shape == (shape[1], shape[0]) and got.dtype == dst and got.is_contiguous()
    assert torch.equal(got, x.t().to(dst))
    strided = torch.randn(shape[0], shape[1] + 5, device="cuda").to(src)[:, 2:2 + shape[1]]
    assert torch.equal(transpose(strided, dst), strided.t().to(dst))
