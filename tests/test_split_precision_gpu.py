"""IEEE fp32 encode on the bf16 tensor cores (B200).

fp32 x with fp32 W_enc and TF32 not allowed asks for IEEE products (the reference's
`input_precision="ieee"`, saeflow/kernels/encode.py:118-120). The default route splits
both operands into three bf16 parts and sums the six significant partial products,
smallest first, on the tensor cores; `config={"variant": "simt"}` pins the CUDA-core
FMA kernel. These tests hold the split route to the fp32 contract against the float64
oracle, compare its error with the CUDA-core kernel's on the same inputs, and check that
non-finite operands hand the call to the CUDA-core kernel (identical results).
"""

import pytest
import torch

import oracle
from oracle import contract
from saeflow_b200.kernels import best_config, dense_to_csr, device_error, encode_csr, fused_encode

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_device_errors():
    device_error()
    yield
    assert device_error() == 0, "a kernel reported a device-side error"


def _operands(M, d_in, d_sae, seed, layout="row"):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W_dec = torch.randn(d_sae, d_in, generator=g, device="cuda")
    W_dec /= W_dec.norm(dim=1, keepdim=True)
    if layout == "row":
        W = W_dec.T.contiguous()
    elif layout == "col":
        W = W_dec.T  # column-major view
    else:  # a column slice of a wider row-major matrix: unaligned base, odd pitch
        wide = torch.zeros(d_in, d_sae + 3, device="cuda")
        wide[:, 1:d_sae + 1] = W_dec.T
        W = wide[:, 1:d_sae + 1]
    b_enc = torch.randn(d_sae, generator=g, device="cuda") * 0.1 - 1.0
    b_dec = torch.randn(d_in, generator=g, device="cuda") * 0.1
    x = torch.randn(M, d_in, generator=g, device="cuda") * 1.5
    return x, W, b_enc, b_dec


def _pre64(x, W, b_enc, b_dec):
    xs = (x.float() - b_dec.float()).double().cpu()
    return xs @ W.double().cpu() + b_enc.double().cpu()


def _errors(got, pre64):
    d = (got.double().cpu() - pre64.clamp_min(0)).abs()
    return d.max().item(), d.pow(2).mean().sqrt().item()


@pytest.mark.parametrize("shape", [(5, 24, 40), (300, 100, 700), (1000, 768, 4099), (257, 1024, 2000)])
@pytest.mark.parametrize("layout", ["row", "col", "sliced"])
def test_split_precision_within_fp32_contract(shape, layout):
    """Every feature outside the 1e-3 cut band within rtol 1e-5 (atol 1e-5) of the float64
    oracle; the error no more than a small factor above the CUDA-core IEEE kernel's. d_in up
    to 1024, the range the "auto" kernel choice sends to this route."""
    M, d_in, d_sae = shape
    x, W, b_enc, b_dec = _operands(M, d_in, d_sae, seed=d_in + d_sae, layout=layout)
    rn = torch.zeros(M, dtype=torch.int32, device="cuda")
    got = fused_encode(x, W, b_enc, b_dec, row_nnz=rn)
    assert best_config()["variant"].startswith("tcgen05") and "split" in best_config()["operands"]
    assert torch.equal(rn, torch.count_nonzero(got, dim=1).int())
    want, _, pre = oracle.fused_encode(x.cpu(), W.cpu(), b_enc.cpu(), b_dec.cpu())
    near = contract.near_cut(pre)
    contract.assert_values_close(got.cpu()[~near], want[~near], torch.float32, what="split-precision encode")

    simt = fused_encode(x, W, b_enc, b_dec, config={"variant": "simt"})
    pre64 = _pre64(x, W, b_enc, b_dec)
    mx, rms = _errors(got, pre64)
    mx_s, rms_s = _errors(simt, pre64)
    assert mx <= 4 * mx_s + 1e-7 and rms <= 3 * rms_s + 1e-8, (mx, rms, mx_s, rms_s)


@pytest.mark.parametrize("x_layout", ["transposed", "sliced"])
def test_split_precision_strided_x_and_b_dec(x_layout):
    """x column-major (the split's scalar path) or a column slice of a wider matrix, b_dec a
    strided fp16 view: same contract against the oracle, and the same values as contiguous
    operands (the split sees the same fp32 differences)."""
    M, d_in, d_sae = 333, 200, 1100
    x, W, b_enc, b_dec = _operands(M, d_in, d_sae, seed=21)
    if x_layout == "transposed":
        xs = x.T.contiguous().T
    else:
        wide = torch.zeros(M, d_in + 5, device="cuda")
        wide[:, 3:d_in + 3] = x
        xs = wide[:, 3:d_in + 3]
    bd16 = torch.zeros(2 * d_in, device="cuda", dtype=torch.float16)
    bd16[::2] = b_dec.half()
    bd = bd16[::2]
    got = fused_encode(xs, W, b_enc, bd)
    ref = fused_encode(x.contiguous(), W, b_enc, bd.contiguous())
    assert torch.equal(got.view(torch.int32), ref.view(torch.int32))
    want, _, pre = oracle.fused_encode(x.cpu(), W.cpu(), b_enc.cpu(), bd.cpu())
    near = contract.near_cut(pre)
    contract.assert_values_close(got.cpu()[~near], want[~near], torch.float32, what=x_layout)


@pytest.mark.parametrize("d_in", [1025, 2304, 4096])
def test_split_precision_k_ranges(d_in):
    """Above d_in 1024 the tensor cores' per-MMA rounding of one running sum would outgrow
    the fp32 tolerance (measured at d_in 4096 in one range: 89 of 51200 features outside
    it), so the route runs K ranges of at most 1024, each accumulated from zero, and adds
    their sums in fp32: within the contract, the error of the order of the CUDA-core IEEE
    kernel's, and the encode straight to CSR identical to the dense route."""
    x, W, b_enc, b_dec = _operands(300, d_in, 1500, seed=d_in)
    rn = torch.zeros(300, dtype=torch.int32, device="cuda")
    got = fused_encode(x, W, b_enc, b_dec, row_nnz=rn)
    assert best_config()["variant"] == "tcgen05" and "split" in best_config()["operands"]
    want, _, pre = oracle.fused_encode(x.cpu(), W.cpu(), b_enc.cpu(), b_dec.cpu())
    near = contract.near_cut(pre)
    contract.assert_values_close(got.cpu()[~near], want[~near], torch.float32, what=f"d_in {d_in}")
    simt = fused_encode(x, W, b_enc, b_dec, config={"variant": "simt"})
    pre64 = _pre64(x, W, b_enc, b_dec)
    mx, rms = _errors(got, pre64)
    mx_s, rms_s = _errors(simt, pre64)
    assert mx <= 4 * mx_s + 1e-7 and rms <= 3 * rms_s + 1e-8, (mx, rms, mx_s, rms_s)
    csr = encode_csr(x, W, b_enc, b_dec)
    ref = dense_to_csr(got, rn)
    for a, b in zip(csr, ref):
        assert torch.equal(a.view(torch.int32) if a.is_floating_point() else a,
                           b.view(torch.int32) if b.is_floating_point() else b)
    single = fused_encode(x, W, b_enc, b_dec, config={"variant": "tcgen05_1cta"})
    contract.assert_values_close(single.cpu()[~near], want[~near], torch.float32, what="single-CTA ranges")


def test_split_precision_nonfinite_in_a_later_k_range():
    """An inf in the last K range's operands: the earlier ranges' partial sums are written,
    the last range's GEMM exits, and the CUDA-core kernel computes the call (identical)."""
    x, W, b_enc, b_dec = _operands(200, 2304, 700, seed=8)
    x[5, 2200] = float("inf")
    rn = torch.zeros(200, dtype=torch.int32, device="cuda")
    got = fused_encode(x, W, b_enc, b_dec, row_nnz=rn)
    rn_s = torch.zeros(200, dtype=torch.int32, device="cuda")
    want = fused_encode(x, W, b_enc, b_dec, row_nnz=rn_s, config={"variant": "simt"})
    assert not torch.isfinite(want).all()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32)) and torch.equal(rn, rn_s)


@pytest.mark.parametrize("variant", ["tcgen05", "tcgen05_1cta"])
def test_split_precision_pair_and_single_cta_kernels_agree(variant):
    """Both tensor-core kernels run the same split schedule: same partial products in the
    same order per output, so the same fp32 results."""
    x, W, b_enc, b_dec = _operands(700, 320, 1500, seed=11)
    got = fused_encode(x, W, b_enc, b_dec, config={"variant": variant})
    ref = fused_encode(x, W, b_enc, b_dec)
    want, _, pre = oracle.fused_encode(x.cpu(), W.cpu(), b_enc.cpu(), b_dec.cpu())
    near = contract.near_cut(pre)
    contract.assert_values_close(got.cpu()[~near], want[~near], torch.float32, what=variant)
    contract.assert_values_close(got.cpu()[~near], ref.cpu()[~near], torch.float32, what="pair vs single")


@pytest.mark.parametrize("where", ["x_inf", "x_nan", "w_inf", "shift_overflow"])
def test_split_precision_nonfinite_operands_use_the_ieee_kernel(where):
    """An inf or NaN in x - b_dec or in W_enc would meet zero parts of the other operand in
    the split products (inf * 0 = NaN where IEEE gives inf). The split flags it and the
    CUDA-core kernel computes the call instead: dense output, row counts and CSR identical
    to the pinned CUDA-core kernel's."""
    M, d_in, d_sae = 300, 96, 600
    x, W, b_enc, b_dec = _operands(M, d_in, d_sae, seed=5)
    if where == "x_inf":
        x[7, 3] = float("inf")
        x[40, 0] = float("-inf")
    elif where == "x_nan":
        x[9, 11] = float("nan")
    elif where == "w_inf":
        W = W.clone()
        W[5, 17] = float("inf")
    else:  # finite x whose shift overflows fp32
        x[3, 2] = 3.0e38
        b_dec = b_dec.clone()
        b_dec[2] = -3.0e38
    rn = torch.zeros(M, dtype=torch.int32, device="cuda")
    got = fused_encode(x, W, b_enc, b_dec, row_nnz=rn)
    rn_s = torch.zeros(M, dtype=torch.int32, device="cuda")
    want = fused_encode(x, W, b_enc, b_dec, row_nnz=rn_s, config={"variant": "simt"})
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    assert torch.equal(rn, rn_s)
    if where != "x_nan":  # a NaN pre-activation stores 0 (max(NaN, 0) = 0, as the reference's tl.maximum)
        assert not torch.isfinite(want).all()  # the case really carries a non-finite output
    csr = encode_csr(x, W, b_enc, b_dec)
    ref = dense_to_csr(want, rn_s)
    for a, b in zip(csr, ref):
        assert torch.equal(a.view(torch.int32) if a.is_floating_point() else a,
                           b.view(torch.int32) if b.is_floating_point() else b)


def test_split_precision_near_fp32_max():
    """Finite operands whose bf16 rounding overflows (|v| above the largest bf16, 3.39e38)
    are split with a truncated high part and stay exact: products near the top of the fp32
    range match the CUDA-core IEEE kernel to the fp32 contract."""
    M, d_in, d_sae = 130, 64, 256
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.zeros(M, d_in, device="cuda")
    cols = torch.randint(0, d_in, (M,), generator=g, device="cuda")
    sign = torch.where(torch.rand(M, generator=g, device="cuda") < 0.5, -1.0, 1.0)
    x[torch.arange(M, device="cuda"), cols] = sign * 3.4e38
    W = (torch.rand(d_in, d_sae, generator=g, device="cuda") - 0.5) * 0.5
    b_enc = torch.zeros(d_sae, device="cuda")
    got = fused_encode(x, W, b_enc, None)
    want = fused_encode(x, W, b_enc, None, config={"variant": "simt"})
    assert torch.isfinite(want).all() and want.abs().max() > 1e37
    contract.assert_values_close(got.cpu(), want.cpu(), torch.float32, what="near FLT_MAX")
