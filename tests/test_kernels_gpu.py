"""CUDA kernels vs the CPU oracle and the reference's golden vectors (B200 only).

Parametrisation follows the reference's tests/test_kernels.py: shapes that are not
tile multiples, fp32 / bf16 / fp16, ReLU and JumpReLU, the cut-exclusion rule, exact
row counts, bit-exact CSR.
"""

import pytest
import torch

import oracle
import saeflow_b200
from oracle import contract
from golden_io import Golden
from saeflow_b200.kernels import (csr_to_dense, dense_to_csr, device_error, encode_csr, fused_encode,
                                  sparse_decode, topk_encode)

pytestmark = pytest.mark.gpu

SHAPES = [(1, 16, 32), (37, 50, 129), (64, 64, 256), (100, 33, 70)]
DTYPES = [torch.float32, torch.bfloat16, torch.float16]
TOL = {torch.float32: 1e-4, torch.bfloat16: 3e-2, torch.float16: 5e-3}


@pytest.fixture(autouse=True)
def _clean_device_errors():
    device_error()
    yield
    assert device_error() == 0, "a kernel reported a device-side error"


def make_sae(d_in, d_sae, activation, dtype, k=None):
    sae = oracle.RefSAE(d_in, d_sae, activation, k=k)
    sae.b_enc.normal_(0, 0.1)
    sae.b_dec.normal_(0, 0.1)
    if activation == "jumprelu":
        sae.threshold.uniform_(0.0, 0.5)
    return sae.to(dtype)


def check_encode(got, x, W, b_enc, b_dec, thr, activation, row_nnz=None, tol_d=None, out_dtype=None):
    """The reference test's rule (test_kernels.py:39-44) against the oracle on the same
    rounded inputs."""
    want, want_nnz, pre = oracle.fused_encode(x.cpu(), W.cpu(), b_enc.cpu(), b_dec.cpu(),
                                              None if thr is None else thr.cpu(), activation, out_dtype=out_dtype)
    got = got.cpu()
    tol_d = tol_d or TOL[x.dtype]
    cut = pre - (thr.cpu().float() if activation == "jumprelu" else 0)
    tol = tol_d * (1 + pre.abs().max())
    keep = cut.abs() > tol
    torch.testing.assert_close(got.float()[keep], want.float()[keep], atol=tol, rtol=tol_d)
    if row_nnz is not None:
        assert torch.equal(row_nnz.cpu(), torch.count_nonzero(got, dim=1).int())


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("activation", ["relu", "jumprelu"])
def test_fused_encode(shape, dtype, activation):
    M, d_in, d_sae = shape
    sae = make_sae(d_in, d_sae, activation, dtype)
    x = torch.randn(M, d_in).to(dtype)
    g = sae.to("cuda")
    row_nnz = torch.zeros(M, device="cuda", dtype=torch.int32)
    got = fused_encode(x.cuda(), g.W_enc, g.b_enc, g.b_dec, g.threshold, activation, row_nnz=row_nnz)
    assert got.dtype == dtype
    check_encode(got, x, g.W_enc, g.b_enc, g.b_dec, g.threshold, activation, row_nnz)


@pytest.mark.parametrize("variant", ["tcgen05", "simt"])
def test_fused_encode_strided_weights(variant):
    sae = make_sae(48, 80, "relu", torch.float32).to("cuda")
    W_t = sae.W_enc.T.contiguous().T  # same values, column-major strides
    x = torch.randn(20, 48, device="cuda")
    got = fused_encode(x, W_t, sae.b_enc, sae.b_dec, config={"variant": variant})
    check_encode(got, x, W_t, sae.b_enc, sae.b_dec, None, "relu", tol_d=1e-4)  # IEEE-grade on both kernels


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("layout", ["row", "col", "sliced", "transposed_rows"])
def test_fused_encode_weight_layouts_tcgen05(dtype, layout):
    """Direct TMA of a row-major (MN-major) W_enc, of a column-major (K-major) one, and
    the repack path for layouts TMA cannot read."""
    d_in, d_sae, M = 192, 520, 300
    sae = make_sae(d_in, d_sae, "jumprelu", dtype).to("cuda")
    W = sae.W_enc
    if layout == "col":
        W = W.T.contiguous().T
    elif layout == "sliced":
        W = torch.randn(d_in, d_sae + 3, device="cuda").to(dtype)[:, 1:d_sae + 1]
    elif layout == "transposed_rows":
        W = torch.randn(d_sae, d_in + 5, device="cuda").to(dtype)[:, :d_in].T
    x = torch.randn(M, d_in, device="cuda").to(dtype)
    row_nnz = torch.zeros(M, device="cuda", dtype=torch.int32)
    got = fused_encode(x, W, sae.b_enc, sae.b_dec, sae.threshold, "jumprelu", row_nnz=row_nnz)
    check_encode(got, x, W, sae.b_enc, sae.b_dec, sae.threshold, "jumprelu", row_nnz)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(129, 64, 256), (300, 200, 700), (1000, 512, 3000), (513, 2304, 1024)])
@pytest.mark.parametrize("colmajor", [False, True])
def test_cta_pair_kernel_matches_single_cta_kernel(dtype, shape, colmajor):
    """The CTA-pair tcgen05 kernel (256 x 256 tiles) and the single-CTA one agree, and both
    match the oracle; shapes leave partial pair tiles in M and N."""
    M, d_in, d_sae = shape
    sae = make_sae(d_in, d_sae, "jumprelu", dtype).to("cuda")
    W = sae.W_enc.T.contiguous().T if colmajor else sae.W_enc
    x = torch.randn(M, d_in, device="cuda").to(dtype)
    outs = []
    for variant in ("tcgen05", "tcgen05_1cta"):
        row_nnz = torch.zeros(M, device="cuda", dtype=torch.int32)
        got = fused_encode(x, W, sae.b_enc, sae.b_dec, sae.threshold, "jumprelu", row_nnz=row_nnz,
                           config={"variant": variant})
        check_encode(got, x, W, sae.b_enc, sae.b_dec, sae.threshold, "jumprelu", row_nnz)
        outs.append(got.float())
    torch.testing.assert_close(outs[0], outs[1], atol=TOL[dtype], rtol=TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bdec_kind", ["none", "same", "fp32", "strided"])
@pytest.mark.parametrize("route", ["dense", "csr", "topk"])
def test_pair_kernel_prologue_independent_of_x_layout(dtype, bdec_kind, route):
    """The CTA-pair kernel gives the same bits for the same values of x whatever x's address
    and dtype (contiguous, a 2-byte-offset view, fp32), for b_dec absent, in x's dtype, in
    fp32 and strided, on the dense, CSR-staging and top-k epilogues, and matches the oracle.
    (Builds with SF_FUSED_SHIFT=1 shift contiguous 16-bit x inside the kernel and the other
    layouts through the shift pass, so there this compares the two prologues.)"""
    M, d_in, d_sae = 300, 264, 1000  # M > 128: the pair kernel; d_in % 64 != 0: a partial K block
    sae = make_sae(d_in, d_sae, "jumprelu", dtype).to("cuda")
    x = torch.randn(M, d_in, device="cuda").to(dtype)
    b = {"none": None, "same": sae.b_dec, "fp32": sae.b_dec.float(),
         "strided": torch.stack([sae.b_dec, -sae.b_dec], 1)[:, 0]}[bdec_kind]
    x_odd = torch.zeros(M, d_in + 1, device="cuda", dtype=dtype)[:, 1:]  # 2-byte offset: shifted-copy path
    x_odd.copy_(x)
    x32 = x.float()  # fp32 x with 16-bit W_enc: shifted-copy path
    b_ref = b if b is not None else torch.zeros(d_in, device="cuda", dtype=dtype)

    def run(xx):
        if route == "dense":
            rn = torch.zeros(M, device="cuda", dtype=torch.int32)
            return [fused_encode(xx, sae.W_enc, sae.b_enc, b, sae.threshold, "jumprelu", row_nnz=rn,
                                 out_dtype=dtype), rn]
        if route == "csr":
            return list(encode_csr(xx, sae.W_enc, sae.b_enc, b, sae.threshold, "jumprelu"))
        return list(topk_encode(xx, sae.W_enc, sae.b_enc, b_ref, 16))

    want = run(x)
    # fp32 x stores CSR / top-k values in fp32, so it is compared on the dense route only
    for other in ((x_odd, x32) if route == "dense" else (x_odd,)):
        got = run(other)
        for u, v in zip(got, want):
            assert u.dtype == v.dtype and u.shape == v.shape
            bits = (lambda t: t.view(torch.int16)) if v.dtype in (torch.bfloat16, torch.float16) else (lambda t: t)
            assert torch.equal(bits(u), bits(v))
    if route == "dense":
        check_encode(want[0], x, sae.W_enc, sae.b_enc, b_ref, sae.threshold, "jumprelu", want[1])


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fused_encode_out_dtype(out_dtype):
    sae = make_sae(96, 300, "relu", torch.bfloat16).to("cuda")
    x = torch.randn(70, 96, device="cuda").to(torch.bfloat16)
    row_nnz = torch.zeros(70, device="cuda", dtype=torch.int32)
    got = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, out_dtype=out_dtype, row_nnz=row_nnz)
    assert got.dtype == out_dtype
    check_encode(got, x, sae.W_enc, sae.b_enc, sae.b_dec, None, "relu", row_nnz, out_dtype=out_dtype)


def test_fused_encode_tf32():
    sae = make_sae(256, 512, "relu", torch.float32).to("cuda")
    x = torch.randn(200, 256, device="cuda")
    got = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, allow_tf32=True)
    check_encode(got, x, sae.W_enc, sae.b_enc, sae.b_dec, None, "relu", tol_d=3e-3)


def test_fused_encode_ieee_fp32_rtol_1e5():
    """fp32 IEEE path at rtol 1e-5 (the north-star fp32 tolerance), d_in=768."""
    sae = make_sae(768, 1024, "relu", torch.float32).to("cuda")
    x = torch.randn(256, 768, device="cuda")
    row_nnz = torch.zeros(256, device="cuda", dtype=torch.int32)
    got = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, row_nnz=row_nnz)
    check_encode(got, x, sae.W_enc, sae.b_enc, sae.b_dec, None, "relu", row_nnz, tol_d=1e-5)


def test_fused_encode_row_nnz_accumulates():
    sae = make_sae(64, 256, "relu", torch.bfloat16).to("cuda")
    x = torch.randn(50, 64, device="cuda").to(torch.bfloat16)
    row_nnz = torch.full((50,), 7, device="cuda", dtype=torch.int32)
    got = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, row_nnz=row_nnz)
    assert torch.equal(row_nnz.cpu(), torch.count_nonzero(got, dim=1).int().cpu() + 7)


def test_fused_encode_empty_and_errors():
    sae = make_sae(32, 64, "relu", torch.bfloat16).to("cuda")
    out = fused_encode(torch.empty(0, 32, device="cuda", dtype=torch.bfloat16), sae.W_enc, sae.b_enc, sae.b_dec)
    assert out.shape == (0, 64)
    with pytest.raises(ValueError):
        fused_encode(torch.randn(3, 31, device="cuda"), sae.W_enc, sae.b_enc, sae.b_dec)
    with pytest.raises(ValueError):
        fused_encode(torch.randn(3, 32, device="cuda"), sae.W_enc, sae.b_enc, sae.b_dec, activation="jumprelu")


# ----------------------------------------------------------------------------- CSR

@pytest.mark.parametrize("shape", [(1, 32), (37, 129), (64, 300)])
def test_dense_to_csr_matches_torch(shape):
    f = torch.relu(torch.randn(*shape, device="cuda") - 1.0)
    f[0] = 0  # an empty row
    indptr, indices, values = dense_to_csr(f)
    want = f.to_sparse_csr()
    assert torch.equal(indptr.cpu(), want.crow_indices().cpu())
    assert torch.equal(indices.long().cpu(), want.col_indices().cpu())
    assert torch.equal(values.cpu(), want.values().cpu())


def test_dense_to_csr_all_zero():
    indptr, indices, values = dense_to_csr(torch.zeros(5, 40, device="cuda"))
    assert indptr.tolist() == [0] * 6 and indices.numel() == 0 and values.numel() == 0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(3, 8), (50, 1000), (33, 4099), (7, 65536)])
@pytest.mark.parametrize("strided", [False, True])
def test_dense_to_csr_vs_oracle(dtype, shape, strided):
    M, N = shape
    base = torch.relu(torch.randn(M, N + (3 if strided else 0)) - 2.0).to(dtype)
    base[0, : min(N, 40)] = 1.0  # a dense run
    f = base[:, 1:N + 1] if strided else base
    fc = base.cuda()[:, 1:N + 1] if strided else base.cuda()
    assert fc.is_contiguous() != strided
    ip, ix, vs = dense_to_csr(fc)
    wip, wix, wvs = oracle.dense_to_csr(f)
    assert torch.equal(ip.cpu(), wip) and torch.equal(ix.cpu(), wix)
    assert torch.equal(vs.cpu().float(), wvs.float())


def test_dense_to_csr_special_values():
    f = torch.zeros(4, 100)
    f[0, 3] = float("nan")
    f[1, 5] = -0.0
    f[2, 7] = float("inf")
    f[3, :] = -1.5  # every feature of a row
    ip, ix, vs = dense_to_csr(f.cuda())
    wip, wix, wvs = oracle.dense_to_csr(f)
    assert torch.equal(ip.cpu(), wip) and torch.equal(ix.cpu(), wix)
    assert torch.equal(vs.cpu().view(torch.int32), wvs.view(torch.int32))


def test_dense_to_csr_given_row_nnz_matches_counted():
    f = torch.relu(torch.randn(200, 3000, device="cuda") - 2.5).to(torch.bfloat16)
    rn = torch.count_nonzero(f, dim=1)  # int64, as torch gives it
    a = dense_to_csr(f, rn)
    b = dense_to_csr(f)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


# ----------------------------------------------------------------------------- encode straight to CSR

def _assert_same_csr(a, b):
    for u, v in zip(a, b):
        assert u.dtype == v.dtype and u.shape == v.shape
        bits = (lambda t: t.view(torch.int16)) if v.element_size() == 2 and v.is_floating_point() else (lambda t: t)
        assert torch.equal(bits(u), bits(v))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("activation", ["relu", "jumprelu"])
@pytest.mark.parametrize("shape", [(1, 16, 32), (37, 50, 129), (300, 128, 1000), (700, 256, 4099), (2000, 512, 8192)])
def test_encode_csr_identical_to_dense_route(dtype, activation, shape):
    """Encode straight to CSR gives bit-for-bit the CSR of fused_encode + dense_to_csr
    (fp32: the CUDA-core encoder's staging epilogue, IEEE products)."""
    M, d_in, d_sae = shape
    sae = make_sae(d_in, d_sae, activation, dtype).to("cuda")
    if activation == "relu":
        sae.b_enc.sub_(1.0)  # sparse features
    x = torch.randn(M, d_in, device="cuda").to(dtype)
    rn = torch.zeros(M, device="cuda", dtype=torch.int32)
    want = dense_to_csr(fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, activation, row_nnz=rn), rn)
    got = encode_csr(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, activation)
    _assert_same_csr(got, want)


def test_encode_csr_dense_rows_and_overflow_fallback():
    """A fully active row, an all-zero row, and a staging capacity too small: the overflow
    is detected and the dense route returns the same CSR."""
    sae = make_sae(64, 600, "relu", torch.bfloat16).to("cuda")
    x = torch.randn(200, 64, device="cuda").to(torch.bfloat16)
    x[3] = 0
    sae.b_enc[:] = -5.0
    sae.b_enc[:300] = 5.0  # every row has >= 300 active features
    rn = torch.zeros(200, device="cuda", dtype=torch.int32)
    want = dense_to_csr(fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, row_nnz=rn), rn)
    _assert_same_csr(encode_csr(x, sae.W_enc, sae.b_enc, sae.b_dec), want)
    _assert_same_csr(encode_csr(x, sae.W_enc, sae.b_enc, sae.b_dec, stage_capacity=1000), want)
    _assert_same_csr(encode_csr(x, sae.W_enc, sae.b_enc, sae.b_dec, stage_capacity=0), want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_encode_csr_values_that_round_to_zero(dtype):
    """Pre-activations just above / at / below half the smallest subnormal of the output
    type: the CSR route keeps exactly the values the dense route stores as nonzero."""
    d_in, d_sae, M = 16, 512, 130
    half_min = 2.0 ** -134 if dtype == torch.bfloat16 else 2.0 ** -25
    x = torch.zeros(M, d_in, device="cuda", dtype=dtype)
    W = torch.zeros(d_in, d_sae, device="cuda", dtype=dtype)
    # x = 0 and W = 0 make pre = b_enc exactly; b_enc is fp32 so it can hold the boundary values
    b_enc = torch.zeros(d_sae, device="cuda", dtype=torch.float32)
    vals = torch.tensor([half_min * f for f in (0.5, 0.999, 1.0, 1.001, 1.5, 2.0, 4.0)], dtype=torch.float64)
    b_enc[: vals.numel()] = vals.to(torch.float32).cuda()
    b_enc[100] = 1.0
    b_dec = torch.zeros(d_in, device="cuda", dtype=dtype)
    thr = torch.full((d_sae,), -1.0, device="cuda")
    thr[101] = float("nan")
    b_enc[101] = 1.0
    for act in ("relu", "jumprelu"):
        rn = torch.zeros(M, device="cuda", dtype=torch.int32)
        want = dense_to_csr(fused_encode(x, W, b_enc, b_dec, thr, act, row_nnz=rn), rn)
        got = encode_csr(x, W, b_enc, b_dec, thr, act)
        _assert_same_csr(got, want)
    assert int(want[1].numel()) > 0


def test_encode_csr_fp32_overflow_and_strided_weights():
    """IEEE fp32 staging: a capacity too small is detected and redone densely, and a
    column-major W_enc gives the same CSR as the dense route."""
    sae = make_sae(96, 700, "relu", torch.float32).to("cuda")
    sae.b_enc[:] = -5.0
    sae.b_enc[:300] = 5.0
    x = torch.randn(300, 96, device="cuda")
    W = sae.W_enc.T.contiguous().T
    rn = torch.zeros(300, device="cuda", dtype=torch.int32)
    want = dense_to_csr(fused_encode(x, W, sae.b_enc, sae.b_dec, row_nnz=rn), rn)
    _assert_same_csr(encode_csr(x, W, sae.b_enc, sae.b_dec), want)
    _assert_same_csr(encode_csr(x, W, sae.b_enc, sae.b_dec, stage_capacity=1000), want)


def test_encode_csr_strided_inputs_and_empty():
    sae = make_sae(96, 513, "jumprelu", torch.bfloat16).to("cuda")
    xb = torch.randn(90, 100, device="cuda").to(torch.bfloat16)
    x = xb[:, 2:98]
    W = sae.W_enc.T.contiguous().T
    rn = torch.zeros(90, device="cuda", dtype=torch.int32)
    want = dense_to_csr(fused_encode(x, W, sae.b_enc, sae.b_dec, sae.threshold, "jumprelu", row_nnz=rn), rn)
    _assert_same_csr(encode_csr(x, W, sae.b_enc, sae.b_dec, sae.threshold, "jumprelu"), want)
    ip, ix, vs = encode_csr(torch.empty(0, 96, device="cuda", dtype=torch.bfloat16), W, sae.b_enc, sae.b_dec,
                            sae.threshold, "jumprelu")
    assert ip.tolist() == [0] and ix.numel() == 0 and vs.numel() == 0


def _sparse_sae(d_in, d_sae, activation, k=None):
    """An SAE whose features fire on ~1% of tokens (well inside the default CSR staging)."""
    sae = make_sae(d_in, d_sae, activation, torch.bfloat16, k=k).to("cuda")
    if activation == "relu":
        sae.b_enc.sub_(2.5)
    elif activation == "jumprelu":
        sae.threshold.add_(2.0)
    return sae


@pytest.mark.parametrize("activation", ["relu", "jumprelu"])
@pytest.mark.parametrize("shape", [(37, 50, 129), (700, 256, 4099), (2000, 512, 8192)])
def test_encode_csr_finish_async_matches_synced_csr(activation, shape):
    """The sync-free finish (capacity-sized outputs) places the same pairs in the same slots
    as the synced finish; indptr is identical and the overflow flag is clear."""
    from saeflow_b200.kernels.encode import encode_csr_finish_async, encode_csr_stage

    M, d_in, d_sae = shape
    sae = _sparse_sae(d_in, d_sae, activation)
    x = torch.randn(M, d_in, device="cuda").to(torch.bfloat16)
    want = encode_csr(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, activation)
    h = encode_csr_stage(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, activation, device_consumer=True)
    ip, ix, vs, ovf = encode_csr_finish_async(h)
    assert int(ovf) == 0
    nnz = int(ip[-1])
    assert ix.numel() >= nnz
    _assert_same_csr((ip, ix[:nnz], vs[:nnz]), want)


def test_forward_overflow_is_redone_and_flagged_csr_is_empty():
    """Staging too small for the batch: the async finish writes an all-empty indptr (a decode
    that follows reads nothing) and raises the flag; forward() redoes the batch correctly."""
    from saeflow_b200 import forward
    from saeflow_b200.kernels.encode import encode_csr_finish_async, encode_csr_stage

    sae = make_sae(64, 600, "relu", torch.bfloat16).to("cuda")
    sae.b_enc[:] = -5.0
    sae.b_enc[:550] = 5.0  # > 512 active features per row: the default staging overflows
    x = torch.randn(300, 64, device="cuda").to(torch.bfloat16)
    h = encode_csr_stage(x, sae.W_enc, sae.b_enc, sae.b_dec, None, "relu", device_consumer=True)
    ip, ix, vs, ovf = encode_csr_finish_async(h)
    assert int(ovf) == 1
    assert int(ip.abs().max()) == 0
    rn = torch.zeros(300, device="cuda", dtype=torch.int32)
    f = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, row_nnz=rn)
    want = sparse_decode(*dense_to_csr(f, rn), sae.W_dec, sae.b_dec)
    got = forward(sae, x)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert device_error() == 0


@pytest.mark.parametrize("activation", ["relu", "jumprelu", "topk"])
@pytest.mark.parametrize("chunk", [64, 1000, 5000])
@pytest.mark.parametrize("whole", [True, False])
def test_forward_host_matches_forward(activation, chunk, whole, monkeypatch):
    """forward_host (pinned host in, host out, chunked with overlapped copies) gives bit for
    bit the device forward() of the same chunks, for chunks smaller and larger than the
    batch, with whole-batch device buffers and with two reused chunk buffers, and the
    whole-batch forward() within the bf16 tolerance."""
    from saeflow_b200 import forward, forward_host, ops

    if not whole:
        monkeypatch.setattr(ops, "WHOLE_BATCH_DEVICE_BYTES", 0)
    M, d_in, d_sae = 1500, 256, 4099
    sae = _sparse_sae(d_in, d_sae, activation, k=16 if activation == "topk" else None)
    x = torch.randn(M, d_in).to(torch.bfloat16)
    from saeflow_b200.ops import _chunk_plan

    bounds = [0]
    for n in _chunk_plan(M, chunk):
        bounds.append(bounds[-1] + n)
    want = torch.cat([forward(sae, x[a:b].cuda()).cpu() for a, b in zip(bounds, bounds[1:])])
    whole_out = forward(sae, x.cuda()).cpu()
    got = forward_host(sae, x.pin_memory(), chunk_tokens=chunk)
    # small chunks run on the single-CTA kernel and the whole batch on the CTA pair: a feature
    # whose pre-activation sits on its cut may flip, moving a row by one feature's term
    torch.testing.assert_close(got.float(), whole_out.float(), atol=0.1, rtol=TOL[torch.bfloat16])
    assert got.dtype == want.dtype and got.shape == want.shape and not got.is_cuda
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    out = torch.empty(M, d_in, dtype=torch.bfloat16).pin_memory()
    forward_host(sae, x, out, chunk_tokens=chunk)  # pageable x is pinned internally
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    with pytest.raises(ValueError):
        forward_host(sae, x.cuda())
    assert device_error() == 0


@pytest.mark.parametrize("whole", [True, False])
def test_forward_host_async_pipelined_calls(whole, monkeypatch):
    """Three forward_host_async calls in flight at once, on different batches and outputs,
    waited in reverse order: each equals forward_host of its own batch bit for bit. A call
    whose CSR staging overflows is redone in wait() like forward_host's."""
    from saeflow_b200 import forward_host, forward_host_async, ops

    if not whole:
        monkeypatch.setattr(ops, "WHOLE_BATCH_DEVICE_BYTES", 0)
    sae = _sparse_sae(256, 4099, "jumprelu")
    xs = [torch.randn(M, 256).to(torch.bfloat16).pin_memory() for M in (3000, 700, 2500)]
    want = [forward_host(sae, x, chunk_tokens=1024) for x in xs]
    outs = [torch.empty(x.shape[0], 256, dtype=torch.bfloat16).pin_memory() for x in xs]
    pend = [forward_host_async(sae, x, o, chunk_tokens=1024) for x, o in zip(xs, outs)]
    for p, o, w in reversed(list(zip(pend, outs, want))):
        assert p.wait() is o
        assert torch.equal(o.view(torch.int16), w.view(torch.int16))
    assert pend[0].wait() is outs[0]  # a second wait returns the same output
    # chunk_tokens=None: forward()'s launches (forward_launch_rows), as forward() on the device
    for x in xs:
        assert torch.equal(forward_host_async(sae, x, chunk_tokens=None).wait().view(torch.int16),
                           ops.forward(sae, x.cuda()).cpu().view(torch.int16))
    dense = make_sae(64, 600, "relu", torch.bfloat16).to("cuda")
    dense.b_enc[:] = -5.0
    dense.b_enc[:550] = 5.0  # > 512 active features per row: the default staging overflows
    x = torch.randn(300, 64).to(torch.bfloat16)
    got = forward_host_async(dense, x).wait()
    rn = torch.zeros(300, device="cuda", dtype=torch.int32)
    f = fused_encode(x.cuda(), dense.W_enc, dense.b_enc, dense.b_dec, row_nnz=rn)
    ref = sparse_decode(*dense_to_csr(f, rn), dense.W_dec, dense.b_dec).cpu()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert device_error() == 0


# ----------------------------------------------------------------------------- decode

@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
def test_sparse_decode(shape, dtype):
    M, d_in, d_sae = shape
    sae = make_sae(d_in, d_sae, "relu", dtype).to("cuda")
    f = torch.relu(torch.randn(M, d_sae, device="cuda") - 1.5).to(dtype)  # ~7% density, variable L0
    got = sparse_decode(*dense_to_csr(f), sae.W_dec, sae.b_dec).float()
    want = f.float() @ sae.W_dec.float() + sae.b_dec.float()
    torch.testing.assert_close(got, want, atol=TOL[dtype] * 4, rtol=TOL[dtype])


@pytest.mark.parametrize("D", [8, 24, 256, 768, 2304, 2310, 4096, 5000])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_sparse_decode_widths_vs_oracle(D, dtype):
    M, d_sae, l0 = 97, 3000, 40
    W = torch.randn(d_sae, D).to(dtype)
    W /= W.float().norm(dim=1, keepdim=True).to(dtype)
    b = (torch.randn(D) * 0.1).to(dtype)
    idx = torch.stack([torch.randperm(d_sae)[:l0].sort().values for _ in range(M)])
    vals = (torch.rand(M, l0) * 2).to(dtype)
    ip = torch.arange(0, M * l0 + 1, l0, dtype=torch.int64)
    ix = idx.flatten().to(torch.int32)
    vs = vals.flatten()
    got = sparse_decode(ip.cuda(), ix.cuda(), vs.cuda(), W.cuda(), b.cuda()).cpu()
    want = oracle.sparse_decode(ip, ix, vs, W, b)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(got.float(), want.float(), atol=tol * l0 ** 0.5, rtol=tol)


def test_sparse_decode_strided_w_no_bias_out_dtype():
    W = torch.randn(500, 70, device="cuda").to(torch.float16).T.contiguous().T  # column-major
    f = torch.relu(torch.randn(30, 500, device="cuda") - 1.0).to(torch.float16)
    got = sparse_decode(*dense_to_csr(f), W, out_dtype=torch.float32)
    assert got.dtype == torch.float32
    torch.testing.assert_close(got, f.float() @ W.float(), atol=2e-2, rtol=5e-3)


def test_sparse_decode_empty_rows_and_zero_nnz():
    W = torch.randn(64, 32, device="cuda")
    b = torch.randn(32, device="cuda")
    ip = torch.zeros(6, dtype=torch.int64, device="cuda")
    got = sparse_decode(ip, torch.zeros(0, dtype=torch.int32, device="cuda"), torch.zeros(0, device="cuda"), W, b)
    torch.testing.assert_close(got, b.expand(5, 32))
    assert sparse_decode(torch.zeros(1, dtype=torch.int64, device="cuda"), torch.zeros(0, dtype=torch.int32,
                         device="cuda"), torch.zeros(0, device="cuda"), W).shape == (0, 32)


def test_sparse_decode_out_of_range_index_is_reported_not_faulted():
    """Bounds-checked gather: a bad index contributes nothing and sets device error bit 2."""
    W = torch.randn(16, 32, device="cuda")
    ip = torch.tensor([0, 2], dtype=torch.int64, device="cuda")
    ix = torch.tensor([3, 99], dtype=torch.int32, device="cuda")
    vs = torch.tensor([1.0, 1.0], device="cuda")
    got = sparse_decode(ip, ix, vs, W)
    assert device_error() == 2
    torch.testing.assert_close(got[0], W[3])


# ----------------------------------------------------------------------------- top-k

def assert_topk_matches(vals, idx, x, W, b_enc, b_dec, k):
    """Index sets per row vs the oracle, excluding rows whose k-th and (k+1)-th values tie."""
    wv, wi = oracle.topk_encode(x.cpu(), W.cpu(), b_enc.cpu(), b_dec.cpu(), k)
    f, _, _ = oracle.fused_encode(x.cpu(), W.cpu(), b_enc.cpu(), b_dec.cpu(), activation="relu")
    srt = f.float().sort(dim=1, descending=True).values
    kth, nxt = srt[:, k - 1], srt[:, k] if f.shape[1] > k else torch.full_like(srt[:, 0], -1)
    tol = 1e-2 * (1 + srt[:, 0].abs())
    clean = (kth - nxt).abs() > tol
    vals, idx = vals.cpu(), idx.cpu()
    got_sets = torch.zeros_like(f, dtype=torch.bool).scatter_(1, idx.long(), True)
    want_sets = torch.zeros_like(f, dtype=torch.bool).scatter_(1, wi.long(), True)
    assert torch.equal(got_sets[clean], want_sets[clean])
    # values are sorted descending and equal the oracle's rounded values where sets agree
    assert (vals.float()[:, :-1] >= vals.float()[:, 1:]).all()
    torch.testing.assert_close(vals.float()[clean], wv.float()[clean], atol=tol.max().item(), rtol=1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape,k", [((33, 40, 150), 8), ((300, 128, 2000), 32), ((130, 64, 700), 1),
                                     ((64, 96, 1030), 64), ((40, 64, 512), 100)])
def test_topk_encode_vs_oracle(dtype, shape, k):
    M, d_in, d_sae = shape
    sae = make_sae(d_in, d_sae, "topk", dtype, k=k).to("cuda")
    x = torch.randn(M, d_in, device="cuda").to(dtype)
    vals, idx = topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, k)
    assert vals.dtype == dtype and idx.dtype == torch.int32 and vals.shape == (M, k)
    assert ((idx >= 0) & (idx < d_sae)).all()
    assert_topk_matches(vals, idx, x, sae.W_enc, sae.b_enc, sae.b_dec, k)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_topk_encode_large_k_dense_route(dtype):
    """k above the fused epilogue's limit: encode densely, then select per row."""
    M, d_in, d_sae, k = 50, 64, 900, 150
    sae = make_sae(d_in, d_sae, "topk", dtype, k=k).to("cuda")
    x = torch.randn(M, d_in, device="cuda").to(dtype)
    vals, idx = topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, k)
    assert_topk_matches(vals, idx, x, sae.W_enc, sae.b_enc, sae.b_dec, k)


def test_topk_encode_fp32_tf32_allowed():
    """fp32 with TF32 allowed takes the fused tensor-core route (the reference's tf32 rule)."""
    sae = make_sae(128, 2000, "topk", torch.float32, k=32).to("cuda")
    x = torch.randn(300, 128, device="cuda")
    vals, idx = topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, 32, allow_tf32=True)
    assert_topk_matches(vals, idx, x, sae.W_enc, sae.b_enc, sae.b_dec, 32)


# ----------------------------------------------------------------------------- ops

@pytest.mark.parametrize("activation", ["relu", "jumprelu", "topk"])
def test_ops_match_reference(activation):
    sae = make_sae(40, 150, activation, torch.float32, k=8)
    x = torch.randn(33, 40)
    g = make_sae(40, 150, activation, torch.float32, k=8).to("cuda")
    g.load_state_dict({k: v.cuda() for k, v in sae.state_dict().items()})
    xc = x.cuda()
    torch.testing.assert_close(saeflow_b200.encode(g, xc).cpu(), sae.encode(x), atol=1e-4, rtol=1e-4)
    csr = saeflow_b200.encode_sparse(g, xc)
    torch.testing.assert_close(csr_to_dense(*csr, 150).cpu(), sae.encode(x), atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(saeflow_b200.forward(g, xc).cpu(), sae(x), atol=1e-4, rtol=1e-4)


def test_product_sae_container_runs_cuda_path():
    torch.manual_seed(3)
    s = saeflow_b200.SAE(64, 512, "jumprelu").to("cuda").to(torch.bfloat16)
    s.threshold.fill_(0.05)
    x = torch.randn(20, 64, device="cuda").to(torch.bfloat16)
    want = oracle.forward(_ref_of(s), x.cpu())
    torch.testing.assert_close(s(x).cpu().float(), want.float(), atol=5e-2, rtol=2e-2)


def _ref_of(s):
    r = oracle.RefSAE(s.d_in, s.d_sae, s.activation, k=s.k).to(s.W_enc.dtype)
    r.load_state_dict({k: v.cpu() for k, v in s.state_dict().items()})
    return r


# ----------------------------------------------------------------------------- golden

ENC = Golden("fused_encode")


@pytest.mark.parametrize("case", range(ENC.int("n")))
def test_golden_fused_encode(case):
    """Our kernel on the reference's own inputs vs the reference's own outputs."""
    p = f"c{case}/"
    act = ENC.str(p + "activation")
    x, W, b_enc, b_dec = (ENC.t(p + n).cuda() for n in ("x", "W_enc", "b_enc", "b_dec"))
    thr = ENC.t(p + "threshold")
    thr = thr.cuda() if thr is not None else None
    if ENC.has(p + "colmajor"):
        W = W.T.contiguous().T
    row_nnz = torch.zeros(x.shape[0], device="cuda", dtype=torch.int32)
    got = fused_encode(x, W, b_enc, b_dec, thr, act, row_nnz=row_nnz).cpu()
    want = ENC.t(p + "out")
    _, _, pre = oracle.fused_encode(x.cpu(), W.cpu(), b_enc.cpu(), b_dec.cpu(), None if thr is None else thr.cpu(), act)
    tol_d = TOL[x.dtype]
    cut = pre - (thr.cpu().float() if act == "jumprelu" else 0)
    tol = tol_d * (1 + pre.abs().max())
    keep = cut.abs() > tol
    torch.testing.assert_close(got.float()[keep], want.float()[keep], atol=tol, rtol=tol_d)
    assert torch.equal(row_nnz.cpu(), torch.count_nonzero(got, dim=1).int())
    if ENC.has(p + "row_nnz"):
        clean = keep.all(dim=1)
        assert torch.equal(row_nnz.cpu()[clean], ENC.t(p + "row_nnz")[clean])


CSR = Golden("dense_to_csr")


@pytest.mark.parametrize("case", range(CSR.int("n")))
def test_golden_dense_to_csr_bit_exact(case):
    p = f"c{case}/"
    ip, ix, vs = dense_to_csr(CSR.t(p + "f").cuda())
    assert torch.equal(ip.cpu(), CSR.t(p + "indptr"))
    assert torch.equal(ix.cpu(), CSR.t(p + "indices"))
    want = CSR.t(p + "values")
    bits = (lambda t: t.view(torch.int16)) if want.element_size() == 2 else (lambda t: t.view(torch.int32))
    assert torch.equal(bits(vs.cpu()), bits(want))


DEC = Golden("sparse_decode")


@pytest.mark.parametrize("case", range(DEC.int("n")))
def test_golden_sparse_decode(case):
    p = f"c{case}/"
    W = DEC.t(p + "W_dec")
    got = sparse_decode(*(DEC.t(p + n).cuda() for n in ("indptr", "indices", "values")), W.cuda(),
                        DEC.t(p + "b_dec").cuda()).cpu()
    want = DEC.t(p + "out")
    torch.testing.assert_close(got.float(), want.float(), atol=TOL[W.dtype] * 4, rtol=TOL[W.dtype])


OPS = Golden("ops")


@pytest.mark.parametrize("activation", ["relu", "jumprelu", "topk"])
def test_golden_ops(activation):
    p = f"{activation}/"
    g = oracle.RefSAE(40, 150, activation, k=8).to("cuda")
    for name in ("W_enc", "W_dec", "b_enc", "b_dec", "threshold"):
        if OPS.has(p + name):
            getattr(g, name).copy_(OPS.t(p + name).cuda())
    x = OPS.t(p + "x").cuda()
    torch.testing.assert_close(saeflow_b200.encode(g, x).cpu(), OPS.t(p + "encode"), atol=1e-4, rtol=1e-4)
    ip, ix, vs = saeflow_b200.encode_sparse(g, x)
    assert torch.equal(ip.cpu(), OPS.t(p + "indptr"))
    if activation != "topk":
        assert torch.equal(ix.cpu(), OPS.t(p + "indices"))
    torch.testing.assert_close(saeflow_b200.forward(g, x).cpu(), OPS.t(p + "forward"), atol=1e-4, rtol=1e-4)
