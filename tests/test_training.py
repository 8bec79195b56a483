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
from saeflow_b200.kernels.backward import csc_gather, csr_sddmm, csr_transpose, matvec, transpose

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
@pytest.mark.parametrize("x_grad", [True, False])
def test_backward_matches_autograd_on_the_active_set(activation, dtype, shape, x_grad):
    M, d_in, d_sae = shape
    sae = _sae(d_in, d_sae, activation, dtype, k=12 if activation == "topk" else None)
    x = (torch.randn(M, d_in, device="cuda") * 1.5).to(dtype).requires_grad_(x_grad)
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
    if not x_grad:
        del want["x"]
    for name, w in want.items():
        g = got[name].float()
        assert g.shape == w.shape, name
        scale = w.abs().max().item() + 1e-6
        err = (g - w).abs().max().item() / scale
        assert err < tol, f"{name}: max error {err:.3g} of the gradient's scale"
    assert device_error() == 0


def _random_csr(M, n_cols, density, full_cols=(), seed=3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dense = (torch.rand(M, n_cols, generator=g, device="cuda") < density).float() * torch.randn(
        M, n_cols, generator=g, device="cuda")
    for j in full_cols:  # columns with an entry in every row: they span several ranges
        dense[:, j] = torch.randn(M, generator=g, device="cuda")
    if n_cols > 60:  # a column with an entry in every fourth row (ranked by one warp up to 128)
        dense[::4, 60] = torch.randn((M + 3) // 4, generator=g, device="cuda")
    if M > 5:
        dense[5] = 0      # an empty row
    if n_cols > 13:
        dense[:, 13] = 0  # an empty column
    dense[:, :2] = 0      # empty columns before the first entry
    dense[:, -3:] = 0     # ... and after the last
    csr = dense.to_sparse_csr()
    return dense, csr.crow_indices(), csr.col_indices().to(torch.int32), csr.values()


def test_csr_transpose_is_the_column_view():
    """The column view is the CSR of the transpose: rows ascend within each column."""
    dense, ip, ix, vs = _random_csr(400, 700, 0.03, full_cols=(40, 41))
    M, n_cols = dense.shape
    col_ptr, row_idx, perm, col_idx = csr_transpose(ip, ix, n_cols)
    csc = dense.to_sparse_csc()
    assert torch.equal(col_ptr, csc.ccol_indices())
    assert torch.equal(row_idx.long(), csc.row_indices())
    assert torch.equal(vs[perm], csc.values())
    rows = torch.repeat_interleave(torch.arange(M, device="cuda"), ip[1:] - ip[:-1])
    assert torch.equal(row_idx.long(), rows[perm])
    cols = torch.repeat_interleave(torch.arange(n_cols, device="cuda"), col_ptr[1:] - col_ptr[:-1])
    assert torch.equal(col_idx.long(), cols)
    assert torch.equal(ix.long()[perm], cols)
    assert device_error() == 0


def test_csr_transpose_long_column_across_bitmap_windows():
    """A column with entries in 600000 rows: the in-column sort works in windows of rows."""
    M = 600_000
    r = torch.arange(M, device="cuda")
    second = 10 + (r * 7919) % 1000          # a second entry per row, in a shuffled column
    idx = torch.stack([torch.full_like(r, 5), second], 1).sort(1).values.reshape(-1).to(torch.int32)
    ip = torch.arange(0, 2 * M + 1, 2, device="cuda")
    col_ptr, row_idx, perm, col_idx = csr_transpose(ip, idx, 1010)
    assert int(col_ptr[6] - col_ptr[5]) == M
    assert torch.equal(row_idx[col_ptr[5]:col_ptr[6]].long(), r)
    rows = torch.repeat_interleave(torch.arange(M, device="cuda"), 2)
    assert torch.equal(row_idx.long(), rows[perm])
    for j in (10, 500, 1009):
        seg = row_idx[col_ptr[j]:col_ptr[j + 1]].long()
        assert torch.equal(seg, r[second == j])
    assert device_error() == 0


@pytest.mark.parametrize("case", [
    # (M, n_cols, D, density, full columns, R dtype, out dtype)
    (400, 700, 96, 0.03, (40, 41), torch.float32, torch.float32),   # columns across ranges
    (800, 3000, 128, 0.01, (7, 2000), torch.bfloat16, torch.bfloat16),
    (300, 500, 64, 0.05, (), torch.float16, torch.float32),
    (50, 90, 40, 0.02, (), torch.bfloat16, torch.float32),            # few entries: one range
    (200, 300, 37, 0.05, (3,), torch.float32, torch.bfloat16),        # unaligned rows: plain kernel
    (64, 200, 4104, 0.05, (9,), torch.float32, torch.float32),        # two D-pieces, dots apart
    (300, 400, 2304, 0.05, (1, 2), torch.bfloat16, torch.bfloat16),   # the benchmark's row width
])
def test_csc_gather_against_torch(case):
    M, n_cols, D, density, full, rdt, odt = case
    dense, ip, ix, vs = _random_csr(M, n_cols, density, full_cols=full)
    vs = vs.to(rdt)
    vs[::7] = 0  # entries whose value is zero get no dot product
    dense = csr_to_dense(ip, ix, vs.float(), n_cols)
    col = csr_transpose(ip, ix, n_cols)
    g = torch.Generator(device="cuda").manual_seed(5)
    R = torch.randn(M, D, generator=g, device="cuda").to(rdt)
    W = torch.randn(n_cols, D, generator=g, device="cuda").to(rdt)
    out, sums, dots = csc_gather(*col, vs, R, W=W, out_dtype=odt, col_sums=True)
    assert out.dtype == odt and out.shape == (n_cols, D)
    want = (dense.double().T @ R.double()).float()
    tol = 2e-5 if odt == torch.float32 else 8e-3
    torch.testing.assert_close(out.float(), want.to(odt).float(), atol=tol * (1 + M ** 0.5), rtol=tol)
    torch.testing.assert_close(sums, dense.double().sum(0).float(), atol=1e-5, rtol=1e-5)
    rows = torch.repeat_interleave(torch.arange(M, device="cuda"), ip[1:] - ip[:-1])
    want_dots = (R.float()[rows] * W.float()[ix.long()]).sum(1) * (vs.float() != 0)
    torch.testing.assert_close(dots, want_dots, atol=2e-4 * D ** 0.5, rtol=1e-4)
    torch.testing.assert_close(dots, csr_sddmm(ip, ix, vs, R, W), atol=2e-4 * D ** 0.5, rtol=1e-4)
    # the sums are taken in the column view's fixed order: the same bits every call, with or
    # without the dot products and column sums
    assert torch.equal(csc_gather(*col, vs, R, out_dtype=odt), out)
    out2, _, dots2 = csc_gather(*col, vs, R, W=W, out_dtype=odt, col_sums=True)
    assert torch.equal(out2, out) and torch.equal(dots2, dots)
    assert device_error() == 0


def test_csc_gather_without_entries():
    M, n_cols, D = 10, 20, 32
    ip = torch.zeros(M + 1, dtype=torch.int64, device="cuda")
    ix = torch.zeros(0, dtype=torch.int32, device="cuda")
    vs = torch.zeros(0, dtype=torch.float32, device="cuda")
    col = csr_transpose(ip, ix, n_cols)
    out, sums = csc_gather(*col, vs, torch.randn(M, D, device="cuda"), out_dtype=torch.bfloat16, col_sums=True)
    assert torch.equal(out, torch.zeros(n_cols, D, dtype=torch.bfloat16, device="cuda"))
    assert torch.equal(sums, torch.zeros(n_cols, device="cuda"))
    assert device_error() == 0


def test_backward_is_deterministic():
    """Two backward passes on the same inputs give the same gradient bits."""
    sae = _sae(256, 2048, "jumprelu", torch.bfloat16)
    x = (torch.randn(1000, 256, device="cuda") * 1.5).to(torch.bfloat16)
    r = torch.randn(1000, 256, device="cuda").to(torch.bfloat16)
    grads = []
    for _ in range(2):
        for name in ("W_enc", "b_enc", "W_dec", "b_dec"):
            getattr(sae, name).grad = None
        training.forward(sae, x).backward(r)
        grads.append([getattr(sae, n).grad.clone() for n in ("W_enc", "b_enc", "W_dec", "b_dec")])
    for a, b in zip(*grads):
        assert torch.equal(a, b)
    assert device_error() == 0


@pytest.mark.parametrize("src,dst", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                     (torch.float16, torch.float32), (torch.float16, torch.bfloat16)])
@pytest.mark.parametrize("shape", [(1, 1), (33, 70), (300, 4099), (64, 130), (130, 4098), (64, 136), (264, 4096)])
def test_transpose_kernel(src, dst, shape):
    x = torch.randn(*shape, device="cuda").to(src)
    got = transpose(x, dst)
    assert got.shape == (shape[1], shape[0]) and got.dtype == dst and got.is_contiguous()
    assert torch.equal(got, x.t().to(dst))
    for extra in (5, 6):  # odd and even row pitch
        strided = torch.randn(shape[0], shape[1] + extra, device="cuda").to(src)[:, 2:2 + shape[1]]
        assert torch.equal(transpose(strided, dst), strided.t().to(dst))
    padded = torch.randn(shape[0], shape[1] + 8, device="cuda").to(src)[:, :shape[1]]  # aligned, pitch + 8
    assert torch.equal(transpose(padded, dst), padded.t().to(dst))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 1), (37, 1000), (2304, 4096)])
def test_matvec(dtype, shape):
    A = torch.randn(*shape, device="cuda").to(dtype)
    x = torch.randn(shape[1], device="cuda")
    want = A.double() @ x.double()
    torch.testing.assert_close(matvec(A, x), want.float(), atol=1e-4 * shape[1] ** 0.5, rtol=1e-4)
    strided = torch.randn(shape[0], shape[1] + 3, device="cuda").to(dtype)[:, 1:1 + shape[1]]
    torch.testing.assert_close(matvec(strided, x), (strided.double() @ x.double()).float(),
                               atol=1e-4 * shape[1] ** 0.5, rtol=1e-4)
