"""CPU restatement of saeflow's SAE hot path — TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Floating-point sums are taken in float64 (the kernels sum in fp32), integer and index
work (nonzero counts, CSR structure, top-k selection order) is exact. Inputs are CPU
torch tensors; outputs are CPU torch tensors.
"""

from __future__ import annotations

import numpy as np
import torch
from torch import nn

ACTIVATIONS = ("relu", "jumprelu", "topk")


class RefSAE(nn.Module):
    """Restatement of saeflow/reference.py:9-52 (plain PyTorch SAE, SAELens names).

    Constructor draws (reference.py:25-33): W_dec ~ N(0,1) rows normalised to unit L2,
    W_enc = W_dec.T (contiguous), b_enc = b_dec = 0, threshold = 0 for JumpReLU.
    """

    def __init__(self, d_in, d_sae, activation="relu", k=None, device=None, dtype=torch.float32):
        super().__init__()
        if activation not in ACTIVATIONS:  # reference.py:19-20
            raise ValueError(f"activation must be one of {ACTIVATIONS}, got {activation!r}")
        if activation == "topk" and not k:  # reference.py:21-22
            raise ValueError("topk activation needs k")
        self.d_in, self.d_sae, self.activation, self.k = d_in, d_sae, activation, k
        W_dec = torch.randn(d_sae, d_in, device=device)
        W_dec /= W_dec.norm(dim=1, keepdim=True)
        self.W_dec = nn.Parameter(W_dec.to(dtype))
        self.W_enc = nn.Parameter(W_dec.T.contiguous().to(dtype))
        self.b_enc = nn.Parameter(torch.zeros(d_sae, device=device, dtype=dtype))
        self.b_dec = nn.Parameter(torch.zeros(d_in, device=device, dtype=dtype))
        self.threshold = (
            nn.Parameter(torch.zeros(d_sae, device=device, dtype=dtype)) if activation == "jumprelu" else None
        )
        self.requires_grad_(False)

    def encode_pre(self, x):  # reference.py:36-37
        return (x - self.b_dec) @ self.W_enc + self.b_enc

    def encode(self, x):  # reference.py:39-46
        pre = self.encode_pre(x)
        if self.activation == "relu":
            return torch.relu(pre)
        if self.activation == "jumprelu":
            return torch.relu(pre) * (pre > self.threshold)
        top = pre.topk(self.k, dim=-1)
        return torch.zeros_like(pre).scatter_(-1, top.indices, torch.relu(top.values))

    def decode(self, f):  # reference.py:48-49
        return f @ self.W_dec + self.b_dec

    def forward(self, x):  # reference.py:51-52
        return self.decode(self.encode(x))


def to_dtype(t, dtype, rounding="nearest"):
    """fp32 -> `dtype`. rounding="truncate" reproduces Triton's CPU interpreter, which
    converts fp32 to bf16 by dropping the low 16 bits (the reference's golden vectors were
    made under it); compiled Triton on a GPU, like these kernels, rounds to nearest even."""
    if rounding == "truncate" and dtype == torch.bfloat16:
        return (t.float().contiguous().view(torch.int32) & ~0xFFFF).view(torch.float32).to(torch.bfloat16)
    if rounding not in ("nearest", "truncate"):
        raise ValueError(f"rounding must be 'nearest' or 'truncate', got {rounding!r}")
    return t.to(dtype)


def _shifted(x, b_dec, w_dtype, rounding="nearest"):
    """(x - b_dec) in fp32, rounded to W_enc's dtype: the reference kernel prologue
    (saeflow/kernels/encode.py:72, `(x.to(fp32) - b_dec.to(fp32)).to(w.dtype)`)."""
    xs = x.float()
    if b_dec is not None:
        xs = xs - b_dec.float()
    return to_dtype(xs, w_dtype, rounding)


def encode_pre(x, W_enc, b_enc, b_dec, chunk=4096, col_chunk=16384, rounding="nearest"):
    """fp32 pre-activation acc + b_enc (encode.py:62-77), products summed in float64.

    W_enc is widened to float64 one block of `col_chunk` columns at a time, so a large SAE
    (4096 x 131072) needs no float64 copy of the whole matrix."""
    xs = _shifted(x, b_dec, W_enc.dtype, rounding).double()
    b = b_enc.float()
    N = W_enc.shape[1]
    out = torch.empty(x.shape[0], N, dtype=torch.float32)
    for c0 in range(0, N, col_chunk):
        c1 = min(N, c0 + col_chunk)
        W = W_enc[:, c0:c1].double()
        for i in range(0, x.shape[0], chunk):
            out[i:i + chunk, c0:c1] = (xs[i:i + chunk] @ W).float() + b[c0:c1]
    return out


def fused_encode(x, W_enc, b_enc, b_dec, threshold=None, activation="relu", out_dtype=None, rounding="nearest"):
    """(out, row_nnz, pre) of the reference fused encoder (encode.py:77-91).

    out = max(pre, 0), zeroed where not (pre > threshold) for JumpReLU, stored in
    `out_dtype or x.dtype`; row_nnz counts the stored nonzeros (int32). `rounding` is the
    fp32 -> bf16 conversion of the shifted input and of the output (see to_dtype)."""
    if activation not in ("relu", "jumprelu"):  # encode.py:107-108
        raise ValueError(f"fused_encode supports ['relu', 'jumprelu'], got {activation!r}")
    if activation == "jumprelu" and threshold is None:  # encode.py:109-110
        raise ValueError("jumprelu needs a threshold")
    pre = encode_pre(x, W_enc, b_enc, b_dec, rounding=rounding)
    out = torch.clamp_min(pre, 0.0)
    if activation == "jumprelu":
        out = torch.where(pre > threshold.float(), out, torch.zeros((), dtype=out.dtype))
    out = to_dtype(out, out_dtype or x.dtype, rounding)
    row_nnz = (out.float() != 0).sum(dim=1).to(torch.int32)
    return out, row_nnz, pre


def dense_to_csr(f, row_nnz=None):
    """Canonical CSR of f's nonzeros (decode.py:77-94 with _compact_kernel :61-74).

    Nonzero test `f != 0.0` (NaN counts, -0.0 does not); indices column-sorted per row;
    indptr int64 [M+1], indices int32, values in f's dtype (bit-exact copies)."""
    fv = f.float().numpy()
    nz = fv != 0.0
    counts = nz.sum(axis=1).astype(np.int64)
    if row_nnz is not None and not np.array_equal(np.asarray(row_nnz, dtype=np.int64), counts):
        raise ValueError("row_nnz disagrees with the nonzeros of f")
    indptr = np.zeros(f.shape[0] + 1, dtype=np.int64)
    np.cumsum(counts, out=indptr[1:])
    rows, cols = np.nonzero(nz)
    values = f[torch.from_numpy(rows), torch.from_numpy(cols)]
    return torch.from_numpy(indptr), torch.from_numpy(cols.astype(np.int32)), values


def sparse_decode(indptr, indices, values, W_dec, b_dec=None, out_dtype=None):
    """b_dec + sum_j values[j] * W_dec[indices[j]] per row (decode.py:28-55), float64 sums.

    The row sums are one float64 CSR x dense product over the W_dec rows the CSR references
    (gathered and renumbered first, so a 2^20-row W_dec is never widened whole); the sum
    order does not matter at float64 precision for these checks. Only indptr's ranges of
    indices / values are read."""
    M = indptr.numel() - 1
    D, N = W_dec.shape[1], W_dec.shape[0]
    ip = indptr.long()
    nnz = int(ip[-1]) if M else 0
    acc = torch.zeros(M, D, dtype=torch.float64)
    if nnz:
        idx = indices[:nnz].long()
        if int(idx.min()) < 0 or int(idx.max()) >= N:
            raise ValueError("sparse_decode: an index is outside W_dec's rows")
        used, local = torch.unique(idx, return_inverse=True)
        with torch.sparse.check_sparse_tensor_invariants(False):
            csr = torch.sparse_csr_tensor(ip, local, values[:nnz].double(), (M, used.numel()))
            acc += torch.sparse.mm(csr, W_dec[used].double())
    if b_dec is not None:
        acc += b_dec.double()
    return acc.to(out_dtype or W_dec.dtype)


def topk_encode(x, W_enc, b_enc, b_dec, k):
    """TopK encode of saeflow/ops.py:12-16: the ReLU output stored in x.dtype, then the k
    largest per row. Returns (values [M,k], indices int32 [M,k]) ordered by value
    descending; equal values are ordered by lower feature index."""
    f, _, pre = fused_encode(x, W_enc, b_enc, b_dec, activation="relu")
    _, order = torch.sort(-f.float(), dim=1, stable=True)
    idx = order[:, :k]
    return f.gather(1, idx), idx.to(torch.int32)


def encode_sparse(sae, x):
    """CSR features (saeflow/ops.py:29-39)."""
    M = x.shape[0]
    if sae.activation == "topk":
        vals, idx = topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.k)
        indptr = torch.arange(0, M * sae.k + 1, sae.k, dtype=torch.int64)
        return indptr, idx.flatten(), vals.flatten()
    f, row_nnz, _ = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation)
    return dense_to_csr(f, row_nnz)


def forward(sae, x):
    """decode_sparse(encode_sparse(x)) (saeflow/ops.py:42-49)."""
    return sparse_decode(*encode_sparse(sae, x), sae.W_dec, sae.b_dec)
