"""Kernel-level backward of the sparse forward (libsaeflow_b200.so, csrc/backward.cu).

The reference has no backward kernels (its roadmap, README.md:244). These ops are what
the gradient of x_hat = decode(encode(x)) needs on a CSR pattern:

- csr_transpose: the column view (col_ptr, row_idx, perm, col_idx) of a CSR pattern, rows
  ascending within each column;
- csc_gather: per-column sums of value-weighted gathered rows (weight gradients), optionally
  with the per-entry dot products of each gathered row with the column's row of a second
  matrix (the gradient at the active features) in the same pass;
- csr_sddmm: those dot products alone, on the CSR pattern;
- transpose: a tiled transpose with a dtype conversion;
- matvec: a matrix-vector product (the token sum of dx, from W_enc and the sums of dpre).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _abi


def transpose(x, dtype=None):
    """x.T as a new row-major tensor in `dtype` (default x's), by a tiled transpose kernel."""
    dev = _abi.require_cuda(("x", x))
    if x.stride(-1) != 1:
        x = x.contiguous()
    out = torch.empty(x.shape[1], x.shape[0], dtype=dtype or x.dtype, device=dev)
    lib = _abi.load()
    with torch.cuda.device(dev):
        _abi.check(lib.sf_transpose(ctypes.byref(_abi.matrix(x, "x")), ctypes.byref(_abi.matrix(out, "out")),
                                    _abi.stream_of(dev)))
    return out


def csr_transpose(indptr, indices, n_cols):
    """(col_ptr int64 [n_cols+1], row_idx int32 [nnz], perm int64 [nnz], col_idx int32 [nnz])
    of a CSR pattern: entry p of the column view is CSR entry perm[p], in row row_idx[p] and
    column col_idx[p]; within a column the rows ascend (the CSR of the transpose)."""
    M, nnz = indptr.numel() - 1, indices.numel()
    dev = _abi.require_cuda(("indptr", indptr), ("indices", indices))
    lib = _abi.load()
    col_ptr = torch.empty(n_cols + 1, dtype=torch.int64, device=dev)
    row_idx = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    perm = torch.empty(max(nnz, 1), dtype=torch.int64, device=dev)
    col_idx = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        need = ctypes.c_size_t(0)
        _abi.check(lib.sf_csr_transpose_workspace(n_cols, nnz, ctypes.byref(need)))
        ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
        _abi.check(lib.sf_csr_transpose(indptr.data_ptr(), M, indices.data_ptr() if nnz else None, nnz, n_cols,
                                        col_ptr.data_ptr(), row_idx.data_ptr(), perm.data_ptr(), col_idx.data_ptr(),
                                        ws.data_ptr(), ws.numel(), _abi.stream_of(dev)))
    return col_ptr, row_idx[:nnz], perm[:nnz], col_idx[:nnz]


def csr_sddmm(indptr, indices, values, G, W):
    """fp32 [nnz]: out[e] = (values[e] != 0) * G[row(e)] . W[indices[e]]."""
    M = indptr.numel() - 1
    dev = _abi.require_cuda(("indptr", indptr), ("indices", indices), ("values", values), ("G", G), ("W", W))
    out = torch.empty(indices.numel(), dtype=torch.float32, device=dev)
    if M == 0 or indices.numel() == 0:
        return out.zero_()
    G = G if G.stride(-1) == 1 else G.contiguous()
    W = W if W.stride(-1) == 1 else W.contiguous()
    if G.dtype != W.dtype:
        G = G.to(W.dtype)
    lib = _abi.load()
    with torch.cuda.device(dev):
        _abi.check(lib.sf_csr_sddmm(indptr.data_ptr(), M, indices.data_ptr(), ctypes.byref(_abi.matrix(G, "G")),
                                    ctypes.byref(_abi.matrix(W, "W")), values.data_ptr(),
                                    _abi.dtype_code(values.dtype, "values"), out.data_ptr(), _abi.stream_of(dev)))
    return out


def matvec(A, x):
    """fp32 [A.shape[0]]: y[i] = sum_j A[i, j] * x[j] (x fp32), fp32 sums in a fixed order."""
    dev = _abi.require_cuda(("A", A), ("x", x))
    A = A if A.stride(-1) == 1 else A.contiguous()
    x = x.to(torch.float32).contiguous()
    if x.numel() != A.shape[1]:
        raise ValueError(f"x has {x.numel()} elements, A has {A.shape[1]} columns")
    y = torch.empty(A.shape[0], dtype=torch.float32, device=dev)
    lib = _abi.load()
    with torch.cuda.device(dev):
        _abi.check(lib.sf_matvec(ctypes.byref(_abi.matrix(A, "A")), x.data_ptr(), y.data_ptr(), _abi.stream_of(dev)))
    return y


def csc_gather(col_ptr, row_idx, perm, col_idx, values, R, *, W=None, out_dtype=torch.float32, col_sums=False):
    """Per-column gather over a column view from csr_transpose (p over column j's entries):

    out [n_cols, R.shape[1]] in out_dtype: out[j] = sum_p values[perm[p]] * R[row_idx[p]]
    (fp32 sums in the view's row order); with col_sums, also fp32 [n_cols]: sum_p values[perm[p]];
    with W [n_cols, R.shape[1]] (R's dtype), also fp32 dots [nnz] in CSR order:
    dots[perm[p]] = (values[perm[p]] != 0) * R[row_idx[p]] . W[j].

    Returns out, then the column sums and the dots when asked for."""
    n_cols = col_ptr.numel() - 1
    nnz = row_idx.numel()
    dev = _abi.require_cuda(("col_ptr", col_ptr), ("row_idx", row_idx), ("perm", perm), ("col_idx", col_idx),
                            ("values", values), ("R", R))
    R = R if R.stride(-1) == 1 else R.contiguous()
    out = torch.empty(n_cols, R.shape[1], dtype=out_dtype, device=dev)
    sums = torch.empty(n_cols, dtype=torch.float32, device=dev) if col_sums else None
    dots = None
    if W is not None:
        _abi.require_cuda(("W", W))
        W = W if W.stride(-1) == 1 else W.contiguous()
        if W.dtype != R.dtype:
            raise ValueError(f"W ({W.dtype}) and R ({R.dtype}) must have one dtype")
        dots = torch.empty(max(nnz, 1), dtype=torch.float32, device=dev)
    lib = _abi.load()
    with torch.cuda.device(dev):
        Rm = _abi.matrix(R, "R")
        need = ctypes.c_size_t(0)
        _abi.check(lib.sf_csc_gather_workspace(nnz, ctypes.byref(Rm), ctypes.byref(need)))
        ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
        Wm = _abi.matrix(W, "W") if W is not None else None
        _abi.check(lib.sf_csc_gather(col_ptr.data_ptr(), n_cols, col_idx.data_ptr() if nnz else None, nnz,
                                     row_idx.data_ptr() if nnz else None, perm.data_ptr() if nnz else None,
                                     values.data_ptr() if nnz else None, _abi.dtype_code(values.dtype, "values"),
                                     ctypes.byref(Rm), ctypes.byref(Wm) if Wm is not None else None,
                                     dots.data_ptr() if dots is not None else None,
                                     ctypes.byref(_abi.matrix(out, "out")),
                                     sums.data_ptr() if sums is not None else None, ws.data_ptr(), ws.numel(),
                                     _abi.stream_of(dev)))
    res = (out,)
    if col_sums:
        res += (sums,)
    if W is not None:
        res += (dots[:nnz],)
    return res[0] if len(res) == 1 else res
