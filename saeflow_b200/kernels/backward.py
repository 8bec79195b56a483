"""Kernel-level backward of the sparse forward (libsaeflow_b200.so, csrc/backward.cu).

The reference has no backward kernels (its roadmap, README.md:244). These three ops are
what the gradient of x_hat = decode(encode(x)) needs on a CSR pattern:

- csr_transpose: the column view (col_ptr, row_idx, perm) of a CSR pattern;
- csr_sddmm: per-entry dot products of a dense row with a dense row (the gradient at the
  active features);
- csc_accumulate: per-column sums of value-weighted gathered rows (weight gradients).
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
    """(col_ptr int64 [n_cols+1], row_idx int32 [nnz], perm int64 [nnz], col_order int32
    [n_cols + 1]) of a CSR pattern. Within a column the entries are in no fixed order;
    col_order lists the columns with more than 256 entries first and ends with their count
    (csc_accumulate's schedule)."""
    M, nnz = indptr.numel() - 1, indices.numel()
    dev = _abi.require_cuda(("indptr", indptr), ("indices", indices))
    lib = _abi.load()
    col_ptr = torch.empty(n_cols + 1, dtype=torch.int64, device=dev)
    row_idx = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    perm = torch.empty(max(nnz, 1), dtype=torch.int64, device=dev)
    order = torch.empty(n_cols + 1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        need = ctypes.c_size_t(0)
        _abi.check(lib.sf_csr_transpose_workspace(n_cols, ctypes.byref(need)))
        ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
        _abi.check(lib.sf_csr_transpose(indptr.data_ptr(), M, indices.data_ptr() if nnz else None, nnz, n_cols,
                                        col_ptr.data_ptr(), row_idx.data_ptr(), perm.data_ptr(), order.data_ptr(),
                                        ws.data_ptr(), ws.numel(), _abi.stream_of(dev)))
    return col_ptr, row_idx[:nnz], perm[:nnz], order


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


def csc_accumulate(col_ptr, row_idx, perm, col_order, values, R, *, col_sums=False):
    """fp32 [n_cols, R.shape[1]] (and optionally fp32 [n_cols] column sums of the values):
    out[j] = sum over column j's entries p of values[perm[p]] * R[row_idx[p]]."""
    n_cols = col_ptr.numel() - 1
    dev = _abi.require_cuda(("col_ptr", col_ptr), ("row_idx", row_idx), ("perm", perm), ("values", values), ("R", R))
    out = torch.empty(n_cols, R.shape[1], dtype=torch.float32, device=dev)
    sums = torch.zeros(n_cols, dtype=torch.float32, device=dev) if col_sums else None
    R = R if R.stride(-1) == 1 else R.contiguous()
    lib = _abi.load()
    with torch.cuda.device(dev):
        _abi.check(lib.sf_csc_accumulate(col_ptr.data_ptr(), n_cols,
                                         col_order.data_ptr() if col_order is not None and n_cols else None,
                                         row_idx.numel(),
                                         row_idx.data_ptr() if row_idx.numel() else None,
                                         perm.data_ptr() if perm.numel() else None,
                                         values.data_ptr() if values.numel() else None,
                                         _abi.dtype_code(values.dtype, "values"), ctypes.byref(_abi.matrix(R, "R")),
                                         out.data_ptr(), out.stride(0), sums.data_ptr() if sums is not None else None,
                                         _abi.stream_of(dev)))
    return (out, sums) if col_sums else out
