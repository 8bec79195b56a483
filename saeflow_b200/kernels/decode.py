"""Sparse SAE decode and the dense -> CSR path, mirroring saeflow/kernels/decode.py.

SAE features are CSR: row m's active features are indices[indptr[m]:indptr[m+1]] with
matching values, and decode computes

    x_hat[m] = b_dec + sum_j values[j] * W_dec[indices[j]]

reading only each token's active W_dec rows. Signatures, dtypes and the single host
sync match the reference (decode.py:77-126); the kernels live in libsaeflow_b200.so.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _abi


def dense_to_csr(f, row_nnz=None):
    """Dense features [M, d_sae] -> (indptr int64 [M+1], indices int32 [nnz], values [nnz]).

    row_nnz: per-row nonzero counts if already known (fused_encode produces them in its
    epilogue); otherwise counted here. One host sync sizes the outputs.
    """
    M, N = f.shape
    dev = _abi.require_cuda(("f", f), ("row_nnz", row_nnz))
    lib = _abi.load()
    fm = _abi.matrix(f, "f")
    with torch.cuda.device(dev):
        s = _abi.stream_of(dev)
        if row_nnz is None:
            row_nnz = torch.empty(M, dtype=torch.int32, device=dev)
            _abi.check(lib.sf_row_nnz(ctypes.byref(fm), row_nnz.data_ptr(), s))
        else:
            if row_nnz.numel() != M:
                raise ValueError(f"row_nnz has {row_nnz.numel()} entries for {M} rows")
            if row_nnz.dtype != torch.int32 or not row_nnz.is_contiguous():
                row_nnz = row_nnz.to(torch.int32).contiguous()
        indptr = torch.empty(M + 1, dtype=torch.int64, device=dev)
        _abi.check(lib.sf_csr_indptr(row_nnz.data_ptr() if M else None, M, indptr.data_ptr(), s))
        nnz = int(indptr[-1])  # the one host sync (decode.py:88)
        indices = torch.empty(nnz, dtype=torch.int32, device=dev)
        values = torch.empty(nnz, dtype=f.dtype, device=dev)
        if nnz:
            _abi.check(lib.sf_dense_to_csr(ctypes.byref(fm), indptr.data_ptr(), indices.data_ptr(),
                                           values.data_ptr(), _abi.dtype_code(f.dtype, "f"), s))
    return indptr, indices, values


def _csr_operands(indptr, indices, values):
    if indptr.dim() != 1 or indices.dim() != 1 or values.dim() != 1:
        raise ValueError("indptr, indices and values must be 1-D")
    if indices.numel() != values.numel():
        raise ValueError(f"indices has {indices.numel()} entries but values has {values.numel()}")
    if indptr.dtype != torch.int64 or not indptr.is_contiguous():
        indptr = indptr.to(torch.int64).contiguous()
    if indices.dtype != torch.int32 or not indices.is_contiguous():
        indices = indices.to(torch.int32).contiguous()
    if not values.is_contiguous():
        values = values.contiguous()
    return indptr, indices, values


def sparse_decode(indptr, indices, values, W_dec, b_dec=None, *, out_dtype=None, config=None, out=None):
    """CSR features @ W_dec (+ b_dec) -> [M, d_in], accumulated in fp32.

    W_dec: [d_sae, d_in], any strides (row-major is the fast case: gathered rows are
    contiguous 16-byte vectors). `config` is accepted for signature parity with the
    reference (decode.py:97) and has no effect: the kernel picks its D-slicing from d_in.
    out: optional [M, d_in] CUDA tensor to write into (any strides; its dtype wins over
    out_dtype). indices / values may be longer than indptr[M]: only indptr's ranges are read.
    """
    del config
    M = indptr.numel() - 1
    D = W_dec.shape[1]
    dev = _abi.require_cuda(("indptr", indptr), ("indices", indices), ("values", values), ("W_dec", W_dec),
                            ("b_dec", b_dec), ("out", out))
    if out is None:
        out = torch.empty(M, D, device=dev, dtype=out_dtype or W_dec.dtype)
    elif tuple(out.shape) != (M, D):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(M, D)}")
    if M == 0:
        return out
    indptr, indices, values = _csr_operands(indptr, indices, values)
    lib = _abi.load()
    wm, om = _abi.matrix(W_dec, "W_dec"), _abi.matrix(out, "out")
    bd = _abi.vector(b_dec, "b_dec")
    with torch.cuda.device(dev):
        _abi.check(lib.sf_sparse_decode(indptr.data_ptr(), M, indices.data_ptr() if indices.numel() else None,
                                        values.data_ptr() if values.numel() else None,
                                        _abi.dtype_code(values.dtype, "values"), ctypes.byref(wm), _abi.ref(bd),
                                        ctypes.byref(om), _abi.stream_of(dev)))
    return out


def csr_to_dense(indptr, indices, values, d_sae):
    """Inverse of dense_to_csr, via torch's own CSR tensor. For tests and inspection
    (decode.py:123-126)."""
    M = indptr.numel() - 1
    return torch.sparse_csr_tensor(indptr, indices.long(), values, (M, d_sae)).to_dense()


def topk_encode(x, W_enc, b_enc, b_dec, k, *, allow_tf32=None):
    """Per-row top-k of relu((x - b_dec) @ W_enc + b_enc), selected in the GEMM epilogue.

    Returns (values [M, k] in x.dtype, indices int32 [M, k]), each row sorted by value
    descending with ties broken by lower feature index. Equivalent to the reference's
    `fused_encode(..., "relu").topk(k)` (saeflow/ops.py:12-16) without writing the dense
    [M, d_sae] output.
    """
    M, K = x.shape
    K_w, N = W_enc.shape
    if K != K_w:
        raise ValueError(f"x has d_in={K} but W_enc has d_in={K_w}")
    if not k or k < 1 or k > N:
        raise ValueError(f"k={k} must be in [1, d_sae={N}]")
    dev = _abi.require_cuda(("x", x), ("W_enc", W_enc), ("b_enc", b_enc), ("b_dec", b_dec))
    values = torch.empty(M, k, device=dev, dtype=x.dtype)
    indices = torch.empty(M, k, device=dev, dtype=torch.int32)
    if M == 0:
        return values, indices
    if allow_tf32 is None:
        allow_tf32 = torch.backends.cuda.matmul.allow_tf32
    lib = _abi.load()
    xm, wm = _abi.matrix(x, "x"), _abi.matrix(W_enc, "W_enc")
    be, bd = _abi.vector(b_enc, "b_enc"), _abi.vector(b_dec, "b_dec")
    with torch.cuda.device(dev):
        need = ctypes.c_size_t(0)
        _abi.check(lib.sf_topk_encode_workspace(ctypes.byref(xm), ctypes.byref(wm), int(k), int(bool(allow_tf32)),
                                                ctypes.byref(need)))
        ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
        _abi.check(lib.sf_topk_encode(ctypes.byref(xm), ctypes.byref(wm), ctypes.byref(be), _abi.ref(bd), int(k),
                                      indices.data_ptr(), values.data_ptr(), _abi.dtype_code(x.dtype, "x"),
                                      int(bool(allow_tf32)), ws.data_ptr(), ws.numel(), _abi.stream_of(dev)))
    return values, indices
