"""Fused SAE encoder: act((x - b_dec) @ W_enc + b_enc), mirroring saeflow/kernels/encode.py.

Same signature, dtype rules and errors as the reference's `fused_encode`
(saeflow/kernels/encode.py:97-139); the work runs in libsaeflow_b200.so:

- 16-bit W_enc, or fp32 with TF32 allowed: a persistent tcgen05/TMEM tensor-core GEMM
  fed by TMA, bias + ReLU/JumpReLU + per-row nonzero count in the epilogue.
- fp32 W_enc with IEEE products (the reference default, encode.py:118-120): a CUDA-core
  GEMM with the same epilogue.

The (x - b_dec) shift is rounded to W_enc's dtype before the product, as the reference
prologue does (encode.py:72 of the kernel body).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _abi

ACTIVATIONS = {"relu": _abi.SF_ACT_RELU, "jumprelu": _abi.SF_ACT_JUMPRELU}

# Tile shapes of the two kernels, reported by best_config().
TCGEN05_PAIR_CONFIG = {"variant": "tcgen05", "BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K_BYTES": 128, "stages": 6,
                       "cta_pair": True, "tmem_accumulators": 2}
TCGEN05_CONFIG = {"variant": "tcgen05_1cta", "BLOCK_M": 128, "BLOCK_N": 256, "BLOCK_K_BYTES": 128, "stages": 4,
                  "cta_pair": False, "tmem_accumulators": 2}
SIMT_CONFIG = {"variant": "simt", "BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_K": 8}
_VARIANTS = {"auto": _abi.SF_VARIANT_AUTO, "tcgen05": _abi.SF_VARIANT_TCGEN05, "simt": _abi.SF_VARIANT_SIMT,
             "tcgen05_1cta": _abi.SF_VARIANT_TCGEN05_SINGLE}

_last_config = None


def _variant(config) -> int:
    """`config` pins the kernel. The reference pins Triton block sizes (encode.py:104);
    here the tile shapes are fixed per kernel, so only {"variant": ...} selects anything
    and block-size keys are accepted without effect."""
    if config is None:
        return _abi.SF_VARIANT_AUTO
    if not isinstance(config, dict):
        raise ValueError(f"config must be a dict, got {type(config).__name__}")
    v = config.get("variant", "auto")
    if v not in _VARIANTS:
        raise ValueError(f"config variant must be one of {list(_VARIANTS)}, got {v!r}")
    return _VARIANTS[v]


SPLIT_PRECISION_RANGE = 1024  # kEmuMaxRangeK of the library: d_in per split-precision K range


def _uses_tensor_cores(x, W_enc, allow_tf32, variant) -> bool:
    """Every kernel choice but "simt" runs on the tensor cores (IEEE fp32 products there
    are split-precision, see _split_precision)."""
    return variant != _abi.SF_VARIANT_SIMT


def _split_precision(x, W_enc, allow_tf32) -> bool:
    """fp32 x and W_enc with TF32 not allowed: the reference's IEEE products
    (encode.py:118-120), computed on the bf16 tensor cores from three-part splits of both
    operands, smallest partial products first, to fp32-class accuracy; a d_in above
    SPLIT_PRECISION_RANGE runs as K ranges whose sums are added in fp32."""
    return W_enc.dtype == torch.float32 and x.dtype == torch.float32 and not allow_tf32


def fused_encode(x, W_enc, b_enc, b_dec, threshold=None, activation="relu", *,
                 out_dtype=None, row_nnz=None, config=None, allow_tf32=None):
    """act((x - b_dec) @ W_enc + b_enc) -> [M, d_sae], accumulated in fp32.

    x: [M, d_in] fp32 / bf16 / fp16. W_enc: [d_in, d_sae], any strides.
    activation: "relu" or "jumprelu" (needs `threshold` [d_sae]).
    row_nnz: optional zeroed int32 [M] buffer; receives each row's nonzero count.
    config: {"variant": "auto" | "tcgen05" | "tcgen05_1cta" | "simt"} to pin the kernel.
    allow_tf32: fp32 inputs only; defaults to torch.backends.cuda.matmul.allow_tf32.
    """
    global _last_config
    if activation not in ACTIVATIONS:
        raise ValueError(f"fused_encode supports {list(ACTIVATIONS)}, got {activation!r}")
    if activation == "jumprelu" and threshold is None:
        raise ValueError("jumprelu needs a threshold")
    M, K = x.shape
    K_w, N = W_enc.shape
    if K != K_w:
        raise ValueError(f"x has d_in={K} but W_enc has d_in={K_w}")
    dev = _abi.require_cuda(("x", x), ("W_enc", W_enc), ("b_enc", b_enc), ("b_dec", b_dec),
                            ("threshold", threshold), ("row_nnz", row_nnz))
    out = torch.empty(M, N, device=dev, dtype=out_dtype or x.dtype)
    if M == 0:
        return out
    if allow_tf32 is None:
        allow_tf32 = torch.backends.cuda.matmul.allow_tf32
    if row_nnz is not None:
        if row_nnz.dtype != torch.int32 or row_nnz.numel() != M or not row_nnz.is_contiguous():
            raise ValueError("row_nnz must be a contiguous int32 tensor with one entry per row")
    variant = _variant(config)
    lib = _abi.load()
    xm, wm, om = _abi.matrix(x, "x"), _abi.matrix(W_enc, "W_enc"), _abi.matrix(out, "out")
    be, bd = _abi.vector(b_enc, "b_enc"), _abi.vector(b_dec, "b_dec")
    th = _abi.vector(threshold, "threshold") if activation == "jumprelu" else None
    with torch.cuda.device(dev):
        need = ctypes.c_size_t(0)
        _abi.check(lib.sf_fused_encode_workspace(ctypes.byref(xm), ctypes.byref(wm), int(bool(allow_tf32)),
                                                 variant, ctypes.byref(need)))
        ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
        _abi.check(lib.sf_fused_encode(
            ctypes.byref(xm), ctypes.byref(wm), _abi.ref(be), _abi.ref(bd), _abi.ref(th), ACTIVATIONS[activation],
            ctypes.byref(om), row_nnz.data_ptr() if row_nnz is not None else None, int(bool(allow_tf32)), variant,
            ws.data_ptr(), ws.numel(), _abi.stream_of(dev)))
    if not _uses_tensor_cores(x, W_enc, allow_tf32, variant):
        _last_config = dict(SIMT_CONFIG)
    elif M > 128 and variant != _abi.SF_VARIANT_TCGEN05_SINGLE:
        _last_config = dict(TCGEN05_PAIR_CONFIG)
    else:
        _last_config = dict(TCGEN05_CONFIG)
    if _split_precision(x, W_enc, allow_tf32) and _last_config["variant"] != "simt":
        _last_config["operands"] = "bf16 x3 split, 6 partial products"
    return out


def best_config():
    """Kernel and tile shape used by the most recent fused_encode call (None before any).

    The reference returns the autotuner's pick (encode.py:142-144); these kernels have
    one tile shape each, so this names the kernel that ran."""
    return _last_config


def encode_csr(x, W_enc, b_enc, b_dec, threshold=None, activation="relu", *, allow_tf32=None,
               stage_capacity=None):
    """CSR features (indptr int64 [M+1], indices int32 [nnz], values [nnz]) of
    act((x - b_dec) @ W_enc + b_enc), without the dense [M, d_sae] output.

    Returns exactly `dense_to_csr(fused_encode(..., row_nnz=r), r)` (the reference's
    encode_sparse, saeflow/ops.py:36-39): the GEMM epilogue stages each row's nonzeros per
    256-column tile (the tensor-core encoder, or the CUDA-core one for IEEE fp32) and a
    placement kernel writes the canonical CSR after the one host sync that sizes it. A
    staging overflow (more nonzeros than `stage_capacity`, default min(d_sae, 512) per row)
    takes the dense route instead.
    """
    staged = encode_csr_stage(x, W_enc, b_enc, b_dec, threshold, activation, allow_tf32=allow_tf32,
                              stage_capacity=stage_capacity)
    return encode_csr_finish(staged)


class _Staged:
    """Device buffers of an encode-straight-to-CSR call between its two steps."""

    __slots__ = ("args", "dev", "M", "N", "dtype", "row_nnz", "tile_cnt", "tile_off", "stage_idx", "stage_val",
                 "state", "csr", "stage_idx_out", "stage_val_out")


def encode_csr_stage(x, W_enc, b_enc, b_dec, threshold=None, activation="relu", *, allow_tf32=None,
                     stage_capacity=None, device_consumer=False):
    """Step 1 of encode_csr: launches the shift pre-pass and the encoder GEMM with the CSR
    staging epilogue (no host sync). Pass the result to encode_csr_finish, or, with
    device_consumer=True (which also allocates capacity-sized CSR outputs), to
    encode_csr_finish_async."""
    if activation not in ACTIVATIONS:
        raise ValueError(f"fused_encode supports {list(ACTIVATIONS)}, got {activation!r}")
    if activation == "jumprelu" and threshold is None:
        raise ValueError("jumprelu needs a threshold")
    M, K = x.shape
    K_w, N = W_enc.shape
    if K != K_w:
        raise ValueError(f"x has d_in={K} but W_enc has d_in={K_w}")
    dev = _abi.require_cuda(("x", x), ("W_enc", W_enc), ("b_enc", b_enc), ("b_dec", b_dec),
                            ("threshold", threshold))
    if allow_tf32 is None:
        allow_tf32 = torch.backends.cuda.matmul.allow_tf32
    h = _Staged()
    h.args = (x, W_enc, b_enc, b_dec, threshold, activation, allow_tf32)
    h.dev, h.M, h.N, h.dtype, h.csr = dev, M, N, x.dtype, None
    if M == 0:
        h.csr = _dense_route(h)
        return h
    n_tiles = (N + _abi.CSR_TILE - 1) // _abi.CSR_TILE
    cap = stage_capacity if stage_capacity is not None else M * min(N, 512)
    cap = int(max(0, min(cap, (1 << 31) - 1)))
    lib = _abi.load()
    xm, wm = _abi.matrix(x, "x"), _abi.matrix(W_enc, "W_enc")
    be, bd = _abi.vector(b_enc, "b_enc"), _abi.vector(b_dec, "b_dec")
    th = _abi.vector(threshold, "threshold") if activation == "jumprelu" else None
    with torch.cuda.device(dev):
        h.row_nnz = torch.zeros(M, dtype=torch.int32, device=dev)
        h.tile_cnt = torch.empty(M * n_tiles, dtype=torch.int32, device=dev)
        h.tile_off = torch.empty(M * n_tiles, dtype=torch.int32, device=dev)
        h.stage_idx = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
        h.stage_val = torch.empty(max(cap, 1), dtype=x.dtype, device=dev)
        h.state = torch.zeros(2, dtype=torch.int32, device=dev)
        if device_consumer:
            h.stage_idx_out = torch.empty_like(h.stage_idx)
            h.stage_val_out = torch.empty_like(h.stage_val)
        need = ctypes.c_size_t(0)
        _abi.check(lib.sf_fused_encode_workspace(ctypes.byref(xm), ctypes.byref(wm), int(bool(allow_tf32)),
                                                 _abi.SF_VARIANT_AUTO, ctypes.byref(need)))
        ws = torch.empty(max(need.value, 16), dtype=torch.uint8, device=dev)
        _abi.check(lib.sf_encode_csr_stage(
            ctypes.byref(xm), ctypes.byref(wm), _abi.ref(be), _abi.ref(bd), _abi.ref(th), ACTIVATIONS[activation],
            _abi.dtype_code(x.dtype, "x"), h.row_nnz.data_ptr(), h.tile_cnt.data_ptr(), h.tile_off.data_ptr(),
            h.stage_idx.data_ptr(), h.stage_val.data_ptr(), cap, h.state.data_ptr(), int(bool(allow_tf32)),
            ws.data_ptr(), ws.numel(), _abi.stream_of(dev)))
    return h


def encode_csr_finish(h):
    """Step 2 of encode_csr: indptr scan, the one host sync (nnz and the overflow flag),
    and the placement kernel. Returns (indptr, indices, values)."""
    if h.csr is not None:
        return h.csr
    lib = _abi.load()
    M, N, dev = h.M, h.N, h.dev
    with torch.cuda.device(dev):
        s = _abi.stream_of(dev)
        indptr = torch.empty(M + 1, dtype=torch.int64, device=dev)
        _abi.check(lib.sf_csr_indptr(h.row_nnz.data_ptr(), M, indptr.data_ptr(), s))
        nnz, overflow = torch.stack([indptr[-1], h.state[1].to(torch.int64)]).tolist()  # the one host sync
        if overflow:
            return _dense_route(h)
        indices = torch.empty(nnz, dtype=torch.int32, device=dev)
        values = torch.empty(nnz, dtype=h.dtype, device=dev)
        if nnz:
            _abi.check(lib.sf_csr_place(h.tile_cnt.data_ptr(), h.tile_off.data_ptr(), M, N, h.stage_idx.data_ptr(),
                                        h.stage_val.data_ptr(), h.stage_idx.numel(), _abi.dtype_code(h.dtype, "values"),
                                        indptr.data_ptr(), indices.data_ptr(), values.data_ptr(), s))
    return indptr, indices, values


def encode_csr_finish_async(h):
    """Step 2 of encode_csr without the host sync, for a CSR consumed on the device:
    (indptr, indices, values, overflow) where indices / values have the staging capacity as
    length (only indptr's ranges are meaningful) and `overflow` is a device int32 scalar.
    If it reads nonzero after the stream work, the staging overflowed, every row of the
    returned CSR is empty, and the caller must redo the rows (encode_csr's dense route)."""
    if h.csr is not None:
        indptr, indices, values = h.csr
        return indptr, indices, values, None
    lib = _abi.load()
    M, N, dev = h.M, h.N, h.dev
    with torch.cuda.device(dev):
        indptr = torch.empty(M + 1, dtype=torch.int64, device=dev)
        _abi.check(lib.sf_csr_finish_async(
            h.row_nnz.data_ptr(), h.tile_cnt.data_ptr(), h.tile_off.data_ptr(), M, N, h.stage_idx.data_ptr(),
            h.stage_val.data_ptr(), h.stage_idx.numel(), _abi.dtype_code(h.dtype, "values"), h.state.data_ptr(),
            indptr.data_ptr(), h.stage_idx_out.data_ptr(), h.stage_val_out.data_ptr(), _abi.stream_of(dev)))
    return indptr, h.stage_idx_out, h.stage_val_out, h.state[1]


def _dense_route(h):
    from .decode import dense_to_csr

    x, W_enc, b_enc, b_dec, threshold, activation, allow_tf32 = h.args
    rn = torch.zeros(h.M, dtype=torch.int32, device=h.dev)
    f = fused_encode(x, W_enc, b_enc, b_dec, threshold, activation, row_nnz=rn, allow_tf32=allow_tf32)
    return dense_to_csr(f, rn)
