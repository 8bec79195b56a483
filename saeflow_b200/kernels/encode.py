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


def _uses_tensor_cores(x, W_enc, allow_tf32, variant) -> bool:
    if variant in (_abi.SF_VARIANT_TCGEN05, _abi.SF_VARIANT_TCGEN05_SINGLE):
        return True
    if variant == _abi.SF_VARIANT_SIMT:
        return False
    return W_enc.dtype != torch.float32 or allow_tf32 or x.dtype != torch.float32


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
    return out


def best_config():
    """Kernel and tile shape used by the most recent fused_encode call (None before any).

    The reference returns the autotuner's pick (encode.py:142-144); these kernels have
    one tile shape each, so this names the kernel that ran."""
    return _last_config
