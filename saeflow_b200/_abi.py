"""ctypes binding of libsaeflow_b200.so (declared in include/saeflow_b200.h).

The library is loaded on first use. There is no fallback: if the shared library is
missing, every op raises ImportError naming the build command; if a tensor is not on a
CUDA device, the op raises ValueError. Python only describes tensors (pointer, dtype
code, shape, strides) and passes torch's current CUDA stream.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# The in-tree build; SAEFLOW_B200_LIB names another build of the same library (e.g. one
# compiled with different tuning flags) to load instead.
LIB_PATH = Path(os.environ.get("SAEFLOW_B200_LIB") or Path(__file__).resolve().parent / "_lib" / "libsaeflow_b200.so")

SF_F32, SF_BF16, SF_F16 = 0, 1, 2
DTYPE_CODES = {torch.float32: SF_F32, torch.bfloat16: SF_BF16, torch.float16: SF_F16}
SF_ACT_RELU, SF_ACT_JUMPRELU = 0, 1
SF_VARIANT_AUTO, SF_VARIANT_TCGEN05, SF_VARIANT_SIMT, SF_VARIANT_TCGEN05_SINGLE = 0, 1, 2, 3

SF_OK, SF_ERR_INVALID, SF_ERR_UNSUPPORTED, SF_ERR_CUDA, SF_ERR_WORKSPACE, SF_ERR_DEVICE = range(6)
ABI_VERSION = 1
CSR_TILE = 256  # SF_CSR_TILE

# Every symbol the header declares, with its ctypes signature.
_c = ctypes
_P = _c.c_void_p


class SfMatrix(_c.Structure):
    _fields_ = [("data", _c.c_void_p), ("dtype", _c.c_int32), ("reserved", _c.c_int32),
                ("rows", _c.c_int64), ("cols", _c.c_int64),
                ("stride_row", _c.c_int64), ("stride_col", _c.c_int64)]


class SfVector(_c.Structure):
    _fields_ = [("data", _c.c_void_p), ("dtype", _c.c_int32), ("reserved", _c.c_int32),
                ("len", _c.c_int64), ("stride", _c.c_int64)]


_MP = _c.POINTER(SfMatrix)
_VP = _c.POINTER(SfVector)
_SIZE_P = _c.POINTER(_c.c_size_t)

SIGNATURES = {
    "sf_last_error": (_c.c_char_p, []),
    "sf_abi_version": (_c.c_int, []),
    "sf_device_error": (_c.c_int, [_c.POINTER(_c.c_uint32)]),
    "sf_fused_encode_workspace": (_c.c_int, [_MP, _MP, _c.c_int, _c.c_int, _SIZE_P]),
    "sf_fused_encode": (_c.c_int, [_MP, _MP, _VP, _VP, _VP, _c.c_int, _MP, _P, _c.c_int, _c.c_int,
                                   _P, _c.c_size_t, _P]),
    "sf_fused_encode_noalloc": (_c.c_int, [_MP, _MP, _VP, _VP, _VP, _c.c_int, _MP, _P, _c.c_int, _c.c_int, _P]),
    "sf_encode_csr_stage": (_c.c_int, [_MP, _MP, _VP, _VP, _VP, _c.c_int, _c.c_int, _P, _P, _P, _P, _P,
                                       _c.c_int64, _P, _c.c_int, _P, _c.c_size_t, _P]),
    "sf_csr_place": (_c.c_int, [_P, _P, _c.c_int64, _c.c_int64, _P, _P, _c.c_int64, _c.c_int, _P, _P, _P, _P]),
    "sf_csr_finish_async": (_c.c_int, [_P, _P, _P, _c.c_int64, _c.c_int64, _P, _P, _c.c_int64, _c.c_int, _P, _P,
                                       _P, _P, _P]),
    "sf_row_nnz": (_c.c_int, [_MP, _P, _P]),
    "sf_csr_indptr": (_c.c_int, [_P, _c.c_int64, _P, _P]),
    "sf_dense_to_csr": (_c.c_int, [_MP, _P, _P, _P, _c.c_int, _P]),
    "sf_sparse_decode": (_c.c_int, [_P, _c.c_int64, _P, _P, _c.c_int, _MP, _VP, _MP, _P]),
    "sf_transpose": (_c.c_int, [_MP, _MP, _P]),
    "sf_csr_transpose_workspace": (_c.c_int, [_c.c_int64, _c.c_int64, _SIZE_P]),
    "sf_csr_transpose": (_c.c_int, [_P, _c.c_int64, _P, _c.c_int64, _c.c_int64, _P, _P, _P, _P, _P, _c.c_size_t,
                                    _P]),
    "sf_csr_sddmm": (_c.c_int, [_P, _c.c_int64, _P, _MP, _MP, _P, _c.c_int, _P, _P]),
    "sf_matvec": (_c.c_int, [_MP, _P, _P, _P]),
    "sf_csc_gather_workspace": (_c.c_int, [_c.c_int64, _MP, _SIZE_P]),
    "sf_csc_gather": (_c.c_int, [_P, _c.c_int64, _P, _c.c_int64, _P, _P, _P, _c.c_int, _MP, _MP, _P, _MP, _P, _P,
                                 _c.c_size_t, _P]),
    "sf_topk_encode_workspace": (_c.c_int, [_MP, _MP, _c.c_int, _c.c_int, _SIZE_P]),
    "sf_topk_encode": (_c.c_int, [_MP, _MP, _VP, _VP, _c.c_int, _P, _P, _c.c_int, _c.c_int, _P,
                                  _c.c_size_t, _P]),
}

_lib = None
_lock = threading.Lock()


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and type the shared library. Raises ImportError if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise ImportError(
                f"saeflow_b200 native library not found at {p}; build it with "
                "`python -m saeflow_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.sf_abi_version() != ABI_VERSION:
            raise ImportError(f"{p} has ABI {lib.sf_abi_version()}, expected {ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


def check(status: int) -> None:
    """Map an sf_status to the reference's exception types (ValueError for bad arguments)."""
    if status == SF_OK:
        return
    msg = load().sf_last_error().decode(errors="replace")
    if status == SF_ERR_INVALID:
        raise ValueError(msg)
    kind = {SF_ERR_UNSUPPORTED: "unsupported", SF_ERR_CUDA: "CUDA error", SF_ERR_WORKSPACE: "workspace",
            SF_ERR_DEVICE: "device error"}.get(status, f"status {status}")
    raise RuntimeError(f"saeflow_b200 {kind}: {msg}")


def dtype_code(dtype: torch.dtype, name: str) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"{name} has dtype {dtype}; expected float32, bfloat16 or float16") from None


def require_cuda(*named: tuple[str, torch.Tensor | None]) -> torch.device:
    """All given tensors must live on one CUDA device; returns it."""
    dev = None
    for name, t in named:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(f"{name} is on {t.device}; saeflow_b200 runs on CUDA devices only")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{name} is on {t.device}, expected {dev}")
    if dev is None:
        raise ValueError("no CUDA tensor given")
    return dev


def matrix(t: torch.Tensor, name: str) -> SfMatrix:
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")
    return SfMatrix(t.data_ptr(), dtype_code(t.dtype, name), 0, t.shape[0], t.shape[1], t.stride(0), t.stride(1))


def vector(t: torch.Tensor | None, name: str) -> SfVector | None:
    if t is None:
        return None
    if t.dim() != 1:
        raise ValueError(f"{name} must be 1-D, got shape {tuple(t.shape)}")
    return SfVector(t.data_ptr(), dtype_code(t.dtype, name), 0, t.shape[0], t.stride(0))


def ref(s):
    """ctypes pointer to a structure, or NULL for None."""
    return ctypes.byref(s) if s is not None else None


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_error(device: torch.device | int | None = None) -> int:
    """Synchronise `device` and return (and clear) its device-side error bits.

    1 = an in-kernel wait timed out, 2 = a CSR index outside [0, d_sae), 4 = an indptr
    inconsistent with the dense rows. 0 means every kernel since the last call was clean.
    """
    lib = load()
    code = ctypes.c_uint32(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        check(lib.sf_device_error(ctypes.byref(code)))
    return code.value
