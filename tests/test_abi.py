"""The C ABI without a GPU: the library loads, exports exactly what include/saeflow_b200.h
declares, validates arguments, and the Python layer refuses CPU tensors (no fallback)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

import saeflow_b200
from saeflow_b200 import _abi
from saeflow_b200.kernels import dense_to_csr, fused_encode, sparse_decode, topk_encode

HEADER = Path(__file__).resolve().parents[1] / "include" / "saeflow_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(sf_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    assert declared_functions() == sorted(_abi.SIGNATURES)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _abi.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.sf_abi_version() == _abi.ABI_VERSION
    assert str(_abi.LIB_PATH) in Path("/proc/self/maps").read_text()


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = _abi.load()
    x = _abi.SfMatrix(None, 7, 0, 4, 8, 8, 1)  # bad dtype code
    W = _abi.SfMatrix(16, 1, 0, 8, 16, 16, 1)
    need = ctypes.c_size_t(0)
    st = lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 0, ctypes.byref(need))
    assert st == _abi.SF_ERR_INVALID
    assert b"dtype" in lib.sf_last_error()
    x = _abi.SfMatrix(16, 1, 0, 4, 9, 9, 1)  # d_in mismatch (placeholder pointers, never dereferenced)
    st = lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 0, ctypes.byref(need))
    assert st == _abi.SF_ERR_INVALID
    assert b"d_in" in lib.sf_last_error()
    with pytest.raises(ValueError):
        _abi.check(st)


def test_workspace_sizes():
    lib = _abi.load()
    need = ctypes.c_size_t(0)
    # bf16 x [16384, 2304], W_enc row-major [2304, 65536]: shifted x copy only, whatever x's
    # dtype and address (fp32 x, a 2-byte-offset base)
    W = _abi.SfMatrix(16, 1, 0, 2304, 65536, 65536, 1)
    for x in (_abi.SfMatrix(16, 1, 0, 16384, 2304, 2304, 1), _abi.SfMatrix(16, 0, 0, 16384, 2304, 2304, 1),
              _abi.SfMatrix(18, 1, 0, 16384, 2304, 2304, 1)):
        assert lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 0, ctypes.byref(need)) == 0
        assert need.value == 16384 * 2304 * 2
    # odd d_sae: W_enc repacked to a 16-byte row pitch
    W = _abi.SfMatrix(16, 1, 0, 2304, 129, 129, 1)
    assert lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 0, ctypes.byref(need)) == 0
    assert need.value == 16384 * 2304 * 2 + 2304 * 136 * 2
    # the CUDA-core kernel is fp32 only
    assert lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 2, ctypes.byref(need)) == \
        _abi.SF_ERR_UNSUPPORTED
    # IEEE fp32 (config 1 shapes): the split x [M, 3 kp] bf16, the fallback's fp32 shifted x, a
    # 256-byte flag, the split W_enc [3 kp, N] bf16 (kp = d_in rounded up to 64); the CUDA-core
    # kernel needs only the fp32 shifted x
    x = _abi.SfMatrix(16, 0, 0, 4096, 768, 768, 1)
    W = _abi.SfMatrix(16, 0, 0, 768, 16384, 16384, 1)
    assert lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 0, ctypes.byref(need)) == 0
    assert need.value == 4096 * 3 * 768 * 2 + 4096 * 768 * 4 + 256 + 3 * 768 * 16384 * 2
    assert lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 2, ctypes.byref(need)) == 0
    assert need.value == 4096 * 768 * 4
    # d_in 2304: three K ranges of 768, plus the fp32 partial sums [M, d_sae rounded up to 256]
    x = _abi.SfMatrix(16, 0, 0, 4096, 2304, 2304, 1)
    W = _abi.SfMatrix(16, 0, 0, 2304, 16384, 16384, 1)
    assert lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 0, ctypes.byref(need)) == 0
    assert need.value == 4096 * 3 * 768 * 2 + 4096 * 2304 * 4 + 256 + 4096 * 16384 * 4 + 3 * 768 * 16384 * 2
    x = _abi.SfMatrix(16, 0, 0, 10, 100, 100, 1)  # d_in 100 -> kp 128; d_sae 129 -> pitch 136
    W = _abi.SfMatrix(16, 0, 0, 100, 129, 129, 1)
    assert lib.sf_fused_encode_workspace(ctypes.byref(x), ctypes.byref(W), 0, 0, ctypes.byref(need)) == 0
    assert need.value == 7680 + 4352 + 256 + 3 * 128 * 136 * 2  # 10x384x2, and 10x104x4 rounded up to 256


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: every op demands CUDA tensors."""
    sae = saeflow_b200.SAE(8, 16, "relu")
    x = torch.randn(3, 8)
    with pytest.raises(ValueError, match="CUDA"):
        fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec)
    with pytest.raises(ValueError, match="CUDA"):
        dense_to_csr(torch.zeros(3, 16))
    with pytest.raises(ValueError, match="CUDA"):
        sparse_decode(torch.zeros(4, dtype=torch.int64), torch.zeros(0, dtype=torch.int32), torch.zeros(0),
                      sae.W_dec)
    with pytest.raises(ValueError, match="CUDA"):
        topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, 4)
    with pytest.raises(ValueError, match="CUDA"):
        saeflow_b200.forward(sae, x)


def test_reference_argument_errors_precede_device_checks():
    """ValueError conventions of saeflow/kernels/encode.py:107-114, raised host-side."""
    x = torch.randn(3, 8)
    W = torch.randn(8, 16)
    b = torch.zeros(16)
    with pytest.raises(ValueError, match="supports"):
        fused_encode(x, W, b, torch.zeros(8), activation="gelu")
    with pytest.raises(ValueError, match="threshold"):
        fused_encode(x, W, b, torch.zeros(8), activation="jumprelu")
    with pytest.raises(ValueError, match="d_in"):
        fused_encode(torch.randn(3, 7), W, b, torch.zeros(8))


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(ImportError, match="saeflow_b200.build"):
        _abi.load(tmp_path / "nope.so")
