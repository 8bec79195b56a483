"""sf_fused_encode_noalloc, the encode entry point that allocates nothing, against the
allocating sf_fused_encode (B200).

The no-alloc entry point serves callers that cannot allocate device memory (a
foreign-language host given only its input and output buffers, a process whose caching
allocator holds the GPU's memory, a loop that cannot take cudaMalloc's synchronisation):
its workspace is a fixed 16 MiB array in the library's device image, which holds the
b_dec-shifted copy of x the encoder reads. This file is
collected last so that a run stopping at the first failure has run every other test.
"""

import ctypes

import pytest
import torch

from oracle import contract
from saeflow_b200 import _abi

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20


def _operands(M, K, N, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W_dec = torch.randn(N, K, generator=g, device="cuda")
    W_dec /= W_dec.norm(dim=1, keepdim=True)
    W = W_dec.T.contiguous().to(torch.bfloat16)
    b_enc = (torch.randn(N, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    b_dec = (torch.randn(K, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    thr = (torch.rand(N, generator=g, device="cuda") * 0.3).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    return x, W, b_enc, b_dec, thr


def _structs(x, W, b_enc, b_dec, thr, out):
    return (_abi.matrix(x, "x"), _abi.matrix(W, "W_enc"), _abi.vector(b_enc, "b_enc"), _abi.vector(b_dec, "b_dec"),
            _abi.vector(thr, "threshold"), _abi.matrix(out, "out"))


def _encode_allocating(lib, x, W, b_enc, b_dec, thr):
    out = torch.empty(x.shape[0], W.shape[1], device="cuda", dtype=torch.bfloat16)
    nnz = torch.zeros(x.shape[0], device="cuda", dtype=torch.int32)
    xm, wm, be, bd, th, om = _structs(x, W, b_enc, b_dec, thr, out)
    need = ctypes.c_size_t(0)
    _abi.check(lib.sf_fused_encode_workspace(ctypes.byref(xm), ctypes.byref(wm), 0, 0, ctypes.byref(need)))
    ws = torch.empty(need.value, device="cuda", dtype=torch.uint8)
    _abi.check(lib.sf_fused_encode(ctypes.byref(xm), ctypes.byref(wm), ctypes.byref(be), ctypes.byref(bd),
                                   ctypes.byref(th), _abi.SF_ACT_JUMPRELU, ctypes.byref(om), nnz.data_ptr(), 0, 0,
                                   ws.data_ptr(), ws.numel(), _abi.stream_of(x.device)))
    return out, nnz, need.value


def _encode_noalloc(lib, x, W, b_enc, b_dec, thr, out, nnz):
    xm, wm, be, bd, th, om = _structs(x, W, b_enc, b_dec, thr, out)
    return lib.sf_fused_encode_noalloc(ctypes.byref(xm), ctypes.byref(wm), ctypes.byref(be), ctypes.byref(bd),
                                       ctypes.byref(th), _abi.SF_ACT_JUMPRELU, ctypes.byref(om), nnz.data_ptr(), 0,
                                       0, _abi.stream_of(x.device))


def test_noalloc_encode_matches_allocating_encode_on_two_calls():
    lib = _abi.load()
    K, N = 512, 4096
    # two calls in a row, different inputs, row counts and x layouts (fp32 x converted to
    # W_enc's bf16, then a column-major bf16 view): the second must not see the first
    # call's scratch contents.
    for M, seed in ((1000, 11), (3000, 12)):
        x, W, b_enc, b_dec, thr = _operands(M, K, N, seed)
        x = x.float() if seed == 11 else x.T.contiguous().T
        want, want_nnz, need = _encode_allocating(lib, x, W, b_enc, b_dec, thr)
        assert 0 < need <= SCRATCH_BYTES
        got = torch.full_like(want, float("nan"))
        nnz = torch.zeros(M, device="cuda", dtype=torch.int32)
        _abi.check(_encode_noalloc(lib, x, W, b_enc, b_dec, thr, got, nnz))
        torch.cuda.synchronize()
        contract.assert_values_close(got.float().cpu(), want.float().cpu(), torch.bfloat16, what="no-alloc encode")
        assert torch.equal(nnz, want_nnz)
        assert torch.equal(nnz.cpu(), torch.count_nonzero(got, dim=1).int().cpu())
    assert _abi.device_error() == 0


def test_noalloc_encode_rejects_operands_beyond_its_scratch():
    lib = _abi.load()
    K, N = 2304, 512
    M = SCRATCH_BYTES // (K * 2) + 1  # one row more than the scratch holds
    x, W, b_enc, b_dec, thr = _operands(M, K, N, 13)
    out = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    nnz = torch.zeros(M, device="cuda", dtype=torch.int32)
    st = _encode_noalloc(lib, x, W, b_enc, b_dec, thr, out, nnz)
    assert st == _abi.SF_ERR_WORKSPACE
    assert b"scratch" in lib.sf_last_error()
    torch.cuda.synchronize()
    assert int(nnz.abs().sum()) == 0 and int(out.float().abs().sum()) == 0  # nothing ran


def test_noalloc_encode_rejects_a_weight_layout_it_would_have_to_copy():
    """An fp32 row-major W_enc on the TF32 path must be repacked K-major; at 2304 x 16384
    that copy alone is 151 MB, so fewer rows cannot help and the message says what layout
    to pass instead."""
    lib = _abi.load()
    K, N, M = 2304, 16384, 8
    g = torch.Generator(device="cuda").manual_seed(14)
    x = torch.randn(M, K, generator=g, device="cuda")
    W = torch.randn(K, N, generator=g, device="cuda")  # row-major fp32: not K-major
    b_enc, b_dec = torch.zeros(N, device="cuda"), torch.zeros(K, device="cuda")
    out = torch.zeros(M, N, device="cuda")
    xm, wm, be, bd, om = (_abi.matrix(x, "x"), _abi.matrix(W, "W_enc"), _abi.vector(b_enc, "b_enc"),
                          _abi.vector(b_dec, "b_dec"), _abi.matrix(out, "out"))
    st = lib.sf_fused_encode_noalloc(ctypes.byref(xm), ctypes.byref(wm), ctypes.byref(be), ctypes.byref(bd), None,
                                     _abi.SF_ACT_RELU, ctypes.byref(om), None, 1, 0, _abi.stream_of(x.device))
    assert st == _abi.SF_ERR_WORKSPACE
    msg = lib.sf_last_error()
    assert b"layout" in msg and b"column-major" in msg
    torch.cuda.synchronize()
    assert int(out.abs().sum()) == 0  # nothing ran


def test_noalloc_ieee_fp32_runs_the_cuda_core_kernel():
    """fp32 x and W_enc with TF32 off: the allocating call splits W_enc into bf16 parts for
    the tensor cores, a copy the static scratch cannot hold, so the no-alloc call runs the
    CUDA-core IEEE kernel (scratch: the shifted x), identical to the allocating call pinned
    to that kernel."""
    lib = _abi.load()
    M, K, N = 700, 256, 2048
    g = torch.Generator(device="cuda").manual_seed(15)
    x = torch.randn(M, K, generator=g, device="cuda")
    W = torch.randn(K, N, generator=g, device="cuda") / 16
    b_enc, b_dec = torch.full((N,), -0.5, device="cuda"), torch.randn(K, generator=g, device="cuda") * 0.1
    xm, wm, be, bd = _abi.matrix(x, "x"), _abi.matrix(W, "W_enc"), _abi.vector(b_enc, "b_enc"), _abi.vector(b_dec, "b_dec")
    outs = []
    for noalloc in (False, True):
        out = torch.full((M, N), float("nan"), device="cuda")
        nnz = torch.zeros(M, device="cuda", dtype=torch.int32)
        om = _abi.matrix(out, "out")
        if noalloc:
            st = lib.sf_fused_encode_noalloc(ctypes.byref(xm), ctypes.byref(wm), ctypes.byref(be), ctypes.byref(bd),
                                             None, _abi.SF_ACT_RELU, ctypes.byref(om), nnz.data_ptr(), 0, 0,
                                             _abi.stream_of(x.device))
        else:
            need = ctypes.c_size_t(0)
            _abi.check(lib.sf_fused_encode_workspace(ctypes.byref(xm), ctypes.byref(wm), 0, _abi.SF_VARIANT_SIMT,
                                                     ctypes.byref(need)))
            ws = torch.empty(need.value, device="cuda", dtype=torch.uint8)
            st = lib.sf_fused_encode(ctypes.byref(xm), ctypes.byref(wm), ctypes.byref(be), ctypes.byref(bd), None,
                                     _abi.SF_ACT_RELU, ctypes.byref(om), nnz.data_ptr(), 0, _abi.SF_VARIANT_SIMT,
                                     ws.data_ptr(), ws.numel(), _abi.stream_of(x.device))
        _abi.check(st)
        torch.cuda.synchronize()
        outs.append((out, nnz))
    assert torch.equal(outs[0][0].view(torch.int32), outs[1][0].view(torch.int32))
    assert torch.equal(outs[0][1], outs[1][1])
    assert _abi.device_error() == 0
