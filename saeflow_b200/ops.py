"""SAE-level entry points, a drop-in for saeflow/ops.py. `sae` is a saeflow_b200.SAE
or anything with the same attributes (W_enc, b_enc, W_dec, b_dec, threshold,
activation, k), e.g. a saeflow.reference.SAE moved to a CUDA device.

Sparse features are CSR tuples (indptr, indices, values); see kernels/decode.py.
"""

import threading

import torch

from .kernels import encode_csr, fused_encode, sparse_decode, topk_encode
from .kernels.encode import encode_csr_finish_async, encode_csr_stage


def _topk(sae, x):
    """(values [M, k], indices int32 [M, k]) of the k largest ReLU'd pre-activations.

    The reference writes the dense ReLU output and calls torch.topk (ops.py:12-16); here
    the selection runs inside the encoder's epilogue and the dense output is never made.
    """
    return topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.k)


def encode(sae, x):
    """Dense feature activations [M, d_sae] (ops.py:19-26)."""
    if sae.activation == "topk":
        values, indices = _topk(sae, x)
        return torch.zeros(x.shape[0], sae.W_enc.shape[1], device=x.device, dtype=x.dtype).scatter_(
            -1, indices.long(), values
        )
    return fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation)


def encode_sparse(sae, x):
    """Feature activations as CSR (indptr, indices, values) (ops.py:29-39)."""
    M = x.shape[0]
    if sae.activation == "topk":
        # TopK is fixed-width: no compaction pass, indptr is arange (ops.py:35).
        values, indices = _topk(sae, x)
        indptr = torch.arange(0, M * sae.k + 1, sae.k, device=x.device, dtype=torch.int64)
        return indptr, indices.flatten(), values.flatten()
    # Same CSR as fused_encode(row_nnz=...) + dense_to_csr (ops.py:37-39), built from the
    # encoder's epilogue without writing or re-reading the dense [M, d_sae] features.
    return encode_csr(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation)


def decode_sparse(sae, csr):
    """Reconstruction [M, d_in] from CSR features (ops.py:42-44)."""
    return sparse_decode(*csr, sae.W_dec, sae.b_dec)


def _forward_async(sae, x, out=None, *, add_b_dec=True, out_dtype=None):
    """forward() with every launch queued and no host sync: returns (x_hat, overflow), where
    overflow is a device int32 scalar (None for routes that cannot overflow). A nonzero
    overflow means the CSR staging ran out of room and x_hat holds only the bias.
    add_b_dec=False gives the partial sum_j f_j W_dec[j] (feature-sharded decode)."""
    b_dec = sae.b_dec if add_b_dec else None
    if sae.activation == "topk":
        csr, overflow = encode_sparse(sae, x), None
    else:
        h = encode_csr_stage(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation,
                             device_consumer=True)
        *csr, overflow = encode_csr_finish_async(h)
    return sparse_decode(*csr, sae.W_dec, b_dec, out=out, out_dtype=out_dtype), overflow


# Rows per encode launch of forward(): larger batches run as consecutive launches. At most
# FORWARD_CHUNK_ROWS, which bounds the CSR staging (M x d_sae/256 tile counts), and at most
# FORWARD_LAUNCH_MACS multiply-adds of the encoder GEMM: long launches meet the 1000 W power
# cap at a lower SM clock. Measured on B200 at config 5 (d_in 2304, d_sae 2^20, one GPU):
# 16384-row launches (4e13 multiply-adds) ran at 1237-1320 MHz, 1418 ms per 262144 tokens;
# 8192-row launches at 1455-1500 MHz, 1275 ms; 4096 and 2048 rows the same as 8192 (one
# 262144-row launch: 960 MHz). Config 2 (16384 x 2304 x 65536 = 2.5e12) stays one launch.
FORWARD_CHUNK_ROWS = 16384
FORWARD_LAUNCH_MACS = 2e13


def forward_launch_rows(sae):
    """Rows per encode launch of forward() for this SAE: a multiple of 1024 (at least 1024)
    up to FORWARD_CHUNK_ROWS, within FORWARD_LAUNCH_MACS multiply-adds."""
    per_row = max(1, sae.W_enc.shape[0] * sae.W_enc.shape[1])
    rows = int(FORWARD_LAUNCH_MACS // per_row) // 1024 * 1024
    return max(1024, min(FORWARD_CHUNK_ROWS, rows))


def forward(sae, x):
    """encode_sparse then decode_sparse: the dense features never reach the decoder (ops.py:47-49).

    The CSR stays on the device between the two, so nothing waits on the host between the
    encoder and the decoder; the one host read (as in the reference, decode.py:88) comes at
    the end and checks that the CSR staging did not overflow (a chunk that overflowed is
    redone through encode_sparse's exact-size route). Batches above forward_launch_rows(sae)
    rows run as consecutive chunks into one output."""
    M = x.shape[0]
    R = forward_launch_rows(sae)
    if M <= R:
        out, overflow = _forward_async(sae, x)
        if overflow is not None and int(overflow):
            out = decode_sparse(sae, encode_sparse(sae, x))
        return out
    out = torch.empty(M, sae.W_dec.shape[1], dtype=sae.W_dec.dtype, device=x.device)
    flags = []
    for r0 in range(0, M, R):
        r1 = min(M, r0 + R)
        _, overflow = _forward_async(sae, x[r0:r1], out[r0:r1])
        if overflow is not None:
            flags.append((r0, r1, overflow))
    bad = torch.stack([f for _, _, f in flags]).tolist() if flags else []
    for (r0, r1, _), ovf in zip(flags, bad):
        if ovf:
            out[r0:r1] = decode_sparse(sae, encode_sparse(sae, x[r0:r1]))
    return out


_copy_streams = {}
_copy_lock = threading.Lock()


def _streams(dev):
    with _copy_lock:
        if dev not in _copy_streams:
            _copy_streams[dev] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        return _copy_streams[dev]


def _even_split(n, cap):
    k = -(-n // cap)
    return [n // k + (1 if i < n % k else 0) for i in range(k)]


# Smallest batch (rows) forward_host splits although it fits one chunk.
SMALL_SPLIT_ROWS = 2048


def _chunk_plan(M, C):
    """Row counts of forward_host's chunks (at most C each): quarter and half chunks at both
    ends, full chunks between. Only the first chunk's copy in and the last chunk's copy out
    are exposed, and every chunk pays a fixed cost (the weights are streamed again, and the
    scans run again: ~0.1 ms at config 2), so the plan keeps both ends short with few chunks.
    Measured on B200 at config 2 (16384 rows, C = 8192): 4.66 ms against 3.94 ms with the
    batch already on the device; plans with more or with smaller end chunks were slower.
    A batch of one chunk or less still splits quarter / half / quarter from SMALL_SPLIT_ROWS
    rows up, so that its copies overlap the compute too."""
    if M <= C:
        if M < SMALL_SPLIT_ROWS:
            return [M]
        q = M // 4
        return [q, M - 2 * q, q]
    ramp = [max(1, C // 4), max(1, C // 2)]
    mid = M - 2 * sum(ramp)
    if mid <= 0:
        return _even_split(M, C)
    return ramp + _even_split(mid, C) + ramp[::-1]


# Device bytes (x and x_hat together) up to which forward_host gives the whole batch device
# buffers, so the copies stream without waiting for a buffer; larger batches cycle through
# two chunk-sized buffers per direction.
WHOLE_BATCH_DEVICE_BYTES = 4 << 30


class HostForward:
    """A forward_host_async call in flight: wait() returns its host output.

    Holds the call's device buffers until its last copy out has finished; the overflow
    flags of its chunks come back through pinned memory, so wait() synchronises on this
    call's own events only, never on work queued after it."""

    def __init__(self, sae, x, out, flags, flags_host, ev_flags, ev_last, keep):
        self._sae, self._x, self._out = sae, x, out
        self._flags, self._flags_host, self._ev_flags, self._ev_last = flags, flags_host, ev_flags, ev_last
        self._keep = keep
        self._done = False

    def wait(self):
        if self._done:
            return self._out
        self._ev_last.synchronize()
        if self._flags:
            self._ev_flags.synchronize()
            dev = self._sae.W_enc.device
            for (r0, r1), ovf in zip(self._flags, self._flags_host.tolist()):
                if ovf:  # the chunk's CSR staging overflowed: redo it on the exact-size route
                    self._out[r0:r1].copy_(forward(self._sae, self._x[r0:r1].to(dev)))
        self._keep = None
        self._done = True
        return self._out


def forward_host(sae, x, out=None, *, chunk_tokens=8192):
    """forward() for a batch held in host memory, returning host memory.

    x: [M, d_in] CPU tensor (pinned for the copies to overlap; pageable x is pinned first).
    out: optional [M, d_in] pinned CPU tensor of W_dec's dtype to write into.
    The batch runs in chunks of at most `chunk_tokens` rows on sae's device: host-to-device
    copies on one stream, encode and decode on the current stream, device-to-host copies on
    a third, each chunk starting as soon as its rows have arrived, so only the first chunk's
    copy in and the last chunk's copy out are not overlapped (the chunk plan keeps those two
    small). Batches up to WHOLE_BATCH_DEVICE_BYTES get device buffers of their own; larger
    ones reuse two chunk buffers per direction. One host wait at the end for the last copy
    and every chunk's overflow flag; a chunk whose CSR staging overflowed is redone through
    forward(). Equivalent to forward_host_async(...).wait().
    """
    return forward_host_async(sae, x, out, chunk_tokens=chunk_tokens).wait()


def forward_host_async(sae, x, out=None, *, chunk_tokens=8192):
    """forward_host() without the host wait: queues the batch's copies and kernels and returns
    a HostForward whose wait() returns `out`. Consecutive calls overlap: a call's copies in
    start while the previous call still computes, and its compute follows the previous
    call's on the current stream, so a stream of host batches keeps only the first copy in
    and the last copy out exposed. x and out must stay untouched until wait() returns.

    chunk_tokens=None: no split for overlap inside the call (each chunk costs ~0.1 ms at
    config 2), only forward()'s launches (forward_launch_rows); the choice for a stream of
    batches, whose copies overlap the neighbouring calls' compute instead."""
    if x.is_cuda:
        raise ValueError("forward_host takes a host tensor; call forward() for a device tensor")
    if x.dim() != 2 or x.shape[1] != sae.W_enc.shape[0]:
        raise ValueError(f"x must be [M, {sae.W_enc.shape[0]}], got {tuple(x.shape)}")
    if chunk_tokens is not None and chunk_tokens < 1:
        raise ValueError("chunk_tokens must be positive or None")
    dev = sae.W_enc.device
    if dev.type != "cuda":
        raise ValueError("the SAE's weights must be on a CUDA device")
    M, K, D, dt = x.shape[0], x.shape[1], sae.W_dec.shape[1], sae.W_dec.dtype
    if out is None:
        out = torch.empty(M, D, dtype=dt, pin_memory=True)
    elif out.is_cuda or tuple(out.shape) != (M, D) or out.dtype != dt:
        raise ValueError(f"out must be a host tensor [M, {D}] of {dt}")
    if M == 0:
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(dev))
        return HostForward(sae, x, out, [], None, done, done, None)
    if not x.is_pinned():
        x = x.pin_memory()
    compute = torch.cuda.current_stream(dev)
    h2d, d2h = _streams(dev)
    whole = M * (K * x.element_size() + D * out.element_size()) <= WHOLE_BATCH_DEVICE_BYTES
    plan = _even_split(M, forward_launch_rows(sae)) if chunk_tokens is None else _chunk_plan(M, chunk_tokens)
    rows = M if whole else max(plan)
    nbuf = 1 if whole else 2
    # Each device buffer comes from the pool of the stream that writes it (x: the copy-in
    # stream, x_hat: the compute stream), so the allocator orders its reuse after that
    # stream's earlier work; record_stream covers the stream that reads it.
    with torch.cuda.stream(h2d):
        xbuf = [torch.empty(rows, K, dtype=x.dtype, device=dev) for _ in range(nbuf)]
    obuf = [torch.empty(rows, D, dtype=dt, device=dev) for _ in range(nbuf)]
    for b in xbuf:
        b.record_stream(compute)
    for b in obuf:
        b.record_stream(d2h)
    bounds = []
    r1 = 0
    for n in plan:
        bounds.append((r1, r1 + n))
        r1 += n

    def slot(i, r0, r1):  # (x slice, x_hat slice) of chunk i in its device buffer
        if whole:
            return xbuf[0][r0:r1], obuf[0][r0:r1]
        return xbuf[i % 2][:r1 - r0], obuf[i % 2][:r1 - r0]

    ev_in = [torch.cuda.Event() for _ in plan]
    ev_done = [torch.cuda.Event() for _ in plan]
    ev_out = [torch.cuda.Event() for _ in plan]

    def copy_in(i):
        r0, r1 = bounds[i]
        with torch.cuda.stream(h2d):
            if not whole and i >= 2:
                h2d.wait_event(ev_done[i - 2])  # chunk i-2 has finished reading this buffer
            slot(i, r0, r1)[0].copy_(x[r0:r1], non_blocking=True)
            ev_in[i].record(h2d)

    if whole:
        for i in range(len(plan)):  # every copy in is queued at once: the copy engine streams
            copy_in(i)
    flags, bounds_f = [], []
    for i, (r0, r1) in enumerate(bounds):
        if not whole:
            copy_in(i)
        xs, os_ = slot(i, r0, r1)
        compute.wait_event(ev_in[i])
        if not whole and i >= 2:
            compute.wait_event(ev_out[i - 2])  # chunk i-2's result has left this buffer
        _, overflow = _forward_async(sae, xs, os_)
        ev_done[i].record(compute)
        if overflow is not None:
            flags.append(overflow)
            bounds_f.append((r0, r1))
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev_done[i])
            out[r0:r1].copy_(os_, non_blocking=True)
            ev_out[i].record(d2h)
    flags_host, ev_flags, stacked = None, None, None
    if flags:
        # The flags come back on the copy-out stream, behind this call's last chunk: a copy on
        # the compute stream would share the copy engine with the previous call's copy out and
        # hold the next call's kernels behind it (measured at config 2: 4.96 against 4.05 ms
        # per batch in a stream of batches).
        stacked = torch.stack(flags)
        ev_stacked = torch.cuda.Event()
        ev_stacked.record(compute)
        flags_host = torch.empty(len(flags), dtype=stacked.dtype, pin_memory=True)
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev_stacked)
            flags_host.copy_(stacked, non_blocking=True)
            ev_flags = torch.cuda.Event()
            ev_flags.record(d2h)
        stacked.record_stream(d2h)
    return HostForward(sae, x, out, bounds_f, flags_host, ev_flags, ev_out[-1], (xbuf, obuf, stacked))
