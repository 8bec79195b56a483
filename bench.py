"""Benchmark of the SAE hot path (encode -> CSR -> decode) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|reference-triton]
                    [--config 1..5] [--partition token|feature] [--route csr|dense]

One step = one forward pass over one batch of synthetic tokens, as saeflow_b200.forward
runs it: the encoder GEMM writing CSR straight from its epilogue, the sync-free indptr scan
and placement, the CSR decode. Default workload: BASELINE config 2, JumpReLU SAE d_in=2304
d_sae=65536 bf16, 16384 tokens per GPU, inputs generated with that config's distributions
(seeded; the reference benchmarks on synthetic data too). `e2e` times
saeflow_b200.forward_host on pinned host tokens (copies inside the timed region).

Multi-GPU (torchrun, one process per GPU, NCCL): token-sharded with replicated weights,
per-GPU work fixed ("weak" scaling), no collective on the data path; the timed region
is bracketed by a barrier + synchronize and the max over ranks is reported. Config 5 is
strong scaling over a fixed 262144-token job, token- or feature-sharded.

--impl reference times the reference's CPU implementation of the path (the CPU
restatement in oracle/: dense torch SAE encode -> to_sparse_csr -> CSR addmm, as the
reference's bench does) on the host cores, on a bounded token sample per step.
--impl reference-triton times the reference's own GPU path (saeflow.forward and its Triton
kernels, installed unmodified in baseline/_ref) on one GPU with this arm's inputs.
"""

from __future__ import annotations

import argparse
import json
import re
import math
import os
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "tokens/s encode->CSR->decode"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

CONFIGS = {
    1: dict(name="cfg1 ReLU fp32 d_in=768 d_sae=16384", activation="relu", d_in=768, d_sae=16384,
            dtype=torch.float32, tokens=4096),
    2: dict(name="cfg2 JumpReLU bf16 d_in=2304 d_sae=65536", activation="jumprelu", d_in=2304, d_sae=65536,
            dtype=torch.bfloat16, tokens=16384, l0=64.0),
    3: dict(name="cfg3 sparse decode bf16 d_in=2304 d_sae=65536", activation="decode", d_in=2304, d_sae=65536,
            dtype=torch.bfloat16, tokens=65536, l0=64.0),
    4: dict(name="cfg4 TopK k=32 bf16 d_in=4096 d_sae=131072", activation="topk", d_in=4096, d_sae=131072,
            dtype=torch.bfloat16, tokens=32768, k=32),
    # tokens = the whole job's batch, split over the ranks (token partition) or run on every
    # rank against its feature slice (feature partition): strong scaling.
    5: dict(name="cfg5 JumpReLU bf16 d_in=2304 d_sae=1048576", activation="jumprelu", d_in=2304, d_sae=1048576,
            dtype=torch.bfloat16, tokens=262144, l0=96.0),
}
CFG5_FEATURE_BLOCK = 65536  # config 5 weights are drawn per block of features (any rank count gets the same W)
TOKEN_CHUNK = 16384  # config 5 tokens are drawn per chunk of rows


# ------------------------------------------------------------------------------ inputs

def unit_rows(d_sae, d_in, gen, device):
    W = torch.randn(d_sae, d_in, generator=gen, device=device)
    W /= W.norm(dim=1, keepdim=True)
    return W


def zipf_probs(d_sae, total, gen, device, s=0.8, cap=0.5):
    """p_i proportional to rank^-s over a random permutation, scaled to sum `total`, each
    clipped to <= cap, iterated to a fixpoint (BASELINE config 2 threshold scheme)."""
    ranks = torch.randperm(d_sae, generator=gen, device=device).double() + 1.0
    w = ranks.pow(-s)
    p = w * (total / w.sum())
    for _ in range(100):
        p = torch.clamp(p, max=cap)
        free = p < cap
        deficit = total - p.sum()
        if deficit.abs() < 1e-9 or not free.any():
            break
        p[free] *= 1.0 + deficit / p[free].sum()
    return p.clamp(max=cap)


def normal_isf(p):
    """Phi^-1(1 - p) via erfinv (the inverse standard-normal survival function)."""
    return math.sqrt(2.0) * torch.erfinv(1.0 - 2.0 * p)


def make_sae(cfg_id, device, seed=0):
    """Weights of a config (identical on every rank: same seed)."""
    from saeflow_b200 import SAE

    c = CONFIGS[cfg_id]
    gen = torch.Generator(device=device).manual_seed(seed)
    act = "relu" if c["activation"] == "decode" else c["activation"]
    sae = SAE.__new__(SAE)
    torch.nn.Module.__init__(sae)
    sae.d_in, sae.d_sae, sae.activation, sae.k = c["d_in"], c["d_sae"], act, c.get("k")
    W_dec = unit_rows(c["d_sae"], c["d_in"], gen, device)
    dt = c["dtype"]
    sae.W_dec = torch.nn.Parameter(W_dec.to(dt), requires_grad=False)
    sae.W_enc = torch.nn.Parameter(W_dec.T.contiguous().to(dt), requires_grad=False)
    del W_dec
    sae.b_enc = torch.nn.Parameter(torch.zeros(c["d_sae"], device=device, dtype=dt), requires_grad=False)
    sae.b_dec = torch.nn.Parameter(torch.zeros(c["d_in"], device=device, dtype=dt), requires_grad=False)
    sae.threshold = None
    if cfg_id == 1:
        sae.b_enc.fill_(-2.66)
    elif cfg_id in (2, 3):
        sae.b_dec.copy_((torch.randn(c["d_in"], generator=gen, device=device) * 0.1).to(dt))
    elif cfg_id == 4:
        sae.b_enc.copy_((torch.randn(c["d_sae"], generator=gen, device=device) * 0.01).to(dt))
    if act == "jumprelu":
        p = zipf_probs(c["d_sae"], c["l0"], gen, device)
        sae.threshold = torch.nn.Parameter(normal_isf(p).float().to(dt), requires_grad=False)
    return sae


def make_sae_cfg5(device, start, stop, seed=0):
    """Config 5 weights restricted to features [start, stop). W_dec rows are drawn per block
    of CFG5_FEATURE_BLOCK features from a generator seeded by the block id, and the threshold
    permutation over all d_sae features from one generator, so every rank count and every
    feature slice sees the same SAE."""
    from saeflow_b200 import SAE

    c = CONFIGS[5]
    dt, d_in, d_sae = c["dtype"], c["d_in"], c["d_sae"]
    sae = SAE.__new__(SAE)
    torch.nn.Module.__init__(sae)
    sae.d_in, sae.d_sae, sae.activation, sae.k = d_in, stop - start, "jumprelu", None
    W_dec = torch.empty(stop - start, d_in, dtype=dt, device=device)
    for b0 in range(start - start % CFG5_FEATURE_BLOCK, stop, CFG5_FEATURE_BLOCK):
        gen = torch.Generator(device=device).manual_seed(seed * 7919 + 5_000_011 + b0 // CFG5_FEATURE_BLOCK)
        blk = unit_rows(CFG5_FEATURE_BLOCK, d_in, gen, device)
        lo, hi = max(start, b0), min(stop, b0 + CFG5_FEATURE_BLOCK)
        W_dec[lo - start:hi - start] = blk[lo - b0:hi - b0].to(dt)
        del blk
    sae.W_dec = torch.nn.Parameter(W_dec, requires_grad=False)
    sae.W_enc = torch.nn.Parameter(W_dec.T.contiguous(), requires_grad=False)
    gen = torch.Generator(device=device).manual_seed(seed * 7919 + 5_000_003)
    sae.b_enc = torch.nn.Parameter(torch.zeros(stop - start, device=device, dtype=dt), requires_grad=False)
    sae.b_dec = torch.nn.Parameter((torch.randn(d_in, generator=gen, device=device) * 0.1).to(dt),
                                   requires_grad=False)
    p = zipf_probs(d_sae, c["l0"], gen, device)[start:stop]
    sae.threshold = torch.nn.Parameter(normal_isf(p).float().to(dt), requires_grad=False)
    sae.feature_start = start
    return sae


def make_token_range(cfg_id, t0, t1, device):
    """Rows [t0, t1) of a config's token stream, drawn per TOKEN_CHUNK rows from a generator
    seeded by the chunk id (the same rows at any rank count)."""
    c = CONFIGS[cfg_id]
    out = torch.empty(t1 - t0, c["d_in"], dtype=c["dtype"], device=device)
    for ch in range(t0 // TOKEN_CHUNK, (t1 + TOKEN_CHUNK - 1) // TOKEN_CHUNK):
        c0 = ch * TOKEN_CHUNK
        gen = torch.Generator(device=device).manual_seed(1_000_003 + 131 * cfg_id + ch)
        rows = torch.randn(TOKEN_CHUNK, c["d_in"], generator=gen, device=device)
        lo, hi = max(t0, c0), min(t1, c0 + TOKEN_CHUNK)
        out[lo - t0:hi - t0] = rows[lo - c0:hi - c0].to(c["dtype"])
    return out


def make_tokens(cfg_id, chunk, device, tokens=None):
    """Token batch `chunk` of a config (seed + chunk id, so a chunk is the same at any GPU count)."""
    c = CONFIGS[cfg_id]
    gen = torch.Generator(device=device).manual_seed(1_000_003 + chunk)
    T = tokens or c["tokens"]
    return torch.randn(T, c["d_in"], generator=gen, device=device).to(c["dtype"])


def make_csr(cfg_id, chunk, device, tokens=None):
    """Config 3 CSR: nnz ~ Poisson(L0) per row, indices without replacement from Zipf(1.1)
    over a random permutation (Gumbel-top-k), sorted; values |N(0,1)|*2."""
    c = CONFIGS[cfg_id]
    gen = torch.Generator(device=device).manual_seed(2_000_003 + chunk)
    T = tokens or c["tokens"]
    d_sae = c["d_sae"]
    perm = torch.randperm(d_sae, generator=gen, device=device)
    logp = torch.empty(d_sae, device=device)
    logp[perm] = -1.1 * torch.log(torch.arange(1, d_sae + 1, device=device, dtype=torch.float32))
    counts = torch.poisson(torch.full((T,), c["l0"], device=device), generator=gen).long().clamp(0, 256)
    kmax = int(counts.max())
    idx_rows = []
    for r0 in range(0, T, 2048):
        r1 = min(T, r0 + 2048)
        u = torch.rand(r1 - r0, d_sae, generator=gen, device=device).clamp_(1e-12, 1 - 1e-7)
        keys = logp - torch.log(-torch.log(u))
        idx_rows.append(keys.topk(kmax, dim=1).indices)
        del u, keys
    top = torch.cat(idx_rows)  # [T, kmax] in key order
    mask = torch.arange(kmax, device=device)[None, :] < counts[:, None]
    sel = torch.where(mask, top, torch.full_like(top, d_sae))  # pad sorts last
    sel = sel.sort(dim=1).values
    indices = sel[mask.sort(dim=1, descending=True).values].to(torch.int32)
    indptr = torch.zeros(T + 1, dtype=torch.int64, device=device)
    indptr[1:] = counts.cumsum(0)
    values = (torch.randn(indices.numel(), generator=gen, device=device).abs() * 2).to(c["dtype"])
    return indptr, indices, values


# ------------------------------------------------------------------------------ measurement helpers

def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """SM clock and throttle reasons of this GPU, sampled every 10 ms through NVML while
    the timed region runs (nvidia-smi's 200 ms loop misses short regions)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index, period_s=0.01):
        self.samples = []
        self.period = period_s
        self.stop = threading.Event()
        self.handle = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            uuid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.nv = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode() if isinstance(uuid, str) else uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - no NVML: report no samples
            self.handle = None

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                util = nv.nvmlDeviceGetUtilizationRates(self.handle).gpu
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                power_w = nv.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                self.samples.append((sm, util, reasons, power_w))
            except Exception:  # noqa: BLE001
                pass
            self.stop.wait(self.period)

    def __enter__(self):
        if self.handle is not None:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.handle is not None:
            self.stop.set()
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in self.samples if s[1] >= 50] or self.samples
        sms = sorted(s[0] for s in loaded)
        seen = 0
        for s in loaded:
            seen |= s[2]
        reasons = sorted(n for n, bit in self.REASONS.items() if seen & bit)
        watts = sorted(s[3] for s in loaded)
        return {"sm_mhz": sms[len(sms) // 2], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "power_w_median": round(watts[len(watts) // 2], 1),
                "samples": len(self.samples), "samples_under_load": len(loaded), "source": "nvml 10 ms"}


def ieee_launches(d_in):
    """Kernels per forward chunk on the IEEE fp32 split route: per K range (at most 1024 of
    d_in, ranges of a multiple of 64 as even as possible) the x split, the W_enc split and
    the GEMM; then the two gated fallback launches, the indptr scan, placement and decode."""
    ranges = -(-d_in // 1024)
    kc = -(-(-(-d_in // ranges)) // 64) * 64 if ranges > 1 else d_in
    return 3 * -(-d_in // kc) + 5


def encode_errors(sae, x, f, rows=4096):
    """Max and rms |error| of encoder output rows f[:rows] against the float64 product of the
    same operands (activation applied to the float64 pre-activations)."""
    xs = x[:rows].double() - sae.b_dec.double()
    pre = xs @ sae.W_enc.double() + sae.b_enc.double()
    want = pre.clamp_min(0)
    if sae.activation == "jumprelu":
        want = torch.where(pre > sae.threshold.double(), want, torch.zeros((), dtype=want.dtype, device=want.device))
    d = (f[:rows].double() - want).abs()
    return {"rows": int(d.shape[0]), "max_abs": float(d.max()), "rms": float(d.pow(2).mean().sqrt())}


def l2_flush(buf):
    buf.add_(1)  # 256 MB read+write: evicts the 126 MB L2 between steps


# ------------------------------------------------------------------------------ our arm

def run_ours(args, rank, world, device):
    from saeflow_b200 import forward_host
    from saeflow_b200.kernels import dense_to_csr, device_error, fused_encode, sparse_decode, topk_encode
    from saeflow_b200.kernels.encode import encode_csr_finish_async, encode_csr_stage

    cfg_id = args.config
    c = CONFIGS[cfg_id]
    T = args.tokens or c["tokens"]
    job_tokens = world * T  # tokens the whole job processes per step (weak scaling)
    sharded = None
    if cfg_id == 5:
        from saeflow_b200.sharded import FeatureShardedSAE, shard_range

        job_tokens = T  # strong scaling: the job's batch is fixed
        if args.partition == "feature":
            f0, f1 = shard_range(c["d_sae"], world, rank)
            sae = make_sae_cfg5(device, f0, f1)
            x = make_token_range(5, 0, T, device)
            sharded = FeatureShardedSAE(sae, chunk_tokens=args.chunk_tokens)
        else:
            t0, t1 = shard_range(T, world, rank)
            sae = make_sae_cfg5(device, 0, c["d_sae"])
            x = make_token_range(5, t0, t1, device)
            T = t1 - t0
    else:
        sae = make_sae(cfg_id, device)
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    quads = 0  # CSR route: CUDA-event quads per step (start, encoded, CSR placed, decoded), one per chunk

    if args.train:
        # A training step on sparse features: the autograd forward and its backward kernels.
        from saeflow_b200 import training

        if cfg_id not in (1, 2, 4):
            raise SystemExit("--train runs configs 1, 2 and 4")
        x = make_tokens(cfg_id, rank, device, T)
        for name in ("W_enc", "b_enc", "W_dec", "b_dec"):
            getattr(sae, name).requires_grad_(True)
        grad_out = (torch.randn(T, c["d_in"], generator=torch.Generator(device=device).manual_seed(7),
                                device=device) * 1e-2).to(c["dtype"])

        def step(ev):
            ev[0].record(stream)
            out = training.forward(sae, x)
            ev[1].record(stream)
            ev[2].record(stream)
            torch.autograd.backward(out, grad_out)
            ev[3].record(stream)
            for name in ("W_enc", "b_enc", "W_dec", "b_dec"):
                getattr(sae, name).grad = None
            return out
        # forward 5 (4 for TopK); backward: count, scan, scatter, 2 in-column sorts, 2 x (gather, carry),
        # transpose of dW_enc, matvec for db_dec (x takes no gradient here)
        launches_per_step = 16
    elif sharded is not None:
        n_chunks = (T + args.chunk_tokens - 1) // args.chunk_tokens

        def step(ev):
            ev[0].record(stream)
            out = sharded.forward(x)
            ev[3].record(stream)
            return out
        launches_per_step = 5 * n_chunks  # per token chunk: shift, encode+stage, indptr scan, place, decode
    elif cfg_id == 3:
        csr = make_csr(cfg_id, rank, device, T)

        def step(ev):
            ev[0].record(stream)
            out = sparse_decode(*csr, sae.W_dec, sae.b_dec)
            ev[3].record(stream)
            return out
        launches_per_step = 1
    elif cfg_id == 4:
        x = make_tokens(cfg_id, rank, device, T)
        indptr = torch.arange(0, T * c["k"] + 1, c["k"], device=device, dtype=torch.int64)

        def step(ev):
            ev[0].record(stream)
            vals, idx = topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, c["k"])
            ev[1].record(stream)
            ev[2].record(stream)
            out = sparse_decode(indptr, idx.view(-1), vals.view(-1), sae.W_dec, sae.b_dec)
            ev[3].record(stream)
            return out
        launches_per_step = 4  # shift, encode+top-k, merge, decode
    elif args.route == "dense":
        # The reference's route: dense features, then compaction.
        x = make_tokens(cfg_id, rank, device, T)
        row_nnz = torch.zeros(T, dtype=torch.int32, device=device)

        def step(ev):
            row_nnz.zero_()
            ev[0].record(stream)
            f = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation, row_nnz=row_nnz)
            ev[1].record(stream)
            csr = dense_to_csr(f, row_nnz)
            ev[2].record(stream)
            out = sparse_decode(*csr, sae.W_dec, sae.b_dec)
            ev[3].record(stream)
            step.nnz = csr[1].numel()
            del f
            return out
        # shift, encode, indptr scan, compact, decode (IEEE fp32: two operand splits and two
        # gated fallback launches in place of the shift)
        launches_per_step = ieee_launches(c["d_in"]) if cfg_id == 1 else 5
    else:
        # Encode straight to CSR (what saeflow_b200.encode_sparse runs): no dense features.
        if cfg_id != 5:
            x = make_tokens(cfg_id, rank, device, T)

        # What saeflow_b200.forward runs: the CSR stays on the device (no host sync mid-step),
        # batches above forward_launch_rows(sae) rows as consecutive chunks into one output.
        from saeflow_b200.ops import forward_launch_rows

        R = forward_launch_rows(sae)
        chunks = [(r0, min(T, r0 + R)) for r0 in range(0, T, R)]
        quads = len(chunks)
        out_buf = torch.empty(T, c["d_in"], dtype=c["dtype"], device=device)

        def step(evs):
            for ev, (r0, r1) in zip(evs, chunks):
                ev[0].record(stream)
                h = encode_csr_stage(x[r0:r1], sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation,
                                     device_consumer=True)
                ev[1].record(stream)
                indptr, indices, values, overflow = encode_csr_finish_async(h)
                ev[2].record(stream)
                sparse_decode(indptr, indices, values, sae.W_dec, sae.b_dec, out=out_buf[r0:r1])
                ev[3].record(stream)
                step.checks.append((indptr[-1], overflow))
            return out_buf
        step.checks = []
        # per chunk: shift, encode+stage, indptr scan, place, decode; IEEE fp32 (config 1): the
        # operand splits of x and W_enc, the encode, the two gated non-finite-fallback launches
        # (no-ops on finite inputs), indptr scan, place, decode
        launches_per_step = (ieee_launches(c["d_in"]) if cfg_id == 1 else 5) * quads

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    def new_quads():
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(max(quads, 1))]
        return evs if quads else evs[0]

    events = [new_quads() for _ in range(args.steps)]
    for _ in range(args.warmup):
        l2_flush(flush)
        step(new_quads())
    barrier()
    with ClockSampler(device.index) as clk:
        barrier()
        wall0 = time.perf_counter()
        for i in range(args.steps):
            l2_flush(flush)
            step(events[i])
        barrier()
        wall = time.perf_counter() - wall0
    if getattr(step, "checks", None):
        nnz_ovf = torch.stack([torch.stack([a, b.to(torch.int64)]) for a, b in step.checks]).cpu()
        if int(nnz_ovf[:, 1].max()):
            raise RuntimeError("CSR staging overflowed inside the timed region: the step did not do the work")
        step.nnz = int(nnz_ovf[-quads:, 0].sum())  # the last step's chunks
        step.checks.clear()
    staged = cfg_id != 3 and sharded is None  # stage events recorded
    if quads:  # one event quad per forward chunk: stage times summed over the chunks
        step_ms = [e[0][0].elapsed_time(e[-1][3]) for e in events]
        stage_ms = [[sum(q[j].elapsed_time(q[j + 1]) for q in e) for j in range(3)] for e in events]
    else:
        step_ms = [e[0].elapsed_time(e[3]) for e in events]
        stage_ms = [[e[j].elapsed_time(e[j + 1]) for j in range(3)] for e in events] if staged else []
    enc_ms = [st[0] for st in stage_ms]
    csr_ms = [st[1] for st in stage_ms] if cfg_id in (1, 2, 5) else []
    dec_ms = [st[2] for st in stage_ms] if staged else (step_ms if cfg_id == 3 else [])
    total_ms = torch.tensor([sum(step_ms)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(total_ms, op=torch.distributed.ReduceOp.MAX)
    total_ms = float(total_ms.item())

    # ---- end to end through the public API with host buffers (H2D in, D2H out, per step)
    e2e = None
    if cfg_id in (1, 2, 4, 5) and not args.no_e2e and not args.train:
        x_host = x.cpu().pin_memory()
        out_host = torch.empty(T, c["d_in"], dtype=c["dtype"]).pin_memory()
        e_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]

        def e2e_step(ev):
            ev[0].record(stream)
            if sharded is not None:
                out_host.copy_(sharded.forward(x_host.to(device, non_blocking=True)), non_blocking=True)
            else:
                forward_host(sae, x_host, out_host, chunk_tokens=args.e2e_chunk)
            ev[1].record(stream)

        for _ in range(max(1, args.warmup)):
            l2_flush(flush)
            e2e_step([torch.cuda.Event(enable_timing=True) for _ in range(2)])
        barrier()
        for i in range(args.steps):
            l2_flush(flush)
            e2e_step(e_ev[i])
        barrier()
        e_tot = torch.tensor([sum(e[0].elapsed_time(e[1]) for e in e_ev)], dtype=torch.float64, device=device)
        if world > 1:
            torch.distributed.all_reduce(e_tot, op=torch.distributed.ReduceOp.MAX)
        e_tot = float(e_tot.item())
        nbytes = T * c["d_in"] * x.element_size()
        api = ("FeatureShardedSAE.forward(x)" if sharded is not None else
               f"saeflow_b200.forward_host(sae, x, out, chunk_tokens={args.e2e_chunk}) (copies overlapped with compute)")
        e2e_sync = {"value": round(job_tokens * args.steps / (e_tot / 1e3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
                    "ms_per_step": round(e_tot / args.steps, 4),
                    "api": f"{api} on pinned host x, result copied to pinned host (bytes per rank), "
                           "one call per step, each waited before the next"}
        e2e = e2e_sync
        if sharded is None:
            # A stream of host batches through forward_host_async with two calls in flight: the
            # next batch's copy in overlaps this batch's compute. Timed from an event before the
            # first step to one after the last step's last copy out (on the copy-out stream),
            # minus the L2 flushes queued between steps (events around each).
            from saeflow_b200 import forward_host_async
            from saeflow_b200.ops import _streams

            outs = [out_host, torch.empty_like(out_host).pin_memory()]
            d2h_stream = _streams(device)[1]

            def pipelined(n, timed):
                fl = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(n)]
                t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0.record(stream)
                pend = None
                for i in range(n):
                    fl[i][0].record(stream)
                    l2_flush(flush)
                    fl[i][1].record(stream)
                    p = forward_host_async(sae, x_host, outs[i % 2], chunk_tokens=None)
                    if pend is not None:
                        pend.wait()
                    pend = p
                t1.record(d2h_stream)
                pend.wait()
                torch.cuda.synchronize(device)
                return t0.elapsed_time(t1) - sum(a.elapsed_time(b) for a, b in fl) if timed else None

            pipelined(max(3, args.warmup), False)
            barrier()
            p_tot = torch.tensor([pipelined(args.steps, True)], dtype=torch.float64, device=device)
            barrier()
            if world > 1:
                torch.distributed.all_reduce(p_tot, op=torch.distributed.ReduceOp.MAX)
            p_tot = float(p_tot.item())
            e2e = {"value": round(job_tokens * args.steps / (p_tot / 1e3), 1), "unit": "tokens/s",
                   "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
                   "ms_per_step": round(p_tot / args.steps, 4),
                   "api": "saeflow_b200.forward_host_async(sae, x, out, chunk_tokens=None), two host batches "
                          "in flight (each step: pinned host x in, x_hat out to pinned host; the next step's "
                          "copies overlap this step's compute); L2 flush time between steps subtracted "
                          "(bytes per rank)",
                   "sync": e2e_sync}

    err = device_error(device)
    if err:
        raise RuntimeError(f"device error bits {err} after the timed region")

    if rank != 0:
        return None

    peaks, peak_src = load_peaks()
    mean = lambda v: sum(v) / len(v) if v else None  # noqa: E731
    e = c["dtype"].itemsize if hasattr(c["dtype"], "itemsize") else torch.finfo(c["dtype"]).bits // 8
    stages = {}
    roofline = None
    if args.train:
        # Forward (encode + CSR + decode) and backward (sddmm, CSR transpose, per-feature
        # accumulations, decode against W_enc^T) of saeflow_b200.training.
        fwd, bwd = mean(enc_ms), mean(dec_ms)
        flops = 2.0 * T * c["d_in"] * c["d_sae"]
        stages = {"step": "training: forward + backward", "forward_ms": round(fwd, 4), "backward_ms": round(bwd, 4),
                  "forward_encode_tflops_incl_decode": round(flops / (fwd / 1e3) / 1e12, 2)}
        nnz = None
        dec_ms = []
    elif sharded is not None:
        # Feature partition: every rank encodes all T tokens against its d_sae / world features;
        # the step (encode + CSR + decode + all-reduce of partials) is timed as a whole.
        n_feat = sharded.stop - sharded.start
        flops = 2.0 * T * c["d_in"] * n_feat
        step_mean = mean(step_ms)
        achieved = flops / (step_mean / 1e3) / 1e12
        tc_peak = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
        roofline = {"kernel": "whole feature-sharded step (encode GEMMs dominate)", "bound": "tensor",
                    "achieved": round(achieved, 2), "peak": tc_peak, "unit": "TFLOP/s",
                    "frac": round(achieved / tc_peak, 4), "traffic": None,
                    "peak_source": f"{peak_src} bf16_tflops_sustained",
                    "algorithmic": f"2*T*d_in*(d_sae/world) = {flops:.4g} FLOP per rank per step"}
        stages["partition"] = f"feature: features [{sharded.start}, {sharded.stop}) on rank 0, " \
                              f"all-reduce of fp32 partials per {args.chunk_tokens}-token chunk"
    elif cfg_id != 3:
        flops = 2.0 * T * c["d_in"] * c["d_sae"]
        enc = mean(enc_ms)
        achieved = flops / (enc / 1e3) / 1e12
        tc_peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        traffic = None
        tp = ROOT / "profiles" / f"traffic_cfg{cfg_id}.json"
        if tp.exists():
            traffic = json.loads(tp.read_text()).get("encode_dram_bytes_per_launch")
        if cfg_id == 1:
            # IEEE fp32 products from three-part bf16 splits of both operands: 6 bf16 partial
            # products per fp32 product on the tensor cores (the executed MMA work).
            mma = 6.0 * flops / (enc / 1e3) / 1e12
            roofline = {"kernel": "fused encode (operand split + tcgen05 GEMM of 6 bf16 partial products + epilogue)",
                        "bound": "tensor", "achieved": round(mma, 2), "peak": tc_peak, "unit": "TFLOP/s",
                        "frac": round(mma / tc_peak, 4), "traffic": traffic,
                        "peak_source": f"{peak_src} bf16_tflops (burst)",
                        "algorithmic": f"6 x 2*T*d_in*d_sae = {6 * flops:.4g} bf16 FLOP per launch "
                                       f"(fp32 work 2*T*d_in*d_sae = {flops:.4g} FLOP)"}
            stages["encode_fp32_equivalent_tflops"] = round(achieved, 2)
        else:
            roofline = {"kernel": "fused encode (shift pre-pass + tcgen05 GEMM + epilogue)",
                        "bound": "tensor", "achieved": round(achieved, 2), "peak": tc_peak, "unit": "TFLOP/s",
                        "frac": round(achieved / tc_peak, 4), "traffic": traffic,
                        "peak_source": f"{peak_src} bf16_tflops (burst)",
                        "algorithmic": f"2*T*d_in*d_sae = {flops:.4g} FLOP per launch"}
        stages["encode_ms"] = round(enc, 4)
        stages["encode_tflops"] = round(achieved, 2)
    dec = mean(dec_ms)
    if args.train:
        pass
    elif sharded is not None:
        nnz = None
    elif cfg_id in (1, 2, 5):
        stages["csr_ms"] = round(mean(csr_ms), 4)
        nnz = step.nnz
        l0 = nnz / T
        if args.route == "dense":
            comp_bytes = T * c["d_sae"] * e + nnz * (4 + e) + (T + 1) * 8
            stages["csr_gbps"] = round(comp_bytes / (mean(csr_ms) / 1e3) / 1e9, 1)
        stages["l0"] = round(l0, 2)
        stages["route"] = "dense+compaction" if args.route == "dense" else "encode straight to CSR"
    elif cfg_id == 3:
        nnz = csr[1].numel()
        l0 = nnz / T
    else:
        l0 = c["k"]
        nnz = T * l0
    if nnz is not None:
        dec_bytes = nnz * (c["d_in"] * e + 4 + e) + T * c["d_in"] * e + (T + 1) * 8
        stages["decode_ms"] = round(dec, 4)
        stages["decode_gbps_requested"] = round(dec_bytes / (dec / 1e3) / 1e9, 1)
    if cfg_id == 3:
        hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        roofline = {"kernel": "sparse decode (CSR gather)", "bound": "hbm",
                    "achieved": stages["decode_gbps_requested"], "peak": hbm, "unit": "GB/s",
                    "frac": round(stages["decode_gbps_requested"] / hbm, 4), "traffic": None,
                    "peak_source": f"{peak_src} hbm_gbs",
                    "algorithmic": "requested bytes L0*(d_in*e+4+e)+d_in*e+8 per token (bench_decode.py:57)"}

    value = job_tokens * args.steps / (total_ms / 1e3)
    if sharded is not None:
        parallelism = f"feature-sharded x{world}: d_sae/{world} features per rank, every rank encodes all " \
                      "tokens, NCCL all-reduce of fp32 partial decodes"
    else:
        parallelism = f"token-sharded x{world}, weights replicated, no data-path collective"
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if cfg_id == 5 else "weak", "vs_baseline": None,
        "dtype": "bf16" if c["dtype"] == torch.bfloat16 else ("fp32" if c["dtype"] == torch.float32 else "fp16"),
        "data": "synthetic (seeded, BASELINE config distributions)",
        "config": {"workload": c["name"], "tokens_per_gpu": T, "global_batch": job_tokens,
                   "parallelism": parallelism,
                   "l2": "flushed between steps (256 MB write, outside the per-step events)"},
        "impl": "ours",
        "stages": stages,
        "roofline": roofline,
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
        "wall_s_timed_region": round(wall, 3),
    }
    if args.accuracy and cfg_id in (1, 2) and sharded is None:
        acc = {"route": encode_errors(sae, x, fused_encode(x[:4096], sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold,
                                                              sae.activation))}
        if c["dtype"] == torch.float32:
            acc["cuda_core_ieee"] = encode_errors(sae, x, fused_encode(x[:4096], sae.W_enc, sae.b_enc, sae.b_dec,
                                                                      sae.threshold, sae.activation,
                                                                      config={"variant": "simt"}))
        line["accuracy"] = acc
    if not args.no_cpu_baseline and world == 1 and cfg_id != 5:
        line["cpu_baseline"] = cpu_baseline(cfg_id, budget_s=args.cpu_seconds)
    return line


# ------------------------------------------------------------------------------ CPU (reference) arm

def cpu_pipeline_setup(cfg_id, tokens):
    """Weights and a token sample on the CPU, from the same generators (CPU RNG)."""
    sae = make_sae(cfg_id, torch.device("cpu"))
    import oracle

    ref = oracle.RefSAE.__new__(oracle.RefSAE)
    torch.nn.Module.__init__(ref)
    ref.d_in, ref.d_sae, ref.activation, ref.k = sae.d_in, sae.d_sae, sae.activation, sae.k
    for name in ("W_enc", "W_dec", "b_enc", "b_dec", "threshold"):
        setattr(ref, name, getattr(sae, name))
    ref.W_dec32, ref.b_dec32 = ref.W_dec.float(), ref.b_dec.float()
    x = make_tokens(cfg_id if cfg_id != 3 else 2, 0, torch.device("cpu"), tokens)
    return ref, x


def cpu_step(ref, x):
    """The reference's CPU path: dense SAE encode -> to_sparse_csr -> addmm(b_dec, csr, W_dec)
    (saeflow/reference.py:36-46, bench/bench_decode.py:61-64,90). The CPU CSR addmm has no
    bf16 kernel, so a 16-bit SAE decodes through fp32 copies of W_dec / b_dec made once at
    set-up (`ref.W_dec32`) and the result is cast back."""
    f = ref.encode(x)
    csr = f.to_sparse_csr()
    if ref.W_dec.dtype == torch.float32:
        return torch.addmm(ref.b_dec.expand(x.shape[0], -1), csr, ref.W_dec)
    csr32 = torch.sparse_csr_tensor(csr.crow_indices(), csr.col_indices(), csr.values().float(), csr.shape)
    return torch.addmm(ref.b_dec32.expand(x.shape[0], -1), csr32, ref.W_dec32).to(ref.W_dec.dtype)


def cpu_model():
    """The host CPU's model name (from /proc/cpuinfo), for the baseline record."""
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def time_cpu(fn, budget_s):
    """Runs fn until `budget_s` seconds have passed (at least once): (iterations, seconds)."""
    t0 = time.perf_counter()
    n = 0
    while True:
        fn()
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return n, time.perf_counter() - t0


def cpu_dense_forward_row(ref, x, budget_s):
    """The second CPU row: the reference's dense SAE.forward, decode(encode(x)) with the dense
    [M, d_sae] features and a dense product with W_dec (saeflow/reference.py:51-52)."""
    ref.forward(x[:16])  # warm-up
    n, dt = time_cpu(lambda: ref.forward(x), budget_s)
    return {"value": round(n * x.shape[0] / dt, 1), "unit": "tokens/s",
            "sample": f"{n} x {x.shape[0]} tokens in {dt:.1f} s (oracle restatement of saeflow.reference.SAE.forward)"}


def cpu_baseline(cfg_id, budget_s=10.0, sample_tokens=None):
    cores = host_threads()
    ref, x = cpu_pipeline_setup(cfg_id, sample_tokens or (1024 if cfg_id != 1 else 4096))
    cpu_step(ref, x[:64])  # warm-up
    n, dt = time_cpu(lambda: cpu_step(ref, x), budget_s)
    return {"value": round(n * x.shape[0] / dt, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
            "cpu_model": cpu_model(), "logical_cpus": os.cpu_count(),
            "sample": f"{n} x {x.shape[0]} tokens of {CONFIGS[cfg_id]['name']} in {dt:.1f} s "
                      "(oracle restatement of the reference CPU path: dense encode -> to_sparse_csr -> addmm)",
            "dense_forward": cpu_dense_forward_row(ref, x, budget_s / 2)}


def run_reference_triton(args, device):
    """The reference's own GPU path (saeflow.forward with its Triton kernels, installed
    unmodified in baseline/_ref) on the same config, inputs and timing as our arm."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "saeflow").is_dir():
        return {"impl": "reference-triton", "unavailable": "baseline/_ref does not hold the reference package"}
    sys.path.insert(0, str(ref_dir))
    import saeflow

    cfg_id = args.config
    if cfg_id not in (1, 2, 4):
        return {"impl": "reference-triton", "unavailable": f"config {cfg_id} has no forward pass to time"}
    c = CONFIGS[cfg_id]
    T = args.tokens or c["tokens"]
    sae = make_sae(cfg_id, device)
    x = make_tokens(cfg_id, 0, device, T)
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    def timed(fn, steps):
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(steps)]
        for ev in evs:
            l2_flush(flush)
            ev[0].record(stream)
            fn()
            ev[1].record(stream)
        torch.cuda.synchronize(device)
        return sum(e[0].elapsed_time(e[1]) for e in evs)

    for _ in range(args.warmup):  # includes the reference's Triton autotuning
        l2_flush(flush)
        saeflow.forward(sae, x)
    with ClockSampler(device.index) as clk:
        total = timed(lambda: saeflow.forward(sae, x), args.steps)
    x_host = x.cpu().pin_memory()
    out_host = torch.empty(T, c["d_in"], dtype=c["dtype"]).pin_memory()
    e_total = timed(lambda: out_host.copy_(saeflow.forward(sae, x_host.to(device, non_blocking=True)),
                                           non_blocking=True), args.steps)
    nbytes = T * c["d_in"] * x.element_size()
    line = {
        "metric": METRIC, "value": round(T * args.steps / (total / 1e3), 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if c["dtype"] == torch.bfloat16 else "fp32", "data": "synthetic (seeded)",
        "config": {"workload": c["name"], "tokens_per_gpu": T,
                   "l2": "flushed between steps (256 MB write, outside the per-step events)"},
        "impl": "reference-triton",
        "api": "saeflow.forward(sae, x) from baseline/_ref (the reference's Triton kernels, unmodified)",
        "e2e": {"value": round(T * args.steps / (e_total / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes},
        "clocks": clk.summary(),
    }
    if args.accuracy and cfg_id in (1, 2):
        f = saeflow.kernels.fused_encode(x[:4096], sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation)
        line["accuracy"] = {"route": encode_errors(sae, x, f)}
    return line


def host_threads():
    """Every host thread this process may run on: torchrun sets OMP_NUM_THREADS=1 per rank, and
    the CPU baselines (rank 0 alone) use the whole host."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    return n


def run_reference(args):
    cfg_id = args.config
    c = CONFIGS[cfg_id]
    sample = args.cpu_tokens
    host_threads()
    ref, x = cpu_pipeline_setup(cfg_id, sample)
    for _ in range(args.warmup):
        cpu_step(ref, x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(ref, x)
    dt = time.perf_counter() - t0
    value = args.steps * sample / dt
    cores = torch.get_num_threads()
    desc = (f"{sample} tokens per step of {c['name']} on {cores} host threads "
            "(oracle restatement of the reference CPU path: dense encode -> to_sparse_csr -> addmm)")
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if c["dtype"] == torch.bfloat16 else "fp32", "data": "synthetic (seeded)",
        "config": {"workload": c["name"], "tokens_per_step": sample, "parallelism": "host CPU, rank 0 only"},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "cpu_model": cpu_model(), "logical_cpus": os.cpu_count(), "sample": desc,
                         "dense_forward": cpu_dense_forward_row(ref, x, args.cpu_seconds / 2)},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------------------ main

def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-triton"], default="ours",
                    help="reference: the reference's CPU path (the driver's reference arm); reference-triton: "
                         "the reference's own GPU kernels from baseline/_ref, one GPU")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=2)
    ap.add_argument("--tokens", type=int, default=None, help="tokens per GPU (default: the config's)")
    ap.add_argument("--cpu-tokens", type=int, default=1024, help="reference arm: tokens per step")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="cpu_baseline time budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--train", action="store_true",
                    help="one step = forward + backward of saeflow_b200.training (configs 1, 2, 4)")
    ap.add_argument("--e2e-chunk", type=int, default=8192, help="forward_host chunk size (tokens)")
    ap.add_argument("--partition", choices=["token", "feature"], default="token",
                    help="config 5: token-sharded (weights replicated) or feature-sharded (d_sae split)")
    ap.add_argument("--chunk-tokens", type=int, default=16384,
                    help="config 5 feature partition: tokens per all-reduced chunk")
    ap.add_argument("--route", choices=["csr", "dense"], default="csr",
                    help="csr: encode straight to CSR (default); dense: dense features + compaction")
    ap.add_argument("--d-in", type=int, default=None, help="configs 1-4: override d_in (same distributions)")
    ap.add_argument("--d-sae", type=int, default=None, help="configs 1-4: override d_sae (same distributions)")
    ap.add_argument("--accuracy", action="store_true",
                    help="fp32 configs: add the encoder's error against a float64 product (and, for this build, "
                         "the CUDA-core IEEE kernel's) on up to 4096 rows")
    args = ap.parse_args(argv)
    if args.d_in or args.d_sae:
        if args.config == 5:
            ap.error("--d-in / --d-sae apply to configs 1-4")
        c = dict(CONFIGS[args.config])
        c["d_in"], c["d_sae"] = args.d_in or c["d_in"], args.d_sae or c["d_sae"]
        c["name"] = re.sub(r"d_in=\d+ d_sae=\d+", f"d_in={c['d_in']} d_sae={c['d_sae']}", c["name"])
        CONFIGS[args.config] = c

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return 0
    if args.impl == "reference-triton":
        if rank == 0:
            device = torch.device("cuda", local_rank)
            torch.cuda.set_device(device)
            print(json.dumps(run_reference_triton(args, device)), flush=True)
        return 0

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    try:
        line = run_ours(args, rank, world, device)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
