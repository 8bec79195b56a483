"""Multi-GPU SAE forward: token sharding and d_sae (feature) sharding.

The reference is single-device; both modes are new.

* Token sharding: tokens are independent rows, so each rank runs the single-GPU path on
  its own contiguous token slice with replicated weights. No collective on the data path.
* Feature sharding (`FeatureShardedSAE`): rank r owns the contiguous feature range
  S_r = [start, stop): W_enc[:, S_r], b_enc[S_r], threshold[S_r], W_dec[S_r, :]
  (b_dec is replicated). Each rank encodes every token against its features, decodes
  its partial reconstruction sum_j f_j W_dec[j] in fp32 without b_dec, and an
  all-reduce(SUM) over the ranks combines the partials; b_dec is added once after it.
  The work is chunked over tokens and the all-reduce of chunk i runs (asynchronously,
  on the process group's stream) while chunk i+1 is encoded.

TopK SAEs are not feature-shardable without a global top-k merge; they are rejected.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced split of range(n): the first n % world ranks get one extra."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def token_shard(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's contiguous slice of the token rows of x."""
    s, e = shard_range(x.shape[0], world, rank)
    return x[s:e]


@dataclass
class _LocalSAE:
    W_enc: torch.Tensor
    b_enc: torch.Tensor
    W_dec: torch.Tensor
    b_dec: torch.Tensor
    threshold: torch.Tensor | None
    activation: str
    k: int | None = None


class _CudaOps:
    """The single-GPU kernels of this package."""

    @staticmethod
    def encode_sparse(sae, x):
        from .ops import encode_sparse

        return encode_sparse(sae, x)

    @staticmethod
    def decode_partial(csr, W_dec):
        from .kernels import sparse_decode

        return sparse_decode(*csr, W_dec, None, out_dtype=torch.float32)

    @staticmethod
    def partial_async(sae, x):
        """fp32 partial decode of x against this rank's features (no b_dec) with the CSR kept
        on the device: (partial, overflow flag as a device scalar or None), no host sync."""
        from .ops import _forward_async

        return _forward_async(sae, x, add_b_dec=False, out_dtype=torch.float32)


class FeatureShardedSAE:
    """d_sae-sharded SAE over a process group (see module docstring).

    sae: an object with the SAE attributes holding the FULL weights (or any object whose
    W_enc / W_dec are already this rank's slices, with `feature_start` set).
    ops: kernel provider (default: this package's CUDA kernels); tests substitute a CPU one.
    """

    def __init__(self, sae, group=None, ops=None, chunk_tokens: int = 4096):
        if sae.activation == "topk":
            raise ValueError("TopK SAEs need a global top-k merge and are not feature-shardable")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        start = getattr(sae, "feature_start", None)
        if start is not None:
            # Already this rank's slice (a caller that never holds the full weights).
            self.start, self.stop = int(start), int(start) + sae.W_enc.shape[1]
            self.local = _LocalSAE(W_enc=sae.W_enc, b_enc=sae.b_enc, W_dec=sae.W_dec, b_dec=sae.b_dec,
                                   threshold=sae.threshold, activation=sae.activation)
        else:
            self.start, self.stop = shard_range(sae.W_enc.shape[1], self.world, self.rank)
            sl = slice(self.start, self.stop)
            thr = sae.threshold[sl].contiguous() if sae.threshold is not None else None
            self.local = _LocalSAE(W_enc=sae.W_enc[:, sl].contiguous(), b_enc=sae.b_enc[sl].contiguous(),
                                   W_dec=sae.W_dec[sl].contiguous(), b_dec=sae.b_dec, threshold=thr,
                                   activation=sae.activation)
        self.ops = ops or _CudaOps()
        self.chunk_tokens = chunk_tokens

    def encode_sparse(self, x):
        """This rank's CSR for every token, with GLOBAL feature ids (local id + start)."""
        indptr, indices, values = self.ops.encode_sparse(self.local, x)
        return indptr, indices + self.start, values

    def _partial(self, x):
        if hasattr(self.ops, "partial_async"):
            return self.ops.partial_async(self.local, x)
        return self.ops.decode_partial(self.ops.encode_sparse(self.local, x), self.local.W_dec), None

    def forward(self, x, out_dtype=None):
        """x_hat for every token: partial decodes all-reduced over the ranks, + b_dec.

        The CSR of each chunk stays on the device (no host sync per chunk); one small
        all-reduce(MAX) of the chunks' CSR-staging overflow flags at the end tells every rank
        which chunks to redo through the exact-size route, so all ranks issue the same
        collectives in the same order."""
        out_dtype = out_dtype or self.local.W_dec.dtype
        M = x.shape[0]
        out = torch.empty(M, self.local.W_dec.shape[1], dtype=out_dtype, device=x.device)
        pending = []  # (work, partial, row slice)
        flags = []
        chunks = [(r0, min(M, r0 + self.chunk_tokens)) for r0 in range(0, M, self.chunk_tokens)]
        for r0, r1 in chunks:
            partial, overflow = self._partial(x[r0:r1])
            flags.append(overflow.reshape(1).to(torch.int32) if overflow is not None
                         else torch.zeros(1, dtype=torch.int32, device=x.device))
            work = dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group, async_op=True) \
                if self.world > 1 else None
            pending.append((work, partial, r0, r1))
            # finish chunks whose reduction had a full chunk of compute to overlap with
            while len(pending) > 1:
                self._finish(pending.pop(0), out)
        while pending:
            self._finish(pending.pop(0), out)
        if flags:
            redo = torch.cat(flags)
            if self.world > 1:
                dist.all_reduce(redo, op=dist.ReduceOp.MAX, group=self.group)
            for (r0, r1), bad in zip(chunks, redo.tolist()):
                if bad:
                    partial = self.ops.decode_partial(self.ops.encode_sparse(self.local, x[r0:r1]), self.local.W_dec)
                    if self.world > 1:
                        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
                    self._finish((None, partial, r0, r1), out)
        return out

    def _finish(self, item, out):
        work, partial, r0, r1 = item
        if work is not None:
            work.wait()
        partial += self.local.b_dec.float()
        out[r0:r1] = partial.to(out.dtype)
