"""Activation caching with on-the-fly SAE encoding: a drop-in for saeflow/cache.py.

The on-disk format, the manifest, the resume rule and the reader's batches are the
reference's (saeflow/cache.py:1-14, :70-137, :140-194), because other tools read this
format; the code that writes and reads it is this package's own:

    manifest.json                                   config + list of finished shards
    <hook>/<shard:05d>.npy                          dense activations [rows, d]
    <hook>/<shard:05d>.{indptr,indices,values}.npy  CSR SAE features [rows, d_sae]

A row is one token position, in sequence-major order; a shard covers
`batches_per_shard` forward batches; bf16 is stored as its raw int16 bits (numpy has no
bf16; the manifest records the dtype). Shard files are fsynced and renamed into place
before the manifest records the shard, so after an interruption the cache holds only
whole shards and a rerun with the same arguments resumes at the first missing one.

What differs is how the GPU is kept busy. The reference copies every batch's result to
the host synchronously and writes each shard before computing the next
(cache.py:118-137). Here:

* encoded hooks run `saeflow_b200.encode_sparse` (the encoder GEMM writing CSR straight
  from its epilogue) on the SAE's device;
* each device-to-host copy (dense activations, the three CSR arrays) is queued on a copy
  stream into pinned host memory, so the next batch's model forward and encode overlap it;
* one writer thread waits for a shard's copies, assembles it, writes and fsyncs its files
  and then the manifest, in shard order, while the next shard is computed. If the
  producer fails, the shards already handed to the writer are still completed before the
  error propagates, so the cache again holds only whole shards.

Several GPUs (the reference's roadmap, README.md:234-235): with `group=` (a
torch.distributed process group, one rank per GPU, all ranks on one filesystem) rank r
caches a contiguous block of whole shards, writing them at their global shard numbers and
recording them in its own manifest (`manifest.rank<r>-of-<n>.json`, so each rank resumes
on its own); when every rank is done, rank 0 merges the rank manifests into
`manifest.json` and removes them. The result is the directory a single process writes.
"""

from __future__ import annotations

import json
import os
import queue
import threading
from pathlib import Path

import numpy as np
import torch

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
_CSR_PARTS = ("indptr", "indices", "values")
_WRITE_AHEAD = 2  # shards that may wait for the writer before the producer blocks


def _encode_sparse(sae, x):
    """The on-the-fly encoder (tests substitute a CPU restatement)."""
    from .ops import encode_sparse

    return encode_sparse(sae, x)


# ----------------------------------------------------------------------------- host side

def _npy_view(t: torch.Tensor) -> np.ndarray:
    """The array a shard file stores for `t`: its values on the host, bf16 as the raw int16
    bit patterns (numpy has no bf16; the manifest's dtype says how to read them back)."""
    host = t.detach().cpu().contiguous()
    if host.dtype == torch.bfloat16:
        host = host.view(torch.int16)
    return host.numpy()


def _tensor_of(arr: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """A writable tensor holding a (read-only, memory-mapped) stored array, bf16 restored."""
    t = torch.from_numpy(np.array(arr, copy=True))
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


def _publish(path: Path, payload) -> None:
    """Write a file so that readers see either nothing or all of it: `payload(fh)` writes a
    sibling `<name>.partial`, which is flushed to stable storage before it is renamed over
    `path`; the directory is then synced so the rename itself survives a crash."""
    staging = path.parent / (path.name + ".partial")
    with open(staging, "wb") as fh:
        payload(fh)
        fh.flush()
        os.fsync(fh.fileno())
    os.replace(staging, path)
    try:
        dir_fd = os.open(path.parent, os.O_RDONLY)
    except OSError:  # a filesystem without directory handles
        return
    try:
        os.fsync(dir_fd)
    except OSError:
        pass
    finally:
        os.close(dir_fd)


def _write_npy(path: Path, t: torch.Tensor) -> None:
    """One shard array as a .npy file (the format np.save writes), published atomically."""
    arr = _npy_view(t)
    _publish(path, lambda fh: np.lib.format.write_array(fh, arr, allow_pickle=False))


def _stack_csr(blocks):
    """Row blocks of CSR (indptr, indices, values) stacked into one CSR: the per-row counts
    of every block, in order, summed into one indptr."""
    counts = torch.cat([ip[1:].to(torch.int64) - ip[:-1].to(torch.int64) for ip, _, _ in blocks])
    indptr = torch.zeros(counts.numel() + 1, dtype=torch.int64)
    torch.cumsum(counts, 0, out=indptr[1:])
    return indptr, torch.cat([ix for _, ix, _ in blocks]), torch.cat([vs for _, _, vs in blocks])


def _layers_to_run(hook_names):
    """How many transformer blocks the forward must run to reach every hook: one past the
    deepest `blocks.<n>.` hook, or None (run the whole model) when any hook lives outside
    the blocks (embeddings, final norm) or no hook is named."""
    deepest = None
    for name in hook_names:
        prefix, _, rest = name.partition(".")
        layer, dot, _ = rest.partition(".")
        if prefix != "blocks" or not dot or not (layer.isascii() and layer.isdigit()):
            return None
        deepest = max(int(layer), -1 if deepest is None else deepest)
    return None if deepest is None else deepest + 1


# ----------------------------------------------------------------------------- async copies

class _HostCopy:
    """A device tensor on its way to pinned host memory (or a host tensor as is)."""

    __slots__ = ("host", "event", "_src")

    def __init__(self, t: torch.Tensor, streams: dict):
        if not t.is_cuda:
            self.host, self.event, self._src = t.detach().contiguous(), None, None
            return
        dev = t.device
        stream = streams.get(dev)
        if stream is None:
            stream = streams[dev] = torch.cuda.Stream(dev)
        src = t.detach().contiguous()
        stream.wait_stream(torch.cuda.current_stream(dev))
        self.host = torch.empty(src.shape, dtype=src.dtype, pin_memory=True)
        with torch.cuda.stream(stream):
            self.host.copy_(src, non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record(stream)
        src.record_stream(stream)  # the allocator must not reuse src before the copy ends
        self._src = src

    def wait(self) -> torch.Tensor:
        if self.event is not None:
            self.event.synchronize()
            self.event, self._src = None, None
        return self.host


class _ShardWriter:
    """One thread that assembles, writes and records shards in submission order.
    `index_shards`: record each shard's global number (rank manifests)."""

    def __init__(self, out_dir: Path, manifest: dict, manifest_path: Path, index_shards: bool = False):
        self.out_dir, self.manifest, self.manifest_path = out_dir, manifest, manifest_path
        self.index_shards = index_shards
        self.jobs: queue.Queue = queue.Queue(maxsize=_WRITE_AHEAD)
        self.error: BaseException | None = None
        self.thread = threading.Thread(target=self._run, name="saeflow-cache-writer", daemon=True)
        self.thread.start()

    def submit(self, job) -> None:
        if self.error is not None:
            raise RuntimeError("the cache writer failed") from self.error
        self.jobs.put(job)

    def close(self) -> None:
        self.jobs.put(None)
        self.thread.join()
        if self.error is not None:
            raise RuntimeError("the cache writer failed") from self.error

    def _run(self) -> None:
        while True:
            job = self.jobs.get()
            if job is None:
                return
            if self.error is not None:
                continue  # drain: nothing after a failed shard may be recorded
            try:
                self._write(*job)
            except BaseException as e:  # noqa: BLE001 - reported to the producer
                self.error = e

    def _write(self, shard: int, parts: dict, hooks_meta: dict, n_seqs: int, n_rows: int) -> None:
        for h, pieces in parts.items():
            if hooks_meta[h]["format"] == "csr":
                csr = _stack_csr([tuple(c.wait() for c in piece) for piece in pieces])
                for name, t in zip(_CSR_PARTS, csr):
                    _write_npy(self.out_dir / h / f"{shard:05d}.{name}.npy", t)
            else:
                _write_npy(self.out_dir / h / f"{shard:05d}.npy", torch.cat([c.wait() for c in pieces]))
            self.manifest["hooks"][h] = hooks_meta[h]
        entry = {"n_seqs": n_seqs, "n_rows": n_rows}
        if self.index_shards:
            entry["index"] = shard
        self.manifest["shards"].append(entry)
        text = json.dumps(self.manifest, indent=2).encode()
        _publish(self.manifest_path, lambda fh: fh.write(text))


# ----------------------------------------------------------------------------- writer API

def _load_manifest(path: Path, config: dict, out_dir: Path) -> dict:
    if path.exists():
        manifest = json.loads(path.read_text())
        if manifest["config"] != config:
            raise ValueError(f"{out_dir} holds a cache with a different config: {manifest['config']}")
        return manifest
    return {"config": config, "hooks": {}, "shards": []}


def _run_shards(model, tokens, hook_names, out_dir, encoders, dtype, batch_size, seqs_per_shard, seq_len,
                first, stop_shard, manifest, manifest_path, index_shards):
    """Compute shards [first, stop_shard) and hand them to a writer that records them in
    `manifest` / `manifest_path`."""
    device = next(model.parameters()).device
    stop = _layers_to_run(hook_names)
    streams: dict = {}
    writer = _ShardWriter(out_dir, manifest, manifest_path, index_shards)
    try:
        for shard in range(first, stop_shard):
            start = shard * seqs_per_shard
            end = min(start + seqs_per_shard, len(tokens))
            parts = {h: [] for h in hook_names}
            meta = {}
            for b in range(start, end, batch_size):
                batch = tokens[b:min(b + batch_size, end)].to(device)
                _, acts = model.run_with_cache(batch, names_filter=hook_names, stop_at_layer=stop, return_type=None)
                for h in hook_names:
                    a = acts[h].flatten(0, 1).flatten(1)  # [batch * pos, d]; per-head hooks are concatenated
                    if h in encoders:
                        sae = encoders[h]
                        indptr, indices, values = _encode_sparse(sae, a.to(sae.W_enc.device, sae.W_enc.dtype))
                        parts[h].append((_HostCopy(indptr, streams), _HostCopy(indices, streams),
                                         _HostCopy(values.to(dtype), streams)))
                        meta[h] = {"format": "csr", "d": int(sae.W_enc.shape[1])}
                    else:
                        parts[h].append(_HostCopy(a.to(dtype), streams))
                        meta[h] = {"format": "dense", "d": int(a.shape[1])}
            writer.submit((shard, parts, meta, end - start, (end - start) * seq_len))
    finally:
        writer.close()


@torch.inference_mode()
def cache_activations(model, tokens, hook_names, out_dir, *, batch_size=8, batches_per_shard=32,
                      dtype=torch.float32, encoders=None, group=None):
    """Run `model` over `tokens` [n_seqs, seq_len] and cache activations at `hook_names`.

    model: a TransformerLens HookedTransformer, or anything with a compatible
      `run_with_cache(batch, names_filter=, stop_at_layer=, return_type=None)` and
      `parameters()`.
    encoders: optional {hook_name: sae}; those hooks are SAE-encoded on the fly on the
      SAE's device and stored as CSR feature activations instead of dense ones.
    group: optional torch.distributed process group: every rank calls with the same
      arguments (its own model and SAEs on its own GPU) and caches its block of shards.
    Calling again with the same arguments after an interruption resumes the run.
    Returns the cache directory as a Path. Same arguments, errors and files as
    saeflow.cache.cache_activations (cache.py:70-137).
    """
    out_dir, hook_names, encoders = Path(out_dir), list(hook_names), encoders or {}
    unknown = set(encoders) - set(hook_names)
    if unknown:
        raise ValueError(f"encoders given for hooks not being cached: {sorted(unknown)}")
    config = {
        "hook_names": hook_names,
        "n_seqs": len(tokens),
        "seq_len": int(tokens.shape[1]),
        "batch_size": batch_size,
        "batches_per_shard": batches_per_shard,
        "dtype": str(dtype).removeprefix("torch."),
        "encoded": sorted(encoders),
    }
    seqs_per_shard = batch_size * batches_per_shard
    n_shards = (len(tokens) + seqs_per_shard - 1) // seqs_per_shard
    manifest_path = out_dir / "manifest.json"
    world, rank = 1, 0
    if group is not None:
        import torch.distributed as dist

        world, rank = dist.get_world_size(group), dist.get_rank(group)
    manifest = _load_manifest(manifest_path, config, out_dir)
    for h in hook_names:
        (out_dir / h).mkdir(parents=True, exist_ok=True)
    args = (model, tokens, hook_names, out_dir, encoders, dtype, batch_size, seqs_per_shard, config["seq_len"])
    if world == 1:
        _run_shards(*args, len(manifest["shards"]), n_shards, manifest, manifest_path, False)
        return out_dir

    import torch.distributed as dist

    from .sharded import shard_range

    done = len(manifest["shards"])  # shards a previous run (of any rank count) already merged
    s0, s1 = shard_range(n_shards, world, rank)
    rank_path = out_dir / f"manifest.rank{rank}-of-{world}.json"
    rank_manifest = _load_manifest(rank_path, {**config, "rank": rank, "world": world}, out_dir)
    if not rank_path.exists():  # recorded even when this rank's block is empty
        text = json.dumps(rank_manifest, indent=2).encode()
        _publish(rank_path, lambda fh: fh.write(text))
    first = max(s0, done, max((e["index"] + 1 for e in rank_manifest["shards"]), default=s0))
    error = None
    try:
        _run_shards(*args, min(first, s1), s1, rank_manifest, rank_path, True)
    except BaseException as e:  # noqa: BLE001 - every rank must reach the barrier
        error = e
    failed = torch.tensor([1 if error is not None else 0], dtype=torch.int32)
    if dist.get_backend(group) == "nccl":
        failed = failed.cuda()
    dist.all_reduce(failed, op=dist.ReduceOp.MAX, group=group)  # also the barrier before the merge
    if error is not None:
        raise error
    if int(failed.item()):
        raise RuntimeError("another rank failed while caching; rerun with the same arguments to resume")
    if rank == 0:
        _merge_rank_manifests(out_dir, manifest, manifest_path, hook_names, world, done)
    dist.barrier(group)
    return out_dir


def _merge_rank_manifests(out_dir: Path, manifest: dict, manifest_path: Path, hook_names, world: int, done: int):
    """Rank 0, after every rank finished: append the ranks' shards (in global order) to the
    manifest, write it, then drop the rank manifests."""
    paths = [out_dir / f"manifest.rank{r}-of-{world}.json" for r in range(world)]
    entries, hooks = [], {}
    for p in paths:
        rm = json.loads(p.read_text())
        entries += [e for e in rm["shards"] if e["index"] >= done]
        hooks.update(rm["hooks"])
    entries.sort(key=lambda e: e["index"])
    if [e["index"] for e in entries] != list(range(done, done + len(entries))):
        raise RuntimeError(f"rank manifests in {out_dir} do not cover consecutive shards")
    for h in hook_names:
        if h in hooks:
            manifest["hooks"][h] = hooks[h]
    manifest["hooks"] = {h: manifest["hooks"][h] for h in hook_names if h in manifest["hooks"]}
    manifest["shards"] += [{"n_seqs": e["n_seqs"], "n_rows": e["n_rows"]} for e in entries]
    text = json.dumps(manifest, indent=2).encode()
    _publish(manifest_path, lambda fh: fh.write(text))
    for p in paths:
        p.unlink()


# ----------------------------------------------------------------------------- reader

class ActivationReader:
    """Streams a cache written by cache_activations (here or by saeflow) back as batches.

    The shards of a hook are one sequence of rows: a row index built once from the
    manifest (the first global row of every shard) locates any global row range, and
    `read_rows` slices it out of the memory-mapped shard files, so batches of any size
    cross shard boundaries without buffering rows. Same constructor, attributes and
    batches as saeflow.cache.ActivationReader (cache.py:140-194)."""

    def __init__(self, path):
        self.path = Path(path)
        self.manifest = json.loads((self.path / "manifest.json").read_text())
        self.dtype = _DTYPES[self.manifest["config"]["dtype"]]
        sizes = np.array([s["n_rows"] for s in self.manifest["shards"]], dtype=np.int64)
        self._first_row = np.concatenate([[0], np.cumsum(sizes)])  # shard i holds [first[i], first[i+1])
        self._maps: dict = {}

    @property
    def hook_names(self):
        return self.manifest["config"]["hook_names"]

    def n_rows(self):
        """Rows (token positions) in the cache, per hook."""
        return int(self._first_row[-1])

    def is_sparse(self, hook):
        """True when `hook` was SAE-encoded on the fly and is stored as CSR features."""
        return self.manifest["hooks"][hook]["format"] == "csr"

    def _shard_arrays(self, hook, i):
        """Memory maps of shard i of `hook`, opened on first use."""
        key = (hook, i)
        if key not in self._maps:
            d = self.path / hook
            if self.is_sparse(hook):
                self._maps[key] = tuple(np.load(d / f"{i:05d}.{part}.npy", mmap_mode="r") for part in _CSR_PARTS)
            else:
                self._maps[key] = np.load(d / f"{i:05d}.npy", mmap_mode="r")
        return self._maps[key]

    def read_rows(self, hook, start, stop):
        """Global rows [start, stop) of `hook`: a [rows, d] tensor, or a CSR (indptr,
        indices, values) tuple for an encoded hook, on the host."""
        if not 0 <= start <= stop <= self.n_rows():
            raise IndexError(f"rows [{start}, {stop}) outside the cache's {self.n_rows()} rows")
        first = int(np.searchsorted(self._first_row, start, side="right")) - 1
        last = int(np.searchsorted(self._first_row, stop, side="left"))
        blocks = []
        for i in range(max(first, 0), min(last, len(self.manifest["shards"]))):
            lo = max(start, int(self._first_row[i])) - int(self._first_row[i])
            hi = min(stop, int(self._first_row[i + 1])) - int(self._first_row[i])
            if hi <= lo:
                continue
            arrays = self._shard_arrays(hook, i)
            if self.is_sparse(hook):
                indptr, indices, values = arrays
                ip = np.array(indptr[lo:hi + 1], dtype=np.int64)
                blocks.append((torch.from_numpy(ip), _tensor_of(indices[ip[0]:ip[-1]], torch.int32),
                               _tensor_of(values[ip[0]:ip[-1]], self.dtype)))
            else:
                blocks.append(_tensor_of(arrays[lo:hi], self.dtype))
        if self.is_sparse(hook):
            if not blocks:
                return (torch.zeros(1, dtype=torch.int64), torch.zeros(0, dtype=torch.int32),
                        torch.zeros(0, dtype=self.dtype))
            return _stack_csr(blocks)
        if not blocks:
            return torch.zeros(0, self.manifest["hooks"][hook]["d"], dtype=self.dtype)
        return blocks[0] if len(blocks) == 1 else torch.cat(blocks)

    def _host_batches(self, hook, batch_size):
        if batch_size < 1:
            raise ValueError("batch_size must be positive")
        total = self.n_rows()
        for start in range(0, total, batch_size):
            yield self.read_rows(hook, start, min(total, start + batch_size))

    def iter_batches(self, hook, batch_size, device=None):
        """Yield `batch_size`-row batches in cache order (the last may be short), crossing
        shard boundaries. Dense hooks yield [rows, d] tensors; encoded hooks yield CSR
        (indptr, indices, values) tuples, which saeflow_b200.decode_sparse takes directly.

        device: None yields host tensors (saeflow.cache.ActivationReader.iter_batches,
        cache.py:178-194). A CUDA device yields tensors already there: each batch is staged
        in pinned memory and copied asynchronously one batch ahead, so reading and the
        copy of batch i+1 overlap the caller's work on batch i.
        """
        if device is None:
            yield from self._host_batches(hook, batch_size)
            return
        device = torch.device(device)
        stream = torch.cuda.Stream(device)

        def upload(item):
            ts = item if isinstance(item, tuple) else (item,)
            with torch.cuda.stream(stream):
                dev = tuple(t.pin_memory().to(device, non_blocking=True) for t in ts)
                ev = torch.cuda.Event()
                ev.record(stream)
            return (dev if isinstance(item, tuple) else dev[0]), ev

        ahead = None
        for item in self._host_batches(hook, batch_size):
            nxt = upload(item)
            if ahead is not None:
                yield self._handoff(ahead, device)
            ahead = nxt
        if ahead is not None:
            yield self._handoff(ahead, device)

    @staticmethod
    def _handoff(staged, device):
        batch, ev = staged
        cur = torch.cuda.current_stream(device)
        cur.wait_event(ev)
        for t in (batch if isinstance(batch, tuple) else (batch,)):
            t.record_stream(cur)
        return batch
