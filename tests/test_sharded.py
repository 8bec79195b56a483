"""Multi-rank host logic on CPU: `gloo` process groups of world size 2, the CPU oracle as
the kernel provider. Covers feature (d_sae) sharding, token sharding, and a rank that
fails before the collective (the survivor must get an error, not hang)."""

import datetime
import multiprocessing as mp
import os
import time
import traceback

import pytest
import torch

from saeflow_b200.sharded import shard_range, token_shard

WORLD = 2


class OracleOps:
    @staticmethod
    def encode_sparse(sae, x):
        import oracle

        return oracle.encode_sparse(sae, x)

    @staticmethod
    def decode_partial(csr, W_dec):
        import oracle

        return oracle.sparse_decode(*csr, W_dec, None, out_dtype=torch.float32)


def _make(activation="jumprelu"):
    import oracle

    torch.manual_seed(0)
    sae = oracle.RefSAE(32, 203, activation)
    sae.b_enc.normal_(0, 0.1)
    sae.b_dec.normal_(0, 0.1)
    if activation == "jumprelu":
        sae.threshold.uniform_(0.0, 0.3)
    x = torch.randn(50, 32)
    return sae, x


class OverflowingOps(OracleOps):
    """Device-style provider whose CSR staging 'overflows' on one chunk of rank 0 only: the
    partial it returns for that chunk is garbage, and its flag says so. Every rank must then
    redo that chunk (the flags are all-reduced) and the result must still be exact."""

    def __init__(self, rank):
        self.rank = rank
        self.calls = 0

    def partial_async(self, sae, x):
        import oracle

        bad = self.rank == 0 and self.calls == 1
        self.calls += 1
        partial = oracle.sparse_decode(*oracle.encode_sparse(sae, x), sae.W_dec, None, out_dtype=torch.float32)
        if bad:
            partial = torch.full_like(partial, 1e6)
        return partial, torch.tensor(int(bad), dtype=torch.int32)


def _worker_overflow(rank, init_file, q):
    try:
        import oracle
        from saeflow_b200.sharded import FeatureShardedSAE

        dist = _init(rank, init_file)
        sae, x = _make("jumprelu")
        fs = FeatureShardedSAE(sae, ops=OverflowingOps(rank), chunk_tokens=16)
        got = fs.forward(x, out_dtype=torch.float32)
        err = (got - oracle.forward(sae, x).float()).abs().max().item()
        dist.destroy_process_group()
        q.put((rank, "ok", err, True))
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc(), False))


def _init(rank, init_file, timeout_s=20):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _worker_forward(rank, init_file, q, activation):
    try:
        import oracle
        from saeflow_b200.sharded import FeatureShardedSAE

        dist = _init(rank, init_file)
        sae, x = _make(activation)
        fs = FeatureShardedSAE(sae, ops=OracleOps(), chunk_tokens=16)
        got = fs.forward(x, out_dtype=torch.float32)
        want = oracle.forward(sae, x).float()
        err = (got - want).abs().max().item()
        # the union of the ranks' CSRs (global ids) is the full CSR, exactly
        ip, ix, vs = fs.encode_sparse(x)
        parts = [None] * WORLD
        dist.all_gather_object(parts, (ip, ix, vs, fs.start, fs.stop))
        fip, fix, fvs = oracle.encode_sparse(sae, x)
        same = True
        for m in range(x.shape[0]):
            cols, vals = [], []
            for pip, pix, pvs, _, _ in parts:
                cols.append(pix[pip[m]:pip[m + 1]])
                vals.append(pvs[pip[m]:pip[m + 1]])
            cols, vals = torch.cat(cols), torch.cat(vals)
            same &= torch.equal(cols, fix[fip[m]:fip[m + 1]]) and torch.equal(vals, fvs[fip[m]:fip[m + 1]])
        dist.destroy_process_group()
        q.put((rank, "ok", err, bool(same)))
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc(), False))


def _worker_fail(rank, init_file, q):
    try:
        from saeflow_b200.sharded import FeatureShardedSAE

        dist = _init(rank, init_file, timeout_s=10)
        sae, x = _make()
        fs = FeatureShardedSAE(sae, ops=OracleOps(), chunk_tokens=16)
        if rank == 1:
            raise SystemExit(3)  # this rank dies before its first collective
        t0 = time.time()
        try:
            fs.forward(x)
            q.put((rank, "no-error", time.time() - t0, False))
        except Exception as e:  # noqa: BLE001
            q.put((rank, "raised", time.time() - t0, type(e).__name__))
    except SystemExit:
        q.put((rank, "exited", 0.0, False))


def _run(target, *args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"sf_gloo_{os.getpid()}_{time.time_ns()}")
    procs = [ctx.Process(target=target, args=(r, init_file, q, *args)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + timeout
    while len(out) < WORLD and time.time() < deadline:
        try:
            item = q.get(timeout=max(0.1, deadline - time.time()))
            out[item[0]] = item
        except Exception:  # noqa: BLE001
            break
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    try:
        os.remove(init_file)
    except OSError:
        pass
    return out


def test_shard_range_partitions():
    for n in (0, 1, 7, 203, 1 << 20):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_token_shard_covers_rows():
    x = torch.arange(23).view(23, 1)
    assert torch.equal(torch.cat([token_shard(x, 4, r) for r in range(4)]), x)


@pytest.mark.parametrize("activation", ["relu", "jumprelu"])
def test_feature_sharded_forward_matches_single_device(activation):
    out = _run(_worker_forward, activation)
    assert sorted(out) == [0, 1], out
    for rank, status, err, same in out.values():
        assert status == "ok", err
        assert err < 1e-5, f"rank {rank}: max error {err}"
        assert same, f"rank {rank}: union of shard CSRs differs from the full CSR"


def test_feature_sharding_rejects_topk():
    import oracle
    from saeflow_b200.sharded import FeatureShardedSAE

    sae = oracle.RefSAE(8, 16, "topk", k=2)
    with pytest.raises(ValueError, match="TopK"):
        FeatureShardedSAE(sae, ops=OracleOps())


def test_dead_rank_surfaces_as_an_error_not_a_hang():
    t0 = time.time()
    out = _run(_worker_fail, timeout=90)
    assert out.get(1, (None, None))[1] == "exited"
    rank0 = out.get(0)
    assert rank0 is not None, "surviving rank never reported (hang)"
    assert rank0[1] == "raised", rank0
    assert time.time() - t0 < 90


def test_feature_sharded_staging_overflow_on_one_rank_is_redone_by_all():
    out = _run(_worker_overflow)
    assert sorted(out) == [0, 1], out
    for rank, status, err, _ in out.values():
        assert status == "ok", err
        assert err < 1e-5, f"rank {rank}: max error {err}"
