"""Activation cache (saeflow_b200.cache), a drop-in for saeflow/cache.py.

The reference's cache tests (tests/test_cache.py of saeflow) need TransformerLens, which
is not installed; tests/cache_fixtures.TinyModel stands in for the model. Files written by
the reference's own cache_activations with that model (tests/golden/cache_ref/, made by
tests/golden/make_golden_cache.py) pin the format byte for byte.
"""

import filecmp
from pathlib import Path

import pytest
import torch

import cache_fixtures as cf
import oracle
from saeflow_b200 import cache as sf_cache
from saeflow_b200.cache import ActivationReader, cache_activations
from saeflow_b200.kernels import csr_to_dense

GOLDEN = Path(__file__).resolve().parent / "golden" / "cache_ref"


@pytest.fixture
def model():
    return cf.TinyModel()


@pytest.fixture
def tokens():
    return cf.tokens()


@pytest.fixture
def cpu_encoder(monkeypatch):
    """The CPU restatement of encode_sparse stands in for the CUDA kernels."""
    monkeypatch.setattr(sf_cache, "_encode_sparse", oracle.encode_sparse)


def read_all(reader, hook, batch_size):
    return torch.cat(list(reader.iter_batches(hook, batch_size)))


def same_tree(a: Path, b: Path):
    fa = sorted(p.relative_to(a) for p in a.rglob("*") if p.is_file())
    fb = sorted(p.relative_to(b) for p in b.rglob("*") if p.is_file())
    assert fa == fb
    for rel in fa:
        assert filecmp.cmp(a / rel, b / rel, shallow=False), f"{rel} differs from the reference's file"


# ------------------------------------------------------------------ format parity with the reference

def test_dense_cache_is_byte_identical_to_the_reference(model, tokens, tmp_path):
    cache_activations(model, tokens, cf.HOOKS, tmp_path / "dense_fp32", batch_size=4, batches_per_shard=2)
    same_tree(tmp_path / "dense_fp32", GOLDEN / "dense_fp32")
    cache_activations(model, tokens, cf.HOOKS[:1], tmp_path / "dense_bf16", batch_size=8, dtype=torch.bfloat16)
    same_tree(tmp_path / "dense_bf16", GOLDEN / "dense_bf16")


def test_encoded_cache_is_byte_identical_to_the_reference(model, tokens, tmp_path, cpu_encoder):
    sae = cf.exact_sae(oracle.RefSAE)
    cache_activations(model, tokens, cf.HOOKS, tmp_path / "csr_fp32", batch_size=4, batches_per_shard=2,
                      encoders={cf.HOOKS[0]: sae})
    same_tree(tmp_path / "csr_fp32", GOLDEN / "csr_fp32")


def test_reader_reads_the_reference_caches(model, tokens):
    reader = ActivationReader(GOLDEN / "dense_fp32")
    assert reader.hook_names == cf.HOOKS and reader.n_rows() == 22 * cf.N_CTX
    for hook in cf.HOOKS:
        assert torch.equal(read_all(reader, hook, 7), cf.expected(model, tokens, hook))
    got = read_all(ActivationReader(GOLDEN / "dense_bf16"), cf.HOOKS[0], 64)
    assert got.dtype == torch.bfloat16 and torch.equal(got, cf.expected(model, tokens, cf.HOOKS[0]).bfloat16())
    reader = ActivationReader(GOLDEN / "csr_fp32")
    sae = cf.exact_sae(oracle.RefSAE)
    dense = torch.cat([csr_to_dense(*csr, 96) for csr in reader.iter_batches(cf.HOOKS[0], 13)])
    assert torch.equal(dense, sae.encode(cf.expected(model, tokens, cf.HOOKS[0])))


def test_read_rows_is_random_access_across_shards():
    """Any global row range, inside one shard or across several, equals the same rows of a
    full read; empty ranges and ranges past the end behave."""
    for name, hook in (("dense_fp32", cf.HOOKS[1]), ("csr_fp32", cf.HOOKS[0])):
        reader = ActivationReader(GOLDEN / name)
        n = reader.n_rows()
        whole = reader.read_rows(hook, 0, n)
        if reader.is_sparse(hook):
            whole = csr_to_dense(*whole, 96)
        for a, b in ((0, 1), (3, 3), (5, 70), (63, 65), (17, n), (n - 1, n), (n, n)):
            got = reader.read_rows(hook, a, b)
            if reader.is_sparse(hook):
                assert got[0][0] == 0 and got[0].numel() == b - a + 1
                got = csr_to_dense(*got, 96)
            assert torch.equal(got, whole[a:b]), (name, a, b)
        with pytest.raises(IndexError):
            reader.read_rows(hook, 0, n + 1)
        with pytest.raises(ValueError):
            next(reader.iter_batches(hook, 0))


def test_layers_to_run():
    assert sf_cache._layers_to_run(["blocks.0.hook_resid_post", "blocks.11.attn.hook_z"]) == 12
    assert sf_cache._layers_to_run(["blocks.2.hook_mlp_out", "hook_embed"]) is None
    assert sf_cache._layers_to_run(["blocks.x.hook"]) is None
    assert sf_cache._layers_to_run([]) is None


# ------------------------------------------------------------------ the reference's cache tests

def test_write_and_read_back_exactly(model, tokens, tmp_path):
    cache_activations(model, tokens, cf.HOOKS, tmp_path, batch_size=4, batches_per_shard=2)
    reader = ActivationReader(tmp_path)
    assert len(reader.manifest["shards"]) == 3
    for hook in cf.HOOKS:
        assert torch.equal(read_all(reader, hook, 7), cf.expected(model, tokens, hook))


def test_resume_after_interruption(model, tokens, tmp_path):
    with pytest.raises(cf.Interrupted):
        cache_activations(cf.FlakyModel(model, 3), tokens, cf.HOOKS, tmp_path, batch_size=4, batches_per_shard=2)
    assert len(ActivationReader(tmp_path).manifest["shards"]) == 1  # the half-computed shard 1 is discarded
    cache_activations(model, tokens, cf.HOOKS, tmp_path, batch_size=4, batches_per_shard=2)
    reader = ActivationReader(tmp_path)
    assert len(reader.manifest["shards"]) == 3
    assert not list(tmp_path.rglob("*.partial"))
    for hook in cf.HOOKS:
        assert torch.equal(read_all(reader, hook, 5), cf.expected(model, tokens, hook))


def test_resume_with_different_config_refuses(model, tokens, tmp_path):
    cache_activations(model, tokens, cf.HOOKS[:1], tmp_path, batch_size=4)
    with pytest.raises(ValueError, match="different config"):
        cache_activations(model, tokens, cf.HOOKS[:1], tmp_path, batch_size=8)


def test_encoders_for_uncached_hooks_refused(model, tokens, tmp_path):
    with pytest.raises(ValueError, match="not being cached"):
        cache_activations(model, tokens, cf.HOOKS[:1], tmp_path, encoders={cf.HOOKS[1]: object()})


def test_bfloat16_storage(model, tokens, tmp_path):
    hook = cf.HOOKS[0]
    cache_activations(model, tokens, [hook], tmp_path, batch_size=8, dtype=torch.bfloat16)
    got = read_all(ActivationReader(tmp_path), hook, 64)
    assert got.dtype == torch.bfloat16
    assert torch.equal(got, cf.expected(model, tokens, hook).bfloat16())


def test_encode_on_the_fly_stores_sparse(model, tokens, tmp_path, cpu_encoder):
    hook = cf.HOOKS[0]
    sae = cf.exact_sae(oracle.RefSAE)
    cache_activations(model, tokens, [hook], tmp_path, batch_size=4, batches_per_shard=2, encoders={hook: sae})
    reader = ActivationReader(tmp_path)
    assert reader.manifest["hooks"][hook] == {"format": "csr", "d": 96}
    dense = torch.cat([csr_to_dense(*csr, 96) for csr in reader.iter_batches(hook, 13)])
    assert torch.equal(dense, sae.encode(cf.expected(model, tokens, hook)))


# ------------------------------------------------------------------ the background writer

def test_failed_shard_write_leaves_only_whole_shards_and_resumes(model, tokens, tmp_path, monkeypatch):
    real_save, calls = sf_cache._write_npy, []

    def flaky_save(path, t):
        calls.append(path)
        if len(calls) == 3:  # shard 1's first file
            raise OSError("disk full")
        real_save(path, t)

    monkeypatch.setattr(sf_cache, "_write_npy", flaky_save)
    with pytest.raises(RuntimeError, match="writer failed"):
        cache_activations(model, tokens, cf.HOOKS, tmp_path, batch_size=4, batches_per_shard=2)
    assert len(ActivationReader(tmp_path).manifest["shards"]) == 1
    monkeypatch.setattr(sf_cache, "_write_npy", real_save)
    cache_activations(model, tokens, cf.HOOKS, tmp_path, batch_size=4, batches_per_shard=2)
    same_tree(tmp_path, GOLDEN / "dense_fp32")


def test_producer_error_still_completes_handed_over_shards(model, tokens, tmp_path):
    # 5 forward passes: shards 0 and 1 (2 batches each) are handed to the writer, then the
    # model dies in shard 2; both finished shards must be on disk and recorded.
    with pytest.raises(cf.Interrupted):
        cache_activations(cf.FlakyModel(model, 5), tokens, cf.HOOKS, tmp_path, batch_size=4, batches_per_shard=2)
    assert len(ActivationReader(tmp_path).manifest["shards"]) == 2


# ------------------------------------------------------------------ GPU: the CUDA encoder

@pytest.mark.gpu
@pytest.mark.parametrize("sae_dtype", [torch.float32, torch.bfloat16])
def test_cuda_encode_on_the_fly_matches_reference_files(tokens, tmp_path, sae_dtype):
    """Model on the GPU, SAE encoded by the CUDA kernels (IEEE fp32: the dense route; bf16:
    encode straight to CSR), D2H copies overlapped: fp32 gives the reference's files byte
    for byte; bf16 gives the CSR of encode_sparse on the same activations."""
    from saeflow_b200 import encode_sparse
    from saeflow_b200.kernels import device_error

    model = cf.TinyModel("cuda")
    sae = cf.exact_sae(oracle.RefSAE).to(sae_dtype).cuda()
    out = tmp_path / "c"
    cache_activations(model, tokens, cf.HOOKS, out, batch_size=4, batches_per_shard=2,
                      encoders={cf.HOOKS[0]: sae})
    if sae_dtype == torch.float32:
        same_tree(out, GOLDEN / "csr_fp32")
    reader = ActivationReader(out)
    got = torch.cat([csr_to_dense(*csr, 96) for csr in reader.iter_batches(cf.HOOKS[0], 50)])
    acts = cf.expected(model, tokens.cuda(), cf.HOOKS[0]).to(sae_dtype)
    want = csr_to_dense(*encode_sparse(sae, acts), 96).float().cpu()
    assert torch.equal(got, want)
    assert device_error() == 0


@pytest.mark.gpu
def test_reader_device_batches_match_host_batches(tmp_path):
    reader = ActivationReader(GOLDEN / "csr_fp32")
    for hook in cf.HOOKS:
        host = list(reader.iter_batches(hook, 29))
        dev = list(reader.iter_batches(hook, 29, device="cuda"))
        assert len(host) == len(dev)
        for h, d in zip(host, dev):
            for a, b in zip(h if isinstance(h, tuple) else (h,), d if isinstance(d, tuple) else (d,)):
                assert b.is_cuda and torch.equal(a, b.cpu())


# ------------------------------------------------------------------ several ranks (gloo, CPU)

def _rank_worker(rank, world, init_file, out_dir, q, encode, flaky_rank):
    import datetime
    import traceback

    try:
        import torch.distributed as dist

        import cache_fixtures as cfx
        import oracle as orc
        from saeflow_b200 import cache as c

        c._encode_sparse = orc.encode_sparse
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=30))
        model = cfx.TinyModel()
        if rank == flaky_rank:
            model = cfx.FlakyModel(model, 1)
        enc = {cfx.HOOKS[0]: cfx.exact_sae(orc.RefSAE)} if encode else None
        try:
            c.cache_activations(model, cfx.tokens(), cfx.HOOKS, out_dir, batch_size=4, batches_per_shard=2,
                                encoders=enc, group=dist.group.WORLD)
            q.put((rank, "ok", ""))
        except Exception as e:  # noqa: BLE001
            q.put((rank, "raised", type(e).__name__))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc()))


def _run_ranks(world, out_dir, encode=False, flaky_rank=-1, timeout=120):
    import multiprocessing as mp
    import os
    import time

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"sf_cache_{os.getpid()}_{time.time_ns()}")
    procs = [ctx.Process(target=_rank_worker, args=(r, world, init_file, str(out_dir), q, encode, flaky_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    out, deadline = {}, time.time() + timeout
    while len(out) < world and time.time() < deadline:
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


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("encode", [False, True])
def test_ranks_write_the_single_process_cache(tmp_path, world, encode):
    """Each rank caches its block of whole shards; after the merge the directory is the one a
    single process writes (byte for byte, against the reference's files). With 4 ranks and 3
    shards one rank has nothing to do."""
    out = _run_ranks(world, tmp_path / "c", encode=encode)
    assert sorted(out) == list(range(world)), out
    assert all(v[1] == "ok" for v in out.values()), out
    ref = GOLDEN / ("csr_fp32" if encode else "dense_fp32")
    same_tree(tmp_path / "c", ref)


def test_rank_failure_is_reported_everywhere_and_resumes(tmp_path):
    out = _run_ranks(2, tmp_path / "c", flaky_rank=1)  # rank 1 dies after one forward pass
    assert sorted(out) == [0, 1], out
    assert out[1][1] == "raised" and out[1][2] == "Interrupted"
    assert out[0][1] == "raised" and out[0][2] == "RuntimeError"
    assert not (tmp_path / "c" / "manifest.json").exists()  # nothing merged
    out = _run_ranks(2, tmp_path / "c")
    assert all(v[1] == "ok" for v in out.values()), out
    same_tree(tmp_path / "c", GOLDEN / "dense_fp32")
