"""Feature (d_sae) sharding on the GPU with the package's own CUDA kernels.

* One process: N feature shards emulated by a loop over shard_range slices, each through
  FeatureShardedSAE's real kernel provider (fp32 partial decode without b_dec, CSR kept on
  the device); the partials summed, b_dec added once, against saeflow_b200.forward on the
  whole SAE. The union of the shards' CSRs (global feature ids) is the whole SAE's CSR.
* Two processes: FeatureShardedSAE.forward with its asynchronous all-reduce of per-chunk
  partials overlapping the next chunk's encode. NCCL with one GPU per rank when the box
  has two; otherwise both ranks share GPU 0 over `gloo`, whose all-reduce is host-side
  (no kernel waits on another rank's kernel).
"""

import datetime
import multiprocessing as mp
import os
import time
import traceback
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

D_IN, D_SAE, TOKENS = 512, 12288, 3000


def make_sae(device):
    """A sparse bf16 JumpReLU SAE (L0 ~ 70) and a token batch, the same in every process."""
    import oracle

    torch.manual_seed(0)  # the constructor draws W_dec from the global generator: same SAE in every process
    g = torch.Generator().manual_seed(0)
    sae = oracle.RefSAE(D_IN, D_SAE, "jumprelu")
    sae.b_enc.copy_(torch.randn(D_SAE, generator=g) * 0.1)
    sae.b_dec.copy_(torch.randn(D_IN, generator=g) * 0.1)
    sae.threshold.copy_(torch.rand(D_SAE, generator=g) + 2.0)
    x = torch.randn(TOKENS, D_IN, generator=g)
    return sae.to(torch.bfloat16).to(device), x.to(torch.bfloat16).to(device)


def shard_view(sae, start, stop):
    """This shard's slices of the weights, as a caller that holds only its features passes them."""
    sl = slice(start, stop)
    return SimpleNamespace(W_enc=sae.W_enc[:, sl].contiguous(), b_enc=sae.b_enc[sl].contiguous(),
                           W_dec=sae.W_dec[sl].contiguous(), b_dec=sae.b_dec, threshold=sae.threshold[sl].contiguous(),
                           activation=sae.activation, k=None, feature_start=start)


@pytest.mark.parametrize("n_shards", [1, 3, 8])
def test_feature_shards_sum_to_the_whole_forward(n_shards):
    import saeflow_b200
    from oracle import contract
    from saeflow_b200.kernels import device_error
    from saeflow_b200.sharded import FeatureShardedSAE, _CudaOps, shard_range

    dev = torch.device("cuda")
    device_error()
    sae, x = make_sae(dev)
    want = saeflow_b200.forward(sae, x)
    whole_csr = saeflow_b200.encode_sparse(sae, x)
    acc = torch.zeros(TOKENS, D_IN, dtype=torch.float32, device=dev)
    shard_csrs = []
    for r in range(n_shards):
        start, stop = shard_range(D_SAE, n_shards, r)
        fs = FeatureShardedSAE(shard_view(sae, start, stop))
        assert isinstance(fs.ops, _CudaOps) and (fs.start, fs.stop) == (start, stop)
        partial, overflow = fs._partial(x)
        assert partial.dtype == torch.float32 and partial.shape == (TOKENS, D_IN)
        assert overflow is None or int(overflow) == 0
        acc += partial
        shard_csrs.append([t.cpu() for t in fs.encode_sparse(x)])
        if n_shards == 1:  # the whole forward of one shard: partial + b_dec, no collective
            torch.testing.assert_close(fs.forward(x, out_dtype=torch.float32), acc + sae.b_dec.float(),
                                       rtol=0, atol=0)
    got = (acc + sae.b_dec.float()).to(torch.bfloat16)
    contract.assert_values_close(got.cpu().float(), want.cpu().float(), torch.bfloat16, what="sharded forward")

    # global feature ids: each row of the whole CSR is the concatenation of the shards' rows
    wip, wix, wvs = (t.cpu() for t in whole_csr)
    for m in range(TOKENS):
        cols = torch.cat([ix[ip[m]:ip[m + 1]] for ip, ix, _ in shard_csrs])
        vals = torch.cat([vs[ip[m]:ip[m + 1]] for ip, _, vs in shard_csrs])
        assert torch.equal(cols, wix[wip[m]:wip[m + 1]]), f"row {m}: feature ids differ"
        assert torch.equal(vals.view(torch.int16), wvs[wip[m]:wip[m + 1]].view(torch.int16)), f"row {m}: values"
    assert device_error() == 0


def _worker(rank, world, init_file, backend, q):
    try:
        import torch.distributed as dist

        import saeflow_b200
        from saeflow_b200.kernels import device_error
        from saeflow_b200.sharded import FeatureShardedSAE

        dev = torch.device("cuda", rank if backend == "nccl" else 0)
        torch.cuda.set_device(dev)
        kw = {"device_id": dev} if backend == "nccl" else {}
        dist.init_process_group(backend, init_method=f"file://{init_file}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), **kw)
        sae, x = make_sae(dev)
        fs = FeatureShardedSAE(sae, chunk_tokens=1024)  # three chunks, two of them overlapped
        got = fs.forward(x)
        want = saeflow_b200.forward(sae, x)
        g, w = got.float().cpu(), want.float().cpu()
        worst = ((g - w).abs() - (1e-4 + 1e-2 * w.abs())).max().item()
        err = device_error(dev)
        dist.destroy_process_group()
        q.put((rank, "ok", worst, err, (fs.start, fs.stop)))
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc(), -1, None))


def test_feature_sharded_forward_two_ranks_all_reduce():
    world = 2
    backend = "nccl" if torch.cuda.device_count() >= world else "gloo"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = os.path.join(os.environ.get("TMPDIR", "/tmp"), f"sf_shard_gpu_{os.getpid()}_{time.time_ns()}")
    procs = [ctx.Process(target=_worker, args=(r, world, init_file, backend, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + 240
    while len(out) < world and time.time() < deadline:
        try:
            item = q.get(timeout=max(0.1, deadline - time.time()))
            out[item[0]] = item
        except Exception:  # noqa: BLE001
            break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    try:
        os.remove(init_file)
    except OSError:
        pass
    assert sorted(out) == [0, 1], out
    spans = []
    for rank, status, worst, err, span in out.values():
        assert status == "ok", worst
        assert worst <= 0, f"rank {rank} ({backend}): outside rtol 1e-2 atol 1e-4 by {worst}"
        assert err == 0, f"rank {rank}: device error bits {err}"
        spans.append(span)
    assert sorted(spans) == [(0, D_SAE // 2), (D_SAE // 2, D_SAE)]
