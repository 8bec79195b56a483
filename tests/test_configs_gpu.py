"""The BASELINE configurations at full size on the GPU, held to the contract's rules.

Inputs come from bench.py's seeded generators (the same tensors the benchmark times).
Every config runs at its full batch on the GPU; the CPU oracle (float64 sums) checks a
spread of sampled rows (all rows for the decode-only config), and size-independent
properties are checked on every row at full size:

* config 1 (ReLU, fp32 IEEE): row counts == nonzeros of the output, the compaction equals
  torch's to_sparse_csr bit for bit, forward == decode(encode_sparse);
* config 2 (JumpReLU, bf16): encode straight to CSR equals the dense route bit for bit,
  forward == decode(encode_sparse);
* config 3 (decode only): every row against the oracle;
* config 4 (TopK k=32): the selected values are the dense ReLU encoder's values at the
  selected ids, and no other feature of the row ranks above the k-th (value, then lower id);
* config 5's feature dimension (d_sae = 2^20) on a 4096-token slice of its batch: encode
  straight to CSR equals the dense route bit for bit, forward == decode(encode_sparse).

The tolerances are oracle/contract.py's: rtol 1e-2 (bf16) / 1e-5 (fp32) with small
absolute floors, features within 1e-3 of their cut excluded, CSR structure bit-exact.
"""

import pytest
import torch

import bench
import oracle
import saeflow_b200
from oracle import contract
from saeflow_b200.kernels import best_config, dense_to_csr, device_error, fused_encode, sparse_decode, topk_encode

pytestmark = pytest.mark.gpu

SAMPLE_ROWS = 256


@pytest.fixture(autouse=True)
def _clean_device_errors():
    device_error()
    yield
    assert device_error() == 0, "a kernel reported a device-side error"


def sample_rows(T, n=SAMPLE_ROWS):
    """n rows spread evenly over the batch, first and last included."""
    return torch.linspace(0, T - 1, n).round().long().unique()


def sub_csr(csr, rows):
    """CPU CSR of the given rows of a (device) CSR triple."""
    ip, ix, vs = (t.cpu() for t in csr)
    starts, ends = ip[rows], ip[rows + 1]
    counts = ends - starts
    out_ip = torch.zeros(rows.numel() + 1, dtype=torch.int64)
    out_ip[1:] = counts.cumsum(0)
    take = torch.cat([torch.arange(int(a), int(b)) for a, b in zip(starts, ends)]) if int(counts.sum()) else \
        torch.zeros(0, dtype=torch.int64)
    return out_ip, ix[take], vs[take]


def bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def assert_same_csr(a, b):
    for u, v in zip(a, b):
        assert u.dtype == v.dtype and u.shape == v.shape
        assert torch.equal(bits(u) if u.is_floating_point() else u, bits(v) if v.is_floating_point() else v)


def check_encoded_rows(sae, x, f_rows, csr, rows):
    """Sampled rows of a dense encode (f_rows, may be None) and of its CSR against the
    oracle: values outside the cut band under the contract, CSR rows of clean rows exact."""
    want_f, want_nnz, pre = oracle.fused_encode(x[rows].cpu(), sae.W_enc.cpu(), sae.b_enc.cpu(), sae.b_dec.cpu(),
                                                None if sae.threshold is None else sae.threshold.cpu(),
                                                sae.activation)
    thr = None if sae.threshold is None else sae.threshold.cpu()
    near = contract.near_cut(pre, thr, sae.activation)
    clean = ~near.any(dim=1)
    assert clean.float().mean() > 0.3, f"only {int(clean.sum())} clean rows of {rows.numel()}"
    dt = x.dtype
    if f_rows is not None:
        contract.assert_values_close(f_rows.cpu()[~near], want_f[~near], dt, what="encoded features")
    got = sub_csr(csr, rows)
    want = oracle.dense_to_csr(want_f)
    contract.assert_csr_rows_match(got, want, torch.nonzero(clean).flatten().tolist(), dt)
    return clean


def check_decoded_rows(sae, out, csr_rows, rows):
    """out[rows] against the oracle's decode of the same CSR rows."""
    want = oracle.sparse_decode(*csr_rows, sae.W_dec.cpu(), sae.b_dec.cpu())
    contract.assert_values_close(out[rows].cpu().float(), want.float(), sae.W_dec.dtype, what="decoded rows")


@pytest.mark.parametrize("variant", ["auto", "simt"])
def test_cfg1_relu_fp32_ieee_full_size(variant):
    """Config 1 under the fp32 contract (rtol 1e-5) on both IEEE-product routes: the default
    split-precision tensor-core GEMM and the CUDA-core kernel."""
    dev = torch.device("cuda")
    sae = bench.make_sae(1, dev)
    x = bench.make_tokens(1, 0, dev)
    T = x.shape[0]
    rn = torch.zeros(T, dtype=torch.int32, device=dev)
    f = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, row_nnz=rn, config={"variant": variant})
    cfg = best_config()
    if variant == "simt":
        assert cfg["variant"] == "simt"
    else:  # IEEE products from split operands on the tensor cores, not TF32
        assert cfg["variant"] == "tcgen05" and "split" in cfg["operands"]
    assert torch.equal(rn, torch.count_nonzero(f, dim=1).int())
    csr = dense_to_csr(f, rn)
    ref = f.to_sparse_csr()
    assert torch.equal(csr[0], ref.crow_indices()) and torch.equal(csr[1].long(), ref.col_indices())
    assert torch.equal(bits(csr[2]), bits(ref.values()))
    l0 = csr[1].numel() / T
    assert 50 < l0 < 80, f"L0 {l0}"  # the config's b_enc = -2.66 gives L0 ~ 64
    rows = sample_rows(T)
    clean = check_encoded_rows(sae, x, f[rows], csr, rows)
    assert torch.equal(rn.cpu()[rows][clean], torch.count_nonzero(f[rows], dim=1).int().cpu()[clean])
    if variant == "auto":  # forward encodes straight to CSR with the same arithmetic
        out = saeflow_b200.forward(sae, x)
        assert torch.equal(bits(out), bits(sparse_decode(*csr, sae.W_dec, sae.b_dec)))
        check_decoded_rows(sae, out, sub_csr(csr, rows), rows)


def test_cfg2_jumprelu_bf16_full_size():
    dev = torch.device("cuda")
    sae = bench.make_sae(2, dev)
    x = bench.make_tokens(2, 0, dev)
    T = x.shape[0]
    csr = saeflow_b200.encode_sparse(sae, x)
    rn = torch.zeros(T, dtype=torch.int32, device=dev)
    f = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, "jumprelu", row_nnz=rn)
    assert_same_csr(csr, dense_to_csr(f, rn))  # CSR route == dense route, every row
    l0 = csr[1].numel() / T
    assert 55 < l0 < 75, f"L0 {l0}"
    out = saeflow_b200.forward(sae, x)
    assert torch.equal(bits(out), bits(sparse_decode(*csr, sae.W_dec, sae.b_dec)))

    rows = sample_rows(T)
    check_encoded_rows(sae, x, f[rows], csr, rows)
    del f
    check_decoded_rows(sae, out, sub_csr(csr, rows), rows)


def test_cfg3_sparse_decode_full_size_every_row():
    dev = torch.device("cuda")
    sae = bench.make_sae(3, dev)
    csr = bench.make_csr(3, 0, dev)
    out = sparse_decode(*csr, sae.W_dec, sae.b_dec)
    assert out.dtype == torch.bfloat16 and out.shape == (csr[0].numel() - 1, 2304)
    want = oracle.sparse_decode(*(t.cpu() for t in csr), sae.W_dec.cpu(), sae.b_dec.cpu())
    contract.assert_values_close(out.cpu().float(), want.float(), torch.bfloat16, what="decoded rows")


def test_cfg4_topk_bf16_full_size():
    dev = torch.device("cuda")
    sae = bench.make_sae(4, dev)
    x = bench.make_tokens(4, 0, dev)
    T, k, N = x.shape[0], sae.k, sae.d_sae
    vals, idx = topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, k)
    assert vals.shape == (T, k) and idx.dtype == torch.int32
    assert ((idx >= 0) & (idx < N)).all()
    assert (vals[:, :-1].float() >= vals[:, 1:].float()).all()  # value-sorted, as torch.topk gives them

    # Every row at full size: the dense ReLU encoder's values at the selected ids, and the
    # selection is the top k of those values ranked by (value, lower id).
    for r0 in range(0, T, 4096):
        r1 = min(T, r0 + 4096)
        f = fused_encode(x[r0:r1], sae.W_enc, sae.b_enc, sae.b_dec, activation="relu")
        ii = idx[r0:r1].long()
        assert torch.equal(bits(f.gather(1, ii)), bits(vals[r0:r1]))
        assert (ii.sort(dim=1).values[:, 1:] != ii.sort(dim=1).values[:, :-1]).all()  # distinct ids
        vmin = vals[r0:r1, -1:].float()
        ff = f.float().scatter_(1, ii, float("-inf"))
        assert (ff <= vmin).all(), "an unselected feature has a larger value than the k-th selected one"
        # an unselected feature tied with the k-th value must have a larger id than every
        # selected feature of that value
        tie_sel = torch.where(f.float().gather(1, ii) == vmin, ii, torch.full_like(ii, -1)).max(dim=1).values
        cols = torch.arange(N, device=dev)
        tie_unsel = torch.where(ff == vmin, cols, torch.full_like(cols, N)).min(dim=1).values
        assert (tie_unsel > tie_sel).all(), "a lower-id feature tied with the k-th value was left out"
        del f, ff

    rows = sample_rows(T)
    pre = oracle.encode_pre(x[rows].cpu(), sae.W_enc.cpu(), sae.b_enc.cpu(), sae.b_dec.cpu())
    wv, wi = oracle.topk_encode(x[rows].cpu(), sae.W_enc.cpu(), sae.b_enc.cpu(), sae.b_dec.cpu(), k)
    amb = contract.topk_ambiguous_rows(pre, k, torch.bfloat16)
    assert amb.float().mean() < 0.5, f"{int(amb.sum())} ambiguous rows of {rows.numel()}"
    got_sets = contract.topk_sets(idx[rows].cpu(), N)
    want_sets = contract.topk_sets(wi, N)
    assert torch.equal(got_sets[~amb], want_sets[~amb])
    gv = torch.zeros(rows.numel(), N).scatter_(1, idx[rows].cpu().long(), vals[rows].cpu().float())
    wvd = torch.zeros(rows.numel(), N).scatter_(1, wi.long(), wv.float())
    sel = want_sets & ~amb[:, None]
    contract.assert_values_close(gv[sel], wvd[sel], torch.bfloat16, what="top-k values")

    out = saeflow_b200.forward(sae, x)
    ip = torch.arange(0, rows.numel() * k + 1, k, dtype=torch.int64)
    check_decoded_rows(sae, out, (ip, idx[rows].cpu().flatten(), vals[rows].cpu().flatten()), rows)


def test_cfg5_jumprelu_2pow20_features_token_slice():
    dev = torch.device("cuda")
    sae = bench.make_sae_cfg5(dev, 0, 1 << 20)
    x = bench.make_token_range(5, 0, 4096, dev)
    T = x.shape[0]
    csr = saeflow_b200.encode_sparse(sae, x)
    rn = torch.zeros(T, dtype=torch.int32, device=dev)
    f = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, "jumprelu", row_nnz=rn)
    assert_same_csr(csr, dense_to_csr(f, rn))
    l0 = csr[1].numel() / T
    assert 85 < l0 < 115, f"L0 {l0}"  # the config's thresholds give L0 ~ 96
    out = saeflow_b200.forward(sae, x)
    assert torch.equal(bits(out), bits(sparse_decode(*csr, sae.W_dec, sae.b_dec)))

    rows = sample_rows(T, 64)
    check_encoded_rows(sae, x, f[rows], csr, rows)
    del f
    check_decoded_rows(sae, out, sub_csr(csr, rows), rows)
