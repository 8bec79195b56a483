"""Pin the CPU oracle against golden vectors produced by the reference saeflow itself.

CPU only. The same tolerance rules as the reference's tests/test_kernels.py: elements
within rounding distance of the ReLU / JumpReLU cut are excluded, everything integer
(row counts, CSR structure) is compared exactly.
"""

import pytest
import torch

import oracle
from golden_io import Golden

TOL = {torch.float32: 1e-4, torch.bfloat16: 3e-2, torch.float16: 5e-3}

ENC = Golden("fused_encode")


@pytest.mark.parametrize("case", range(ENC.int("n")))
def test_oracle_fused_encode_matches_reference(case):
    p = f"c{case}/"
    act = ENC.str(p + "activation")
    x, W, b_enc, b_dec = ENC.t(p + "x"), ENC.t(p + "W_enc"), ENC.t(p + "b_enc"), ENC.t(p + "b_dec")
    thr = ENC.t(p + "threshold")
    if ENC.has(p + "colmajor"):
        W = W.T.contiguous().T
    want = ENC.t(p + "out")
    got, row_nnz, pre = oracle.fused_encode(x, W, b_enc, b_dec, thr, act)
    assert got.dtype == want.dtype and got.shape == want.shape
    tol_d = TOL[x.dtype]
    cut = pre - (thr.float() if act == "jumprelu" else 0)
    tol = tol_d * (1 + pre.abs().max())
    keep = cut.abs() > tol
    torch.testing.assert_close(got.float()[keep], want.float()[keep], atol=tol, rtol=tol_d)
    # the oracle's count is exactly the nonzeros it stores
    assert torch.equal(row_nnz, torch.count_nonzero(got, dim=1).int())
    if ENC.has(p + "row_nnz"):
        ref_nnz = ENC.t(p + "row_nnz")
        assert torch.equal(ref_nnz, torch.count_nonzero(want, dim=1).int())  # the reference's own invariant
        clean = keep.all(dim=1)  # rows with no element on the cut agree exactly
        assert torch.equal(row_nnz[clean], ref_nnz[clean])


CSR = Golden("dense_to_csr")


def _bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


@pytest.mark.parametrize("case", range(CSR.int("n")))
def test_oracle_dense_to_csr_bit_exact(case):
    p = f"c{case}/"
    f = CSR.t(p + "f")
    ip, ix, vs = oracle.dense_to_csr(f)
    assert torch.equal(ip, CSR.t(p + "indptr"))
    assert torch.equal(ix, CSR.t(p + "indices"))
    want = CSR.t(p + "values")
    assert vs.dtype == want.dtype
    assert torch.equal(_bits(vs), _bits(want))


DEC = Golden("sparse_decode")


@pytest.mark.parametrize("case", range(DEC.int("n")))
def test_oracle_sparse_decode_matches_reference(case):
    p = f"c{case}/"
    W = DEC.t(p + "W_dec")
    got = oracle.sparse_decode(DEC.t(p + "indptr"), DEC.t(p + "indices"), DEC.t(p + "values"), W, DEC.t(p + "b_dec"))
    want = DEC.t(p + "out")
    assert got.dtype == want.dtype
    torch.testing.assert_close(got.float(), want.float(), atol=TOL[W.dtype] * 4, rtol=TOL[W.dtype])


OPS = Golden("ops")


@pytest.mark.parametrize("activation", ["relu", "jumprelu", "topk"])
def test_oracle_ops_match_reference(activation):
    p = f"{activation}/"
    sae = oracle.RefSAE(40, 150, activation, k=8)
    for name in ("W_enc", "W_dec", "b_enc", "b_dec", "threshold"):
        if OPS.has(p + name):
            getattr(sae, name).copy_(OPS.t(p + name))
    x = OPS.t(p + "x")
    # the reference's dense SAE and the restated one agree
    torch.testing.assert_close(sae.encode(x), OPS.t(p + "sae_encode"), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(sae(x), OPS.t(p + "sae_forward"), atol=1e-5, rtol=1e-5)
    ip, ix, vs = oracle.encode_sparse(sae, x)
    if activation == "topk":
        assert torch.equal(ip, OPS.t(p + "indptr"))
        # index sets per row (the reference orders by value, ops.py:16)
        got = torch.zeros(33, 150).scatter_(1, ix.view(33, 8).long(), vs.view(33, 8))
        want = torch.zeros(33, 150).scatter_(1, OPS.t(p + "indices").view(33, 8).long(), OPS.t(p + "values").view(33, 8))
        torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
    else:
        assert torch.equal(ip, OPS.t(p + "indptr"))
        assert torch.equal(ix, OPS.t(p + "indices"))
        torch.testing.assert_close(vs, OPS.t(p + "values"), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(oracle.forward(sae, x), OPS.t(p + "forward"), atol=1e-5, rtol=1e-5)


def test_sae_constructor_draws_match_reference():
    """Same seed -> same weights as saeflow.reference.SAE (reference.py:25-33), for the
    oracle's restatement and for the product's parameter container."""
    from saeflow_b200 import SAE

    g = Golden("sae_init")
    for cls in (oracle.RefSAE, SAE):
        torch.manual_seed(0)
        s = cls(24, 64, "jumprelu")
        for name in ("W_enc", "W_dec", "b_enc", "b_dec", "threshold"):
            assert torch.equal(getattr(s, name), g.t(name)), (cls.__name__, name)


def test_constructor_errors():
    from saeflow_b200 import SAE

    for cls in (oracle.RefSAE, SAE):
        with pytest.raises(ValueError):
            cls(4, 8, "gelu")
        with pytest.raises(ValueError):
            cls(4, 8, "topk")


def test_oracle_encode_errors():
    x = torch.randn(3, 4)
    W = torch.randn(4, 5)
    b = torch.zeros(5)
    with pytest.raises(ValueError):
        oracle.fused_encode(x, W, b, torch.zeros(4), activation="gelu")
    with pytest.raises(ValueError):
        oracle.fused_encode(x, W, b, torch.zeros(4), activation="jumprelu")


@pytest.mark.parametrize("case", range(ENC.int("n")))
def test_reference_outputs_meet_the_contract_tolerances(case):
    """The contract's rules (oracle/contract.py: rtol 1e-2 bf16 / 1e-5 fp32 with small
    absolute floors, 1e-3 cut band, exact CSR rows) hold between the reference's own
    outputs and the oracle: the oracle is pinned to the reference at the tolerances the GPU
    tests hold the kernels to."""
    from oracle import contract

    p = f"c{case}/"
    act = ENC.str(p + "activation")
    x, W, b_enc, b_dec = ENC.t(p + "x"), ENC.t(p + "W_enc"), ENC.t(p + "b_enc"), ENC.t(p + "b_dec")
    thr = ENC.t(p + "threshold")
    if ENC.has(p + "colmajor"):
        W = W.T.contiguous().T
    want = ENC.t(p + "out")
    # The golden vectors come from Triton's CPU interpreter, which converts fp32 to bf16 by
    # truncation; the oracle restates that conversion for the bf16 cases (the GPU kernels,
    # like compiled Triton, round to nearest and are checked against the default oracle).
    rounding = "truncate" if x.dtype == torch.bfloat16 else "nearest"
    got, _, pre = oracle.fused_encode(x, W, b_enc, b_dec, thr, act, rounding=rounding)
    near = contract.near_cut(pre, thr, act)
    contract.assert_values_close(want[~near].float(), got[~near].float(), x.dtype, what="reference vs oracle")
    clean = torch.nonzero(~near.any(dim=1)).flatten().tolist()
    contract.assert_csr_rows_match(oracle.dense_to_csr(want), oracle.dense_to_csr(got), clean, x.dtype)


def test_contract_cut_band_and_topk_ambiguity():
    from oracle import contract

    pre = torch.tensor([[0.0005, 0.5, 1.2], [0.3, -0.0002, 2.0]])
    thr = torch.tensor([-1.0, 0.5004, 1.0])
    # JumpReLU: the cut is max(threshold, 0); ReLU: the cut is 0
    assert contract.near_cut(pre, thr, "jumprelu").tolist() == [[True, True, False], [False, False, False]]
    assert contract.near_cut(pre, None, "relu").tolist() == [[True, False, False], [False, True, False]]
    assert contract.clean_rows(pre, None, "relu").tolist() == [False, False]
    # a bf16 rounding midpoint next to the k-th value makes a row ambiguous; a wide gap does not
    mid = 1.0 + 2.0 ** -8  # halfway between the bf16 neighbours 1.0 and 1.0078125
    rows = torch.tensor([[3.0, 2.0, mid, 0.1], [3.0, 2.0, 1.0, 0.1]])
    assert contract.topk_ambiguous_rows(rows, 3, torch.bfloat16).tolist() == [True, False]
    with pytest.raises(AssertionError, match="outside rtol"):
        contract.assert_values_close(torch.tensor([1.02]), torch.tensor([1.0]), torch.bfloat16)
    contract.assert_values_close(torch.tensor([1.0078125, 5e-5]), torch.tensor([1.0, 0.0]), torch.bfloat16)


def test_bf16_golden_outputs_are_the_truncating_conversion_bit_for_bit():
    """Every bf16 golden output away from the cut is reproduced bit for bit by the oracle
    with the interpreter's truncating fp32 -> bf16 conversion, and not by round-to-nearest:
    the one difference between the golden vectors and the GPU contract is that rounding mode."""
    from oracle import contract

    n_trunc_diff = n_rn_diff = 0
    for case in range(ENC.int("n")):
        p = f"c{case}/"
        x = ENC.t(p + "x")
        if x.dtype != torch.bfloat16:
            continue
        act = ENC.str(p + "activation")
        W, b_enc, b_dec, thr = ENC.t(p + "W_enc"), ENC.t(p + "b_enc"), ENC.t(p + "b_dec"), ENC.t(p + "threshold")
        if ENC.has(p + "colmajor"):
            W = W.T.contiguous().T
        want = ENC.t(p + "out").view(torch.int16)
        tr, _, pre = oracle.fused_encode(x, W, b_enc, b_dec, thr, act, rounding="truncate")
        rn, _, _ = oracle.fused_encode(x, W, b_enc, b_dec, thr, act)
        # a truncation boundary within fp32 summation error of pre is the only other way to differ
        edge = (oracle.to_dtype(pre - 1e-5, torch.bfloat16, "truncate") !=
                oracle.to_dtype(pre + 1e-5, torch.bfloat16, "truncate"))
        keep = ~contract.near_cut(pre, thr, act) & ~edge
        n_trunc_diff += int((tr.view(torch.int16) != want)[keep].sum())
        n_rn_diff += int((rn.view(torch.int16) != want)[keep].sum())
    assert n_trunc_diff == 0
    assert n_rn_diff > 0
