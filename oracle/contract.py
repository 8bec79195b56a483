"""Parity rules of the SAE hot path — TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The contract the CUDA path is held to, against the CPU restatement in sae_oracle.py on
the same rounded inputs (the pattern of the reference test, tests/test_kernels.py:33-63):

* floating-point outputs: |got - want| <= ATOL + RTOL * |want| with RTOL 1e-2 for 16-bit
  storage and 1e-5 for fp32 (IEEE products);
* features whose pre-activation lies within CUT_BAND = 1e-3 of their cut (max(threshold, 0)
  for JumpReLU, 0 for ReLU) are excluded, and with them every CSR check of their row;
* CSR structure (row counts, column indices) bit-exact on the remaining rows.

The absolute floors are not slack for the 16-bit cases: two correct results of a
16-bit output differ by at most one rounding step (2^-7 relative for bf16), far inside
RTOL; ATOL only covers values near zero. For fp32 the floor is needed: an fp32 sum of
d_in products differs from the float64 sum by a few units of 1e-6 at config 1 (d_in=768,
measured 6.7e-6 worst over 16k active features), so a purely relative 1e-5 would fail
for small features whatever the summation order.
"""

from __future__ import annotations

import torch

CUT_BAND = 1e-3
RTOL = {torch.bfloat16: 1e-2, torch.float16: 5e-3, torch.float32: 1e-5}
ATOL = {torch.bfloat16: 1e-4, torch.float16: 1e-4, torch.float32: 1e-5}


def tolerance(dtype):
    """(rtol, atol) of the contract for outputs stored in `dtype`."""
    return RTOL[dtype], ATOL[dtype]


def near_cut(pre, threshold=None, activation="relu", band=CUT_BAND):
    """Boolean mask of pre-activations within `band` of the point where the output switches
    between zero and nonzero: 0 for ReLU, max(threshold, 0) for JumpReLU (relu(pre) is
    kept where pre > threshold, so a negative threshold leaves the ReLU's 0 as the cut)."""
    if activation == "jumprelu":
        cut = torch.clamp_min(threshold.float(), 0.0)
        return (pre - cut).abs() < band
    return pre.abs() < band


def clean_rows(pre, threshold=None, activation="relu", band=CUT_BAND):
    """Rows with no feature near its cut: their CSR must match exactly."""
    return ~near_cut(pre, threshold, activation, band).any(dim=1)


def assert_values_close(got, want, dtype, what="values"):
    """The contract's floating-point rule, element-wise, with the worst offender reported."""
    rtol, atol = tolerance(dtype)
    g, w = got.double(), want.double()
    bad = (g - w).abs() > atol + rtol * w.abs()
    bad |= torch.isnan(g) != torch.isnan(w)
    if bool(bad.any()):
        err = ((g - w).abs() - rtol * w.abs()).nan_to_num(float("inf"))
        i = int(err.flatten().argmax())
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.numel()} elements outside rtol {rtol} atol {atol}; "
                             f"worst got {g.flatten()[i].item()!r} want {w.flatten()[i].item()!r}")


def csr_row(indptr, indices, values, r):
    """(indices, values) of row r of a CSR triple (CPU tensors)."""
    a, b = int(indptr[r]), int(indptr[r + 1])
    return indices[a:b], values[a:b]


def assert_csr_rows_match(got, want, rows, dtype):
    """Row r of `got` equals row r of `want` for every r in `rows`: same count and column
    indices bit for bit, values under the contract's rule. CSR triples on the CPU."""
    for r in rows:
        gi, gv = csr_row(*got, r)
        wi, wv = csr_row(*want, r)
        if gi.numel() != wi.numel() or not torch.equal(gi.long(), wi.long()):
            raise AssertionError(f"row {r}: columns differ ({gi.numel()} vs {wi.numel()} nonzeros)")
        assert_values_close(gv, wv, dtype, what=f"row {r} values")


def round_to(t, dtype):
    """fp32 values rounded to `dtype` and back (the kernels' output rounding)."""
    return t.to(dtype).float()


def topk_ambiguous_rows(pre, k, dtype, delta=2e-4):
    """Rows whose top-k set could legitimately differ between two correct fp32 sums, for
    values stored in a 16-bit `dtype`.

    Both the reference (dense ReLU output in `dtype`, then torch.topk, saeflow/ops.py:12-16)
    and the kernels rank the ROUNDED values, ties by lower feature index, so the set is a
    function of the rounded values. It can change only if an element near the k-th rounded
    value (within one rounding step of it) has a pre-activation within `delta` of a rounding
    midpoint, where a sum error can flip its rounding. Such rows are excluded; this is
    stricter than excluding every row whose k-th and (k+1)-th values lie within 1e-3."""
    f = torch.clamp_min(pre.float(), 0.0)
    r = round_to(f, dtype)
    kth = r.sort(dim=1, descending=True).values[:, k - 1:k]
    step = kth.abs() * (2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10) * 1.01
    close = (r - kth).abs() <= step
    # distance of f to the nearest rounding midpoint: rounding f -/+ delta gives different values
    risky = round_to(f - delta, dtype) != round_to(f + delta, dtype)
    return (close & risky & (f > 0)).any(dim=1)


def topk_sets(indices, n_cols):
    """Boolean [M, n_cols] membership of each row's selected feature ids."""
    m = torch.zeros(indices.shape[0], n_cols, dtype=torch.bool)
    return m.scatter_(1, indices.long(), True)
