"""CPU oracle of the saeflow SAE hot path — TEST INFRASTRUCTURE ONLY.

A plain restatement, on the CPU, of the reference algorithm (iamartyaa/saeflow:
saeflow/kernels/encode.py, saeflow/kernels/decode.py, saeflow/ops.py,
saeflow/reference.py). Only tests/, __graft_entry__.smoke() and the cpu_baseline /
reference arm of bench.py may import it, and only as the checker or the timed CPU
baseline. The product (saeflow_b200) never imports it.

Parity pin: the restatement is checked against golden vectors produced by the
reference itself (tests/golden/make_golden.py, run where the reference is importable;
its Triton kernels executed by Triton's CPU interpreter). See tests/test_oracle_golden.py.
"""

from .sae_oracle import (  # noqa: F401
    RefSAE,
    dense_to_csr,
    encode_pre,
    encode_sparse,
    forward,
    fused_encode,
    sparse_decode,
    to_dtype,
    topk_encode,
)
