"""Kernel-level API, a drop-in for saeflow.kernels (saeflow/kernels/__init__.py:1-9).

There is no interpreter mode: every op runs a CUDA kernel of libsaeflow_b200.so on
sm_100a, so INTERPRET is always False.
"""

from .._abi import device_error
from .decode import csr_to_dense, dense_to_csr, sparse_decode, topk_encode
from .encode import best_config, encode_csr, fused_encode

INTERPRET = False

__all__ = ["INTERPRET", "best_config", "csr_to_dense", "dense_to_csr", "device_error", "encode_csr",
           "fused_encode", "sparse_decode", "topk_encode"]
