"""saeflow_b200: the saeflow SAE hot path (encode -> CSR -> decode) on B200 (sm_100a).

Drop-in for saeflow's `encode / encode_sparse / decode_sparse / forward` and
`saeflow.kernels`, backed by hand-written CUDA kernels in libsaeflow_b200.so.
"""

from .ops import HostForward, decode_sparse, encode, encode_sparse, forward, forward_host, forward_host_async
from .sae import SAE

__version__ = "0.1.0"
__all__ = ["SAE", "HostForward", "decode_sparse", "encode", "encode_sparse", "forward", "forward_host",
           "forward_host_async"]
