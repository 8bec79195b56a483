"""SAE parameter container with saeflow's constructor and SAELens parameter names.

Mirrors the constructor of saeflow/reference.py:9-33: W_dec [d_sae, d_in] has
unit-norm Gaussian rows, W_enc = W_dec.T (contiguous), b_enc = b_dec = 0, and a
threshold [d_sae] for JumpReLU. The random draws are made in the same order, so a
given torch seed yields the same weights as the reference class.

Its compute methods run the CUDA path of this package (the reference's are the plain
PyTorch ground truth); `decode` takes dense features and decodes them through CSR.
"""

import torch
from torch import nn

ACTIVATIONS = ("relu", "jumprelu", "topk")


class SAE(nn.Module):
    """x -> f = act((x - b_dec) @ W_enc + b_enc) -> x_hat = f @ W_dec + b_dec.

    activation: "relu", "jumprelu" (per-feature `threshold`) or "topk" (keep the `k`
    largest pre-activations per token). W_enc [d_in, d_sae], W_dec [d_sae, d_in].
    """

    def __init__(self, d_in, d_sae, activation="relu", k=None, device=None, dtype=torch.float32):
        super().__init__()
        if activation not in ACTIVATIONS:
            raise ValueError(f"activation must be one of {ACTIVATIONS}, got {activation!r}")
        if activation == "topk" and not k:
            raise ValueError("topk activation needs k")
        self.d_in, self.d_sae, self.activation, self.k = d_in, d_sae, activation, k

        W_dec = torch.randn(d_sae, d_in, device=device)
        W_dec /= W_dec.norm(dim=1, keepdim=True)
        self.W_dec = nn.Parameter(W_dec.to(dtype))
        self.W_enc = nn.Parameter(W_dec.T.contiguous().to(dtype))
        self.b_enc = nn.Parameter(torch.zeros(d_sae, device=device, dtype=dtype))
        self.b_dec = nn.Parameter(torch.zeros(d_in, device=device, dtype=dtype))
        self.threshold = (
            nn.Parameter(torch.zeros(d_sae, device=device, dtype=dtype)) if activation == "jumprelu" else None
        )
        self.requires_grad_(False)

    def encode(self, x):
        from . import ops

        return ops.encode(self, x)

    def encode_sparse(self, x):
        from . import ops

        return ops.encode_sparse(self, x)

    def decode_sparse(self, csr):
        from . import ops

        return ops.decode_sparse(self, csr)

    def decode(self, f):
        from .kernels import dense_to_csr, sparse_decode

        return sparse_decode(*dense_to_csr(f), self.W_dec, self.b_dec)

    def forward(self, x):
        from . import ops

        return ops.forward(self, x)
