"""SAE-level entry points, a drop-in for saeflow/ops.py. `sae` is a saeflow_b200.SAE
or anything with the same attributes (W_enc, b_enc, W_dec, b_dec, threshold,
activation, k), e.g. a saeflow.reference.SAE moved to a CUDA device.

Sparse features are CSR tuples (indptr, indices, values); see kernels/decode.py.
"""

import torch

from .kernels import encode_csr, fused_encode, sparse_decode, topk_encode


def _topk(sae, x):
    """(values [M, k], indices int32 [M, k]) of the k largest ReLU'd pre-activations.

    The reference writes the dense ReLU output and calls torch.topk (ops.py:12-16); here
    the selection runs inside the encoder's epilogue and the dense output is never made.
    """
    return topk_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.k)


def encode(sae, x):
    """Dense feature activations [M, d_sae] (ops.py:19-26)."""
    if sae.activation == "topk":
        values, indices = _topk(sae, x)
        return torch.zeros(x.shape[0], sae.W_enc.shape[1], device=x.device, dtype=x.dtype).scatter_(
            -1, indices.long(), values
        )
    return fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation)


def encode_sparse(sae, x):
    """Feature activations as CSR (indptr, indices, values) (ops.py:29-39)."""
    M = x.shape[0]
    if sae.activation == "topk":
        # TopK is fixed-width: no compaction pass, indptr is arange (ops.py:35).
        values, indices = _topk(sae, x)
        indptr = torch.arange(0, M * sae.k + 1, sae.k, device=x.device, dtype=torch.int64)
        return indptr, indices.flatten(), values.flatten()
    # Same CSR as fused_encode(row_nnz=...) + dense_to_csr (ops.py:37-39), built from the
    # encoder's epilogue without writing or re-reading the dense [M, d_sae] features.
    return encode_csr(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, sae.activation)


def decode_sparse(sae, csr):
    """Reconstruction [M, d_in] from CSR features (ops.py:42-44)."""
    return sparse_decode(*csr, sae.W_dec, sae.b_dec)


def forward(sae, x):
    """encode_sparse then decode_sparse: the dense features never reach the decoder (ops.py:47-49)."""
    return decode_sparse(sae, encode_sparse(sae, x))
