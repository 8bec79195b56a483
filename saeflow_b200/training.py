"""Differentiable sparse forward for training SAEs on sparse features (saeflow's roadmap,
README.md:244: "Backward kernels for training SAEs on sparse features"; the reference has
none).

`forward(sae, x)` returns x_hat = decode(encode_sparse(x)) like saeflow_b200.forward and
supports autograd for x, W_enc, b_enc, W_dec and b_dec. Only the active features carry
gradient (ReLU / JumpReLU: the stored nonzeros; TopK: the selected positive values). The
JumpReLU threshold receives no gradient here: the step function has zero derivative almost
everywhere, and a straight-through estimator for it is a training choice left to the
caller.

Backward, with g = dL/dx_hat and the forward's CSR (indptr, indices, values), over the
column view of the CSR (csr_transpose, rows ascending within each column, so every sum is
taken in one fixed order and the gradients are the same from run to run):
    dW_dec   = per feature, sum of value * g[row]           } one csc_gather pass over the
    dpre     = g[row] . W_dec[col] at each active entry     } gathered rows of g
    dW_enc^T = per feature, sum of dpre * (x - b_dec)[row], db_enc = per feature sum of dpre
                                                              (a second csc_gather pass)
    dx       = dpre @ W_enc^T (the CSR decode against W_enc^T), db_dec = sum_rows (g - dx);
               without a gradient for x, db_dec = sum_rows g - W_enc @ db_enc (matvec), and dx
               is never formed
(x - b_dec) is taken rounded to W_enc's dtype, the operand the encoder multiplied.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .kernels import sparse_decode
from .kernels.backward import csc_gather, csr_sddmm, csr_transpose, matvec, transpose


@dataclass
class _Params:
    W_enc: torch.Tensor
    b_enc: torch.Tensor
    W_dec: torch.Tensor
    b_dec: torch.Tensor
    threshold: torch.Tensor | None
    activation: str
    k: int | None


class _SparseForward(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, W_enc, b_enc, W_dec, b_dec, threshold, activation, k):
        from .ops import encode_sparse

        p = _Params(W_enc.detach(), b_enc.detach(), W_dec.detach(), b_dec.detach(),
                    threshold.detach() if threshold is not None else None, activation, k)
        indptr, indices, values = encode_sparse(p, x.detach())
        out = sparse_decode(indptr, indices, values, p.W_dec, p.b_dec)
        ctx.save_for_backward(x.detach(), p.W_enc, p.W_dec, p.b_dec, indptr, indices, values)
        return out

    @staticmethod
    def backward(ctx, g):
        x, W_enc, W_dec, b_dec, indptr, indices, values = ctx.saved_tensors
        need_x, need_we, need_be, need_wd, need_bd = ctx.needs_input_grad[:5]
        g = g.contiguous()
        if g.dtype != W_dec.dtype:
            g = g.to(W_dec.dtype)
        d_sae = W_enc.shape[1]
        dx = dW_enc = db_enc = dW_dec = db_dec = None
        need_dpre = need_x or need_bd or need_we or need_be
        col = csr_transpose(indptr, indices, d_sae) if (need_wd or need_we or need_be) else None
        dpre = None
        if need_wd and need_dpre:
            dW_dec, dpre = csc_gather(*col, values, g, W=W_dec, out_dtype=W_dec.dtype)
        elif need_wd:
            dW_dec = csc_gather(*col, values, g, out_dtype=W_dec.dtype)
        elif need_dpre:
            dpre = csr_sddmm(indptr, indices, values, g, W_dec)
        sums = None  # fp32 per-feature sums of dpre
        if need_we or need_be:
            if x.dtype == b_dec.dtype == W_enc.dtype:
                xs = x - b_dec  # torch subtracts 16-bit operands in fp32 and rounds once, as below
            else:
                xs = (x.float() - b_dec.float()).to(W_enc.dtype)
            dW_enc_t, sums = csc_gather(*col, dpre, xs, out_dtype=W_enc.dtype, col_sums=True)
            dW_enc = transpose(dW_enc_t) if need_we else None
            db_enc = sums.to(W_enc.dtype) if need_be else None
        if need_x or (need_bd and sums is None):
            dx = sparse_decode(indptr, indices, dpre, transpose(W_enc), None, out_dtype=torch.float32)
            if need_bd:
                db_dec = (g.sum(0, dtype=torch.float32) - dx.sum(0)).to(b_dec.dtype)
            dx = dx.to(x.dtype) if need_x else None
        elif need_bd:
            # sum over tokens of dx = W_enc @ (per-feature sums of dpre): no dx, no W_enc^T
            db_dec = (g.sum(0, dtype=torch.float32) - matvec(W_enc, sums)).to(b_dec.dtype)
        return dx, dW_enc, db_enc, dW_dec, db_dec, None, None, None


def forward(sae, x):
    """x_hat = sae's sparse forward, differentiable in x and the SAE parameters (not the
    JumpReLU threshold). `sae` has the SAELens-named attributes (W_enc, b_enc, W_dec, b_dec,
    threshold, activation, k), e.g. saeflow_b200.SAE with requires_grad parameters."""
    return _SparseForward.apply(x, sae.W_enc, sae.b_enc, sae.W_dec, sae.b_dec, getattr(sae, "threshold", None),
                                sae.activation, getattr(sae, "k", None))
