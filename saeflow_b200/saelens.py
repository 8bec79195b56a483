"""SAELens SAE objects on this package's kernels (saeflow's roadmap item "take sae_lens.SAE
objects directly (architecture and activation-normalisation handling)", README.md:236-238;
the reference's own bench adapter goes the other way, bench/common.py:107-129).

A SAELens SAE holds the parameters this package already names after SAELens: W_enc
[d_in, d_sae], b_enc [d_sae], W_dec [d_sae, d_in], b_dec [d_in] and, for JumpReLU,
threshold [d_sae]; its `cfg` carries d_in, d_sae, apply_b_dec_to_input and
normalize_activations, and names the architecture (`cfg.architecture` as a string, or a
`cfg.architecture()` method) and, for TopK, k (`cfg.k` or `cfg.activation_fn_kwargs["k"]`).

SAELens computes

    x_n   = norm_in(x)
    f     = act((x_n - b_dec * apply_b_dec_to_input) @ W_enc + b_enc)
    x_hat = norm_out(f @ W_dec + b_dec)

with these run-time normalisations (per token row):
    "none", "expected_average_only_in"   identity (the constant dataset scale of the latter
                                         is applied by the activation store or folded into
                                         the weights, not at run time)
    "constant_norm_rescale"              x * sqrt(d_in) / ||x||;  out / that factor
    "layer_norm"                         (x - mean) / (std + 1e-5);  out * std + mean
Architectures "standard" (ReLU), "jumprelu" and "topk" map onto the kernels; others raise
ValueError. The normalisations are elementwise host glue around the kernels.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

_ARCH = {"standard": "relu", "relu": "relu", "jumprelu": "jumprelu", "topk": "topk"}
_NORMS = ("none", "expected_average_only_in", "constant_norm_rescale", "layer_norm")
_LN_EPS = 1e-5


@dataclass
class SAELensView:
    """The kernels' view of a SAELens SAE. `b_dec_in` is the encoder's input shift (b_dec
    when the SAE applies it to its input, zeros otherwise); `b_dec` is the decoder bias."""

    W_enc: torch.Tensor
    b_enc: torch.Tensor
    W_dec: torch.Tensor
    b_dec: torch.Tensor
    b_dec_in: torch.Tensor
    threshold: torch.Tensor | None
    activation: str
    k: int | None
    normalize_activations: str

    def _encoder(self):
        return _Params(self.W_enc, self.b_enc, self.W_dec, self.b_dec_in, self.threshold, self.activation, self.k)


@dataclass
class _Params:
    W_enc: torch.Tensor
    b_enc: torch.Tensor
    W_dec: torch.Tensor
    b_dec: torch.Tensor
    threshold: torch.Tensor | None
    activation: str
    k: int | None


def _architecture(sae, cfg) -> str:
    arch = getattr(cfg, "architecture", None)
    if callable(arch):
        arch = arch()
    if arch is None and callable(getattr(sae, "architecture", None)):
        arch = sae.architecture()
    if arch is None:
        arch = "jumprelu" if getattr(sae, "threshold", None) is not None else "standard"
    return str(arch).lower()


def adapt(sae) -> SAELensView:
    """Read a SAELens SAE (or any object with its attributes) into a SAELensView.

    The tensors are the SAE's own (no copies). Raises ValueError for an architecture or a
    normalisation these kernels do not implement, or a TopK SAE without k."""
    cfg = getattr(sae, "cfg", None)
    arch = _architecture(sae, cfg)
    if arch not in _ARCH:
        raise ValueError(f"SAELens architecture {arch!r} is not supported (standard, jumprelu, topk)")
    activation = _ARCH[arch]
    act_fn = str(getattr(cfg, "activation_fn_str", "") or "").lower()
    if act_fn == "topk":
        activation = "topk"
    k = None
    if activation == "topk":
        k = getattr(cfg, "k", None)
        if k is None:
            k = (getattr(cfg, "activation_fn_kwargs", None) or {}).get("k")
        if not k:
            raise ValueError("a TopK SAELens SAE must name k (cfg.k or cfg.activation_fn_kwargs['k'])")
        k = int(k)
    norm = str(getattr(cfg, "normalize_activations", "none") or "none")
    if norm not in _NORMS:
        raise ValueError(f"normalize_activations={norm!r} is not supported {_NORMS}")
    threshold = getattr(sae, "threshold", None) if activation == "jumprelu" else None
    if activation == "jumprelu" and threshold is None:
        raise ValueError("a JumpReLU SAELens SAE must have a threshold")
    apply_b_dec = bool(getattr(cfg, "apply_b_dec_to_input", True))
    b_dec = sae.b_dec
    b_dec_in = b_dec if apply_b_dec else torch.zeros_like(b_dec)
    return SAELensView(W_enc=sae.W_enc, b_enc=sae.b_enc, W_dec=sae.W_dec, b_dec=b_dec, b_dec_in=b_dec_in,
                       threshold=threshold, activation=activation, k=k, normalize_activations=norm)


def _norm_in(view: SAELensView, x: torch.Tensor):
    """(normalised x in x's dtype, state for norm_out)."""
    mode = view.normalize_activations
    if mode == "constant_norm_rescale":
        xf = x.float()
        scale = math.sqrt(x.shape[-1]) / xf.norm(dim=-1, keepdim=True)
        return (xf * scale).to(x.dtype), ("scale", scale)
    if mode == "layer_norm":
        xf = x.float()
        mu = xf.mean(dim=-1, keepdim=True)
        xc = xf - mu
        std = xc.std(dim=-1, keepdim=True)
        return (xc / (std + _LN_EPS)).to(x.dtype), ("ln", mu, std)
    return x, None


def _norm_out(x_hat: torch.Tensor, state):
    if state is None:
        return x_hat
    if state[0] == "scale":
        return (x_hat.float() / state[1]).to(x_hat.dtype)
    _, mu, std = state
    return (x_hat.float() * std + mu).to(x_hat.dtype)


def _view(sae) -> SAELensView:
    return sae if isinstance(sae, SAELensView) else adapt(sae)


def encode(sae, x):
    """Dense features [M, d_sae] of a SAELens SAE (SAE.encode)."""
    from . import ops

    v = _view(sae)
    xn, _ = _norm_in(v, x)
    return ops.encode(v._encoder(), xn)


def encode_sparse(sae, x):
    """CSR features (indptr, indices, values) of a SAELens SAE."""
    from . import ops

    v = _view(sae)
    xn, _ = _norm_in(v, x)
    return ops.encode_sparse(v._encoder(), xn)


def decode_sparse(sae, csr, x=None):
    """Reconstruction from CSR features (SAE.decode). Row normalisations need the input
    rows they came from: pass `x` when the SAE normalises its activations."""
    from .kernels import sparse_decode

    v = _view(sae)
    state = None
    if v.normalize_activations in ("constant_norm_rescale", "layer_norm"):
        if x is None:
            raise ValueError(f"normalize_activations={v.normalize_activations!r}: decode_sparse needs x")
        _, state = _norm_in(v, x)
    return _norm_out(sparse_decode(*csr, v.W_dec, v.b_dec), state)


def forward(sae, x):
    """x_hat = SAE(x) through the sparse path: encode straight to CSR, then the CSR decode."""
    v = _view(sae)
    xn, state = _norm_in(v, x)
    from . import ops

    enc = v._encoder()
    if v.activation == "topk":
        csr = ops.encode_sparse(enc, xn)
    else:
        from .kernels.encode import encode_csr_finish_async, encode_csr_stage

        h = encode_csr_stage(xn, enc.W_enc, enc.b_enc, enc.b_dec, enc.threshold, enc.activation, device_consumer=True)
        *csr, overflow = encode_csr_finish_async(h)
        if overflow is not None and int(overflow):
            csr = ops.encode_sparse(enc, xn)
    from .kernels import sparse_decode

    return _norm_out(sparse_decode(*csr, v.W_dec, v.b_dec), state)
