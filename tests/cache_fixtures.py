"""Shared by the activation-cache tests and tests/golden/make_golden_cache.py.

TinyModel stands in for a TransformerLens model (only `run_with_cache` and `parameters`
are used by the cache, saeflow/cache.py:109-115). Its activations are exact in fp32 and
bf16 (sums and products of multiples of 1/8 with few terms), and the SAE below has
weights on the same grid, so every backend (torch CPU, Triton's interpreter, the CUDA
kernels) computes bit-identical activations and features, whatever its summation order.
"""

import torch

HOOKS = ["blocks.0.hook_resid_post", "blocks.1.attn.hook_z"]
D_MODEL, N_HEADS, D_HEAD, D_VOCAB, N_CTX = 32, 4, 8, 100, 16


class TinyModel(torch.nn.Module):
    def __init__(self, device="cpu"):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        emb = torch.randint(-8, 9, (D_VOCAB, D_MODEL), generator=g).float() / 8
        self.emb = torch.nn.Parameter(emb.to(device), requires_grad=False)
        self.perm = torch.randperm(D_MODEL, generator=g).to(device)

    def run_with_cache(self, tokens, names_filter=None, stop_at_layer=None, return_type=None):
        x = self.emb[tokens]                                     # [batch, pos, d_model]
        resid0 = x * 2 + 0.125
        cache = {HOOKS[0]: resid0}
        if stop_at_layer is None or stop_at_layer > 1:
            z = (resid0[..., self.perm] - x).view(*x.shape[:2], N_HEADS, D_HEAD)  # per-head hook
            cache[HOOKS[1]] = z
        names = set(names_filter) if names_filter is not None else set(cache)
        return None, {k: v for k, v in cache.items() if k in names}


class Interrupted(Exception):
    pass


class FlakyModel:
    """Delegates to a model but dies after `n` forward passes."""

    def __init__(self, model, n):
        self.model, self.n = model, n

    def parameters(self):
        return self.model.parameters()

    def run_with_cache(self, *args, **kwargs):
        if self.n == 0:
            raise Interrupted
        self.n -= 1
        return self.model.run_with_cache(*args, **kwargs)


def tokens():
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, D_VOCAB, (22, N_CTX), generator=g)  # last shard and last batch partial


def expected(model, toks, hook):
    with torch.inference_mode():
        _, acts = model.run_with_cache(toks, names_filter=[hook])
    return acts[hook].flatten(0, 1).flatten(1)


def exact_sae(sae_cls, d_sae=96):
    """A JumpReLU SAE whose parameters are multiples of 1/8 (W_enc entries in {-1/8, 0, 1/8})."""
    g = torch.Generator().manual_seed(2)
    sae = sae_cls(D_MODEL, d_sae, "jumprelu")
    with torch.no_grad():
        sae.W_enc.copy_(torch.randint(-1, 2, (D_MODEL, d_sae), generator=g).float() / 8)
        sae.W_dec.copy_(sae.W_enc.T)
        sae.b_enc.copy_(torch.randint(-4, 5, (d_sae,), generator=g).float() / 8)
        sae.b_dec.copy_(torch.randint(-2, 3, (D_MODEL,), generator=g).float() / 8)
        sae.threshold.fill_(0.5)
    return sae
