"""Write the activation-cache fixtures of tests/golden/cache_ref/ with the reference's own
saeflow.cache.cache_activations (saeflow/cache.py:70-137).

Run where the reference package is importable (a checkout of iamartyaa/saeflow):

    python tests/golden/make_golden_cache.py --reference /path/to/saeflow

The model is tests/cache_fixtures.TinyModel (the cache only calls `run_with_cache` and
`parameters`); its activations and the encoder SAE's features are exact on a 1/8 grid,
so the files are what any correct implementation writes, byte for byte. The on-the-fly
encoder runs the reference's Triton kernels through Triton's CPU interpreter
(TRITON_INTERPRET=1, as the reference's CI does). Three caches are written:

    dense_fp32/  both hooks dense, fp32, batch_size=4, batches_per_shard=2 (3 shards)
    dense_bf16/  hook 0 dense, stored as bf16 raw bits, batch_size=8
    csr_fp32/    hook 0 encoded on the fly (JumpReLU SAE, d_sae=96), hook 1 dense
"""

from __future__ import annotations

import argparse
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "cache_ref"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory holding the saeflow package")
    args = ap.parse_args(argv)
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(Path(args.reference).resolve()))
    sys.path.insert(0, str(HERE.parent))
    import torch
    from saeflow.cache import cache_activations
    from saeflow.reference import SAE

    import cache_fixtures as cf

    if OUT.exists():
        shutil.rmtree(OUT)
    model, toks = cf.TinyModel(), cf.tokens()
    cache_activations(model, toks, cf.HOOKS, OUT / "dense_fp32", batch_size=4, batches_per_shard=2)
    cache_activations(model, toks, cf.HOOKS[:1], OUT / "dense_bf16", batch_size=8, dtype=torch.bfloat16)
    sae = cf.exact_sae(SAE)
    cache_activations(model, toks, cf.HOOKS, OUT / "csr_fp32", batch_size=4, batches_per_shard=2,
                      encoders={cf.HOOKS[0]: sae})
    for p in sorted(OUT.rglob("*")):
        if p.is_file():
            print(p.relative_to(HERE), p.stat().st_size)
    return 0


if __name__ == "__main__":
    sys.exit(main())
