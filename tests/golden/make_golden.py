"""Generate the golden vectors of tests/golden/*.npz from the reference saeflow itself.

Run where the reference package is importable (a checkout of iamartyaa/saeflow):

    python tests/golden/make_golden.py --reference /path/to/saeflow

The reference's Triton kernels run on the CPU through Triton's interpreter
(TRITON_INTERPRET=1, as the reference's own CI does), so every output here is what
saeflow computes: fused_encode outputs and row counts, dense_to_csr structure,
sparse_decode outputs, and the ops-level encode / encode_sparse / forward results.
Inputs are seeded; the fixtures hold inputs and outputs, bf16 stored as raw uint16 bits.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _pack(store: dict, key: str, t) -> None:
    import torch

    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        store[key] = t.view(torch.int16).numpy().view(np.uint16)
        store[key + ".dtype"] = np.array("bfloat16")
    else:
        store[key] = t.numpy()
        store[key + ".dtype"] = np.array(str(t.dtype).replace("torch.", ""))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory holding the saeflow package")
    a = ap.parse_args(argv)
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(Path(a.reference).resolve()))
    import torch

    import saeflow
    from saeflow.kernels import dense_to_csr, fused_encode, sparse_decode
    from saeflow.reference import SAE

    SHAPES = [(1, 16, 32), (37, 50, 129), (64, 64, 256), (100, 33, 70)]
    DTYPES = [torch.float32, torch.bfloat16, torch.float16]

    def make_sae(d_in, d_sae, activation, dtype, k=None):
        sae = SAE(d_in, d_sae, activation, k=k)
        sae.b_enc.normal_(0, 0.1)
        sae.b_dec.normal_(0, 0.1)
        if activation == "jumprelu":
            sae.threshold.uniform_(0.0, 0.5)
        return sae.to(dtype)

    # ---- fused_encode
    enc = {}
    case = 0
    for shape in SHAPES:
        for dtype in DTYPES:
            for activation in ("relu", "jumprelu"):
                torch.manual_seed(1000 + case)
                M, d_in, d_sae = shape
                sae = make_sae(d_in, d_sae, activation, dtype)
                x = torch.randn(M, d_in).to(dtype)
                row_nnz = torch.zeros(M, dtype=torch.int32)
                out = fused_encode(x, sae.W_enc, sae.b_enc, sae.b_dec, sae.threshold, activation, row_nnz=row_nnz)
                p = f"c{case}/"
                enc[p + "activation"] = np.array(activation)
                for name, t in (("x", x), ("W_enc", sae.W_enc), ("b_enc", sae.b_enc), ("b_dec", sae.b_dec),
                                ("out", out), ("row_nnz", row_nnz)):
                    _pack(enc, p + name, t)
                if activation == "jumprelu":
                    _pack(enc, p + "threshold", sae.threshold)
                case += 1
    # column-major W_enc (test_kernels.py:47-52)
    torch.manual_seed(2000)
    sae = make_sae(48, 80, "relu", torch.float32)
    W_t = sae.W_enc.T.contiguous().T
    x = torch.randn(20, 48)
    out = fused_encode(x, W_t, sae.b_enc, sae.b_dec)
    p = f"c{case}/"
    enc[p + "activation"] = np.array("relu")
    enc[p + "colmajor"] = np.array(1)
    for name, t in (("x", x), ("W_enc", sae.W_enc), ("b_enc", sae.b_enc), ("b_dec", sae.b_dec), ("out", out)):
        _pack(enc, p + name, t)
    case += 1
    enc["n"] = np.array(case)
    np.savez_compressed(HERE / "fused_encode.npz", **enc)

    # ---- dense_to_csr
    csr = {}
    cases = []
    for i, shape in enumerate([(1, 32), (37, 129), (64, 300)]):
        torch.manual_seed(3000 + i)
        f = torch.relu(torch.randn(*shape) - 1.0)
        f[0] = 0
        cases.append(f)
    cases.append(torch.zeros(5, 40))
    torch.manual_seed(3100)
    g = torch.relu(torch.randn(6, 70) - 0.5)
    g[1, 3] = float("nan")
    g[2, 5] = -0.0
    g[3, 7] = float("inf")
    g[4, :] = 0.5  # every feature active
    cases.append(g)
    torch.manual_seed(3200)
    cases.append((torch.relu(torch.randn(9, 77) - 1.0)).to(torch.bfloat16))
    cases.append((torch.relu(torch.randn(9, 77) - 1.0)).to(torch.float16))
    for i, f in enumerate(cases):
        ip, ix, vs = dense_to_csr(f)
        p = f"c{i}/"
        for name, t in (("f", f), ("indptr", ip), ("indices", ix), ("values", vs)):
            _pack(csr, p + name, t)
    csr["n"] = np.array(len(cases))
    np.savez_compressed(HERE / "dense_to_csr.npz", **csr)

    # ---- sparse_decode
    dec = {}
    case = 0
    for shape in SHAPES:
        for dtype in DTYPES:
            torch.manual_seed(4000 + case)
            M, d_in, d_sae = shape
            sae = make_sae(d_in, d_sae, "relu", dtype)
            f = torch.relu(torch.randn(M, d_sae) - 1.5).to(dtype)
            ip, ix, vs = dense_to_csr(f)
            out = sparse_decode(ip, ix, vs, sae.W_dec, sae.b_dec)
            p = f"c{case}/"
            for name, t in (("indptr", ip), ("indices", ix), ("values", vs), ("W_dec", sae.W_dec),
                            ("b_dec", sae.b_dec), ("out", out)):
                _pack(dec, p + name, t)
            case += 1
    dec["n"] = np.array(case)
    np.savez_compressed(HERE / "sparse_decode.npz", **dec)

    # ---- ops (saeflow.encode / encode_sparse / forward), 33 x 40 -> 150, k=8
    ops = {}
    for i, activation in enumerate(("relu", "jumprelu", "topk")):
        torch.manual_seed(5000 + i)
        sae = make_sae(40, 150, activation, torch.float32, k=8)
        x = torch.randn(33, 40)
        dense = saeflow.encode(sae, x)
        ip, ix, vs = saeflow.encode_sparse(sae, x)
        xh = saeflow.forward(sae, x)
        p = f"{activation}/"
        for name, t in (("x", x), ("W_enc", sae.W_enc), ("W_dec", sae.W_dec), ("b_enc", sae.b_enc),
                        ("b_dec", sae.b_dec), ("encode", dense), ("indptr", ip), ("indices", ix),
                        ("values", vs), ("forward", xh), ("sae_encode", sae.encode(x)), ("sae_forward", sae(x))):
            _pack(ops, p + name, t)
        if activation == "jumprelu":
            _pack(ops, p + "threshold", sae.threshold)
    np.savez_compressed(HERE / "ops.npz", **ops)

    # ---- SAE constructor draws (reference.py:25-33) at seed 0
    torch.manual_seed(0)
    s = SAE(24, 64, "jumprelu")
    init = {}
    for name in ("W_enc", "W_dec", "b_enc", "b_dec", "threshold"):
        _pack(init, name, getattr(s, name))
    np.savez_compressed(HERE / "sae_init.npz", **init)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))
    return 0


if __name__ == "__main__":
    sys.exit(main())
