"""Build libsaeflow_b200.so (sm_100a) in-tree with nvcc.

    python -m saeflow_b200.build [--force] [-v]

Each csrc/*.cu compiles to an object under saeflow_b200/_build/ (in parallel, skipped
when newer than its sources), then one shared library is linked into
saeflow_b200/_lib/. The CUDA runtime is linked statically; the driver API
(cuTensorMapEncodeTiled) is reached through cudaGetDriverEntryPoint, so no libcuda
is needed at link time and the library builds on machines without a GPU.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libsaeflow_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set $NVCC")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every kernel source for sm_100a and link the shared library. Returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    extra += os.environ.get("SAEFLOW_B200_NVCC_FLAGS", "").split()  # e.g. -DSF_RASTER_GROUP_MB=32

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if force or ptxas_verbose or _stale(obj, [src, *headers]):
            cmd = [cc, *ARCH, *FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
            if (verbose or ptxas_verbose) and (r.stdout or r.stderr):
                print(r.stdout + r.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))

    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print registers / spills per kernel")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas))
    return 0


if __name__ == "__main__":
    sys.exit(main())
