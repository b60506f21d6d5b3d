"""Build the native library ``liblongspark_b200.so`` in-tree with nvcc (sm_100a).

    python -m longspark_b200.build [--force]

Sources: ``longspark_b200/csrc/*.cu``.  Output:
``longspark_b200/_native/liblongspark_b200.so`` (kept out of git, shipped with
the source tree).  The CUDA runtime is linked statically and the driver API is
reached through ``cudaGetDriverEntryPoint``, so the library loads on a machine
without a GPU driver (the symbols can be inspected there; kernels need a B200).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_native"
LIB = OUT_DIR / "liblongspark_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def _nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the native library needs the CUDA 12.9 toolkit")
    return cand


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date():
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + headers() + [Path(__file__)])


def build(force=False, verbose=False, ptxas_info=False):
    """Compile every ``csrc/*.cu`` for sm_100a and link the shared library."""
    if not force and up_to_date():
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    obj_dir = OUT_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src):
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
        if verbose or ptxas_info:
            sys.stderr.write(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
