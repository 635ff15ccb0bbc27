"""Build libsluice_sm100.so (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: ``python -m sluice_b200.csrc.build [--force] [--verbose]``. Objects go to
``_build/`` at the repository root; the library lands next to the package
(``sluice_b200/libsluice_sm100.so``). Rebuilds only when a source or header is
newer than the library.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libsluice_sm100.so")
BUILD = os.path.join(ROOT, "_build")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
              "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(HERE, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    flags = NVCC_FLAGS + GENCODE + (extra or [])

    def compile_one(src: str) -> str:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        cmd = [cc, *flags, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB + ".tmp"
    cmd = [cc, *GENCODE, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem use")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_v else None
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=extra))
    return 0


if __name__ == "__main__":
    sys.exit(main())
