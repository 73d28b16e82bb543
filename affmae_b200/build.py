"""Build the sm_100a shared library ``affmae_b200/_lib/libaffmae_b200.so``.

The library is plain CUDA C++ with an ``extern "C"`` interface (declared in
``include/affmae_b200.h``); it does not link against torch.  Objects are
compiled in parallel and relinked only when a source or header changed.

Usage: ``python -m affmae_b200.build [--force] [--verbose] [--ptxas-verbose]``.
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
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libaffmae_b200.so"
OBJ_DIR = ROOT / "_build" / "obj"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
] + ARCH


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the affmae_b200 CUDA library cannot be built")
    return cand


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    hdrs = sorted(list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))
    flags = NVCC_FLAGS + list(extra_flags or []) + os.environ.get("AFFB_NVCC_EXTRA", "").split()
    jobs, objs = [], []
    for src in sorted(CSRC.glob("*.cu")):
        obj = OBJ_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            jobs.append((src, [cc, *flags, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, flush=True)
        return src

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            for f in [ex.submit(run, j) for j in jobs]:
                f.result()
    if force or jobs or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    lib = build(force=a.force or a.ptxas_verbose, verbose=a.verbose or a.ptxas_verbose,
                extra_flags=extra)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
