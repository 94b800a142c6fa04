"""Builds libtilemaxsim_b200.so in-tree with nvcc for sm_100a (no torch, no JIT cache).

    python -m tilemaxsim_b200.build [--verbose] [--force]

Every ``csrc/*.cu`` is compiled to an object under ``csrc/_build/`` and linked (static cudart)
into ``tilemaxsim_b200/libtilemaxsim_b200.so``. Objects are rebuilt when the source or any header
is newer.
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
BUILD = CSRC / "_build"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libtilemaxsim_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fvisibility=hidden"]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build tilemaxsim_b200")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _compile(nvcc: str, src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)
    return obj


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> Path:
    nvcc = nvcc_path()
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    todo = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        if force or ptxas_info or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            todo.append(src)
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 1))) as ex:
        list(ex.map(lambda s: _compile(nvcc, s, verbose or ptxas_info, extra), todo))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if force or todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills/smem per kernel")
    a = ap.parse_args(argv)
    print(build(verbose=a.verbose, force=a.force, ptxas_info=a.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
