"""Builds and runs the microbenchmarks in this directory (nvcc, sm_100a; needs a B200).

    python -m tilemaxsim_b200.microbench.run tmem_read    # tcgen05.ld bandwidth per SM
    python -m tilemaxsim_b200.microbench.run tmem_store   # tcgen05.st bandwidth, alone / beside loads
    python -m tilemaxsim_b200.microbench.run handoff      # cycles per mbarrier pipeline hand-off
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

from ..build import ARCH, nvcc_path

HERE = Path(__file__).resolve().parent


def main(argv: list[str]) -> int:
    name = argv[0] if argv else "tmem_read"
    out = HERE.parent / "csrc" / "_build" / name
    out.parent.mkdir(exist_ok=True)
    subprocess.run([nvcc_path(), *ARCH, "-O3", "-std=c++17", str(HERE / f"{name}.cu"), "-o", str(out)],
                   check=True)
    return subprocess.run([str(out)]).returncode


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
