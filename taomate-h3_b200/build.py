"""Build libh3sa.so (the C-ABI library) from csrc/ for sm_100a with nvcc.

Objects go to taomate-h3_b200/_build/, the shared library next to the Python package
(taomate-h3_b200/h3sa/libh3sa.so) so it travels with the source tree. Rebuilds only the
translation units whose sources or headers changed.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
INCLUDE = HERE.parent / "include"
LIB = HERE / "h3sa" / "libh3sa.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    headers = _headers()
    objects = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if not force and not _stale(obj, [src, *headers]):
            continue
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd[1:1] = ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or _stale(LIB, objects):
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               *[str(o) for o in objects], "-o", str(LIB)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(args.verbose, args.ptxas_info, args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
