"""Build the in-tree engine library ``scmp_vit_b200/libscmp_b200.so``.

nvcc compiles every ``csrc/*.cu`` for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``) into one shared object with a plain C ABI
(``include/scmp_b200.h``).  No torch headers are involved; Python binds the
library with ctypes (``scmp_vit_b200/_lib.py``).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libscmp_b200.so"
ROOT = PKG.parent

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
    # IEEE float everywhere: the rescale must match the oracle bit for bit.
    "-prec-div=true", "-prec-sqrt=true", "-fmad=false", "-ftz=false",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; cannot build the sm_100a engine")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "scmp_b200.h"]
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"),
           *[str(s) for s in sources()], "-o", str(LIB) + ".tmp"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
