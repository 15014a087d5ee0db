"""Build the CUDA library of this package in-tree with nvcc (sm_100a only).

``python -m minigpt_train_infra_b200._build`` compiles ``csrc/*.cu`` into
``lib/libb200_optim.so``.  The library is a plain C-ABI shared object (``include/b200_optim.h``)
with the CUDA runtime linked statically, so it loads next to PyTorch's own runtime and needs no
Python extension machinery.  Flags: no fast-math, IEEE division and square root, denormals kept
(the step must reproduce the CPU reference's fp32 rounding).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = PKG / "lib"
LIB_NAME = "libb200_optim.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-ftz=false",
              "-prec-div=true", "-prec-sqrt=true", "-cudart", "static"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the library")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def lib_path() -> Path:
    return LIB_DIR / LIB_NAME


def needs_build() -> bool:
    out = lib_path()
    if not out.exists():
        return True
    mtime = out.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile (if stale) and return the path of the shared library."""
    out = lib_path()
    if not force and not needs_build():
        return out
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc_path(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-shared",
           "-o", str(tmp), *map(str, sources())]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
