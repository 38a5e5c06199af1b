"""Build the in-tree CUDA library libanchorkv_b200.so for sm_100a with nvcc.

    python dynamic-quantization_b200/build.py [--force]

The library is a plain C-ABI shared object (include/anchorkv_b200.h) linked
against the static CUDA runtime; Python loads it with ctypes.  It is written
next to the package (anchorkv_b200/lib/) so it travels with the source tree.
Never add fast-math flags: the codec is bit-exact only with IEEE division.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OUT = HERE / "anchorkv_b200" / "lib" / "libanchorkv_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build anchorkv_b200")
    return found


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    built = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in sources() + headers() + [Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(ROOT / "include"), "-I", str(CSRC),
           *map(str, sources()), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout, proc.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
