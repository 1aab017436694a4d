"""Build recipe for libljx.so: nvcc, sm_100a only, in-tree next to this file.

    python -c "import importlib.util as u, sys; ..."   # or __graft_entry__.build()

The library holds every kernel (csrc/*.cu) and the bundle loader (csrc/bundle.cpp) behind the
C ABI of include/ljx.h, include/ljx_neigh.h, include/ljx_pair.h and include/ljx_md.h.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libljx.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-Wall", "-shared"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in deps)


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the ljx library is compiled for sm_100a with nvcc")


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile libljx.so for sm_100a unless it is newer than every source."""
    if not force and not _stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(tmp),
           *[str(s) for s in sources()]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + proc.stdout + proc.stderr)
    if verbose:
        print(proc.stdout + proc.stderr)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build_library(force=True, verbose=True))
