"""Build libpagekv.so in-tree with nvcc for sm_100a (B200).

    python -m pagellm_b200.build          # rebuild if any source is newer than the .so
    python -m pagellm_b200.build --force  # always rebuild

nvcc cross-compiles without a GPU, so this runs on CPU-only machines too. The CUDA runtime
is linked statically: the library needs only the NVIDIA driver at run time.
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
LIB = PKG / "libpagekv.so"

SOURCES = ["pk_api.cu", "pk_kernels.cu", "pk_attn_tc.cu", "pk_attn_wide.cu", "pk_block_manager.cpp", "pk_static.cu",
           "pk_peer.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "-DPK_BUILD", f"-I{INCLUDE}", f"-I{CSRC}",
        *(["-Xptxas", "-v"] if verbose else []),
        "-o", str(tmp), *map(str, sources()),
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
