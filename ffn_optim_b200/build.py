"""Builds the in-tree CUDA library ``ffn_optim_b200/_lib/libffn_b200.so`` for sm_100a.

The library is the C-ABI declared in ``include/ffn_b200.h``; the Python host layer loads it
with ctypes.  It is built with nvcc directly (no torch extension machinery), so the result
is a plain shared object that any host language can bind.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "_lib"
LIB = LIBDIR / "libffn_b200.so"
SOURCES = [CSRC / "ffn_capi.cu", CSRC / "ffn_noalloc.cu", CSRC / "ffn_placement.cu", CSRC / "ffn_quant.cu"]
HEADERS = [CSRC / "ffn_kernel.cuh", CSRC / "ffn_rowblock.cuh", CSRC / "ffn_hslice.cuh", ROOT / "include" / "ffn_b200.h"]
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the ffn_b200 CUDA library cannot be built")


def source_digest() -> str:
    h = hashlib.sha256()
    for path in SOURCES + HEADERS:
        h.update(path.read_bytes())
    return h.hexdigest()


def stamp_path() -> Path:
    return LIBDIR / "libffn_b200.sha256"


def up_to_date() -> bool:
    return LIB.exists() and stamp_path().exists() and stamp_path().read_text().strip() == source_digest()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if its sources changed; returns the library path."""
    if not force and up_to_date():
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-Xptxas", "-v" if verbose else "-O3",
           "-I", str(ROOT / "include"), "-o", str(tmp)] + [str(s) for s in SOURCES]
    # -fvisibility=hidden keeps the template kernels private; the extern "C" API is exported
    # through the FFN_B200_EXPORT default-visibility attribute in the header.
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    tmp.replace(LIB)
    stamp_path().write_text(source_digest() + "\n")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
