"""Build the in-tree CUDA library ``librnn_kernel_b200.so`` for sm_100a.

``python -m rnn_kernel_b200.build`` (or ``build()``) compiles every ``.cu`` in
``csrc/`` with nvcc into one shared library next to this file.  The library
has a plain C ABI (``include/rnn_kernel_b200.h``) and is loaded with ctypes.
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
# RNN_KERNEL_B200_VARIANT=timeline selects an instrumented build of the same
# sources (-DGRU_TIMELINE: the time loops record clock64() at the phases of a
# few steps, read back by gru_timeline_read) in a library of its own; it is
# slower by a few percent and only used for profiling (bench.py --timeline).
VARIANT = os.environ.get("RNN_KERNEL_B200_VARIANT", "")
if VARIANT not in ("", "timeline"):
    raise ValueError(f"RNN_KERNEL_B200_VARIANT must be unset or 'timeline', got {VARIANT!r}")
LIB_NAME = "librnn_kernel_b200_timeline.so" if VARIANT else "librnn_kernel_b200.so"
LIB_PATH = PKG / LIB_NAME
VARIANT_FLAGS = ["-DGRU_TIMELINE"] if VARIANT == "timeline" else []

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build rnn_kernel_b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    mtime = LIB_PATH.stat().st_mtime
    deps = list(CSRC.glob("*")) + list((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, *VARIANT_FLAGS, *(extra or []), "-I", str(ROOT / "include"),
           *map(str, sources()), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None)
