"""Build the sm_100a shared library ``libmarathon_shift.so`` in-tree with nvcc.

The library is the whole native product: the CUDA kernels of the shift path
plus their ``extern "C"`` entry points (declared in ``include/marathon_shift.h``).
It links the CUDA runtime statically and depends on nothing from torch, so a
non-Python host can ``dlopen`` it directly.

    python -m marathon_b200.build          # build if sources are newer
    python -m marathon_b200.build --force  # rebuild
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
SOURCES = [PKG / "csrc" / "shift_kernels.cu"]
HEADERS = [ROOT / "include" / "marathon_shift.h"]
LIB = PKG / "libmarathon_shift.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def command(out: Path = LIB, extra: list[str] | None = None) -> list[str]:
    return [
        nvcc(),
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "-shared",
        "-cudart=static",
        f"-I{ROOT / 'include'}",
        *(extra or []),
        "-o",
        str(out),
        *map(str, SOURCES),
    ]


def stale(out: Path = LIB) -> bool:
    if not out.exists():
        return True
    built = out.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources."""
    if not force and not stale():
        return LIB
    cmd = command()
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    tmp = LIB.with_suffix(".so.tmp")
    cmd[cmd.index("-o") + 1] = str(tmp)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
