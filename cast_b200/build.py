"""Builds ``cast_b200/libcast_b200.so`` (sm_100a only) with nvcc.

Usage: ``python -m cast_b200.build [--verbose]``.  The library is built in the
source tree so that it travels with the repository snapshot; it links only the
CUDA runtime (the TMA descriptor encoder is fetched through
``cudaGetDriverEntryPoint``, so no libcuda link is needed).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc", "cast_b200.cu")
OUT = os.path.join(HERE, "libcast_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    d = os.path.join(HERE, "csrc")
    return [os.path.join(d, f) for f in sorted(os.listdir(d))] + [
        os.path.join(os.path.dirname(HERE), "include", "cast_b200.h")
    ]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
        "-o", OUT + ".tmp", SRC, "-lcudart",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True)
    print(OUT)
