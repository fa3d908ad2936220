"""Compile the CUDA library (csrc/lib.cu) for sm_100a into ``libbsgemm.so``.

    python <package dir>/build.py            # writes <package dir>/libbsgemm.so

nvcc cross-compiles without a GPU.  No ``--use_fast_math``: the quantisers
rely on IEEE division and RNE conversions to match the reference bit for bit.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc", "lib.cu")
OUT = os.path.join(HERE, "libbsgemm.so")
DEPS = [os.path.join(HERE, "csrc", f) for f in ("lib.cu", "common.cuh", "quant.cu", "dequant.cu", "hc.cu", "attn.cu", "gemm.cu", "gemm_pair.cu", "capi.cu", "moe.cu", "peer.cu", "moe_fused.cu", "gate.cu", "noalloc.cu")]
DEPS.append(os.path.join(os.path.dirname(HERE), "include", "bsgemm.h"))


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(d) <= t for d in DEPS if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
           "-Xcompiler", "-fPIC", "-shared", "-o", OUT + ".tmp", SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
