"""Build libgdn_b200.so in-tree for sm_100a.

    python -m gateddeltanet_b200.build          # or __graft_entry__.build()

nvcc compiles the CUDA kernel and the C-ABI host layer into one shared
library next to this file (gateddeltanet_b200/libgdn_b200.so), linked against
the static CUDA runtime so it does not depend on torch's copy of libcudart.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libgdn_b200.so")
SOURCES = ["gdn_decode.cu", "gdn_recurrence.cu", "gdn_batch.cu", "gdn_score.cu", "gdn_host.cu", "gdn_batch_host.cu",
           "gdn_abi_host.cpp"]
HEADERS = ["gdn_engine.h", "gdn_batch.h", "gdn_synth.h", "gdn_math.h", "exports.map"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the B200 engine cannot be built")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps += [os.path.join(REPO, "include", f) for f in ("gdn_model.h", "gdn_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O3,-ffp-contract=off",
           "-I", os.path.join(REPO, "include"), "-I", CSRC, "-o", tmp,
           *[os.path.join(CSRC, s) for s in SOURCES], "-lpthread",
           "-Xlinker", "--version-script=" + os.path.join(CSRC, "exports.map")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
