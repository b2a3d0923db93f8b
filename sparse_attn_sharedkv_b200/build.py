"""Build ``libsas.so`` (sm_100a CUDA kernels + C ABI) in-tree.

The library is compiled with nvcc straight from ``csrc/`` into
``sparse_attn_sharedkv_b200/_lib/libsas.so``; nothing is installed elsewhere
and no JIT cache is used, so the built file travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIB_DIR, "libsas.so")
INCLUDE = os.path.join(REPO, "include")

SOURCES = ["sas_capi.cu", "sas_fwd.cu", "sas_fwd_pair.cu", "sas_combine.cu", "sas_noalloc.cu", "sas_kvwrite.cu",
           "sas_plan_dev.cu", "sas_plan.cpp", "sas_metadata.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def sources_newer_than(target: str) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(INCLUDE, "sas.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libsas.so if it is missing or older than its sources."""
    if not force and not sources_newer_than(LIB):
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc_path(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-O3", "-shared", "-I" + INCLUDE, "-I" + CSRC,
           *[os.path.join(CSRC, s) for s in SOURCES], "-o", tmp]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
