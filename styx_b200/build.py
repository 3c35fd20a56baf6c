"""Builds libstyx_moe.so (in-tree, next to this file) with nvcc for sm_100a.

    python -m styx_b200.build            # incremental
    python -m styx_b200.build --force    # rebuild everything

Objects go to styx_b200/_build/; the shared library links the CUDA runtime
statically so it carries no dependency on the runtime torch ships.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libstyx_moe.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          f"-I{os.path.join(ROOT, 'include')}", "--expt-relaxed-constexpr"]
# per-source extra flags: the synthetic quantiser must round like the C oracle
EXTRA = {"synth.cu": ["-fmad=false"]}
SOURCES = ["moe_kernels.cu", "moe_fused.cu", "moe_cluster.cu", "batch.cu", "attn.cu", "attn_fused.cu", "attn_cluster.cu", "synth.cu", "api.cu", "residency.cpp", "gguf.cpp"]
HEADERS = ["common.cuh", "qdot.cuh", "kernels.h", "moe_common.cuh", "cluster.cuh", "ep_sync.cuh"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", h)
                                                         for h in ("styx_moe.h", "styx_residency.h", "styx_gguf.h",
                                                                   "styx_attn.h")]
    objs = []
    for src in SOURCES:
        sp = os.path.join(CSRC, src)
        op = os.path.join(OUT_DIR, os.path.splitext(src)[0] + ".o")
        objs.append(op)
        if force or _stale(op, [sp] + hdrs):
            cmd = [nvcc()] + ARCH + COMMON + EXTRA.get(src, []) + ["-c", sp, "-o", op]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
