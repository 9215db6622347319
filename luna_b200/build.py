"""Build the engine's shared library in-tree with nvcc for sm_100a.

    python -m luna_b200.build          # -> luna_b200/_lib/libluna_b200.so
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIBDIR, "libluna_b200.so")
SOURCES = ["kernels.cu", "conv_kernels.cu", "tc_gemm.cu", "tc_conv.cu", "engine.cpp", "capi.cpp", "noalloc.cu",
           "shard.cpp", "property.cu", "graph_canon.cpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _needs_rebuild() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(ROOT, "include", "luna_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _needs_rebuild():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    def compile_one(src):
        obj = os.path.join(LIBDIR, src.replace(".", "_") + ".o")
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
               "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
               "-I", os.path.join(ROOT, "include"), "-x", "cu",
               "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB + ".tmp"
    subprocess.run([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart", "-ldl"], check=True)
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
