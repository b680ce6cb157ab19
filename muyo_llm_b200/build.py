"""In-tree build of libmuyo_cuda.so (and the oracle, when asked) for sm_100a only.

nvcc cross-compiles without a GPU, so this runs in the CPU container as well as on a GPU box. The
library goes to muyo_llm_b200/_lib/libmuyo_cuda.so; objects to muyo_llm_b200/_build/.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libmuyo_cuda.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["runtime.cu", "ops.cu", "decode.cu", "sampler.cu"]
CPP_SOURCES = ["gguf_loader.cpp"]
HOST = os.path.join(PKG, "host")
HOST_SOURCES = ["checks.cpp", "forward.cpp", "main.cpp", "gguf_meta.cpp", "tokenizer.cpp"]
HOST_BIN = os.path.join(LIBDIR, "muyo-llm")  # the C++ command line over the library
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, "muyo_cuda.h"), os.path.abspath(__file__)]


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if _newer(obj, [src] + _headers()):
        cmd = [nvcc()] + ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", INCLUDE,
                                 "-c", src, "-o", obj] + extra
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES + CPP_SOURCES]
    with cf.ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        objs = list(ex.map(lambda s: _compile(s, ["-Xptxas", "-v"] if verbose and s.endswith(".cu") else []), srcs))
    if _newer(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        subprocess.run(cmd, check=True)
    build_host()
    return LIB


def build_host() -> str:
    """The muyo-llm command line (host/): g++ against include/ and libmuyo_cuda.so (found beside it
    through $ORIGIN), with the CUDA runtime for its own device buffers."""
    srcs = [os.path.join(HOST, f) for f in HOST_SOURCES]
    deps = srcs + [os.path.join(HOST, f) for f in ("host.h", "gguf_meta.h", "tokenizer.h", "unicode_classes.inc")]
    deps += [os.path.join(INCLUDE, "muyo_cuda.h"), LIB]
    if _newer(HOST_BIN, deps):
        cxx = shutil.which("g++") or "g++"
        cmd = [cxx, "-O2", "-std=c++17", "-Wall", "-I", INCLUDE, "-I", HOST, "-I", os.path.join(CUDA_HOME, "include")]
        cmd += srcs + ["-o", HOST_BIN, "-L", LIBDIR, "-lmuyo_cuda", "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart",
                       "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + os.path.join(CUDA_HOME, "lib64")]
        subprocess.run(cmd, check=True)
    return HOST_BIN


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
