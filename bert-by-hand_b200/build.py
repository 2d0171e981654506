"""Build libbbh.so in-tree with nvcc for sm_100a (python bert-by-hand_b200/build.py).

Each .cu in csrc/ is compiled to an object (in parallel), then linked into a shared
library with the CUDA runtime linked statically, so the library loads on a machine
without a GPU driver (its calls then fail with BBH_ERR_CUDA / BBH_ERR_UNSUPPORTED).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libbbh.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + os.path.join(HERE, "..", "include")]
SOURCES = ["gemm_tc.cu", "gemm_pair.cu", "gemm_ln.cu", "attention_tc.cu", "rowwise.cu", "capi.cu", "corpus.cu", "similarity.cu", "blob.cu", "tokenizer.cu"]


def _needs(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(HERE, "..", "include", "bbh.h"))
    return hs


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(OBJ, os.path.splitext(src)[0] + ".o")
    deps = [os.path.join(CSRC, src)] + _headers()
    if _needs(obj, deps):
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), SOURCES))
    if _needs(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


EXAMPLE_SRC = os.path.join(HERE, "examples", "bert_embed_main.cpp")
EXAMPLE_BIN = os.path.join(OBJ, "bert_embed_main")


def build_example() -> str:
    """The C++ drop-in example, linked against libbbh.so (rpath = its folder)."""
    build()
    deps = [EXAMPLE_SRC, LIB, os.path.join(HERE, "..", "include", "bert_by_hand.hpp")]
    if _needs(EXAMPLE_BIN, deps):
        cmd = [NVCC, "-std=c++17", "-O2", "-I" + os.path.join(HERE, "..", "include"), EXAMPLE_SRC, "-o", EXAMPLE_BIN,
               "-L" + HERE, "-lbbh", "-Xlinker", "-rpath=" + HERE, "-Xlinker", "-rpath=$ORIGIN/.."]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"example build failed:\n{r.stdout}\n{r.stderr}")
    return EXAMPLE_BIN


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
    print(build_example())
