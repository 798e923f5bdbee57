"""Builds libsemantica_b200.so in-tree for sm_100a.

CUDA sources are compiled with --fmad=false (the element-wise kernels restate
the reference's unfused float32 arithmetic bit for bit) and without fast-math.
Usage: python go-semantica_b200/build.py [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsemantica_b200.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xcompiler", "-fPIC", "-ccbin", CXX,
                     "-Xptxas", "-warn-spills"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function", f"-I{CUDA_HOME}/include"]

CU_SOURCES = ["model_kernels.cu", "gemm_q8.cu", "gemm_split.cu", "gemm_dp4a.cu", "attention.cu", "attention_short.cu",
              "brute_kernels.cu", "gemm_noalloc.cu", "search_tc.cu"]
CPP_SOURCES = ["host/gguf.cpp", "host/model.cpp", "host/brute.cpp", "host/group.cpp"]
HEADERS = ["common.cuh", "sm100.cuh", "tmap.h", "kernels.h", "host/internal.h", "host/gguf.h"]


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    deps = [src] + [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "semantica_b200.h")]
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool) -> str:
    path = os.path.join(CSRC, src)
    obj = os.path.join(OUT_DIR, src.replace("/", "_") + ".o")
    if force or _stale(obj, path):
        if src.endswith(".cu"):
            cmd = [NVCC] + NVCC_FLAGS + ["-c", path, "-o", obj]
        else:
            cmd = [CXX] + CXX_FLAGS + ["-c", path, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False) -> str:
    if not os.path.exists(NVCC):
        raise RuntimeError(f"nvcc not found at {NVCC}")
    os.makedirs(OUT_DIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), CU_SOURCES + CPP_SOURCES))
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC] + ARCH + ["-shared", "-ccbin", CXX, "-o", tmp] + objs + ["-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        shutil.move(tmp, LIB)
    return LIB


TEST_SRC = os.path.join(ROOT, "tests", "kernels", "test_kernels.cu")
TEST_LIB = os.path.join(ROOT, "tests", "_build", "libsemantica_testkernels.so")


def build_test_kernels(force: bool = False) -> str:
    """The tests' kernel library (tests/kernels/test_kernels.cu): the product's
    device helpers applied element by element, and a bounded pipeline wait
    that nothing completes. Test infrastructure; the product never links it."""
    deps = [TEST_SRC] + [os.path.join(CSRC, h) for h in HEADERS]
    if force or not os.path.exists(TEST_LIB) or any(os.path.getmtime(d) > os.path.getmtime(TEST_LIB) for d in deps):
        os.makedirs(os.path.dirname(TEST_LIB), exist_ok=True)
        cmd = [NVCC] + NVCC_FLAGS + ["-shared", TEST_SRC, "-o", TEST_LIB]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return TEST_LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
    print(build_test_kernels(force="--force" in sys.argv))
