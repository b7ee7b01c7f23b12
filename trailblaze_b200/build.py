"""Build libtb_cuda_sm100.so in-tree with nvcc for sm_100a.

The shared library is the product: the C ABI of include/tb_gguf_dequant.h over
hand-written sm_100a kernels.  It is built in place (next to this file) so it
travels with the repository snapshot and is the file the tests and the bench
load.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtb_cuda_sm100.so")
BUILD_DIR = os.path.join(HERE, "_build")

SOURCES = ["tb_matvec.cu", "tb_dequant.cu", "tb_abi.cu", "tb_decode.cu", "tb_qgemm.cu", "tb_sample.cu",
           "tb_loader.cu", "tb_prefill.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-I", os.path.join(REPO, "include"),
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; cannot build libtb_cuda_sm100.so")
    return cand


def _deps() -> list[str]:
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files.append(os.path.join(REPO, "include", "tb_gguf_dequant.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu of csrc/ for sm_100a and link libtb_cuda_sm100.so."""
    if not force and up_to_date():
        return LIB
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)

    def compile_one(src: str) -> str:
        obj = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
        cmd = [nvcc, *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs,
           "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
