"""Build the in-tree native libraries of flashcart_b200.

* ``flashcart_b200/_lib/libflashcart_b200.so``: the product, every kernel compiled
  with ``nvcc -gencode arch=compute_100a,code=sm_100a`` (static cudart, no torch);
* ``flashcart_b200/_lib/libflashcart_b200_emu.so``: the same sources compiled by the
  host C++ compiler with ``-DFC_HOST_EMU`` so that the CPU test suite can execute the
  generated per-thread arithmetic and the C ABI without a GPU. Only tests load it.

Objects go to ``_build/`` at the repository root and are rebuilt when the source or
any header is newer. Usage: ``python -m flashcart_b200.build_ext [--no-emu] [-j N]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys
from typing import List

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "_lib")
BUILD_DIR = os.path.join(ROOT, "_build")
CUDA_LIB = os.path.join(LIB_DIR, "libflashcart_b200.so")
EMU_LIB = os.path.join(LIB_DIR, "libflashcart_b200_emu.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-DNDEBUG",
]
EMU_FLAGS = ["-x", "c++", "-std=c++17", "-DFC_HOST_EMU", "-O1", "-fPIC"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> List[str]:
    gen = sorted(glob.glob(os.path.join(CSRC, "gen", "*.cu")))
    own = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    return own + gen


def _headers() -> List[str]:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "gen", "*.cuh"))
    hs += glob.glob(os.path.join(CSRC, "gen", "*.inc")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _stale(obj: str, src: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _obj_name(src: str, tag: str) -> str:
    rel = os.path.relpath(src, CSRC).replace(os.sep, "__")
    return os.path.join(BUILD_DIR, tag, rel[:-3] + ".o")


def _run(cmd: List[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"command failed ({res.returncode}): {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def generate() -> None:
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from flashcart_b200.codegen import emit

    emit.write_all()


def _compile_all(tag: str, compile_cmd, jobs: int) -> List[str]:
    os.makedirs(os.path.join(BUILD_DIR, tag), exist_ok=True)
    newest = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    objs, todo = [], []
    for src in sources():
        obj = _obj_name(src, tag)
        objs.append(obj)
        if _stale(obj, src, newest):
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = [ex.submit(_run, compile_cmd(src, obj)) for src, obj in todo]
            for f in cf.as_completed(futs):
                f.result()
    return objs


def build_cuda(jobs: int = 8) -> str:
    nvcc = _nvcc()
    objs = _compile_all("cuda", lambda s, o: [nvcc, *NVCC_FLAGS, "-c", s, "-o", o], jobs)
    os.makedirs(LIB_DIR, exist_ok=True)
    if not os.path.exists(CUDA_LIB) or max(os.path.getmtime(o) for o in objs) > os.path.getmtime(CUDA_LIB):
        tmp = CUDA_LIB + ".tmp"
        _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
              "-o", tmp, *objs])
        os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_emu(jobs: int = 8) -> str:
    cxx = os.environ.get("CXX", "g++")
    objs = _compile_all("emu", lambda s, o: [cxx, *EMU_FLAGS, "-c", s, "-o", o], jobs)
    os.makedirs(LIB_DIR, exist_ok=True)
    if not os.path.exists(EMU_LIB) or max(os.path.getmtime(o) for o in objs) > os.path.getmtime(EMU_LIB):
        tmp = EMU_LIB + ".tmp"
        _run([cxx, "-shared", "-o", tmp, *objs])
        os.replace(tmp, EMU_LIB)
    return EMU_LIB


def build(cuda: bool = True, emu: bool = True, jobs: int = 0) -> None:
    jobs = jobs or max(1, os.cpu_count() or 1)
    generate()
    if emu:
        build_emu(jobs)
    if cuda:
        build_cuda(jobs)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--no-emu", action="store_true")
    ap.add_argument("--no-cuda", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    a = ap.parse_args()
    build(cuda=not a.no_cuda, emu=not a.no_emu, jobs=a.j)
    print("built:", CUDA_LIB if not a.no_cuda else "", EMU_LIB if not a.no_emu else "")


if __name__ == "__main__":
    main()
