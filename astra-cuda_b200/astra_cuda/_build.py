"""Builds the CUDA library ``_lib/libastra_market.so`` for sm_100a.

``python -m astra_cuda._build`` (or ``__graft_entry__.build()``) compiles
``csrc/am_engine.cu`` with nvcc into the package, in-tree, with the CUDA
runtime linked statically.  A digest of the sources is stored beside the
library so an up-to-date build is not repeated.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)                 # astra-cuda_b200/
REPO_DIR = os.path.dirname(ROOT_DIR)
CSRC_DIR = os.path.join(ROOT_DIR, "csrc")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libastra_market.so")
HEADERS = ("astra_market.h", "astra_trading.h")  # the C ABI
DIGEST_PATH = LIB_PATH + ".digest"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              "-cudart", "static", "-Xptxas", "-warn-spills"]


def _sources():
    srcs = sorted(os.path.join(CSRC_DIR, f) for f in os.listdir(CSRC_DIR)
                  if f.endswith((".cu", ".cuh", ".h")))
    srcs += [os.path.join(INCLUDE_DIR, h) for h in HEADERS]
    return srcs


def source_digest() -> str:
    h = hashlib.sha256()
    for p in _sources():
        h.update(os.path.basename(p).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()


def is_current() -> bool:
    if not os.path.exists(LIB_PATH) or not os.path.exists(DIGEST_PATH):
        return False
    with open(DIGEST_PATH) as f:
        return f.read().strip() == source_digest()


def nvcc() -> str | None:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    p = "/usr/local/cuda/bin/nvcc"
    return p if os.path.exists(p) else None


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if the sources changed; return its path."""
    if not force and is_current():
        return LIB_PATH
    exe = nvcc()
    if exe is None:
        raise RuntimeError("nvcc not found: cannot build the astra_cuda CUDA library")
    os.makedirs(LIB_DIR, exist_ok=True)
    import fcntl
    with open(os.path.join(LIB_DIR, ".build.lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)  # one builder when several ranks start together
        if not force and is_current():
            return LIB_PATH
        return _compile(exe, verbose)


def _compile(exe: str, verbose: bool) -> str:
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    cmd = [exe, *NVCC_FLAGS, *ARCH_FLAGS, "-I", INCLUDE_DIR, "-I", CSRC_DIR,
           "-o", tmp, os.path.join(CSRC_DIR, "am_engine.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed building libastra_market.so:\n" + res.stderr[-4000:])
    os.replace(tmp, LIB_PATH)
    with open(DIGEST_PATH, "w") as f:
        f.write(source_digest())
    return LIB_PATH


# ---- the C++ host side (cpp/vec_market.*): VecMarket for C++ callers ----

CPP_DIR = os.path.join(ROOT_DIR, "cpp")
CPP_LIB_PATH = os.path.join(LIB_DIR, "libastra_vec_market.so")


def torch_paths():
    """Include and library directories of the installed torch (C++ API, c10/cuda)."""
    import torch
    base = os.path.dirname(torch.__file__)
    inc = [os.path.join(base, "include"), os.path.join(base, "include", "torch", "csrc", "api",
                                                        "include"), "/usr/local/cuda/include"]
    return inc, os.path.join(base, "lib")


def build_cpp(verbose: bool = False) -> str:
    """Compile the C++ host library (VecMarket, FillBatch, BBOBatch of market.h,
    and the player-trading step, over the C ABI) with g++, linked against the
    CUDA library and torch."""
    lib = build()
    units = [os.path.join(CPP_DIR, f) for f in ("vec_market.cpp", "high_low_trading_step.cpp")]
    srcs = units + [os.path.join(CPP_DIR, f) for f in ("vec_market.h", "high_low_trading_step.h")]
    stamp = CPP_LIB_PATH + ".digest"
    h = hashlib.sha256()
    for p in srcs + [os.path.join(INCLUDE_DIR, x) for x in HEADERS]:
        with open(p, "rb") as f:
            h.update(f.read())
    digest = h.hexdigest()
    if os.path.exists(CPP_LIB_PATH) and os.path.exists(stamp):
        with open(stamp) as f:
            if f.read().strip() == digest:
                return CPP_LIB_PATH
    inc, tlib = torch_paths()
    tmp = CPP_LIB_PATH + f".tmp{os.getpid()}"
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-I", INCLUDE_DIR, "-I", CPP_DIR]
    for d in inc:
        cmd += ["-isystem", d]
    # --no-as-needed keeps libtorch_cuda loaded: nothing references its symbols
    # directly, but it registers torch's CUDA backend
    cmd += [*units, "-o", tmp, "-L", LIB_DIR, "-lastra_market",
            "-L", tlib, "-Wl,--no-as-needed", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10",
            "-lc10_cuda", "-Wl,--as-needed", f"-Wl,-rpath,{LIB_DIR}", f"-Wl,-rpath,{tlib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError("g++ failed building libastra_vec_market.so:\n" + res.stderr[-4000:])
    os.replace(tmp, CPP_LIB_PATH)
    with open(stamp, "w") as f:
        f.write(digest)
    del lib
    return CPP_LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    if "--cpp" in sys.argv:
        print(build_cpp(verbose=True))
