"""Build libkvattn.so in-tree with nvcc for sm_100a.

Usage: python rk3588-npu_b200/build.py [--force]

Sources: csrc/*.cu (kernels + host runtime + C ABI) and csrc/*.cpp (host-only
C ABI parts, compiled through nvcc's host compiler).  Output:
lib/libkvattn.so next to this file, and bin/qwen2_chat (frontend/qwen2_chat.cpp,
the line-protocol front end of the device model, linked against it).  cudart is linked statically, so the
library needs only the CUDA driver at run time; streams and device pointers
from any other runtime in the process (e.g. torch's) are interchangeable
with it because they are driver objects.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libkvattn.so")
CHAT_SRC = os.path.join(HERE, "frontend", "qwen2_chat.cpp")
CHAT = os.path.join(HERE, "bin", "qwen2_chat")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h")) + [os.path.abspath(__file__)]


def up_to_date() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(CHAT):
        return False
    t = min(os.path.getmtime(LIB), os.path.getmtime(CHAT))
    return all(os.path.getmtime(d) <= t for d in _deps() + [CHAT_SRC])


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, f"-I{INCLUDE}", "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs, "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    os.makedirs(os.path.dirname(CHAT), exist_ok=True)
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", f"-I{INCLUDE}", CHAT_SRC, "-o", CHAT + ".tmp",
           f"-L{LIBDIR}", "-lkvattn", "-Wl,-rpath,$ORIGIN/../lib"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(CHAT + ".tmp", CHAT)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
