"""The C++ adapter (include/kvattn_kvcache.hpp) used from a C++ program the
way Qwen2Model uses KVCache: compiled with nvcc against the library, run as
a subprocess.  Host-only bookkeeping on CPU; on the GPU its decode outputs,
cache rows and op_attention shim against the oracle."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT

LIBDIR = os.path.join(ROOT, "rk3588-npu_b200", "lib")
SRC = os.path.join(ROOT, "tests", "cpp", "kvcache_adapter.cpp")


@pytest.fixture(scope="module")
def adapter_bin(tmp_path_factory):
    from conftest import load_pkg
    load_pkg().load()  # builds lib/libkvattn.so if needed
    out = str(tmp_path_factory.mktemp("cpp") / "kvcache_adapter")
    subprocess.run(["nvcc", "-std=c++14", "-O2", f"-I{os.path.join(ROOT, 'include')}", SRC,
                    f"-L{LIBDIR}", "-lkvattn", "-Xlinker", f"-rpath,{LIBDIR}", "-o", out],
                   check=True)
    return out


def test_adapter_host_bookkeeping(adapter_bin):
    r = subprocess.run([adapter_bin, "host"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stderr


@pytest.mark.gpu
def test_adapter_gpu_matches_oracle(adapter_bin, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    path = str(tmp_path / "run.bin")
    r = subprocess.run([adapter_bin, "gpu", path], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stderr
    L, KVD, HID, P, STEPS, CAP = 2, 256, 1536, 40, 5, 64
    T = P + STEPS
    raw = open(path, "rb").read()
    nf = L * 2 * P * KVD + STEPS * L * (HID + 2 * KVD + HID) + 2 * 3 * HID
    f = np.frombuffer(raw[:nf * 4], np.float32)
    u = np.frombuffer(raw[nf * 4:], np.uint16)
    o = 0

    def take(n):
        nonlocal o
        a = f[o:o + n]
        o += n
        return a

    kc = [np.zeros((CAP, KVD), np.uint16) for _ in range(L)]
    vc = [np.zeros((CAP, KVD), np.uint16) for _ in range(L)]
    for li in range(L):
        k = take(P * KVD).reshape(P, KVD).copy()
        v = take(P * KVD).reshape(P, KVD).copy()
        orc.lib().orc_rope_append(np.zeros(P * HID, np.float32), k.reshape(-1), v.reshape(-1),
                                  kc[li].reshape(-1), vc[li].reshape(-1), P, 0, 12, 2, 128, 1e6, 0)
    worst = 0.0
    for s in range(STEPS):
        for li in range(L):
            q = take(HID).reshape(1, HID)
            k = take(KVD).reshape(1, KVD)
            v = take(KVD).reshape(1, KVD)
            out = take(HID)
            ref, _, _ = orc.layer_step(q, k, v, kc[li], vc[li], P + s)
            g = out.reshape(-1, 128).astype(np.float64)
            rr = ref[0].reshape(-1, 128).astype(np.float64)
            worst = max(worst, float((np.abs(g - rr).max(1) / np.abs(rr).max(1)).max()))
    assert worst <= 1e-3, worst
    q3 = take(3 * HID).reshape(3, HID)
    o3 = take(3 * HID).reshape(3, HID)
    kh = u[:T * KVD].reshape(T, KVD)
    vh = u[T * KVD:].reshape(T, KVD)
    assert np.array_equal(kh, kc[0][:T]) and np.array_equal(vh, vc[0][:T])  # gather: bit-exact
    ref3 = orc.attention(q3, kc[0], vc[0], 3, T, 12, 2, 128, T - 3)
    g = o3.reshape(-1, 128).astype(np.float64)
    rr = np.asarray(ref3).reshape(-1, 128).astype(np.float64)
    assert float((np.abs(g - rr).max(1) / np.abs(rr).max(1)).max()) <= 1e-3
