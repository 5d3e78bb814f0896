"""Generate golden vectors from the REFERENCE's own functions.

The reference ships no tests or golden data for this path, so these fixtures
are produced by its unmodified op_rope / op_attention / op_softmax and half.h
conversions, compiled from its sources by oracle/Makefile (`make ref`) into
oracle/_ref/libkvref.so, on seeded inputs.  Run from the repository root:

    make -C oracle ref && python tests/golden/gen_golden.py

Outputs (committed): tests/golden/ref_cases.npz
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402

NH, NKV, HD, THETA = 12, 2, 128, 1e6
KVD = NKV * HD


def special_floats() -> np.ndarray:
    vals = [0.0, -0.0, 1.0, -1.0, 0.5, 65504.0, 65519.0, 65520.0, 65536.0, -70000.0, 6.1035156e-05,
            6.0e-05, 3.0e-08, 1e-40, -1e-40, np.inf, -np.inf, np.nan, 1.0009766, 1.0004883,
            3.14159265, -2.71828, 1e-5, 123.456, 2.0 ** -14, 2.0 ** -15, 2.0 ** -24, 2.0 ** -25]
    rng = np.random.default_rng(11)
    vals += list(rng.standard_normal(64).astype(np.float32) * 10.0)
    return np.array(vals, np.float32)


def main() -> None:
    R = O.ref()
    out = {}
    # ---- conversions (half.h) ----
    x = special_floats()
    f16 = np.empty(x.shape, np.uint16)
    R.ref_f32_to_f16(x, f16, x.size)
    bf16 = np.empty(x.shape, np.uint16)
    R.ref_f32_to_bf16(x, bf16, x.size)
    out["conv_x"] = x
    out["conv_f16"] = f16
    out["conv_bf16"] = bf16
    allcodes = np.arange(65536, dtype=np.uint16)
    dec16 = np.empty(65536, np.float32)
    R.ref_f16_to_f32(allcodes, dec16, 65536)
    decb = np.empty(65536, np.float32)
    R.ref_bf16_to_f32(allcodes, decb, 65536)
    out["dec_f16_sha256"] = np.frombuffer(hashlib.sha256(dec16.view(np.uint32).tobytes()).digest(), np.uint8)
    out["dec_bf16_sha256"] = np.frombuffer(hashlib.sha256(decb.view(np.uint32).tobytes()).digest(), np.uint8)

    # ---- RoPE at assorted positions (op_rope.cpp) ----
    rng = np.random.default_rng(7)
    positions = np.array([0, 1, 2, 17, 511, 4095, 32767, 131071], np.int32)
    rq = rng.standard_normal((len(positions), NH * HD)).astype(np.float32)
    rk = rng.standard_normal((len(positions), KVD)).astype(np.float32)
    oq, ok = rq.copy(), rk.copy()
    for i, p in enumerate(positions):
        qi, ki = oq[i].copy(), ok[i].copy()
        R.ref_rope(qi, ki, NH, NKV, HD, int(p), THETA)
        oq[i], ok[i] = qi, ki
    out.update(rope_pos=positions, rope_q=rq, rope_k=rk, rope_q_out=oq, rope_k_out=ok)

    # ---- layer steps: RoPE + append + op_attention (qwen2_model.cpp:180-206) ----
    cases = [(0, 1), (1, 1), (15, 1), (16, 1), (37, 1), (300, 1), (11, 5), (0, 7)]
    rng = np.random.default_rng(1234)
    for ci, (pos, seq) in enumerate(cases):
        cap = pos + seq
        k0 = np.zeros((cap, KVD), np.uint16)
        v0 = np.zeros((cap, KVD), np.uint16)
        if pos:
            R.ref_f32_to_f16(rng.standard_normal(pos * KVD).astype(np.float32), k0[:pos].reshape(-1), pos * KVD)
            R.ref_f32_to_f16(rng.standard_normal(pos * KVD).astype(np.float32), v0[:pos].reshape(-1), pos * KVD)
        q = rng.standard_normal((seq, NH * HD)).astype(np.float32)
        k = rng.standard_normal((seq, KVD)).astype(np.float32)
        v = rng.standard_normal((seq, KVD)).astype(np.float32)
        kc, vc = k0.copy(), v0.copy()
        o, qr, kr = O.ref_layer_step(q, k, v, kc, vc, pos)
        assert np.array_equal(kc[:pos], k0[:pos]) and np.array_equal(vc[:pos], v0[:pos])
        pre = f"step{ci}_"
        out.update({pre + "pos": np.int32(pos), pre + "k0": k0[:pos], pre + "v0": v0[:pos],
                    pre + "q": q, pre + "k": k, pre + "v": v, pre + "out": o,
                    pre + "k_app": kc[pos:], pre + "v_app": vc[pos:], pre + "q_rot": qr})
    out["n_steps"] = np.int32(len(cases))
    path = os.path.join(HERE, "ref_cases.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
