"""Pin the oracle: the C restatement (oracle/kvattn_oracle.c) must reproduce
the reference's golden vectors bit-for-bit, and match the reference's own
compiled functions live where they were built."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

NH, NKV, HD, THETA = 12, 2, 128, 1e6
KVD = NKV * HD


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint16)


def test_conversions_match_golden(orc, golden):
    x = golden["conv_x"]
    assert np.array_equal(orc.encode(x, orc.F16), golden["conv_f16"])
    assert np.array_equal(orc.encode(x, orc.BF16), golden["conv_bf16"])
    codes = np.arange(65536, dtype=np.uint16)
    for dt, key in ((orc.F16, "dec_f16_sha256"), (orc.BF16, "dec_bf16_sha256")):
        dig = hashlib.sha256(orc.decode(codes, dt).view(np.uint32).tobytes()).digest()
        assert dig == golden[key].tobytes()


def test_f16_encoder_truncates_and_flushes(orc):
    # half.h:24-32: no rounding, exp<=0 -> signed zero, exp>=31 (and NaN) -> inf.
    f = orc.lib().orc_f32_to_f16
    assert f(1.0009765625) == 0x3C01          # exactly representable
    assert f(1.00146484375) == 0x3C01         # 1.5 ulp: truncated, not rounded up
    assert f(6.0e-05) == 0x0000               # below 2^-14: flushed
    assert f(-6.0e-05) == 0x8000
    assert f(65536.0) == 0x7C00
    assert f(float("nan")) == 0x7C00
    assert f(float("-inf")) == 0xFC00


def test_rope_matches_golden(orc, golden):
    L = orc.lib()
    for i, p in enumerate(golden["rope_pos"]):
        q = golden["rope_q"][i].copy()
        k = golden["rope_k"][i].copy()
        L.orc_rope(q, k, NH, NKV, HD, int(p), THETA)
        assert np.array_equal(bits(q), bits(golden["rope_q_out"][i]))
        assert np.array_equal(bits(k), bits(golden["rope_k_out"][i]))


@pytest.mark.parametrize("ci", range(8))
def test_layer_step_matches_golden(orc, golden, ci):
    g = {k[len(f"step{ci}_"):]: v for k, v in golden.items() if k.startswith(f"step{ci}_")}
    pos = int(g["pos"])
    seq = g["q"].shape[0]
    kc = np.zeros((pos + seq, KVD), np.uint16)
    vc = np.zeros((pos + seq, KVD), np.uint16)
    kc[:pos], vc[:pos] = g["k0"], g["v0"]
    out, q_rot, _ = orc.layer_step(g["q"], g["k"], g["v"], kc, vc, pos)
    assert np.array_equal(kc[pos:], g["k_app"])
    assert np.array_equal(vc[pos:], g["v_app"])
    assert np.array_equal(bits(q_rot), bits(g["q_rot"]))
    assert np.array_equal(bits(out), bits(g["out"]))


def test_rope_table_matches_rotation(orc):
    # The table the product builds uses the same three libm calls; spot-check
    # that rotating with table values equals the oracle's rotation.
    c, s = orc.rope_table(THETA, HD, 4090, 8)
    rng = np.random.default_rng(3)
    k = rng.standard_normal(KVD).astype(np.float32)
    for j in range(8):
        q = np.zeros(NH * HD, np.float32)
        kk = k.copy()
        orc.lib().orc_rope(q, kk, NH, NKV, HD, 4090 + j, THETA)
        a, b = k[:64], k[64:128]
        with np.errstate(all="ignore"):
            r0 = (a * c[j]).astype(np.float32) - (b * s[j]).astype(np.float32)
            r1 = (a * s[j]).astype(np.float32) + (b * c[j]).astype(np.float32)
        assert np.array_equal(bits(r0.astype(np.float32)), bits(kk[:64]))
        assert np.array_equal(bits(r1.astype(np.float32)), bits(kk[64:128]))


def test_lse_combine_equals_unsplit_attention(orc):
    rng = np.random.default_rng(5)
    T = 70
    kc = orc.encode(rng.standard_normal((T, KVD)).astype(np.float32))
    vc = orc.encode(rng.standard_normal((T, KVD)).astype(np.float32))
    q = rng.standard_normal((1, NH * HD)).astype(np.float32)
    full = orc.attention(q, kc, vc, 1, T, NH, NKV, HD, T - 1)
    # Split positions [0,30) and [30,70): compute each part's (m, l, o) by hand.
    ms, ls, os_ = [], [], []
    kd = orc.decode(kc)
    vd = orc.decode(vc)
    for lo, hi in ((0, 30), (30, 70)):
        m = np.empty(NH, np.float32)
        l = np.empty(NH, np.float32)
        o = np.empty((NH, HD), np.float32)
        for h in range(NH):
            kh = h // (NH // NKV)
            sc = (kd[lo:hi, kh * HD:(kh + 1) * HD] @ q[0, h * HD:(h + 1) * HD]) / np.sqrt(HD)
            m[h] = sc.max()
            w = np.exp(sc - m[h])
            l[h] = w.sum()
            o[h] = (w @ vd[lo:hi, kh * HD:(kh + 1) * HD]) / l[h]
        ms.append(m)
        ls.append(l)
        os_.append(o)
    comb = orc.lse_combine(np.stack(ms), np.stack(ls), np.stack(os_))
    np.testing.assert_allclose(comb.reshape(-1), full.reshape(-1), rtol=0, atol=1e-5)


@pytest.mark.skipif("not __import__('oracle').have_ref()")
def test_restatement_equals_reference_live(orc):
    rng = np.random.default_rng(99)
    for pos, seq in ((0, 1), (63, 1), (64, 3), (200, 1)):
        cap = pos + seq
        kc = orc.encode(rng.standard_normal((cap, KVD)).astype(np.float32))
        vc = orc.encode(rng.standard_normal((cap, KVD)).astype(np.float32))
        kc2, vc2 = kc.copy(), vc.copy()
        q = rng.standard_normal((seq, NH * HD)).astype(np.float32)
        k = (rng.standard_normal((seq, KVD)) * 30000).astype(np.float32)  # some encode to inf
        v = rng.standard_normal((seq, KVD)).astype(np.float32)
        o1, q1, _ = orc.layer_step(q, k, v, kc, vc, pos)
        o2, q2, _ = orc.ref_layer_step(q, k, v, kc2, vc2, pos)
        assert np.array_equal(kc, kc2) and np.array_equal(vc, vc2)
        assert np.array_equal(bits(q1), bits(q2))
        assert np.array_equal(bits(o1), bits(o2))


def test_int8_quantiser_properties(orc):
    """orc_quantize_i8: scale = max|x| / 127, codes round-half-away(x / scale)
    in [-127, 127], every element within half a step of its dequantised
    value; an all-zero row has scale 0 and zero codes."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((64, 128)).astype(np.float32) * rng.uniform(0.01, 100, (64, 1)).astype(np.float32)
    x[3] = 0.0
    x[5, 7] = -x[5].__abs__().max() * 2  # a negative extreme
    q, s = orc.quantize_i8(x)
    assert q.dtype == np.int8 and s.shape == (64,)
    amax = np.abs(x).max(axis=1)
    assert np.array_equal(s, (amax / np.float32(127)).astype(np.float32))
    assert s[3] == 0 and not q[3].any()
    nz = s > 0
    assert (np.abs(q[nz]).max(axis=1) == 127).all()
    err = np.abs(q.astype(np.float32) * s[:, None] - x)
    assert (err <= s[:, None] * 0.5 * (1 + 1e-6) + 1e-30).all()
    # exact halves round away from zero: 2.5 steps -> 3, -2.5 -> -3
    row = np.zeros((1, 128), np.float32)
    row[0, 0], row[0, 1], row[0, 2] = 127.0, 2.5, -2.5
    q1, s1 = orc.quantize_i8(row)
    assert s1[0] == 1.0 and q1[0, 0] == 127 and q1[0, 1] == 3 and q1[0, 2] == -3


def test_int8_attention_close_to_fp32(orc):
    """The INT8 layer step against the same step on unquantised fp32 caches:
    quantisation error only (informational bound, per-row scales)."""
    rng = np.random.default_rng(6)
    T, kvd, hid = 200, 256, 1536
    k = rng.standard_normal((T, kvd)).astype(np.float32)
    v = rng.standard_normal((T, kvd)).astype(np.float32)
    kq = np.zeros((T + 1, kvd), np.int8)
    vq = np.zeros((T + 1, kvd), np.int8)
    ks = np.zeros((T + 1, 2), np.float32)
    vs = np.zeros((T + 1, 2), np.float32)
    for t in range(T):
        for h in range(2):
            kq[t, h * 128:(h + 1) * 128], ks[t, h] = [a[0] for a in orc.quantize_i8(k[t:t + 1, h * 128:(h + 1) * 128])]
            vq[t, h * 128:(h + 1) * 128], vs[t, h] = [a[0] for a in orc.quantize_i8(v[t:t + 1, h * 128:(h + 1) * 128])]
    q = rng.standard_normal((1, hid)).astype(np.float32)
    kn = rng.standard_normal((1, kvd)).astype(np.float32)
    vn = rng.standard_normal((1, kvd)).astype(np.float32)
    out = orc.layer_step_i8(q, kn, vn, kq, ks, vq, vs, T)
    assert np.isfinite(out).all() and np.abs(out).max() > 0
    # the appended row is the quantised RoPE'd k / plain v
    assert np.abs(vq[T].astype(np.float32) * np.repeat(vs[T], 128) - vn[0]).max() <= vs[T].max() * 0.5001


def test_int8_prefill_step_matches_numpy(orc):
    """The INT8 layer step with a multi-token chunk (seq = n, the prefill
    attention's oracle) against an independent float64 numpy computation:
    NeoX RoPE at positions pos..pos+n-1, causal GQA attention over the
    dequantised caches (the context's codes and the chunk's appended codes);
    the appended k / v rows decode to the rotated k and to v within half a
    quantisation step."""
    rng = np.random.default_rng(8)
    C, n, qh, kvh, hd = 150, 37, 12, 2, 128
    kvd, hid, G = kvh * hd, qh * hd, qh // kvh
    kq = np.zeros((C + n, kvd), np.int8)
    vq = np.zeros((C + n, kvd), np.int8)
    ks = np.zeros((C + n, kvh), np.float32)
    vs = np.zeros((C + n, kvh), np.float32)
    kq[:C] = rng.integers(-127, 128, (C, kvd))
    vq[:C] = rng.integers(-127, 128, (C, kvd))
    ks[:C] = rng.uniform(0.001, 0.05, (C, kvh))
    vs[:C] = rng.uniform(0.001, 0.05, (C, kvh))
    q = rng.standard_normal((n, hid)).astype(np.float32)
    k = rng.standard_normal((n, kvd)).astype(np.float32)
    v = rng.standard_normal((n, kvd)).astype(np.float32)
    out = orc.layer_step_i8(q, k, v, kq, ks, vq, vs, C)

    def rope(x, heads):  # NeoX pairs (i, i + 64), theta 1e6, float64
        x = x.astype(np.float64).reshape(n, heads, hd)
        pos = np.arange(C, C + n, dtype=np.float64)[:, None]
        ang = pos * (1e6 ** (-np.arange(64, dtype=np.float64) * 2 / hd))[None, :]
        c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
        a, b = x[..., :64], x[..., 64:]
        return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)

    qr, kr = rope(q, qh), rope(k, kvh)
    kd = kq.astype(np.float64).reshape(C + n, kvh, hd) * ks[..., None]
    vd = vq.astype(np.float64).reshape(C + n, kvh, hd) * vs[..., None]
    # the chunk's appended rows (the oracle rotates in fp32: ~3e-5 from float64)
    step_k = ks[C:, :, None] * 0.5 * (1 + 1e-5) + 1e-4
    assert (np.abs(kd[C:] - kr) <= step_k).all()
    assert (np.abs(vd[C:] - v.astype(np.float64).reshape(n, kvh, hd)) <= vs[C:, :, None] * 0.5 * (1 + 1e-5) + 1e-7).all()
    ref = np.zeros((n, qh, hd))
    for h in range(qh):
        kh, vh = kd[:, h // G], vd[:, h // G]
        sc = qr[:, h] @ kh.T / np.sqrt(hd)
        sc[np.arange(C + n)[None, :] > (C + np.arange(n))[:, None]] = -np.inf
        p = np.exp(sc - sc.max(axis=1, keepdims=True))
        ref[:, h] = (p / p.sum(axis=1, keepdims=True)) @ vh
    got = out.reshape(n, qh, hd).astype(np.float64)
    rel = (np.abs(got - ref).max(axis=2) / np.abs(ref).max(axis=2)).max()
    assert rel <= 5e-4, rel  # fp32 vs float64; a wrong mask, group or scale is O(1)
