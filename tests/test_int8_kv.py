"""INT8 KV cache (KV_I8): the FP16 -> INT8 compression the reference plans
(docs/work_division.md:72), on the device decode path, against the oracle's
restatement of the scheme (oracle/kvattn_oracle.c: orc_quantize_i8,
orc_attention_i8, orc_layer_step_i8):
  * codes and scales bit-exact, through kv_append_chunk and through the
    fused append of the decode launch (K quantised after RoPE);
  * attention within 1e-3 relative per (sequence, query head) row of the
    oracle's attention over the dequantised caches, for decode steps and for
    prompt chunks (the mma.sync prefill kernel reading the compact tiles).
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from conftest import load_pkg  # noqa: E402

HD = 128
TOL = 1e-3


def rel_err(gpu, ref):
    g = gpu.reshape(-1, HD).astype(np.float64)
    r = ref.reshape(-1, HD).astype(np.float64)
    den = np.maximum(np.abs(r).max(axis=1), 1e-30)
    return float((np.abs(g - r).max(axis=1) / den).max())


def rope_k(orc, k, pos0, kvh, theta=1e6):
    """Rows of k [n, kvh*128] rotated at positions pos0.. by the oracle's RoPE."""
    out = np.array(k, np.float32, order="C")
    qd = np.zeros(HD, np.float32)
    for r in range(out.shape[0]):
        orc.lib().orc_rope(qd, out[r], 1, kvh, HD, pos0 + r, theta)
    return out


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.gpu
def test_int8_append_chunk_bit_exact(kv, orc):
    need_gpu()
    kvh = 2
    rng = np.random.default_rng(1)
    P = kv.Pool(0, 1, 64, num_q_heads=12, num_kv_heads=kvh, dtype=kv.KV_I8, max_seqs=1, max_seq_len=1024)
    s = P.seq_alloc()
    P.reserve(s, 337)
    k = rng.standard_normal((337, kvh * HD)).astype(np.float32) * rng.uniform(0.1, 10, (337, 1)).astype(np.float32)
    v = rng.standard_normal((337, kvh * HD)).astype(np.float32)
    k[5] = 0.0  # an all-zero row: scale 0, codes 0
    for pos0, n in ((0, 300), (300, 37)):
        P.append_chunk(0, s, pos0, torch.from_numpy(k[pos0:pos0 + n]).cuda(), torch.from_numpy(v[pos0:pos0 + n]).cuda())
    P.set_cur_pos(s, 337)
    kc, vc, ks, vs = [t.cpu().numpy() for t in P.gather_i8(0, s)]
    kr = rope_k(orc, k, 0, kvh)
    qk, sk = orc.quantize_i8(kr.reshape(337, kvh, HD))
    qv, sv = orc.quantize_i8(v.reshape(337, kvh, HD))
    assert np.array_equal(kc, qk.reshape(337, -1)) and np.array_equal(ks, sk)
    assert np.array_equal(vc, qv.reshape(337, -1)) and np.array_equal(vs, sv)
    assert P.device_status() == 0
    P.close()


@pytest.mark.gpu
@pytest.mark.parametrize("merge", ["grid", "cluster"])
@pytest.mark.parametrize("lens,layers,seed", [([0, 1, 15, 16, 17, 33, 300, 1000], 2, 2), ([5000, 40, 2100], 1, 3)])
def test_int8_decode_matches_oracle(kv, orc, lens, layers, seed, merge):
    """Context imported as codes + scales, then three decode steps (fused
    RoPE + INT8 append + attention) on a batch with ragged lengths; split
    heads merged by the merge launch, or inside 8-CTA clusters where the
    planner can keep them there (the first case)."""
    need_gpu()
    qh, kvh = 12, 2
    kvd, hid = kvh * HD, qh * HD
    steps = 3
    rng = np.random.default_rng(seed)
    nb = sum(-(-(L + steps) // 16) for L in lens) + 8
    P = kv.Pool(0, layers, nb, num_q_heads=qh, num_kv_heads=kvh, dtype=kv.KV_I8, max_seqs=len(lens),
                max_seq_len=max(lens) + 64)
    P.set_merge_mode(kv.KVP_MERGE_CLUSTER if merge == "cluster" else kv.KVP_MERGE_GRID)
    ids, caches = [], []
    for L in lens:
        s = P.seq_alloc()
        P.reserve(s, L + steps)
        per_layer = []
        for y in range(layers):
            kq = np.zeros((L + steps, kvd), np.int8)
            vq = np.zeros((L + steps, kvd), np.int8)
            ks = np.zeros((L + steps, kvh), np.float32)
            vs = np.zeros((L + steps, kvh), np.float32)
            if L:
                kq[:L] = rng.integers(-127, 128, (L, kvd))
                vq[:L] = rng.integers(-127, 128, (L, kvd))
                ks[:L] = rng.uniform(0.001, 0.05, (L, kvh))
                vs[:L] = rng.uniform(0.001, 0.05, (L, kvh))
                P.import_i8(y, s, 0, torch.from_numpy(kq[:L]).cuda(), torch.from_numpy(vq[:L]).cuda(),
                            torch.from_numpy(ks[:L]).cuda(), torch.from_numpy(vs[:L]).cuda())
            per_layer.append((kq, ks, vq, vs))
        P.set_cur_pos(s, L)
        ids.append(s)
        caches.append(per_layer)
    worst = 0.0
    clustered = 0
    for step in range(steps):
        P.plan(ids)
        clustered += P.plan_clusters()[0]
        for y in range(layers):
            q = rng.standard_normal((len(lens), hid)).astype(np.float32)
            k = rng.standard_normal((len(lens), kvd)).astype(np.float32)
            v = rng.standard_normal((len(lens), kvd)).astype(np.float32)
            out = torch.empty((len(lens), hid), device="cuda")
            P.decode_layer(y, torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), out)
            got = out.cpu().numpy()
            for i, L in enumerate(lens):
                kq, ks, vq, vs = caches[i][y]
                ref = orc.layer_step_i8(q[i:i + 1], k[i:i + 1], v[i:i + 1], kq, ks, vq, vs, L + step)
                worst = max(worst, rel_err(got[i], ref))
        P.commit()
    assert worst <= TOL, worst
    if merge == "grid":
        assert clustered == 0
    elif seed == 2:  # short contexts: the planner keeps every split inside one cluster
        assert clustered == steps
    for i, L in enumerate(lens):
        for y in range(layers):
            kc, vc, ks, vs = [t.cpu().numpy() for t in P.gather_i8(y, ids[i])]
            kq, ksr, vq, vsr = caches[i][y]
            n = L + steps
            assert np.array_equal(kc, kq[:n]) and np.array_equal(ks, ksr[:n])
            assert np.array_equal(vc, vq[:n]) and np.array_equal(vs, vsr[:n])
    assert P.device_status() == 0
    P.close()


@pytest.mark.gpu
@pytest.mark.parametrize("batched", [True, False], ids=["batch", "per_chunk"])
def test_int8_prefill_matches_oracle(kv, orc, batched):
    """Prompt chunks over INT8 caches: imported context (codes + scales),
    then the chunks' quantising append and causal attention (attn_prefill_batch,
    or attn_prefill per chunk): attention within 1e-3 of the oracle's over
    the dequantised caches, codes and scales bit-exact.  A chunk at position
    0, a one-token chunk, and a 512-token chunk after 3000 tokens (key splits)."""
    need_gpu()
    qh, kvh = 12, 2
    kvd, hid = kvh * HD, qh * HD
    ctx, chunks = [0, 37, 3000], [100, 1, 512]
    rng = np.random.default_rng(7)
    nb = sum(-(-(c + n) // 16) for c, n in zip(ctx, chunks)) + 8
    P = kv.Pool(0, 1, nb, num_q_heads=qh, num_kv_heads=kvh, dtype=kv.KV_I8, max_seqs=len(ctx),
                max_seq_len=max(ctx) + max(chunks) + 16)
    ids, caches = [], []
    for c, n in zip(ctx, chunks):
        s = P.seq_alloc()
        P.reserve(s, c + n)
        kq = np.zeros((c + n, kvd), np.int8)
        vq = np.zeros((c + n, kvd), np.int8)
        ks = np.zeros((c + n, kvh), np.float32)
        vs = np.zeros((c + n, kvh), np.float32)
        if c:
            kq[:c] = rng.integers(-127, 128, (c, kvd))
            vq[:c] = rng.integers(-127, 128, (c, kvd))
            ks[:c] = rng.uniform(0.001, 0.05, (c, kvh))
            vs[:c] = rng.uniform(0.001, 0.05, (c, kvh))
            P.import_i8(0, s, 0, torch.from_numpy(kq[:c]).cuda(), torch.from_numpy(vq[:c]).cuda(),
                        torch.from_numpy(ks[:c]).cuda(), torch.from_numpy(vs[:c]).cuda())
        P.set_cur_pos(s, c)
        ids.append(s)
        caches.append((kq, ks, vq, vs))
    R = sum(chunks)
    q = rng.standard_normal((R, hid)).astype(np.float32)
    k = rng.standard_normal((R, kvd)).astype(np.float32)
    v = rng.standard_normal((R, kvd)).astype(np.float32)
    out = torch.full((R, hid), float("nan"), device="cuda")
    qd, kd, vd = torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    if batched:
        P.append_chunk_batch(0, ids, ctx, kd, vd, ns=chunks)
        P.prefill_batch(0, ids, ctx, chunks, qd, out)
    else:
        r0 = 0
        for s, c, n in zip(ids, ctx, chunks):
            P.append_chunk(0, s, c, kd[r0:r0 + n], vd[r0:r0 + n])
            P.prefill(0, s, c, qd[r0:r0 + n], out[r0:r0 + n])
            r0 += n
    got = out.cpu().numpy()
    worst, r0 = 0.0, 0
    for i, (c, n) in enumerate(zip(ctx, chunks)):
        kq, ks, vq, vs = caches[i]
        ref = orc.layer_step_i8(q[r0:r0 + n], k[r0:r0 + n], v[r0:r0 + n], kq, ks, vq, vs, c)
        worst = max(worst, rel_err(got[r0:r0 + n], ref))
        P.set_cur_pos(ids[i], c + n)
        kc, vc, ksd, vsd = [t.cpu().numpy() for t in P.gather_i8(0, ids[i])]
        assert np.array_equal(kc, kq) and np.array_equal(ksd, ks)
        assert np.array_equal(vc, vq) and np.array_equal(vsd, vs)
        r0 += n
    assert worst <= TOL, worst
    assert P.device_status() == 0
    P.close()


@pytest.mark.gpu
def test_int8_pool_rejects_16bit_paths(kv):
    need_gpu()
    P = kv.Pool(0, 1, 8, dtype=kv.KV_I8, max_seqs=1, max_seq_len=128)
    s = P.seq_alloc()
    P.reserve(s, 32)
    with pytest.raises(kv.KVError) as e:
        P.import_rows(0, s, 0, torch.zeros((4, 256), dtype=torch.int16, device="cuda"),
                      torch.zeros((4, 256), dtype=torch.int16, device="cuda"))
    assert e.value.status == kv.KV_ERR_INVAL
    P.close()
    Q = kv.Pool(0, 1, 8, dtype=kv.KV_BF16, max_seqs=1, max_seq_len=128)
    t = Q.seq_alloc()
    Q.reserve(t, 16)
    with pytest.raises(kv.KVError) as e:
        Q.import_i8(0, t, 0, torch.zeros((4, 256), dtype=torch.int8, device="cuda"),
                    torch.zeros((4, 256), dtype=torch.int8, device="cuda"),
                    torch.zeros((4, 2), device="cuda"), torch.zeros((4, 2), device="cuda"))
    assert e.value.status == kv.KV_ERR_INVAL
    Q.close()
