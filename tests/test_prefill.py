"""Chunked-prefill attention over the pool (attn_prefill) against the oracle's
op_attention with seq = n (worker/src/ops/op_attention.cpp:9-56): kv_append_chunk
then attn_prefill per layer must equal the oracle's RoPE + append + attention
step, outputs within 1e-3 relative per (token, head) row, cache bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_pkg

HD = 128
TOL = 1e-3


def rel_err(gpu, ref):
    g = gpu.reshape(-1, HD).astype(np.float64)
    r = ref.reshape(-1, HD).astype(np.float64)
    den = np.maximum(np.abs(r).max(axis=1), 1e-30)
    return float((np.abs(g - r).max(axis=1) / den).max())


def run_case(kv, orc, L0, chunks, dtype, layers=1, qh=12, kvh=2, seed=0, kernel="tc"):
    rng = np.random.default_rng(seed)
    kvd, hid = kvh * HD, qh * HD
    total = L0 + sum(chunks)
    P = kv.Pool(0, layers, -(-total // 16) + 4, num_q_heads=qh, num_kv_heads=kvh, dtype=dtype,
                max_seqs=1, max_seq_len=total + 16)
    s = P.seq_alloc()
    P.reserve(s, total)
    caches = []
    for y in range(layers):
        kc = np.zeros((total, kvd), np.uint16)
        vc = np.zeros((total, kvd), np.uint16)
        if L0:
            kc[:L0] = orc.encode(rng.standard_normal((L0, kvd)).astype(np.float32), dtype)
            vc[:L0] = orc.encode(rng.standard_normal((L0, kvd)).astype(np.float32), dtype)
            P.import_rows(y, s, 0, torch.from_numpy(kc[:L0].view(np.int16)).cuda(),
                          torch.from_numpy(vc[:L0].view(np.int16)).cuda())
        caches.append((kc, vc))
    P.set_cur_pos(s, L0)
    worst, pos = 0.0, L0
    for n in chunks:
        for y in range(layers):
            q = rng.standard_normal((n, hid)).astype(np.float32)
            k = rng.standard_normal((n, kvd)).astype(np.float32)
            v = rng.standard_normal((n, kvd)).astype(np.float32)
            out = torch.empty((n, hid), device="cuda")
            P.append_chunk(y, s, pos, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
            P.prefill(y, s, pos, torch.from_numpy(q).cuda(), out, kernel=kernel)
            kc, vc = caches[y]
            ref, _, _ = orc.layer_step(q, k, v, kc, vc, pos, qh, kvh, HD, 1e6, dtype)
            worst = max(worst, rel_err(out.cpu().numpy(), ref))
        pos += n
        P.set_cur_pos(s, pos)
    for y in range(layers):
        kd, vd = P.gather(y, s)
        assert np.array_equal(kd.cpu().numpy().view(np.uint16), caches[y][0][:pos])
        assert np.array_equal(vd.cpu().numpy().view(np.uint16), caches[y][1][:pos])
    assert P.device_status() == 0
    return worst


KERNELS = ["tc", "mma"]  # tcgen05 (attn_prefill) and the mma.sync baseline (attn_prefill_mma)


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("dtype", [0, 1], ids=["f16", "bf16"])
def test_prefill_ragged_chunks(kv, orc, dtype, kernel):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    # first chunk at position 0, then ragged sizes and offsets off the block grid
    assert run_case(kv, orc, 0, [1, 15, 16, 17, 100], dtype, layers=2, seed=dtype, kernel=kernel) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", KERNELS)
def test_prefill_512_chunks_after_context(kv, orc, kernel):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert run_case(kv, orc, 1003, [512, 512], 1, seed=3, kernel=kernel) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", KERNELS)
def test_prefill_long_context_many_splits(kv, orc, kernel):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert run_case(kv, orc, 6000, [64, 33], 0, seed=4, kernel=kernel) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("qh,kvh", [(16, 2), (4, 4), (8, 1), (6, 1), (10, 2)])
def test_prefill_group_sizes(kv, orc, qh, kvh, kernel):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert run_case(kv, orc, 300, [40], 1, qh=qh, kvh=kvh, seed=qh, kernel=kernel) <= TOL


def test_prefill_rejects_bad_calls():
    kv = load_pkg()
    P = kv.Pool(kv.KVP_HOST_ONLY, 1, 8, max_seqs=1, max_seq_len=128)
    s = P.seq_alloc()
    P.reserve(s, 32)
    with pytest.raises(kv.KVError) as e:
        kv.call("attn_prefill", P.h, 0, s, 0, 4, 16, 16, None)
    assert e.value.status == kv.KV_ERR_STATE          # no device storage
    with pytest.raises(kv.KVError) as e:
        kv.call("attn_prefill", P.h, 0, s + 1, 0, 4, 16, 16, None)
    assert e.value.status == kv.KV_ERR_BADSEQ


def run_batch(kv, orc, ctx, chunks, dtype, seed, qh=12, kvh=2):
    """Every sequence i holds ctx[i] imported tokens, then one batched append +
    attention of chunks[i] tokens per sequence; each against the oracle."""
    rng = np.random.default_rng(seed)
    kvd, hid = kvh * HD, qh * HD
    nseq = len(ctx)
    nb = sum(-(-(c + n) // 16) for c, n in zip(ctx, chunks)) + 8
    P = kv.Pool(0, 1, nb, num_q_heads=qh, num_kv_heads=kvh, dtype=dtype, max_seqs=nseq,
                max_seq_len=max(c + n for c, n in zip(ctx, chunks)) + 16)
    ids, caches = [], []
    for c, n in zip(ctx, chunks):
        s = P.seq_alloc()
        P.reserve(s, c + n)
        kc = np.zeros((c + n, kvd), np.uint16)
        vc = np.zeros((c + n, kvd), np.uint16)
        if c:
            kc[:c] = orc.encode(rng.standard_normal((c, kvd)).astype(np.float32), dtype)
            vc[:c] = orc.encode(rng.standard_normal((c, kvd)).astype(np.float32), dtype)
            P.import_rows(0, s, 0, torch.from_numpy(kc[:c].view(np.int16)).cuda(),
                          torch.from_numpy(vc[:c].view(np.int16)).cuda())
        P.set_cur_pos(s, c)
        ids.append(s)
        caches.append((kc, vc))
    R = sum(chunks)
    q = rng.standard_normal((R, hid)).astype(np.float32)
    k = rng.standard_normal((R, kvd)).astype(np.float32)
    v = rng.standard_normal((R, kvd)).astype(np.float32)
    out = torch.full((R, hid), float("nan"), device="cuda")
    P.append_chunk_batch(0, ids, ctx, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), ns=chunks)
    P.prefill_batch(0, ids, ctx, chunks, torch.from_numpy(q).cuda(), out)
    got = out.cpu().numpy()
    worst, r0 = 0.0, 0
    for i, (c, n) in enumerate(zip(ctx, chunks)):
        kc, vc = caches[i]
        if n:
            ref, _, _ = orc.layer_step(q[r0:r0 + n], k[r0:r0 + n], v[r0:r0 + n], kc, vc, c, qh, kvh, HD, 1e6, dtype)
            worst = max(worst, rel_err(got[r0:r0 + n], ref))
        P.set_cur_pos(ids[i], c + n)
        kd, vd = P.gather(0, ids[i])
        assert np.array_equal(kd.cpu().numpy().view(np.uint16), kc[:c + n])
        assert np.array_equal(vd.cpu().numpy().view(np.uint16), vc[:c + n])
        r0 += n
    assert P.device_status() == 0
    P.close()
    return worst


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [0, 1], ids=["f16", "bf16"])
def test_prefill_batch_mixed_chunks(kv, orc, dtype):
    """One launch over ragged chunks and contexts: a chunk at position 0, a
    one-token chunk, an empty chunk, 512-token chunks after long contexts
    (split and unsplit in the same launch)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = [0, 37, 2000, 5000, 16, 700, 3000]
    chunks = [100, 1, 512, 512, 0, 33, 512]
    assert run_batch(kv, orc, ctx, chunks, dtype, seed=10 + dtype) <= TOL


@pytest.mark.gpu
def test_prefill_batch_more_chunks_than_one_launch(kv, orc):
    """40 chunks: two launches of at most 32 chunks each."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(12)
    ctx = [int(x) for x in rng.integers(0, 300, 40)]
    chunks = [int(x) for x in rng.integers(1, 40, 40)]
    assert run_batch(kv, orc, ctx, chunks, 1, seed=12) <= TOL


def test_prefill_batch_rejects_bad_calls():
    kv = load_pkg()
    P = kv.Pool(kv.KVP_HOST_ONLY, 1, 8, max_seqs=2, max_seq_len=128)
    a, b = P.seq_alloc(), P.seq_alloc()
    P.reserve(a, 32)
    P.reserve(b, 32)
    ints = kv._ints
    for fn in ("attn_prefill_batch", "kv_append_chunk_batch"):
        with pytest.raises(kv.KVError) as e:  # no device storage
            kv.call(fn, P.h, 0, 2, ints([a, b]), ints([0, 0]), ints([4, 4]), 16, 16, None)
        assert e.value.status == kv.KV_ERR_STATE
        with pytest.raises(kv.KVError) as e:  # a dead sequence
            kv.call(fn, P.h, 0, 2, ints([b + 1, a]), ints([0, 0]), ints([4, 4]), 16, 16, None)
        assert e.value.status == kv.KV_ERR_BADSEQ
        with pytest.raises(kv.KVError) as e:  # the same sequence twice
            kv.call(fn, P.h, 0, 2, ints([a, a]), ints([0, 4]), ints([4, 4]), 16, 16, None)
        assert e.value.status in (kv.KV_ERR_STATE, kv.KV_ERR_INVAL)
        with pytest.raises(kv.KVError) as e:  # past the reserved blocks
            kv.call(fn, P.h, 0, 1, ints([b]), ints([30]), ints([4]), 16, 16, None)
        assert e.value.status in (kv.KV_ERR_STATE, kv.KV_ERR_RANGE)
    P.close()
