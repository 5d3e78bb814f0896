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
