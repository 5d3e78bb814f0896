"""attn_contig_noalloc: attention for callers that cannot allocate device
memory (a host that owns all GPU memory in its own arena, or a decode loop
that may not call the allocator).  It creates no pool and no buffers; its
split-KV partials live in a fixed device array inside the library.

Checked here against the existing entry point (attn_decode_append over the
paged pool) on the same data, within the tolerance the other GPU tests use,
for two decode steps in a row, so the second call runs on a scratch array
that still holds the first call's contents; and against the oracle's
attention for prompt-style calls (several query rows, causal limits, empty
key splits, the largest problem the array takes) in fp16 and bf16.  This
file is collected last."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-3
HD, NQ, NKV = 128, 12, 2


def rel_err(gpu, ref):
    g = gpu.reshape(-1, HD).astype(np.float64)
    r = ref.reshape(-1, HD).astype(np.float64)
    return float((np.abs(g - r).max(axis=1) / np.maximum(np.abs(r).max(axis=1), 1e-30)).max())


@pytest.mark.parametrize("dtype", [0, 1], ids=["f16", "bf16"])
def test_noalloc_matches_paged_decode_two_steps(kv, orc, dtype):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(77 + dtype)
    lens = [1, 300, 2000]
    P = kv.Pool(0, 1, 256, dtype=dtype, max_seqs=4, max_seq_len=4096)
    ids = []
    for L in lens:
        s = P.seq_alloc()
        P.reserve(s, L + 8)
        k0 = orc.encode(rng.standard_normal((L, 256)).astype(np.float32), dtype)
        v0 = orc.encode(rng.standard_normal((L, 256)).astype(np.float32), dtype)
        P.import_rows(0, s, 0, torch.from_numpy(k0.view(np.int16)).cuda(),
                      torch.from_numpy(v0.view(np.int16)).cuda())
        P.set_cur_pos(s, L)
        ids.append(s)
    lib = kv.load()
    stream = torch.cuda.current_stream().cuda_stream
    for step in range(2):
        pos = [P.cur_pos(s) for s in ids]
        q = rng.standard_normal((len(ids), NQ * HD)).astype(np.float32)
        k = rng.standard_normal((len(ids), NKV * HD)).astype(np.float32)
        v = rng.standard_normal((len(ids), NKV * HD)).astype(np.float32)
        ref = torch.empty((len(ids), NQ * HD), device="cuda")
        P.plan(ids)
        P.decode_layer(0, torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                       torch.from_numpy(v).cuda(), ref)
        P.commit()
        ref = ref.cpu().numpy()
        for i, s in enumerate(ids):
            kc, vc = P.gather(0, s)  # contiguous rows, new token included
            qr = q[i].copy()
            kk = k[i].copy()
            lib_o = orc.lib()
            lib_o.orc_rope(qr, kk, NQ, NKV, HD, pos[i], 1e6)  # the rotation the pool applied
            qd = torch.from_numpy(qr).cuda()
            out = torch.full((1, NQ * HD), float("nan"), device="cuda")
            rc = lib.attn_contig_noalloc(qd.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), 1,
                                         pos[i] + 1, NQ, NKV, HD, pos[i], dtype, stream)
            assert rc == 0
            got = out.cpu().numpy()[0]
            assert np.all(np.isfinite(got))
            assert rel_err(got, ref[i]) <= TOL, (step, i)


@pytest.mark.parametrize("dtype", [0, 1], ids=["f16", "bf16"])
@pytest.mark.parametrize("seq,pos_base,extra", [(1, 0, 0), (1, 2999, 0), (3, 700, 5), (64, 1500, 0), (504, 500, 0)],
                         ids=["first-token", "decode-3000", "rows3-past-end", "rows64-empty-splits", "rows504-one-split"])
def test_noalloc_matches_oracle(kv, orc, dtype, seq, pos_base, extra):
    """Against the oracle's attention (the reference's loops) on contiguous
    caches: query row s attends keys 0 .. pos_base + s.  Rows 64 at position
    1500 leave the last key split empty for the early rows (their merge must
    skip it); 504 rows x 2 KV heads is the largest problem the fixed array
    takes (one split per row and KV head).  Two calls in a row: the second
    reads a scratch array that still holds the first call's states."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(1000 * seq + pos_base + dtype)
    total = pos_base + seq + extra
    kc = orc.encode(rng.standard_normal((total, NKV * HD)).astype(np.float32), dtype)
    vc = orc.encode(rng.standard_normal((total, NKV * HD)).astype(np.float32), dtype)
    kd = torch.from_numpy(kc.view(np.int16)).cuda()
    vd = torch.from_numpy(vc.view(np.int16)).cuda()
    lib = kv.load()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        q = rng.standard_normal((seq, NQ * HD)).astype(np.float32)
        ref = orc.attention(q, kc, vc, seq, total, NQ, NKV, HD, pos_base, dtype)
        out = torch.full((seq, NQ * HD), float("nan"), device="cuda")
        qd = torch.from_numpy(q).cuda()
        rc = lib.attn_contig_noalloc(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), seq, total, NQ,
                                     NKV, HD, pos_base, dtype, stream)
        assert rc == kv.KV_OK, rc
        got = out.cpu().numpy()
        assert np.all(np.isfinite(got)), call
        assert rel_err(got, ref) <= TOL, (call, rel_err(got, ref))


def test_noalloc_rejects_unaligned_and_bad_arguments(kv):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = kv.load()
    x = torch.zeros(4096, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    p = x.data_ptr()
    # caches must be 16-byte aligned (one vector load per lane per row)
    assert lib.attn_contig_noalloc(p, p + 8, p, p, 1, 1, NQ, NKV, HD, 0, 0, st) == kv.KV_ERR_INVAL
    assert lib.attn_contig_noalloc(p, p, p, p, 1, 1, NQ, NKV, 64, 0, 0, st) == kv.KV_ERR_INVAL  # head_dim
    assert lib.attn_contig_noalloc(p, p, p, p, 1, 1, NQ, NKV, HD, 0, 2, st) == kv.KV_ERR_INVAL  # INT8 not served
    assert lib.attn_contig_noalloc(p, p, p, p, 1, 1, 18, NKV, HD, 0, 0, st) == kv.KV_ERR_INVAL  # group of 9


def test_noalloc_rejects_oversized_problem(kv):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = kv.load()
    x = torch.zeros(16, device="cuda")
    # seq * n_kv_heads > 1008 partial states do not fit the fixed array
    rc = lib.attn_contig_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 600, 1000, 12, 2,
                                 HD, 0, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == kv.KV_ERR_RANGE
