"""Continuous batching (serving.Server): placement, chunked prefill, decode,
completion.  Host logic on CPU with two gloo ranks and bookkeeping-only
pools; on the GPU, every decode output and every prefill chunk's attention
against the oracle and every cached row bit-exact through admissions,
completions and block reuse."""
from __future__ import annotations

import os
import socket
from importlib import import_module

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT, load_pkg


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stream(seed, n, lo, hi, glo, ghi):
    rng = np.random.default_rng(seed)
    return [(int(rng.integers(lo, hi + 1)), int(rng.integers(glo, ghi + 1))) for _ in range(n)]


def _host_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kv = load_pkg()
        srv_mod = import_module("rk3588_npu_b200.serving")
        nb = 900
        P = kv.Pool(kv.KVP_HOST_ONLY, 2, nb, max_seqs=64, max_seq_len=4096)
        S = kv.Scheduler([nb] * world)
        srv = srv_mod.Server(P, S, rank, world, chunk=64, prefill_slots=3)
        for i, (L, g) in enumerate(_stream(11, 10, 100, 900, 2, 30)):
            srv.add_resident(srv_mod.Request(i, L, g))
        for i, (L, g) in enumerate(_stream(12, 40, 30, 1000, 1, 40)):
            srv.submit(srv_mod.Request(100 + i, L, g))
        counts = []
        for _ in range(400):
            counts.append(srv.step())
            if not (srv.queue or srv.prefilling or srv.decoding):
                break
        mine = sorted(r.rid for r in srv.finished if r.gpu == rank)
        q.put((rank, srv.placements, counts, mine, P.free_blocks(), len(srv.finished)))
    finally:
        dist.destroy_process_group()


def test_serving_host_logic_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_host_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, pl0, c0, mine0, free0, n0), (_, pl1, c1, mine1, free1, n1) = out
    glob = lambda cs: [(c["decode_tokens"], c["prefill_tokens"], c["completed"]) for c in cs]
    assert pl0 == pl1 and glob(c0) == glob(c1)  # replicated state agrees without communication
    assert sum(c["local_decode"] for c in c0 + c1) == sum(c["decode_tokens"] for c in c0)
    assert n0 == n1 == 50                    # every request completed
    assert not set(mine0) & set(mine1)       # each executed on exactly one rank
    assert sorted(mine0 + mine1) == sorted(rid for rid, _ in pl0)
    assert {g for _, g in pl0} == {0, 1}     # both GPUs used
    assert free0 == free1 == 900             # every block returned
    assert max(c["prefill_tokens"] for c in c0) <= 3 * 64


def test_placement_balances_resident_blocks():
    kv = load_pkg()
    srv_mod = import_module("rk3588_npu_b200.serving")
    P = kv.Pool(kv.KVP_HOST_ONLY, 1, 10000, max_seqs=256, max_seq_len=9000)
    S = kv.Scheduler([10000] * 4)
    srv = srv_mod.Server(P, S, 0, 4)
    for i, (L, g) in enumerate(_stream(4, 128, 512, 8192, 16, 256)):
        srv.add_resident(srv_mod.Request(i, L, g))
    loads = [S.load(g)[0] for g in range(4)]
    assert max(loads) - min(loads) <= -(-(8192 + 256) // 16)  # within one request's footprint


def test_admission_waits_for_room():
    kv = load_pkg()
    srv_mod = import_module("rk3588_npu_b200.serving")
    P = kv.Pool(kv.KVP_HOST_ONLY, 1, 40, max_seqs=8, max_seq_len=2000)
    S = kv.Scheduler([40])
    srv = srv_mod.Server(P, S, 0, 1, chunk=64, prefill_slots=4)
    srv.submit(srv_mod.Request(1, 300, 20))   # 20 blocks
    srv.submit(srv_mod.Request(2, 300, 20))   # 20 blocks
    srv.submit(srv_mod.Request(3, 16, 1))     # 2 blocks: must wait behind 1 and 2
    srv.step()
    assert [r.rid for r in srv.prefilling] == [1, 2] and [r.rid for r in srv.queue] == [3]
    while any(r.rid in (1, 2) for r in srv.prefilling + srv.decoding):
        srv.step()
    srv.step()
    assert 3 in [r.rid for r in srv.prefilling + srv.decoding + srv.finished]


# ------------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("batched", [False, True], ids=["per_request", "batched_prefill"])
def test_serving_gpu_matches_oracle_with_block_reuse(batched):
    """batched: the step's prompt chunks go through kv_append_chunk_batch +
    attn_prefill_batch (Server.step's prefill_batch_io) instead of one call
    per request."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    kv = load_pkg()
    srv_mod = import_module("rk3588_npu_b200.serving")
    dtype, layers, kvd, hid = 1, 2, 256, 1536
    nb = 260                                   # tight: completions must free blocks for admissions
    P = kv.Pool(0, layers, nb, dtype=dtype, max_seqs=32, max_seq_len=2048)
    S = kv.Scheduler([nb])
    srv = srv_mod.Server(P, S, 0, 1, chunk=48, prefill_slots=3)
    rng = np.random.default_rng(21)
    mirror = {}                                # rid -> [layer] (k_cache, v_cache)

    def new_mirror(req):
        cap = req.prompt + req.gen + 1
        mirror[req.rid] = [(np.zeros((cap, kvd), np.uint16), np.zeros((cap, kvd), np.uint16))
                           for _ in range(layers)]

    def load(req):
        new_mirror(req)
        for y in range(layers):
            kc, vc = mirror[req.rid][y]
            kc[:req.prompt] = orc.encode(rng.standard_normal((req.prompt, kvd)).astype(np.float32), dtype)
            vc[:req.prompt] = orc.encode(rng.standard_normal((req.prompt, kvd)).astype(np.float32), dtype)
            P.import_rows(y, req.seq, 0, torch.from_numpy(kc[:req.prompt].view(np.int16)).cuda(),
                          torch.from_numpy(vc[:req.prompt].view(np.int16)).cuda())

    for i, (L, g) in enumerate(_stream(31, 5, 40, 700, 2, 9)):
        srv.add_resident(srv_mod.Request(i, L, g), load)
    for i, (L, g) in enumerate(_stream(32, 12, 20, 400, 1, 8)):
        srv.submit(srv_mod.Request(100 + i, L, g))

    worst = 0.0
    state = {}

    def decode_io(layer, reqs):
        n = len(reqs)
        qh = rng.standard_normal((n, hid)).astype(np.float32)
        kh = rng.standard_normal((n, kvd)).astype(np.float32)
        vh = rng.standard_normal((n, kvd)).astype(np.float32)
        out = torch.empty((n, hid), device="cuda")
        state[layer] = (reqs, qh, kh, vh, out)
        return (torch.from_numpy(qh).cuda(), torch.from_numpy(kh).cuda(), torch.from_numpy(vh).cuda(), out)

    prefill_checks = []

    def prefill_kv(layer, req, pos0, n):
        """The chunk's k/v and q; the oracle appends and attends the same
        chunk (op_attention with seq = n) on the mirror."""
        if req.rid not in mirror:
            new_mirror(req)
        qh = rng.standard_normal((n, hid)).astype(np.float32)
        kh = rng.standard_normal((n, kvd)).astype(np.float32)
        vh = rng.standard_normal((n, kvd)).astype(np.float32)
        kc, vc = mirror[req.rid][layer]
        ref, _, _ = orc.layer_step(qh, kh, vh, kc, vc, pos0, dtype=dtype)
        out = torch.empty((n, hid), device="cuda")
        prefill_checks.append((out, ref))
        return (torch.from_numpy(kh).cuda(), torch.from_numpy(vh).cuda(), torch.from_numpy(qh).cuda(), out)

    def prefill_batch_io(layer, chunks):
        """All chunks' rows concatenated; each chunk's slice of the shared
        output is checked against its oracle step."""
        parts = [prefill_kv(layer, r, p0, n) for r, p0, n in chunks]
        out = torch.empty((sum(n for _, _, n in chunks), hid), device="cuda")
        first, o = len(prefill_checks) - len(chunks), 0
        for i, (_, _, n) in enumerate(chunks):
            prefill_checks[first + i] = (out[o:o + n], prefill_checks[first + i][1])
            o += n
        return (torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts]),
                torch.cat([p[2] for p in parts]), out)

    reused = False
    for step in range(200):
        if not (srv.queue or srv.prefilling or srv.decoding):
            break
        before = {r.rid: r.length for r in srv.decoding}
        state.clear()
        prefill_checks.clear()
        if batched:
            srv.step(decode_io, prefill_batch_io=prefill_batch_io)
        else:
            srv.step(decode_io, prefill_kv)
        reused = reused or bool(srv.finished and (srv.prefilling or srv.decoding))
        for out, ref in prefill_checks:  # chunk attention against the oracle
            g = out.cpu().numpy().reshape(-1, 128).astype(np.float64)
            rr = ref.reshape(-1, 128).astype(np.float64)
            worst = max(worst, float((np.abs(g - rr).max(1) / np.abs(rr).max(1)).max()))
        for layer, (reqs, qh, kh, vh, out) in state.items():
            got = out.cpu().numpy()
            for i, r in enumerate(reqs):
                kc, vc = mirror[r.rid][layer]
                ref, _, _ = orc.layer_step(qh[i:i + 1], kh[i:i + 1], vh[i:i + 1], kc, vc, before[r.rid],
                                           dtype=dtype)
                g = got[i].reshape(-1, 128).astype(np.float64)
                rr = ref[0].reshape(-1, 128).astype(np.float64)
                worst = max(worst, float((np.abs(g - rr).max(1) / np.abs(rr).max(1)).max()))
        # every live sequence's cache equals its mirror, bit for bit
        for r in srv.decoding + srv.prefilling:
            for y in range(layers):
                kd, vd = P.gather(y, r.seq)
                kc, vc = mirror[r.rid][y]
                assert np.array_equal(kd.cpu().numpy().view(np.uint16), kc[:r.length]), (step, r.rid)
                assert np.array_equal(vd.cpu().numpy().view(np.uint16), vc[:r.length]), (step, r.rid)
    assert not (srv.queue or srv.prefilling or srv.decoding)
    assert len(srv.finished) == 17 and reused
    assert P.free_blocks() == nb
    assert worst <= 1e-3, worst
    assert P.device_status() == 0
