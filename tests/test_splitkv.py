"""Split-KV across ranks: host logic on CPU (gloo, host-only pools) and the
full step on one GPU with two processes (gloo), against the unsplit oracle."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT, load_pkg
from importlib import import_module


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _host_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kv = load_pkg()
        from importlib import import_module
        sk_mod = import_module("rk3588_npu_b200.splitkv")
        P = kv.Pool(kv.KVP_HOST_ONLY, 1, 4096, max_seqs=4, max_seq_len=40000)
        lens = [1000, 33, 20000]
        S = sk_mod.SplitKV(P, lens, rank, world)
        S.reserve(8)
        for i, (lo, hi) in enumerate(S.bounds):
            P.set_cur_pos(S.ids[i], hi - lo)
        res = []
        for step in range(3):
            S.begin_step()
            info = P.plan_info()
            res.append((info["npatch"], [P.cur_pos(s) for s in S.ids]))
            S.end_step()
        # the slices tile [0, L) exactly
        gathered = [None] * world
        dist.all_gather_object(gathered, S.bounds)
        q.put((rank, res, gathered, S.lengths))
    finally:
        dist.destroy_process_group()


def test_splitkv_host_logic_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_host_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out.sort()
    lens = [1000, 33, 20000]
    for rank, res, gathered, final_lens in out:
        assert final_lens == [L + 3 for L in lens]
        for i, L in enumerate(lens):
            assert gathered[0][i][0] == 0 and gathered[-1][i][1] == L
            assert gathered[0][i][1] == gathered[1][i][0]
        lengths = [r[1] for r in res]
        if rank == 0:  # never appends
            assert lengths[0] == lengths[-1]
        else:  # the last rank grows by one per step
            assert [x - lengths[0][j] for j, x in enumerate(lengths[-1])] == [2, 2, 2]


def _gpu_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as orc
        kv = load_pkg()
        from importlib import import_module
        sk_mod = import_module("rk3588_npu_b200.splitkv")
        rng = np.random.default_rng(5)
        lens = [700, 2500]
        dtype = 1
        full_k = [orc.encode(rng.standard_normal((L + 4, 256)).astype(np.float32), dtype) for L in lens]
        full_v = [orc.encode(rng.standard_normal((L + 4, 256)).astype(np.float32), dtype) for L in lens]
        P = kv.Pool(0, 1, 600, dtype=dtype, max_seqs=4, max_seq_len=4096)
        # two ranks on one GPU: NCCL needs one GPU per rank, so the states
        # go through torch.distributed's gloo all-gather
        S = sk_mod.SplitKV(P, lens, rank, world, transport="collective")
        S.reserve(4)
        for i, (lo, hi) in enumerate(S.bounds):
            k = torch.from_numpy(full_k[i][lo:hi].view(np.int16)).cuda()
            v = torch.from_numpy(full_v[i][lo:hi].view(np.int16)).cuda()
            S.load_slice(0, i, k, v)
        worst = 0.0
        for step in range(2):
            qh = rng.standard_normal((2, 1536)).astype(np.float32)
            kh = rng.standard_normal((2, 256)).astype(np.float32)
            vh = rng.standard_normal((2, 256)).astype(np.float32)
            out = torch.empty((2, 1536), device="cuda")
            S.begin_step()
            S.layer(0, torch.from_numpy(qh).cuda(), torch.from_numpy(kh).cuda(),
                    torch.from_numpy(vh).cuda(), out)
            pos = list(S.lengths)
            S.end_step()
            got = out.cpu().numpy()
            for i in range(2):
                ref, _, _ = orc.layer_step(qh[i:i + 1], kh[i:i + 1], vh[i:i + 1], full_k[i], full_v[i],
                                           pos[i], dtype=dtype)
                g = got[i].reshape(-1, 128).astype(np.float64)
                r = ref[0].reshape(-1, 128).astype(np.float64)
                worst = max(worst, float((np.abs(g - r).max(1) / np.abs(r).max(1)).max()))
        q.put((rank, worst, P.device_status()))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_splitkv_two_ranks_one_gpu_matches_unsplit():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, worst, status in out:
        assert status == 0
        assert worst <= 1e-3, (rank, worst)


def _p2p_worker(rank, world, port, q, transport="p2p"):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as orc
        kv = load_pkg()
        sk_mod = import_module("rk3588_npu_b200.splitkv")
        rng = np.random.default_rng(6)
        lens = [900, 3100, 17]
        dtype = 1
        full_k = [orc.encode(rng.standard_normal((L + 8, 256)).astype(np.float32), dtype) for L in lens]
        full_v = [orc.encode(rng.standard_normal((L + 8, 256)).astype(np.float32), dtype) for L in lens]
        P = kv.Pool(rank, 2, 600, dtype=dtype, max_seqs=4, max_seq_len=4096)
        S = sk_mod.SplitKV(P, lens, rank, world, transport=transport)
        S.reserve(8)
        for layer in range(2):
            for i, (lo, hi) in enumerate(S.bounds):
                k = torch.from_numpy(full_k[i][lo:hi].view(np.int16)).cuda()
                v = torch.from_numpy(full_v[i][lo:hi].view(np.int16)).cuda()
                S.load_slice(layer, i, k, v)
        worst = 0.0
        caches = [[(full_k[i].copy(), full_v[i].copy()) for i in range(3)] for _ in range(2)]
        for step in range(3):
            pos = list(S.lengths)
            S.begin_step()
            for layer in range(2):
                qh = rng.standard_normal((3, 1536)).astype(np.float32)
                kh = rng.standard_normal((3, 256)).astype(np.float32)
                vh = rng.standard_normal((3, 256)).astype(np.float32)
                out = torch.empty((3, 1536), device="cuda")
                S.layer(layer, torch.from_numpy(qh).cuda(), torch.from_numpy(kh).cuda(),
                        torch.from_numpy(vh).cuda(), out)
                got = out.cpu().numpy()
                for i in range(3):
                    kc, vc = caches[layer][i]
                    ref, _, _ = orc.layer_step(qh[i:i + 1], kh[i:i + 1], vh[i:i + 1], kc, vc, pos[i],
                                               dtype=dtype)
                    g = got[i].reshape(-1, 128).astype(np.float64)
                    r = ref[0].reshape(-1, 128).astype(np.float64)
                    worst = max(worst, float((np.abs(g - r).max(1) / np.abs(r).max(1)).max()))
            S.end_step()
        status = P.device_status()
        S.close()
        q.put((rank, worst, status))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_splitkv_p2p_exchange_two_gpus_matches_unsplit():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_p2p_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, worst, status in out:
        assert status == 0
        assert worst <= 1e-3, (rank, worst)


@pytest.mark.gpu
def test_splitkv_nccl_two_gpus_matches_unsplit():
    """The library's NCCL path (attn_decode_append_nccl: local decode, NCCL
    all-gather of the packed states, merge) on two GPUs, 2 layers x 3 steps,
    against the unsplit oracle."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_p2p_worker, args=(r, 2, port, q, "nccl")) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, worst, status in out:
        assert status == 0
        assert worst <= 1e-3, (rank, worst)


@pytest.mark.gpu
def test_nccl_call_with_one_rank_equals_local_decode():
    """A one-rank NCCL communicator (a single-GPU box still runs the NCCL
    path): the decode states go through the communicator's buffers, a
    one-rank all-gather and the merge; the output must match the ordinary
    decode.  A plan with more rows than the communicator holds is refused."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ctypes as C
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    kv = load_pkg()
    rng = np.random.default_rng(8)
    lens = [5, 700, 4000]
    P = kv.Pool(0, 1, 400, dtype=1, max_seqs=3, max_seq_len=4200)
    ids = []
    for L in lens:
        s = P.seq_alloc()
        P.reserve(s, L + 4)
        kc = orc.encode(rng.standard_normal((L, 256)).astype(np.float32), 1)
        vc = orc.encode(rng.standard_normal((L, 256)).astype(np.float32), 1)
        P.import_rows(0, s, 0, torch.from_numpy(kc.view(np.int16)).cuda(),
                      torch.from_numpy(vc.view(np.int16)).cuda())
        P.set_cur_pos(s, L)
        ids.append(s)
    uid = (C.c_char * kv.KVN_UNIQUE_ID_BYTES)()
    kv.call("kvn_unique_id", uid)
    c = kv._vp()
    kv.call("kvn_create", 0, 0, 1, uid, 3 * 12, C.byref(c))
    q = torch.randn((3, 1536), device="cuda")
    k = torch.randn((3, 256), device="cuda")
    v = torch.randn((3, 256), device="cuda")
    ref = torch.empty((3, 1536), device="cuda")
    got = torch.empty((3, 1536), device="cuda")
    P.plan(ids, rope_pos=lens, append=[0, 0, 0])
    P.decode_layer(0, q, k, v, ref)
    for _ in range(2):
        kv.call("attn_decode_append_nccl", P.h, 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), got.data_ptr(), c,
                None)
        torch.cuda.synchronize()
        assert torch.allclose(got, ref, rtol=1e-5, atol=1e-6)
    kv.call("kvn_destroy", c)
    # a communicator for one sequence's rows cannot take this 3-sequence plan
    kv.call("kvn_unique_id", uid)
    small = kv._vp()
    kv.call("kvn_create", 0, 0, 1, uid, 12, C.byref(small))
    rc = kv.load().attn_decode_append_nccl(P.h, 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), got.data_ptr(),
                                           small, None)
    assert rc == kv.KV_ERR_RANGE
    kv.call("kvn_destroy", small)
    P.commit()
    assert P.device_status() == 0


@pytest.mark.gpu
def test_xgpu_call_with_one_rank_equals_local_decode():
    """A one-rank exchange: the decode states go through this rank's slot of
    the exchange area and the exchange kernel's merge of a single state must
    reproduce the ordinary decode output exactly."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ctypes as C
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    kv = load_pkg()
    rng = np.random.default_rng(7)
    lens = [5, 700, 4000]
    P = kv.Pool(0, 1, 400, dtype=0, max_seqs=3, max_seq_len=4200)
    ids = []
    for L in lens:
        s = P.seq_alloc()
        P.reserve(s, L + 4)
        kc = orc.encode(rng.standard_normal((L, 256)).astype(np.float32), 0)
        vc = orc.encode(rng.standard_normal((L, 256)).astype(np.float32), 0)
        P.import_rows(0, s, 0, torch.from_numpy(kc.view(np.int16)).cuda(),
                      torch.from_numpy(vc.view(np.int16)).cuda())
        P.set_cur_pos(s, L)
        ids.append(s)
    x = kv._vp()
    kv.call("kvx_create", 0, 0, 1, 3 * 12, C.byref(x))
    q = torch.randn((3, 1536), device="cuda")
    k = torch.randn((3, 256), device="cuda")
    v = torch.randn((3, 256), device="cuda")
    ref = torch.empty((3, 1536), device="cuda")
    got = torch.empty((3, 1536), device="cuda")
    for s, L in zip(ids, lens):
        P.set_cur_pos(s, L)
    P.plan(ids, rope_pos=lens, append=[0, 0, 0])
    P.decode_layer(0, q, k, v, ref)
    for _ in range(3):  # both buffers of the exchange area
        kv.call("attn_decode_append_xgpu", P.h, 0, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                got.data_ptr(), x, None)
        torch.cuda.synchronize()
        assert torch.allclose(got, ref, rtol=1e-6, atol=1e-7)
    P.commit()
    assert P.device_status() == 0
    kv.call("kvx_destroy", x)


def _skip_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kv = load_pkg()
        sk_mod = import_module("rk3588_npu_b200.splitkv")
        P = kv.Pool(rank, 1, 64, dtype=1, max_seqs=1, max_seq_len=1024)
        S = sk_mod.SplitKV(P, [300], rank, world, transport="p2p")
        S.reserve(4)
        lo, hi = S.bounds[0]
        z = torch.zeros((hi - lo, 256), dtype=torch.int16, device="cuda")
        S.load_slice(0, 0, z, z)
        q_ = torch.randn((1, 1536), device="cuda")
        k_ = torch.randn((1, 256), device="cuda")
        out = torch.empty((1, 1536), device="cuda")
        S.begin_step()
        S.layer(0, q_, k_, k_, out)       # both ranks: a completed exchange
        torch.cuda.synchronize()
        ok_status = P.device_status()
        dist.barrier()
        if rank == 0:                     # rank 1 skips this call: nothing sets its words
            S.layer(0, q_, k_, k_, out)
            torch.cuda.synchronize()
        status = P.device_status()
        dist.barrier()
        q.put((rank, ok_status, status, bool(torch.all(out == 0)) if rank == 0 else None))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_xgpu_timeout_when_peer_skips_call():
    """A peer that never makes its layer call: the exchange's bounded wait
    gives up (~1 s) and reports KV_ERR_TIMEOUT; no hang, outputs zeroed."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_skip_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, ok0, st0, zero0), (_, ok1, st1, _) = out
    assert ok0 == 0 and ok1 == 0
    assert st0 == 7 and zero0          # KV_ERR_TIMEOUT on the rank that waited
    assert st1 == 0
