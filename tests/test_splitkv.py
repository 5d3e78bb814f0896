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
        S = sk_mod.SplitKV(P, lens, rank, world)
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
