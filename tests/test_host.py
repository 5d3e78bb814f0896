"""Host logic on CPU: block allocator, block tables, lengths and the decode
planner of a bookkeeping-only pool (KVP_HOST_ONLY), checked bit-exactly
against a small model allocator, plus the C ABI's exported symbols."""
from __future__ import annotations

import os
import re

import numpy as np
import pytest

from conftest import ROOT


class ModelPool:
    """Model of the documented allocation policy: a LIFO stack of free ids
    that hands out 0, 1, 2, ... initially; freeing pushes a sequence's blocks
    last-to-first; an explicit take swaps the top into the taken id's place;
    sequence ids are the lowest non-live slot."""

    def __init__(self, nblocks, max_seqs):
        self.free = [nblocks - 1 - i for i in range(nblocks)]
        self.seqs = [None] * max_seqs  # None or [len, blocks]

    def pop(self):
        return self.free.pop()

    def take(self, b):
        i = self.free.index(b)
        last = self.free[-1]
        self.free[i] = last
        self.free.pop()

    def alloc(self):
        i = self.seqs.index(None)
        self.seqs[i] = [0, []]
        return i

    def release(self, s):
        for b in reversed(self.seqs[s][1]):
            self.free.append(b)
        self.seqs[s] = None

    def reserve(self, s, n):
        need = -(-n // 16) - len(self.seqs[s][1])
        if need > len(self.free):
            return False
        for _ in range(max(0, need)):
            self.seqs[s][1].append(self.pop())
        return True

    def plan(self, ids):
        for s in ids:
            ln, bl = self.seqs[s]
            if ln // 16 >= len(bl):
                bl.append(self.pop())

    def commit(self, ids):
        for s in ids:
            self.seqs[s][0] += 1


PIECE_COST = 8  # block-equivalents the planner charges per piece (kPieceCost)


def host_pool(kv, nblocks=64, max_seqs=8, max_seq_len=4096, kv_heads=2):
    return kv.Pool(kv.KVP_HOST_ONLY, 1, nblocks, num_q_heads=6 * kv_heads, num_kv_heads=kv_heads,
                   max_seqs=max_seqs, max_seq_len=max_seq_len)


def test_abi_exports_every_declared_symbol(kv):
    import ctypes
    decl = set()
    inc = os.path.join(ROOT, "include")
    for fn in os.listdir(inc):
        if fn.endswith(".h"):
            txt = open(os.path.join(inc, fn)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            txt = re.sub(r"^\s*typedef[^;]*;", "", txt, flags=re.M)  # function-pointer types
            decl |= set(re.findall(r"^\s*(?:const\s+)?\w+\s*\**\s*(\w+)\s*\(", txt, flags=re.M))
    decl -= {"if", "while", "for", "return", "sizeof"}
    assert len(decl) >= 25
    lib = ctypes.CDLL(kv.LIB_PATH)
    missing = [n for n in sorted(decl) if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.kv_version
    assert set(kv._SIGS) <= decl


def test_create_rejects_unsupported_shapes(kv):
    with pytest.raises(kv.KVError) as e:
        kv.Pool(kv.KVP_HOST_ONLY, 1, 8, num_q_heads=12, num_kv_heads=1)  # group 12 > 8
    assert e.value.status == kv.KV_ERR_INVAL
    with pytest.raises(kv.KVError):
        kv.Pool(kv.KVP_HOST_ONLY, 1, 8, num_q_heads=12, num_kv_heads=5)
    with pytest.raises(kv.KVError):
        kv.Pool(kv.KVP_HOST_ONLY, 0, 8)


def test_allocator_matches_model_random_ops(kv):
    rng = np.random.default_rng(0)
    for trial in range(5):
        P = host_pool(kv, nblocks=48, max_seqs=6)
        M = ModelPool(48, 6)
        live = []
        for step in range(300):
            op = rng.integers(0, 5)
            if op == 0 and len(live) < 6:
                s = P.seq_alloc()
                assert s == M.alloc()
                live.append(s)
            elif op == 1 and live:
                s = live[rng.integers(len(live))]
                n = int(rng.integers(0, 200))
                ok = M.reserve(s, n)
                if ok:
                    P.reserve(s, n)
                else:
                    with pytest.raises(kv.KVError) as e:
                        P.reserve(s, n)
                    assert e.value.status == kv.KV_ERR_OOM
            elif op == 2 and live:
                s = live.pop(rng.integers(len(live)))
                P.seq_free(s)
                M.release(s)
            elif op == 3 and live:
                s = live[rng.integers(len(live))]
                free_now = list(M.free)
                k = int(rng.integers(0, min(4, len(free_now)) + 1))
                pick = list(rng.permutation(free_now)[:k]) if k else []
                P.set_blocks(s, pick)
                for b in pick:
                    M.take(int(b))
                    M.seqs[s][1].append(int(b))
            elif op == 4 and live:
                ids = [s for s in live if len(M.seqs[s][1]) * 16 < 4096]
                ids = ids[: int(rng.integers(1, len(ids) + 1))] if ids else []
                need = sum(1 for s in ids if M.seqs[s][0] // 16 >= len(M.seqs[s][1]))
                if ids and need <= len(M.free):
                    P.plan(ids)
                    M.plan(ids)
                    P.commit()
                    M.commit(ids)
            for s in live:
                assert P.blocks(s) == M.seqs[s][1]
                assert P.cur_pos(s) == M.seqs[s][0]
            assert P.free_blocks() == len(M.free)
        P.close()


def test_reserve_is_all_or_nothing(kv):
    P = host_pool(kv, nblocks=10)
    a = P.seq_alloc()
    P.reserve(a, 16 * 8)
    b = P.seq_alloc()
    with pytest.raises(kv.KVError) as e:
        P.reserve(b, 16 * 3)
    assert e.value.status == kv.KV_ERR_OOM
    assert P.blocks(b) == [] and P.free_blocks() == 2
    P.reserve(b, 16 * 2)
    assert P.free_blocks() == 0


def test_set_blocks_validation(kv):
    P = host_pool(kv, nblocks=16)
    a = P.seq_alloc()
    P.set_blocks(a, [5, 3, 9])
    assert P.blocks(a) == [5, 3, 9]
    b = P.seq_alloc()
    for bad in ([3], [1, 1], [16], [-1]):
        with pytest.raises(kv.KVError) as e:
            P.set_blocks(b, bad)
        assert e.value.status == kv.KV_ERR_INVAL
    assert P.blocks(b) == [] and P.free_blocks() == 13


def test_lengths_and_errors(kv):
    P = host_pool(kv, nblocks=16, max_seqs=2, max_seq_len=100)
    a = P.seq_alloc()
    P.reserve(a, 20)
    P.set_cur_pos(a, 32)
    assert P.cur_pos(a) == 32
    with pytest.raises(kv.KVError) as e:
        P.set_cur_pos(a, 33)
    assert e.value.status == kv.KV_ERR_RANGE
    with pytest.raises(kv.KVError) as e:
        P.reserve(a, 101)
    assert e.value.status == kv.KV_ERR_RANGE
    with pytest.raises(kv.KVError) as e:
        P.cur_pos(1)
    assert e.value.status == kv.KV_ERR_BADSEQ
    P.seq_alloc()
    with pytest.raises(kv.KVError) as e:
        P.seq_alloc()
    assert e.value.status == kv.KV_ERR_OOM
    with pytest.raises(kv.KVError) as e:
        P.plan([a, a])
    assert e.value.status == kv.KV_ERR_INVAL
    with pytest.raises(kv.KVError) as e:
        P.commit()
    assert e.value.status == kv.KV_ERR_STATE


def test_plan_pieces_cover_every_block_once_balanced(kv):
    P = host_pool(kv, nblocks=40000, max_seqs=40, max_seq_len=32768)
    P.set_merge_mode(kv.KVP_MERGE_GRID)
    rng = np.random.default_rng(1)
    lens = [0, 1, 15, 16, 17, 255, 256, 257] + list(rng.integers(1, 20000, 24))
    ids = []
    for L in lens:
        s = P.seq_alloc()
        P.reserve(s, int(L))
        P.set_cur_pos(s, int(L))
        ids.append(s)
    P.plan(ids)
    info = P.plan_info()
    items, cs = info["items"], info["cta_start"]
    assert cs[0] == 0 and cs[-1] == info["nitems"] == len(items)
    assert info["grid"] == len(cs) - 1 <= 148 * 3
    # every (slot, head, block) covered exactly once, pieces in flat order
    cover = {}
    for (slot, h, b0, b1) in items:
        assert 0 <= b0 <= b1
        for b in range(b0, b1):
            assert (slot, h, b) not in cover
            cover[(slot, h, b)] = 1
    want = {(i, h, b) for i, L in enumerate(lens) for h in range(2) for b in range(-(-(L + 1) // 16))}
    assert set(cover) == want
    # balance: with PIECE_COST block-equivalents charged per piece, every CTA but the
    # last carries the same cost to within one piece overhead
    cost = [sum(b1 - b0 + PIECE_COST for (_, _, b0, b1) in items[cs[g]:cs[g + 1]]) for g in range(info["grid"])]
    assert max(cost) - min(cost[:-1]) <= PIECE_COST
    assert all(cs[g + 1] - cs[g] <= 64 for g in range(info["grid"]))
    # one new block for every sequence whose next position starts a block
    assert info["npatch"] == sum(1 for L in lens if L % 16 == 0)
    P.commit()
    assert [P.cur_pos(s) for s in ids] == [L + 1 for L in lens]


def _plan_costs(info):
    items, cs = info["items"], info["cta_start"]
    return [sum(b1 - b0 + PIECE_COST for (_, _, b0, b1) in items[cs[g]:cs[g + 1]]) for g in range(info["grid"])]


@pytest.mark.parametrize("lens", [
    [int(x) + 1 for x in np.random.default_rng(1).integers(256, 4097, 32)],   # batch 32, U[256,4096]
    [3, 100, 513],                                                          # one cluster
    [int(min(8192, x)) for x in np.random.default_rng(2).lognormal(np.log(2048.0), 0.8, 200)],
], ids=["batch32", "small", "lognormal200"])
def test_plan_cluster_merge_keeps_segments_in_clusters(kv, lens):
    """Merging inside 8-CTA clusters: every (slot, head, block) once, every
    split segment's pieces in consecutive CTAs of ONE cluster (each later
    piece its CTA's first), and CTA costs close to the grid-wide cut."""
    def mk(mode):
        P = host_pool(kv, nblocks=sum(-(-(L + 1) // 16) for L in lens) + 8, max_seqs=len(lens), max_seq_len=8300)
        P.set_merge_mode(mode)
        ids = []
        for L in lens:
            s = P.seq_alloc()
            P.reserve(s, int(L))
            P.set_cur_pos(s, int(L))
            ids.append(s)
        P.plan(ids)
        return P, P.plan_info()
    Pg, grid_info = mk(kv.KVP_MERGE_GRID)
    assert Pg.plan_clusters() == (0, 1)
    P, info = mk(kv.KVP_MERGE_CLUSTER)
    assert P.plan_clusters() == (1, 1)
    items, cs = info["items"], info["cta_start"]
    assert info["grid"] % 8 == 0 and info["grid"] <= 320
    cover, where = {}, {}
    for g in range(info["grid"]):
        for j, (slot, h, b0, b1) in enumerate(items[cs[g]:cs[g + 1]]):
            for b in range(b0, b1):
                assert (slot, h, b) not in cover
                cover[(slot, h, b)] = 1
            where.setdefault((slot, h), []).append((g, j, b0, b1))
    want = {(i, h, b) for i, L in enumerate(lens) for h in range(2) for b in range(-(-(L + 1) // 16))}
    assert set(cover) == want
    for pieces in where.values():
        gs = [g for g, _, _, _ in pieces]
        assert len({g // 8 for g in gs}) == 1                      # one cluster
        assert gs == list(range(gs[0], gs[0] + len(gs)))           # consecutive CTAs
        assert pieces[0][2] == 0 and all(j == 0 for _, j, _, _ in pieces[1:])
        assert all(pieces[u][3] == pieces[u + 1][2] for u in range(len(pieces) - 1))
    assert all(cs[g + 1] - cs[g] <= 64 for g in range(info["grid"]))
    gmax = max(_plan_costs(grid_info))
    assert max(_plan_costs(info)) <= gmax + gmax // 10 + 4 + PIECE_COST


def test_merge_mode_arguments(kv):
    P = host_pool(kv)
    with pytest.raises(kv.KVError) as e:
        P.plan_clusters()  # no active plan
    assert e.value.status == kv.KV_ERR_STATE
    with pytest.raises(kv.KVError) as e:
        P.set_merge_mode(7)
    assert e.value.status == kv.KV_ERR_INVAL
    # a plan with no split head stays a single grid-wide launch in either mode
    a = P.seq_alloc()
    P.set_merge_mode(kv.KVP_MERGE_CLUSTER)
    P.plan([a])
    assert P.plan_clusters() == (0, 1) and P.plan_info()["grid"] == 1
    P.commit()


def test_plan_small_workload_uses_few_ctas(kv):
    P = host_pool(kv, nblocks=64)
    a = P.seq_alloc()
    P.plan([a])
    info = P.plan_info()
    assert info["grid"] == 1 and info["items"] == [(0, 0, 0, 1), (0, 1, 0, 1)]


def test_plan_ex_no_append_reserves_nothing(kv):
    P = host_pool(kv, nblocks=8)
    a = P.seq_alloc()
    P.reserve(a, 32)
    P.set_cur_pos(a, 32)
    P.plan([a], rope_pos=[1000], append=[0])
    assert P.plan_info()["npatch"] == 0 and P.free_blocks() == 6
    P.commit()
    assert P.cur_pos(a) == 32
    with pytest.raises(kv.KVError) as e:
        P.plan([a], rope_pos=[4096], append=[0])  # outside the table
    assert e.value.status == kv.KV_ERR_RANGE


def test_plan_oom_changes_nothing(kv):
    P = host_pool(kv, nblocks=2)
    a, b, c = P.seq_alloc(), P.seq_alloc(), P.seq_alloc()
    P.plan([a, b])
    P.commit()
    assert P.free_blocks() == 0
    with pytest.raises(kv.KVError) as e:
        P.plan([c])
    assert e.value.status == kv.KV_ERR_OOM
    assert P.blocks(c) == [] and P.cur_pos(c) == 0


def test_device_calls_refused_on_host_only_pool(kv):
    P = host_pool(kv)
    a = P.seq_alloc()
    P.plan([a])
    with pytest.raises(kv.KVError) as e:
        kv.call("attn_decode_append", P.h, 0, 8, 8, 8, 8, None)  # pointers are never touched
    assert e.value.status in (kv.KV_ERR_STATE, kv.KV_ERR_INVAL)


def test_nccl_unique_id_and_argument_checks(kv):
    """The NCCL communicator's set-up calls that need no GPU: a unique id
    (NCCL loaded at run time) and the argument checks of kvn_create."""
    import ctypes as C
    L = kv.load()
    uid = (C.c_char * kv.KVN_UNIQUE_ID_BYTES)()
    if L.kvn_unique_id(uid) != kv.KV_OK:
        pytest.skip("NCCL not loadable here: " + L.kv_last_error().decode())
    assert any(bytes(uid))
    c = kv._vp()
    assert L.kvn_create(0, 2, 2, uid, 10, C.byref(c)) == kv.KV_ERR_INVAL   # rank outside the world
    assert L.kvn_create(0, 0, 1, uid, 0, C.byref(c)) == kv.KV_ERR_INVAL    # no rows
    assert L.kvn_create(0, 0, 1, None, 10, C.byref(c)) == kv.KV_ERR_INVAL  # no id
    assert L.kvn_destroy(None) == kv.KV_OK
