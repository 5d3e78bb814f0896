"""Placement of requests onto GPUs (kvs_* C ABI): least resident KV blocks
among GPUs with room, ties to the lowest index, all-or-nothing errors.
Checked against a Python model of the rule on random operation streams."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import load_pkg


class ModelSched:
    """The placement rule restated in Python (test model)."""

    def __init__(self, caps, bt=16):
        self.caps, self.bt = list(caps), bt
        self.res = [0] * len(caps)
        self.cnt = [0] * len(caps)
        self.reqs = {}

    def blocks(self, tokens):
        return -(-tokens // self.bt)

    def place(self, r, tokens):
        if r in self.reqs:
            return "inval"
        need = self.blocks(tokens)
        cands = [g for g in range(len(self.caps)) if self.res[g] + need <= self.caps[g]]
        if not cands:
            return "oom"
        g = min(cands, key=lambda i: (self.res[i], i))
        self.res[g] += need
        self.cnt[g] += 1
        self.reqs[r] = [g, need]
        return g

    def resize(self, r, tokens):
        if r not in self.reqs:
            return "badseq"
        g, have = self.reqs[r]
        need = self.blocks(tokens)
        if need > have and self.res[g] + need - have > self.caps[g]:
            return "oom"
        self.res[g] += need - have
        self.reqs[r][1] = need
        return None

    def release(self, r):
        if r not in self.reqs:
            return "badseq"
        g, have = self.reqs.pop(r)
        self.res[g] -= have
        self.cnt[g] -= 1
        return None


def test_least_loaded_and_ties():
    kv = load_pkg()
    S = kv.Scheduler([100, 100, 50])
    assert S.place(1, 160) == 0      # all empty: lowest index
    assert S.place(2, 16) == 1
    assert S.place(3, 17) == 2       # 2 blocks on GPU 2 (0 resident)
    assert S.load(0) == (10, 1) and S.load(1) == (1, 1) and S.load(2) == (2, 1)
    assert S.place(4, 1) == 1        # GPU 1 holds 1 block, the fewest
    assert S.gpu_of(3) == 2
    S.release(1)
    assert S.load(0) == (0, 0)
    assert S.place(5, 48 * 16) == 0  # 48 blocks: GPU 0 is now emptiest
    with pytest.raises(kv.KVError) as e:
        S.place(6, 200 * 16)         # fits nowhere
    assert e.value.status == kv.KV_ERR_OOM
    with pytest.raises(kv.KVError) as e:
        S.place(5, 1)                # already placed
    assert e.value.status == kv.KV_ERR_INVAL
    with pytest.raises(kv.KVError) as e:
        S.release(99)
    assert e.value.status == kv.KV_ERR_BADSEQ
    S.resize(4, 64)                  # 1 -> 4 blocks on GPU 1
    assert S.load(1) == (5, 2)
    with pytest.raises(kv.KVError) as e:
        S.resize(4, 101 * 16)
    assert e.value.status == kv.KV_ERR_OOM
    assert S.load(1) == (5, 2)       # unchanged by the failed resize
    S.close()


def test_skips_full_gpu():
    kv = load_pkg()
    S = kv.Scheduler([4, 100])
    assert S.place(1, 64) == 0       # 4 blocks: GPU 0 now full
    assert S.place(2, 16) == 1
    assert S.place(3, 1) == 1        # GPU 1 holds fewer blocks (1 < 4)
    S.release(2)
    S.release(3)
    assert S.place(4, 16) == 1       # GPU 1 empty (0 < 4)
    S.close()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_streams_match_model(seed):
    kv = load_pkg()
    rng = np.random.default_rng(seed)
    caps = [int(c) for c in rng.integers(50, 400, int(rng.integers(1, 9)))]
    S, M = kv.Scheduler(caps), ModelSched(caps)
    status = {kv.KV_ERR_OOM: "oom", kv.KV_ERR_INVAL: "inval", kv.KV_ERR_BADSEQ: "badseq"}
    live = []
    for op in range(3000):
        kind = rng.integers(0, 10)
        if kind < 5 or not live:
            r = int(rng.integers(0, 10**12)) if rng.random() < 0.98 or not live else live[0]
            tokens = int(rng.integers(0, 2000))
            want = M.place(r, tokens)
            try:
                got = S.place(r, tokens)
            except kv.KVError as e:
                got = status[e.status]
            assert got == want, (op, r, tokens)
            if isinstance(want, int):
                live.append(r)
        elif kind < 8:
            r = live[int(rng.integers(0, len(live)))]
            tokens = int(rng.integers(0, 3000))
            want = M.resize(r, tokens)
            try:
                S.resize(r, tokens)
                got = None
            except kv.KVError as e:
                got = status[e.status]
            assert got == want, (op, r, tokens)
        else:
            r = live.pop(int(rng.integers(0, len(live))))
            assert M.release(r) is None
            S.release(r)
        for g in range(len(caps)):
            assert S.load(g) == (M.res[g], M.cnt[g])
    for r in live:
        assert S.gpu_of(r) == M.reqs[r][0]
    S.close()
