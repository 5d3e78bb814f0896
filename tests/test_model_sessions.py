"""Sessions, multi-turn, batch and async generation of the device model (the
interfaces the reference plans on top of LLMEngine, docs/api_requirements.md:
90-151) against one-session greedy decoding of the same model.

A batched step runs one forward over every session (shared projections, one
planned decode-attention launch for the one-token rows, prompt chunks beside
them), so its rounding differs from a one-session forward's; each generated
id must therefore be the one-session greedy choice, or a near-tie of it
(within 2e-3 of the largest |logit|), when the same tokens are replayed
teacher-forced on a fresh session.
"""
from __future__ import annotations

import threading

import numpy as np
import pytest
import torch

from conftest import load_pkg

SMALL = dict(hidden=256, layers=2, q_heads=2, kv_heads=1, head_dim=128, intermediate=512, vocab=1000,
             rms_eps=1e-6, rope_theta=1e6, max_position=512)
NEAR = 2e-3


def q2():
    load_pkg()
    import importlib
    return importlib.import_module("rk3588_npu_b200.qwen2")


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def model():
    need_gpu()
    m = q2()
    M = m.Model(0, SMALL, max_sessions=8)
    for name, a in m.synth_weights(SMALL, seed=21):
        M.set_tensor(name, a)
    yield M
    M.close()


def prompt(n, seed):
    return [int(x) for x in np.random.default_rng(seed).integers(0, SMALL["vocab"], n)]


def replay_consistent(M, tokens_before, ids):
    """Teacher-forced replay on a fresh session: every id is the greedy choice
    (or a near-tie) after the tokens before it."""
    s = M.create_session()
    try:
        logits, am = M.forward_session(s, tokens_before)
        for t in ids:
            if t != am:
                assert logits[t] >= logits.max() - NEAR * np.abs(logits).max(), (t, am)
            logits, am = M.forward_session(s, [t])
    finally:
        M.destroy_session(s)


@pytest.mark.gpu
def test_session_lifecycle():
    need_gpu()
    m = q2()
    kv = load_pkg()
    M = m.Model(0, SMALL, max_sessions=3)
    assert M.session_exists(0) and not M.session_exists(1)
    a, b = M.create_session(), M.create_session()
    assert {a, b} == {1, 2}
    with pytest.raises(kv.KVError) as e:
        M.create_session()
    assert e.value.status == kv.KV_ERR_OOM
    M.destroy_session(a)
    assert not M.session_exists(a)
    assert M.create_session() == a
    with pytest.raises(kv.KVError) as e:
        M.destroy_session(7)
    assert e.value.status == kv.KV_ERR_BADSEQ
    with pytest.raises(kv.KVError) as e:
        M.forward_session(2, [1])
    assert e.value.status == kv.KV_ERR_STATE  # weights not set
    M.close()


@pytest.mark.gpu
def test_generate_batch_matches_one_session_greedy(model):
    M = model
    sessions = [M.create_session() for _ in range(4)]
    prompts = [prompt(5, 1), prompt(40, 2), prompt(300, 3), prompt(1, 4)]  # 300: two 256-token chunks
    reqs = [dict(session=s, input_ids=p, max_new_tokens=16) for s, p in zip(sessions, prompts)]
    out = M.generate_batch(reqs)
    for s, p, (ids, res) in zip(sessions, prompts, out):
        assert res["status"] == 0 and res["n_out"] == 16 and len(ids) == 16
        assert res["prefill_tokens"] == len(p) and res["decode_tokens"] == 16
        assert M.session_len(s) == len(p) + 16  # every emitted id was forwarded
        replay_consistent(M, p, ids)
    for s in sessions:
        M.destroy_session(s)


@pytest.mark.gpu
def test_generate_batch_stops_and_repetition(model):
    """Same request alone on a fresh session each time (same rounding), with
    and without a stop token / repetition window."""
    M = model

    def run(**kw):
        s = M.create_session()
        try:
            return M.generate_batch([dict(session=s, input_ids=prompt(9, 5), max_new_tokens=24, **kw)])[0]
        finally:
            M.destroy_session(s)

    free, _ = run()
    stop = free[6]
    cut = free.index(stop)
    a, ra = run(stop_tokens=(stop,))
    assert ra["hit_stop"] == 1 and a == free[:cut]
    # repetition: checked after each push (llm_engine.cpp:83-90)
    w = 4
    n = next((k for k in range(w, len(free) + 1)
              if any(k - w - p >= 0 and all(free[i] == free[i - p] for i in range(k - w, k))
                     for p in range(1, w // 2 + 1))), len(free))
    b, rb = run(repetition_window=w)
    assert b == free[:n] and rb["hit_repetition"] == int(n < len(free))


@pytest.mark.gpu
def test_multi_turn_session_continues_its_cache(model):
    M = model
    s = M.create_session()
    p1, p2 = prompt(30, 6), prompt(12, 7)
    ids1, r1 = M.generate_session(s, p1, 8)
    assert M.session_len(s) == 30 + 8
    ids2, r2 = M.generate_session(s, p2, 8)
    assert M.session_len(s) == 30 + 8 + 12 + 8 and r2["prefill_tokens"] == 12
    replay_consistent(M, p1, ids1)
    replay_consistent(M, p1 + ids1 + p2, ids2)
    M.destroy_session(s)


@pytest.mark.gpu
def test_async_submit_wait_and_cancel(model):
    M = model
    kv = load_pkg()
    sessions = [M.create_session() for _ in range(3)]
    prompts = [prompt(7, 8), prompt(64, 9), prompt(2, 10)]
    seen = {s: [] for s in sessions}
    lock = threading.Lock()

    def on_token(session, step, tok, ms):
        with lock:
            seen[session].append((step, tok))

    jobs = [M.submit(s, p, 12, on_token=on_token) for s, p in zip(sessions, prompts)]
    for s, p, j in zip(sessions, prompts, jobs):
        ids, res = M.wait(j)
        assert res["status"] == 0 and len(ids) == 12
        assert seen[s] == list(enumerate(ids))  # TokenCallback: (step, id) after each forward
        replay_consistent(M, p, ids)
    with pytest.raises(kv.KVError) as e:
        M.wait(jobs[0])  # retired
    assert e.value.status == kv.KV_ERR_INVAL
    # cancel: ends at the next step (or the request finished first)
    j = M.submit(sessions[0], prompt(3, 11), 200)
    M.cancel(sessions[0])
    ids, res = M.wait(j, timeout_ms=60000)
    assert res["cancelled"] == 1 or len(ids) == 200
    M.forward_session(sessions[0], [1])  # the session is free again
    for s in sessions:
        M.destroy_session(s)


@pytest.mark.gpu
def test_int8_kv_model_tracks_fp16_cache():
    """The model with an INT8 KV cache (qw2_create_kv, KV_I8): the same prompt
    (one chunk) and teacher-forced decode steps as the fp16-cache model; the
    logits differ only by the cache's quantisation error (not at all would
    mean the INT8 path did not run)."""
    need_gpu()
    m = q2()
    models = [m.Model(0, SMALL, kv_dtype=dt) for dt in (0, 2)]
    for M in models:
        for name, a in m.synth_weights(SMALL, seed=21):
            M.set_tensor(name, a)
    p = prompt(40, 12)
    follow = prompt(8, 13)
    worst, moved = 0.0, False
    for toks in [p] + [[t] for t in follow]:
        (l16, _), (l8, _) = [M.forward_session(0, toks) for M in models]
        d = float(np.abs(l8 - l16).max() / np.abs(l16).max())
        worst = max(worst, d)
        moved = moved or d > 0.0
    assert moved and worst <= 5e-2, worst
    for M in models:
        assert M.session_len(0) == 48
        M.close()
