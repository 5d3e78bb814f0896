"""qwen2_chat: the reference's line-protocol REPL (worker/src/chat_main.cpp:
4-23) on the device model.  On a reduced model written as model.safetensors
+ config.json, every request's "OK ..." line must equal LLMEngine::generate's
ids from the Python binding (single turn: the cache cleared first; stop ids
151645/151643, repetition window 6)."""
from __future__ import annotations

import json
import os
import subprocess

import numpy as np
import pytest
import torch

from conftest import ROOT, load_pkg

CHAT = os.path.join(ROOT, "rk3588-npu_b200", "bin", "qwen2_chat")
SMALL = dict(hidden=256, layers=2, q_heads=2, kv_heads=1, head_dim=128, intermediate=512, vocab=1000,
             rms_eps=1e-6, rope_theta=1e6, max_position=128)


def q2():
    load_pkg()
    import importlib
    return importlib.import_module("rk3588_npu_b200.qwen2")


def test_chat_usage_without_arguments():
    if not os.path.exists(CHAT):
        pytest.skip("front end not built")
    r = subprocess.run([CHAT], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "Usage" in r.stderr


@pytest.mark.gpu
def test_chat_protocol_matches_engine(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    m = q2()
    d = str(tmp_path)
    m.write_safetensors(os.path.join(d, "model.safetensors"), m.tensor_specs(SMALL), m.synth_weights(SMALL, seed=31))
    json.dump({"hidden_size": 256, "num_hidden_layers": 2, "num_attention_heads": 2, "num_key_value_heads": 1,
               "intermediate_size": 512, "vocab_size": 1000, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0,
               "max_position": 128}, open(os.path.join(d, "config.json"), "w"))
    prompts = [[int(x) for x in np.random.default_rng(s).integers(0, 1000, n)] for s, n in ((1, 5), (2, 33), (3, 1))]
    lines = [" ".join(map(str, prompts[0])), "", "RESET", "not ids", " ".join(map(str, prompts[1])) + "  ",
             " ".join(map(str, prompts[2])), "EXIT", "7 8 9"]
    r = subprocess.run([CHAT, d, "9"], input="\n".join(lines) + "\n", capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    out = r.stdout.strip().split("\n")
    assert out[0] == "READY"
    assert out[2] == "OK" and out[3] == "ERR empty_input" and len(out) == 6  # nothing after EXIT
    M = m.Model(0, SMALL)
    for name, a in m.synth_weights(SMALL, seed=31):
        M.set_tensor(name, a)
    for line, p in zip((out[1], out[4], out[5]), prompts):
        M.reset()
        ids = M.generate(p, 9, stop_tokens=(151645, 151643), repetition_window=6)
        assert line == "OK" + "".join(f" {i}" for i in ids)
    M.close()
