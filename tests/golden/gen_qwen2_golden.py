"""Generate tests/golden/qwen2_greedy.npz: the reference's own Qwen2 model and
engine (oracle/_ref/libqwen2ref.so: Qwen2Model + LLMEngine compiled from the
reference sources with a CPU stand-in for the NPU linear) run on the seeded
random-init weights and prompt of the 1.5B config:

  weights  rk3588-npu_b200/qwen2.py synth_weights(seed=0): N(0, 0.02) fp32
           matrices/embedding/biases, RMSNorm weights 1, written as an F32
           model.safetensors that the reference loader converts to fp16;
  prompt   128 ids uniform in [0, 151936) from default_rng(0);
  run      LLMEngine::generate, 128 new tokens, no stop tokens, repetition
           window 0 (llm_engine.cpp:53-103), and the same loop step by step
           through Qwen2Model::forward to record logits.

Stored: prompt, output ids, the prefill logits (fp16 bit patterns: every
logit is an fp16 value widened to fp32) and, for every decode step, the 64
largest logits with their ids.  Also the model's rounding-noise floor: the
same reference run again with only the stand-in linear's fp32 sums taken in
reverse k order (ref_set_sum_order(1)), fed the same tokens; its relative
logit difference from the first run (prefill: max |diff| / max |ref| over the
vocabulary; each decode step: over the stored top 64) is what any other
summation order, a parallel one included, must be expected to meet.  The
reversed-sum run's teacher-forced argmaxes and its own free-running greedy
stream are stored too: where the reference's top-2 margin is inside that
floor, its own greedy choice flips with the summation order.

Run here (needs the reference sources for `make -C oracle model`):
    python tests/golden/gen_qwen2_golden.py [--dir /tmp/qwen2_synth_s0]
"""
import argparse
import ctypes as C
import importlib.util
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def load_synth():
    """The package's qwen2 module (its directory name has a hyphen, so it is
    loaded by path as `rk3588_npu_b200`)."""
    import importlib
    name = "rk3588_npu_b200"
    pkg_dir = os.path.join(ROOT, "rk3588-npu_b200")
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(pkg_dir, "__init__.py"),
                                                      submodule_search_locations=[pkg_dir])
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return importlib.import_module(name + ".qwen2")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dir", default="/tmp/qwen2_synth_s0")
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    args = ap.parse_args()
    q2 = load_synth()
    cfg = q2.QWEN2_1_5B
    os.makedirs(args.dir, exist_ok=True)
    st = os.path.join(args.dir, "model.safetensors")
    if not os.path.exists(st):
        t = time.time()
        q2.write_safetensors(st, q2.tensor_specs(cfg), q2.synth_weights(cfg, seed=0))
        print(f"wrote {st} in {time.time() - t:.1f}s", flush=True)
    prompt = q2.synth_prompt(128, cfg["vocab"], seed=0)

    so = os.path.join(ROOT, "oracle", "_ref", "libqwen2ref.so")
    R = C.CDLL(so)
    R.ref_qwen2_load.restype = C.c_void_p
    R.ref_qwen2_load.argtypes = [C.c_char_p]
    R.ref_qwen2_forward.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.c_int, C.c_void_p, C.c_int]
    R.ref_greedy_sample.argtypes = [C.c_void_p, C.c_int]
    R.ref_qwen2_free.argtypes = [C.c_void_p]
    R.ref_engine_load.restype = C.c_void_p
    R.ref_engine_load.argtypes = [C.c_char_p]
    R.ref_engine_generate.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.c_int, C.c_int, C.POINTER(C.c_int),
                                      C.c_int, C.c_int, C.POINTER(C.c_int), C.c_int]
    R.ref_engine_free.argtypes = [C.c_void_p]
    R.ref_set_sum_order.argtypes = [C.c_int]
    R.ref_set_threads(args.threads)
    V = cfg["vocab"]

    t = time.time()
    m = R.ref_qwen2_load(args.dir.encode())
    assert m, "reference load failed"
    print(f"model loaded in {time.time() - t:.1f}s", flush=True)
    logits = np.empty(V, np.float32)

    def fwd(ids):
        a = (C.c_int * len(ids))(*[int(x) for x in ids])
        assert R.ref_qwen2_forward(m, a, len(ids), logits.ctypes.data_as(C.c_void_p), V) == V
        return R.ref_greedy_sample(logits.ctypes.data_as(C.c_void_p), V)

    t = time.time()
    nxt = fwd(prompt)
    prefill_logits = logits.copy()
    print(f"prefill {time.time() - t:.1f}s", flush=True)
    out, top_idx, top_val = [], [], []
    t = time.time()
    for step in range(args.steps):  # llm_engine.cpp:76-98 without stops / repetition check
        out.append(nxt)
        nxt = fwd([nxt])
        o = np.argsort(-logits, kind="stable")[:64]
        top_idx.append(o.astype(np.int32))
        top_val.append(logits[o].copy())
    print(f"{args.steps} decode steps {time.time() - t:.1f}s", flush=True)
    R.ref_qwen2_free(m)

    e = R.ref_engine_load(args.dir.encode())
    assert e
    ids = (C.c_int * len(prompt))(*[int(x) for x in prompt])
    eo = (C.c_int * args.steps)()
    k = R.ref_engine_generate(e, ids, len(prompt), args.steps, None, 0, 0, eo, args.steps)
    R.ref_engine_free(e)
    eng = [eo[i] for i in range(k)]
    assert eng == out, "LLMEngine::generate and the forward loop disagree"

    # rounding-noise floor: the same model, sums in reverse k order, same tokens
    R.ref_set_sum_order(1)
    m = R.ref_qwen2_load(args.dir.encode())
    assert m
    fwd(prompt)
    den = np.abs(prefill_logits.astype(np.float64)).max()
    floor_prefill = float(np.abs(logits.astype(np.float64) - prefill_logits).max() / den)
    argmax_reversed = [int(np.argmax(logits))]
    floor_steps = []
    for step, tok in enumerate(out):
        argmax_reversed.append(fwd([tok]))
        val = top_val[step].astype(np.float64)
        floor_steps.append(float(np.abs(logits[top_idx[step]] - val).max() / np.abs(val).max()))
    R.ref_qwen2_free(m)
    # the free-running greedy stream of the reversed-sum reference
    e = R.ref_engine_load(args.dir.encode())
    assert e
    eo = (C.c_int * args.steps)()
    k = R.ref_engine_generate(e, ids, len(prompt), args.steps, None, 0, 0, eo, args.steps)
    R.ref_engine_free(e)
    stream_reversed = [eo[i] for i in range(k)]
    R.ref_set_sum_order(0)
    same = next((i for i, (a, b) in enumerate(zip(stream_reversed, out)) if a != b), None)
    print(f"reversed-sum stream first differs at {same}", flush=True)
    print(f"noise floor: prefill {floor_prefill:.3g}, decode max {max(floor_steps):.3g}", flush=True)

    bits = prefill_logits.view(np.uint32)
    # every logit is an fp16 value (f16_to_f32 of the lm_head output): keep its fp16 bits
    h16 = ((bits >> 16) & 0x8000) | ((((bits >> 23) & 0xFF).astype(np.int64) - 112).clip(0, 31).astype(np.uint32) << 10) \
        | ((bits & 0x7FFFFF) >> 13)
    h16 = np.where((bits & 0x7FFFFFFF) == 0, (bits >> 16) & 0x8000, h16).astype(np.uint16)
    dst = os.path.join(ROOT, "tests", "golden", "qwen2_greedy.npz")
    np.savez_compressed(dst, prompt=prompt, output_ids=np.array(out, np.int32), prefill_logits_f16=h16,
                        top_idx=np.stack(top_idx), top_val=np.stack(top_val).astype(np.float32),
                        weights_seed=np.int32(0), prompt_seed=np.int32(0), std=np.float32(0.02),
                        floor_prefill=np.float64(floor_prefill), floor_steps=np.array(floor_steps, np.float64),
                        argmax_reversed=np.array(argmax_reversed[:-1], np.int32),
                        stream_reversed=np.array(stream_reversed, np.int32))
    print("wrote", dst, "first ids", out[:8])


if __name__ == "__main__":
    main()
