"""Qwen2 model on the device: host binding of the ``qw2_*`` C ABI (include/qwen2_engine.h).

Mirrors the reference's model and engine:
  Qwen2Model  worker/include/model/qwen2_model.h:23-56   -> Model (load / reset / forward)
  LLMEngine   worker/include/api/llm_engine.h            -> Model.generate
  Qwen2Config worker/include/core/model_config.h:8-23     -> QWEN2_1_5B

``synth_weights`` produces the seeded random-init weights used when no
checkpoint is available: every projection matrix, the embedding and every bias
drawn N(0, 0.02) in fp32 from ``numpy.random.default_rng(seed)`` in the
reference's load order (qwen2_model.cpp:70-112), the RMSNorm weights 1.  The
loader rules of weight_loader.cpp:164-235 then apply (fp32 matrices become
fp16 by the truncating f32_to_f16).
"""
from __future__ import annotations

import ctypes as C
import json
import struct

import numpy as np

from . import KVError, _check, load

QW2_F16, QW2_BF16, QW2_F32 = 0, 1, 2

QWEN2_1_5B = dict(hidden=1536, layers=28, q_heads=12, kv_heads=2, head_dim=128, intermediate=8960,
                  vocab=151936, rms_eps=1e-6, rope_theta=1e6, max_position=512)


class Qw2Config(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("q_heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("intermediate", C.c_int), ("vocab", C.c_int),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float), ("max_position", C.c_int)]


def tensor_specs(cfg: dict = QWEN2_1_5B):
    """(name, shape, init) in the reference's load order; init is "normal" or "ones"."""
    H, kvd, IS, V = cfg["hidden"], cfg["kv_heads"] * cfg["head_dim"], cfg["intermediate"], cfg["vocab"]
    specs = [("model.embed_tokens.weight", (V, H), "normal")]
    for i in range(cfg["layers"]):
        p = f"model.layers.{i}."
        specs += [
            (p + "input_layernorm.weight", (H,), "ones"),
            (p + "self_attn.q_proj.weight", (H, H), "normal"),
            (p + "self_attn.q_proj.bias", (H,), "normal"),
            (p + "self_attn.k_proj.weight", (kvd, H), "normal"),
            (p + "self_attn.k_proj.bias", (kvd,), "normal"),
            (p + "self_attn.v_proj.weight", (kvd, H), "normal"),
            (p + "self_attn.v_proj.bias", (kvd,), "normal"),
            (p + "self_attn.o_proj.weight", (H, H), "normal"),
            (p + "post_attention_layernorm.weight", (H,), "ones"),
            (p + "mlp.gate_proj.weight", (IS, H), "normal"),
            (p + "mlp.up_proj.weight", (IS, H), "normal"),
            (p + "mlp.down_proj.weight", (H, IS), "normal"),
        ]
    specs.append(("model.norm.weight", (H,), "ones"))
    return specs


def synth_weights(cfg: dict = QWEN2_1_5B, seed: int = 0, std: float = 0.02):
    """Yield (name, fp32 ndarray) for every tensor, seeded, in load order."""
    rng = np.random.default_rng(seed)
    scale = np.float32(std)
    for name, shape, init in tensor_specs(cfg):
        if init == "ones":
            yield name, np.ones(shape, np.float32)
        else:
            a = rng.standard_normal(shape, dtype=np.float32)
            a *= scale
            yield name, a


def synth_prompt(n: int = 128, vocab: int = QWEN2_1_5B["vocab"], seed: int = 0) -> np.ndarray:
    """n token ids uniform in [0, vocab) from default_rng(seed)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.int32)


def f32_to_f16_trunc(a: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bits by the reference's truncating f32_to_f16
    (worker/include/core/half.h:24-32): mantissa truncated, exponent <= 0 ->
    signed zero, >= 31 -> signed infinity."""
    x = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    sign = ((x >> 16) & 0x8000).astype(np.uint16)
    e = ((x >> 23) & 0xFF).astype(np.int32) - 112
    mant = ((x & 0x7FFFFF) >> 13).astype(np.uint16)
    out = sign | (np.clip(e, 0, 31).astype(np.uint16) << 10) | mant
    out = np.where(e <= 0, sign, out)
    return np.where(e >= 31, sign | np.uint16(0x7C00), out).astype(np.uint16)


def write_safetensors(path: str, specs, tensors, dtype: str = "F32") -> None:
    """Write a safetensors file in the format weight_loader.cpp:77-153 parses
    (8-byte header length, JSON header, data).  `specs` gives (name, shape,
    ...) in file order; `tensors` yields (name, fp32 ndarray) in the same
    order (streamed, never all in memory).  dtype "F16" stores matrices as
    fp16 by the loader's own F32 -> F16 rule (so the loaded model is the same)
    and keeps vectors F32."""
    header, off = {}, 0
    kinds = []
    for sp in specs:
        dt = "F16" if dtype == "F16" and len(sp[1]) == 2 else "F32"
        n = int(np.prod(sp[1])) * (2 if dt == "F16" else 4)
        header[sp[0]] = {"dtype": dt, "shape": list(sp[1]), "data_offsets": [off, off + n]}
        kinds.append(dt)
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for (name, a), sp, dt in zip(tensors, specs, kinds):
            assert name == sp[0] and a.shape == tuple(sp[1]), name
            f.write(f32_to_f16_trunc(a).tobytes() if dt == "F16" else np.ascontiguousarray(a, np.float32).tobytes())


class Qw2GenConfig(C.Structure):
    _fields_ = [("max_new_tokens", C.c_int), ("repetition_window", C.c_int), ("stop_tokens", C.POINTER(C.c_int)),
                ("n_stop", C.c_int)]


class Qw2Result(C.Structure):
    _fields_ = [("n_out", C.c_int), ("prefill_tokens", C.c_int), ("decode_tokens", C.c_int),
                ("prefill_ms", C.c_float), ("decode_ms", C.c_float), ("hit_stop", C.c_int),
                ("hit_repetition", C.c_int), ("cancelled", C.c_int), ("status", C.c_int)]

    def as_dict(self) -> dict:
        return {f: getattr(self, f) for f, _ in self._fields_}


TOKEN_CB = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float)


class Qw2Request(C.Structure):
    _fields_ = [("session", C.c_int), ("input_ids", C.POINTER(C.c_int)), ("n_input", C.c_int),
                ("cfg", Qw2GenConfig), ("out_ids", C.POINTER(C.c_int)), ("out_cap", C.c_int),
                ("on_token", TOKEN_CB), ("user", C.c_void_p)]


_SIGS = {
    "qw2_config_default": [C.POINTER(Qw2Config)],
    "qw2_create_sessions": [C.c_int, C.POINTER(Qw2Config), C.c_int, C.POINTER(C.c_void_p)],
    "qw2_create_kv": [C.c_int, C.POINTER(Qw2Config), C.c_int, C.c_int, C.POINTER(C.c_void_p)],
    "qw2_session_create": [C.c_void_p, C.POINTER(C.c_int)],
    "qw2_session_destroy": [C.c_void_p, C.c_int],
    "qw2_session_exists": [C.c_void_p, C.c_int, C.POINTER(C.c_int)],
    "qw2_session_len": [C.c_void_p, C.c_int, C.POINTER(C.c_int)],
    "qw2_session_seq": [C.c_void_p, C.c_int, C.POINTER(C.c_int)],
    "qw2_forward_session": [C.c_void_p, C.c_int, C.POINTER(C.c_int), C.c_int, C.c_void_p, C.POINTER(C.c_int)],
    "qw2_generate_session": [C.c_void_p, C.c_int, C.POINTER(C.c_int), C.c_int, C.POINTER(Qw2GenConfig),
                             C.POINTER(C.c_int), C.c_int, C.POINTER(Qw2Result)],
    "qw2_generate_batch": [C.c_void_p, C.c_int, C.POINTER(Qw2Request), C.POINTER(Qw2Result)],
    "qw2_submit": [C.c_void_p, C.POINTER(Qw2Request), C.POINTER(C.c_int)],
    "qw2_wait": [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int), C.c_int, C.POINTER(Qw2Result)],
    "qw2_cancel": [C.c_void_p, C.c_int],
    "qw2_create": [C.c_int, C.POINTER(Qw2Config), C.POINTER(C.c_void_p)],
    "qw2_destroy": [C.c_void_p],
    "qw2_set_tensor": [C.c_void_p, C.c_char_p, C.c_int, C.POINTER(C.c_longlong), C.c_int, C.c_void_p],
    "qw2_load_safetensors": [C.c_void_p, C.c_char_p],
    "qw2_ready": [C.c_void_p],
    "qw2_reset": [C.c_void_p],
    "qw2_cur_pos": [C.c_void_p, C.POINTER(C.c_int)],
    "qw2_forward": [C.c_void_p, C.POINTER(C.c_int), C.c_int, C.c_void_p, C.POINTER(C.c_int)],
    "qw2_generate": [C.c_void_p, C.POINTER(C.c_int), C.c_int, C.c_int, C.POINTER(C.c_int), C.c_int, C.c_int,
                     C.POINTER(C.c_int), C.c_int, C.POINTER(C.c_int)],
    "qw2_kv_pool": [C.c_void_p, C.POINTER(C.c_void_p)],
    "qw2_weight_bytes": [C.c_void_p, C.POINTER(C.c_longlong)],
    "qw2_set_stream": [C.c_void_p, C.c_void_p],
    "qw2_set_exact": [C.c_void_p, C.c_int],
}


def _lib():
    L = load()
    if not getattr(L, "_qw2_bound", False):
        for n, a in _SIGS.items():
            f = getattr(L, n)
            f.argtypes = a
            f.restype = C.c_int
        L._qw2_bound = True
    return L


def _ints(xs):
    a = (C.c_int * max(1, len(xs)))(*[int(x) for x in xs])
    return a


class Model:
    """Qwen2Model + LLMEngine on one GPU (weights, KV pool and scratch on the
    device), with up to `max_sessions` sessions sharing the weights.
    kv_dtype: the KV cache's element type (0 fp16 as in the reference, 1
    bf16, 2 INT8 codes + per-row scales)."""

    def __init__(self, device: int = 0, cfg: dict = QWEN2_1_5B, max_sessions: int = 1, kv_dtype: int = 0):
        self.L = _lib()
        c = Qw2Config(**cfg)
        h = C.c_void_p()
        _check(self.L.qw2_create_kv(device, C.byref(c), max_sessions, kv_dtype, C.byref(h)), "qw2_create_kv")
        self.h = h
        self.cfg = dict(cfg)
        self._keep = {}  # ctypes objects an async job still points at

    def close(self) -> None:
        if self.h:
            self.L.qw2_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, name: str, a: np.ndarray) -> None:
        """One weight from host memory: fp32, or fp16/bf16 given as a uint16 array
        with dtype QW2_F16/QW2_BF16 via set_tensor_raw."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        self.set_tensor_raw(name, QW2_F32, a)

    def set_tensor_raw(self, name: str, dtype: int, a: np.ndarray) -> None:
        a = np.ascontiguousarray(a)
        shape = (C.c_longlong * max(1, a.ndim))(*a.shape)
        _check(self.L.qw2_set_tensor(self.h, name.encode(), dtype, shape, a.ndim, a.ctypes.data_as(C.c_void_p)),
               "qw2_set_tensor")

    def load_synthetic(self, seed: int = 0) -> None:
        for name, a in synth_weights(self.cfg, seed):
            self.set_tensor(name, a)
        _check(self.L.qw2_ready(self.h), "qw2_ready")

    def load_safetensors(self, path: str) -> None:
        _check(self.L.qw2_load_safetensors(self.h, path.encode()), "qw2_load_safetensors")

    def reset(self) -> None:
        _check(self.L.qw2_reset(self.h), "qw2_reset")

    def set_exact(self, on: bool) -> None:
        """qw2_set_exact: forwards in the reference's operation order (a parity
        mode whose logits match the reference's bit for bit wherever the C
        library's expf is correctly rounded; far slower)."""
        _check(self.L.qw2_set_exact(self.h, int(on)), "qw2_set_exact")

    def cur_pos(self) -> int:
        p = C.c_int()
        _check(self.L.qw2_cur_pos(self.h, C.byref(p)), "qw2_cur_pos")
        return p.value

    def forward(self, tokens) -> tuple[np.ndarray, int]:
        """Qwen2Model::forward: logits of the last token (fp32 [vocab]) and their
        greedy argmax."""
        ids = _ints(tokens)
        logits = np.empty(self.cfg["vocab"], np.float32)
        am = C.c_int()
        _check(self.L.qw2_forward(self.h, ids, len(tokens), logits.ctypes.data_as(C.c_void_p), C.byref(am)),
               "qw2_forward")
        return logits, am.value

    def generate(self, prompt, max_new: int, stop_tokens=(151645, 151643), repetition_window: int = 6):
        """LLMEngine::generate: the generated ids (prompt excluded)."""
        ids = _ints(prompt)
        stops = _ints(stop_tokens)
        out = (C.c_int * max(1, max_new))()
        n = C.c_int()
        _check(self.L.qw2_generate(self.h, ids, len(prompt), max_new, stops, len(stop_tokens), repetition_window,
                                   out, max_new, C.byref(n)), "qw2_generate")
        return [out[i] for i in range(n.value)]

    # ---------------------------------------------------------- sessions
    def create_session(self) -> int:
        sid = C.c_int()
        _check(self.L.qw2_session_create(self.h, C.byref(sid)), "qw2_session_create")
        return sid.value

    def destroy_session(self, session: int) -> None:
        _check(self.L.qw2_session_destroy(self.h, session), "qw2_session_destroy")

    def session_exists(self, session: int) -> bool:
        e = C.c_int()
        _check(self.L.qw2_session_exists(self.h, session, C.byref(e)), "qw2_session_exists")
        return bool(e.value)

    def session_len(self, session: int) -> int:
        n = C.c_int()
        _check(self.L.qw2_session_len(self.h, session, C.byref(n)), "qw2_session_len")
        return n.value

    def forward_session(self, session: int, tokens) -> tuple[np.ndarray, int]:
        ids = _ints(tokens)
        logits = np.empty(self.cfg["vocab"], np.float32)
        am = C.c_int()
        _check(self.L.qw2_forward_session(self.h, session, ids, len(tokens), logits.ctypes.data_as(C.c_void_p),
                                          C.byref(am)), "qw2_forward_session")
        return logits, am.value

    def _request(self, session, input_ids, max_new_tokens, stop_tokens=(), repetition_window=0, on_token=None,
                 out_cap=None):
        ids = _ints(input_ids)
        stops = _ints(stop_tokens)
        cap = max_new_tokens if out_cap is None else out_cap
        out = (C.c_int * max(1, cap))()
        cb = TOKEN_CB(lambda user, s, step, tok, ms: on_token(s, step, tok, ms)) if on_token else TOKEN_CB()
        r = Qw2Request(session, ids, len(input_ids), Qw2GenConfig(max_new_tokens, repetition_window, stops,
                                                                  len(stop_tokens)), out, cap, cb, None)
        return r, (ids, stops, out, cb)

    def generate_session(self, session: int, input_ids, max_new_tokens: int, stop_tokens=(),
                         repetition_window: int = 0):
        """generate_session: (generated ids, result dict); the session keeps its cache."""
        r, keep = self._request(session, input_ids, max_new_tokens, stop_tokens, repetition_window)
        res = Qw2Result()
        _check(self.L.qw2_generate_session(self.h, session, r.input_ids, r.n_input, C.byref(r.cfg), r.out_ids,
                                           r.out_cap, C.byref(res)), "qw2_generate_session")
        return [keep[2][i] for i in range(min(res.n_out, r.out_cap))], res.as_dict()

    def generate_batch(self, requests):
        """generate_batch: requests are dicts (session, input_ids, max_new_tokens,
        stop_tokens=(), repetition_window=0, on_token=None); returns a list of
        (ids, result dict)."""
        built = [self._request(q["session"], q["input_ids"], q["max_new_tokens"], q.get("stop_tokens", ()),
                               q.get("repetition_window", 0), q.get("on_token")) for q in requests]
        arr = (Qw2Request * max(1, len(built)))(*[b[0] for b in built])
        res = (Qw2Result * max(1, len(built)))()
        _check(self.L.qw2_generate_batch(self.h, len(built), arr, res), "qw2_generate_batch")
        return [([b[1][2][i] for i in range(min(res[k].n_out, b[0].out_cap))], res[k].as_dict())
                for k, b in enumerate(built)]

    def submit(self, session: int, input_ids, max_new_tokens: int, stop_tokens=(), repetition_window: int = 0,
               on_token=None) -> int:
        """generate_async: returns a job id at once (a worker thread runs it)."""
        r, keep = self._request(session, input_ids, max_new_tokens, stop_tokens, repetition_window, on_token)
        job = C.c_int()
        _check(self.L.qw2_submit(self.h, C.byref(r), C.byref(job)), "qw2_submit")
        self._keep[job.value] = (keep, max_new_tokens)
        return job.value

    def wait(self, job: int, timeout_ms: int = -1):
        cap = self._keep.get(job, (None, 1))[1]
        out = (C.c_int * max(1, cap))()
        res = Qw2Result()
        _check(self.L.qw2_wait(self.h, job, timeout_ms, out, cap, C.byref(res)), "qw2_wait")
        self._keep.pop(job, None)
        return [out[i] for i in range(min(res.n_out, cap))], res.as_dict()

    def cancel(self, session: int) -> None:
        _check(self.L.qw2_cancel(self.h, session), "qw2_cancel")

    def weight_bytes(self) -> int:
        b = C.c_longlong()
        _check(self.L.qw2_weight_bytes(self.h, C.byref(b)), "qw2_weight_bytes")
        return b.value

    def kv_pool(self) -> int:
        p = C.c_void_p()
        _check(self.L.qw2_kv_pool(self.h, C.byref(p)), "qw2_kv_pool")
        return p.value


__all__ = ["Model", "KVError", "QWEN2_1_5B", "QW2_F16", "QW2_BF16", "QW2_F32", "synth_weights", "synth_prompt",
           "tensor_specs", "write_safetensors", "f32_to_f16_trunc"]
