"""numpy bindings for the checker libraries (TEST INFRASTRUCTURE ONLY).

Loaded only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg.  Two libraries:

* ``liboracle.so`` -- the C restatement in ``kvattn_oracle.c`` (always
  buildable with gcc; it is the checker the GPU tests compare against);
* ``_ref/libkvref.so`` -- the reference's own functions compiled from its
  sources by ``oracle/Makefile`` (``make ref``); present where the reference
  sources were available at build time, used to pin the restatement and as
  the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libkvref.so")
# Root of the reference checkout (Bobchasm/rk3588-npu): KVATTN_REFERENCE, else
# the location this build's recipe reads it from.  Only the build of the
# reference shim needs it; the tests use the prebuilt libraries.
REF_ROOT = os.environ.get("KVATTN_REFERENCE", "/root/reference")
REF_SRC = os.path.join(REF_ROOT, "worker")

F16, BF16 = 0, 1

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")


def build(ref: bool = True) -> None:
    """Compile liboracle.so (and the reference shim when its sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if ref and os.path.isdir(REF_SRC):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF_DIR={REF_SRC}"], check=True)


_lib = None
_ref = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(
            os.path.join(HERE, "kvattn_oracle.c")
        ):
            build(ref=False)
        L = C.CDLL(ORACLE_SO)
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_f32_to_bf16.argtypes = [C.c_float]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_bf16_to_f32.restype = C.c_float
        L.orc_bf16_to_f32.argtypes = [C.c_uint16]
        L.orc_encode.argtypes = [_f32p, _u16p, C.c_long, C.c_int]
        L.orc_decode.argtypes = [_u16p, _f32p, C.c_long, C.c_int]
        L.orc_rope.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        L.orc_rope_table.argtypes = [C.c_float, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
        L.orc_softmax.argtypes = [_f32p, C.c_int, C.c_int]
        L.orc_attention.restype = C.c_int
        L.orc_attention.argtypes = [_f32p, _u16p, _u16p, _f32p] + [C.c_int] * 7
        L.orc_rope_append.argtypes = [_f32p, _f32p, _f32p, _u16p, _u16p] + [C.c_int] * 5 + [
            C.c_float, C.c_int]
        L.orc_layer_step.restype = C.c_int
        L.orc_layer_step.argtypes = [_f32p, _f32p, _f32p, _u16p, _u16p, _f32p] + [C.c_int] * 5 + [
            C.c_float, C.c_int]
        L.orc_lse_combine.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_quantize_i8.argtypes = [_f32p, C.c_int, _i8p, _f32p]
        L.orc_attention_i8.restype = C.c_int
        L.orc_attention_i8.argtypes = [_f32p, _i8p, _f32p, _i8p, _f32p, _f32p] + [C.c_int] * 6
        L.orc_layer_step_i8.restype = C.c_int
        L.orc_layer_step_i8.argtypes = [_f32p, _f32p, _f32p, _i8p, _f32p, _i8p, _f32p, _f32p] + [C.c_int] * 5 + [
            C.c_float]
        _lib = L
    return _lib


def have_ref() -> bool:
    return os.path.exists(REF_SO)


def ref() -> C.CDLL:
    """The reference's own functions (raises if the shim was never built)."""
    global _ref
    if _ref is None:
        if not have_ref():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference sources)")
        R = C.CDLL(REF_SO)
        for n in ("ref_f32_to_f16", "ref_f32_to_bf16"):
            getattr(R, n).argtypes = [_f32p, _u16p, C.c_long]
        for n in ("ref_f16_to_f32", "ref_bf16_to_f32"):
            getattr(R, n).argtypes = [_u16p, _f32p, C.c_long]
        R.ref_rope.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        R.ref_softmax.argtypes = [_f32p, C.c_int, C.c_int]
        R.ref_attention.argtypes = [_f32p, _u16p, _u16p, _f32p] + [C.c_int] * 6
        R.ref_kvc_create.restype = C.c_void_p
        R.ref_kvc_create.argtypes = [C.c_int, C.c_int, C.c_int]
        R.ref_kvc_destroy.argtypes = [C.c_void_p]
        R.ref_kvc_reset.argtypes = [C.c_void_p]
        R.ref_kvc_cur_pos.restype = C.c_int
        R.ref_kvc_cur_pos.argtypes = [C.c_void_p]
        R.ref_kvc_set_cur_pos.argtypes = [C.c_void_p, C.c_int]
        R.ref_kvc_capacity.restype = C.c_int
        R.ref_kvc_capacity.argtypes = [C.c_void_p]
        R.ref_kvc_k_ptr.restype = C.c_void_p
        R.ref_kvc_k_ptr.argtypes = [C.c_void_p, C.c_int]
        R.ref_kvc_v_ptr.restype = C.c_void_p
        R.ref_kvc_v_ptr.argtypes = [C.c_void_p, C.c_int]
        R.ref_layer_step.argtypes = [_f32p, _f32p, _f32p, C.c_void_p, C.c_void_p, _f32p] + [
            C.c_int] * 5 + [C.c_float]
        R.ref_batch_step.argtypes = [_f32p, _f32p, _f32p, C.c_void_p, C.c_void_p, _f32p,
                                     C.c_void_p] + [C.c_int] * 4 + [C.c_float, C.c_int]
        _ref = R
    return _ref


# ---------------------------------------------------------------- wrappers
def encode(x: np.ndarray, dtype: int = F16) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_encode(x.reshape(-1), out.reshape(-1), x.size, dtype)
    return out


def decode(h: np.ndarray, dtype: int = F16) -> np.ndarray:
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_decode(h.reshape(-1), out.reshape(-1), h.size, dtype)
    return out


def rope_table(theta: float, head_dim: int, pos0: int, npos: int):
    half = head_dim // 2
    c = np.empty((npos, half), np.float32)
    s = np.empty((npos, half), np.float32)
    lib().orc_rope_table(theta, head_dim, pos0, npos, c.reshape(-1), s.reshape(-1))
    return c, s


def attention(q, k_cache, v_cache, seq, total_len, n_heads, n_kv_heads, head_dim, pos_base,
              dtype=F16) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32).reshape(-1)
    out = np.empty(seq * n_heads * head_dim, np.float32)
    rc = lib().orc_attention(q, np.ascontiguousarray(k_cache).reshape(-1),
                             np.ascontiguousarray(v_cache).reshape(-1), out, seq, total_len,
                             n_heads, n_kv_heads, head_dim, pos_base, dtype)
    assert rc == 0
    return out.reshape(seq, n_heads * head_dim)


def layer_step(q, k, v, k_cache, v_cache, pos, n_heads=12, n_kv_heads=2, head_dim=128,
               theta=1e6, dtype=F16):
    """RoPE + append + attention of one layer (qwen2_model.cpp:180-206).

    q [seq, n_heads*head_dim], k/v [seq, kv_dim] float32 (copied, not modified);
    k_cache/v_cache [capacity, kv_dim] uint16 contiguous, modified in place.
    Returns (out [seq, hidden], q_rotated, k_rotated)."""
    q = np.array(q, np.float32, order="C")
    k = np.array(k, np.float32, order="C")
    v = np.ascontiguousarray(v, np.float32)
    seq = q.shape[0]
    out = np.empty((seq, n_heads * head_dim), np.float32)
    assert k_cache.flags.c_contiguous and v_cache.flags.c_contiguous
    rc = lib().orc_layer_step(q.reshape(-1), k.reshape(-1), v.reshape(-1), k_cache.reshape(-1),
                              v_cache.reshape(-1), out.reshape(-1), seq, pos, n_heads,
                              n_kv_heads, head_dim, theta, dtype)
    assert rc == 0
    return out, q, k


def quantize_i8(x):
    """INT8 KV codes and scales of rows [n, head_dim] (orc_quantize_i8)."""
    x = np.ascontiguousarray(x, np.float32)
    rows = x.reshape(-1, x.shape[-1])
    q = np.empty(rows.shape, np.int8)
    s = np.empty(rows.shape[0], np.float32)
    for i in range(rows.shape[0]):
        lib().orc_quantize_i8(rows[i], rows.shape[1], q[i], s[i:i + 1])
    return q.reshape(x.shape), s.reshape(x.shape[:-1])


def layer_step_i8(q, k, v, kq, ks, vq, vs, pos, n_heads=12, n_kv_heads=2, head_dim=128, theta=1e6):
    """RoPE + INT8 append + attention of one layer over INT8 caches.

    kq/vq [capacity, kv_dim] int8 and ks/vs [capacity, n_kv_heads] float32,
    modified in place.  Returns out [seq, hidden]."""
    q = np.array(q, np.float32, order="C")
    k = np.array(k, np.float32, order="C")
    v = np.ascontiguousarray(v, np.float32)
    seq = q.shape[0]
    out = np.empty((seq, n_heads * head_dim), np.float32)
    for a in (kq, ks, vq, vs):
        assert a.flags.c_contiguous
    rc = lib().orc_layer_step_i8(q.reshape(-1), k.reshape(-1), v.reshape(-1), kq.reshape(-1), ks.reshape(-1),
                                 vq.reshape(-1), vs.reshape(-1), out.reshape(-1), seq, pos, n_heads, n_kv_heads,
                                 head_dim, theta)
    assert rc == 0
    return out


def lse_combine(m, l, o):
    """m, l [G, rows]; o [G, rows, dim] -> combined [rows, dim]."""
    m = np.ascontiguousarray(m, np.float32)
    l = np.ascontiguousarray(l, np.float32)
    o = np.ascontiguousarray(o, np.float32)
    G, rows, dim = o.shape
    out = np.empty((rows, dim), np.float32)
    lib().orc_lse_combine(m.reshape(-1), l.reshape(-1), o.reshape(-1), G, rows, dim,
                          out.reshape(-1))
    return out


def ref_layer_step(q, k, v, k_cache, v_cache, pos, n_heads=12, n_kv_heads=2, head_dim=128,
                   theta=1e6):
    """The reference's own RoPE + append + op_attention (fp16 caches only)."""
    R = ref()
    q = np.array(q, np.float32, order="C")
    k = np.array(k, np.float32, order="C")
    v = np.ascontiguousarray(v, np.float32)
    seq = q.shape[0]
    out = np.empty((seq, n_heads * head_dim), np.float32)
    R.ref_layer_step(q.reshape(-1), k.reshape(-1), v.reshape(-1), k_cache.ctypes.data,
                     v_cache.ctypes.data, out.reshape(-1), seq, pos, n_heads, n_kv_heads,
                     head_dim, theta)
    return out, q, k


def ref_batch_step(q, k, v, k_caches, v_caches, pos, threads, n_heads=12, n_kv_heads=2,
                   head_dim=128, theta=1e6):
    """One decode step (seq=1 each) of many sequences through the reference's
    own functions, `threads` host threads taking whole sequences."""
    R = ref()
    nseq = len(k_caches)
    q = np.array(q, np.float32, order="C")
    k = np.array(k, np.float32, order="C")
    v = np.ascontiguousarray(v, np.float32)
    out = np.empty((nseq, n_heads * head_dim), np.float32)
    kp = (C.c_void_p * nseq)(*[c.ctypes.data for c in k_caches])
    vp = (C.c_void_p * nseq)(*[c.ctypes.data for c in v_caches])
    pos = np.ascontiguousarray(pos, np.int32)
    R.ref_batch_step(q.reshape(-1), k.reshape(-1), v.reshape(-1), kp, vp, out.reshape(-1),
                     pos.ctypes.data, nseq, n_heads, n_kv_heads, head_dim, theta, threads)
    return out


def orc_batch_step(q, k, v, k_caches, v_caches, pos, n_heads=12, n_kv_heads=2, head_dim=128,
                   theta=1e6, dtype=F16):
    """The C restatement of one decode step for many sequences (1 thread)."""
    outs = []
    for i in range(len(k_caches)):
        o, _, _ = layer_step(q[i:i + 1], k[i:i + 1], v[i:i + 1], k_caches[i], v_caches[i],
                             int(pos[i]), n_heads, n_kv_heads, head_dim, theta, dtype)
        outs.append(o[0])
    return np.stack(outs)
