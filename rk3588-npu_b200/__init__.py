"""Python host binding of the B200 decode hot path (ctypes over include/kvattn.h).

The product is the C ABI in ``lib/libkvattn.so`` (CUDA kernels for sm_100a +
C++ host runtime).  This module only marshals arguments: device tensors are
torch tensors (used for device memory and streams), everything else is plain
Python.  There is no fallback: if the library is missing, ``load()`` raises.

Reference interfaces mirrored (Bobchasm/rk3588-npu):
  KVCache        worker/include/model/kv_cache.h:19-41  -> Pool + sequences
  op_rope + append loop + op_attention
                 worker/src/model/qwen2_model.cpp:180-206 -> Pool.plan / decode_layer / commit
  (no counterpart) placement of requests onto GPUs      -> Scheduler
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libkvattn.so")

KV_OK, KV_ERR_INVAL, KV_ERR_OOM, KV_ERR_BADSEQ, KV_ERR_CUDA, KV_ERR_RANGE, KV_ERR_STATE, \
    KV_ERR_TIMEOUT = range(8)
KV_F16, KV_BF16, KV_I8 = 0, 1, 2
KVP_HOST_ONLY = -1
KVP_MERGE_GRID, KVP_MERGE_CLUSTER = 0, 1
HEAD_DIM = 128
BLOCK_TOKENS = 16
KVX_HANDLE_BYTES = 64
KVN_UNIQUE_ID_BYTES = 128

_vp = C.c_void_p
_ip = C.POINTER(C.c_int)

# name -> argtypes (all return int status unless listed in _RESTYPE)
_SIGS = {
    "kv_last_error": [],
    "kv_status_str": [C.c_int],
    "kv_version": [],
    "kv_kernel_count": [C.POINTER(C.c_longlong)],
    "kvp_create": [C.c_int] * 10 + [C.c_float, C.POINTER(_vp)],
    "kvp_destroy": [_vp],
    "kvp_reset": [_vp, _vp],
    "kvp_free_blocks": [_vp, _ip],
    "kvp_num_blocks": [_vp, _ip],
    "kvp_storage": [_vp, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(C.c_size_t)],
    "kvp_seq_alloc": [_vp, _ip],
    "kvp_seq_free": [_vp, C.c_int],
    "kvp_seq_reserve": [_vp, C.c_int, C.c_int],
    "kvp_seq_set_blocks": [_vp, C.c_int, _ip, C.c_int],
    "kvp_seq_len": [_vp, C.c_int, _ip],
    "kvp_seq_set_len": [_vp, C.c_int, C.c_int],
    "kvp_seq_blocks": [_vp, C.c_int, _ip, C.c_int, _ip],
    "kvp_import": [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp],
    "kvp_gather": [_vp, C.c_int, C.c_int, _vp, _vp, _vp],
    "kvp_import_i8": [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp],
    "kvp_gather_i8": [_vp, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp],
    "kv_append_chunk": [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp],
    "attn_prefill": [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp],
    "attn_prefill_mma": [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp],
    "kv_append_chunk_batch": [_vp, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp],
    "attn_prefill_batch": [_vp, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp],
    "attn_decode_plan": [_vp, C.c_int, _ip, _vp],
    "attn_decode_plan_ex": [_vp, C.c_int, _ip, _ip, _ip, _vp],
    "attn_decode_append": [_vp, C.c_int, _vp, _vp, _vp, _vp, _vp],
    "attn_decode_append_partial": [_vp, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "attn_decode_commit": [_vp],
    "attn_combine_lse": [C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp],
    "attn_combine_lse_packed": [C.c_int, C.c_int, C.c_int, _vp, _vp, _vp],
    "kvp_device_status": [_vp, _vp, _ip],
    "kvp_plan_info": [_vp, _ip, _ip, _ip, _ip, _ip, _ip, _ip, C.c_int],
    "kvp_plan_cta_start": [_vp, _ip, C.c_int],
    "kvp_launch_info": [_vp, _ip, _ip],
    "kvp_timing_enable": [_vp, C.c_int],
    "kvp_set_overlap": [_vp, C.c_int],
    "kvp_set_merge_mode": [_vp, C.c_int],
    "kvp_plan_clusters": [_vp, _ip, _ip],
    "attn_contig_noalloc": [_vp, _vp, _vp, _vp] + [C.c_int] * 7 + [_vp],
    "kvp_timing_read": [_vp, C.POINTER(C.c_double), _ip],
    "kvx_create": [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)],
    "kvx_handle": [_vp, _vp],
    "kvx_open": [_vp, C.c_int, _vp],
    "kvx_destroy": [_vp],
    "attn_decode_append_xgpu": [_vp, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp],
    "kvn_unique_id": [_vp],
    "kvn_create": [C.c_int, C.c_int, C.c_int, _vp, C.c_int, C.POINTER(_vp)],
    "kvn_destroy": [_vp],
    "attn_decode_append_nccl": [_vp, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp],
    "kvs_create": [C.c_int, C.c_int, C.POINTER(C.c_longlong), C.POINTER(_vp)],
    "kvs_destroy": [_vp],
    "kvs_place": [_vp, C.c_longlong, C.c_int, _ip],
    "kvs_resize": [_vp, C.c_longlong, C.c_int],
    "kvs_release": [_vp, C.c_longlong],
    "kvs_gpu_of": [_vp, C.c_longlong, _ip],
    "kvs_load": [_vp, C.c_int, C.POINTER(C.c_longlong), _ip],
}
_RESTYPE = {"kv_last_error": C.c_char_p, "kv_status_str": C.c_char_p, "kv_version": C.c_char_p}

_lib = None


class KVError(RuntimeError):
    def __init__(self, status: int, fn: str, msg: str):
        self.status = status
        super().__init__(f"{fn}: {_lib.kv_status_str(status).decode()} ({msg})")


def load() -> C.CDLL:
    """Load libkvattn.so (build it with rk3588-npu_b200/build.py).  Raises
    FileNotFoundError when it is absent: there is no other implementation."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing; build it with `python rk3588-npu_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = _RESTYPE.get(name, C.c_int)
        _lib = L
    return _lib


def _check(rc: int, fn: str) -> None:
    if rc != KV_OK:
        raise KVError(rc, fn, _lib.kv_last_error().decode())


def call(fn: str, *args) -> None:
    """Call a status-returning C entry point, raising KVError on failure."""
    _check(getattr(load(), fn)(*args), fn)


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _ints(xs):
    xs = list(int(x) for x in xs)
    return (C.c_int * max(1, len(xs)))(*xs)


class Pool:
    """A paged KV pool on one GPU (or a host-only bookkeeping pool).

    Method names follow KVCache where one exists (kv_cache.h:19-41):
    ``reset``, ``cur_pos``/``set_cur_pos`` (per sequence), ``capacity``."""

    def __init__(self, device: int, num_layers: int, num_blocks: int, *, num_q_heads: int = 12,
                 num_kv_heads: int = 2, dtype: int = KV_F16, max_seqs: int = 256,
                 max_seq_len: int = 32768, rope_theta: float = 1e6):
        L = load()
        h = _vp()
        _check(L.kvp_create(device, num_layers, num_q_heads, num_kv_heads, HEAD_DIM, BLOCK_TOKENS,
                            num_blocks, dtype, max_seqs, max_seq_len, rope_theta, C.byref(h)),
               "kvp_create")
        self.h = h
        self.device = device
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.q_heads = num_q_heads
        self.kv_heads = num_kv_heads
        self.kv_dim = num_kv_heads * HEAD_DIM
        self.hidden = num_q_heads * HEAD_DIM
        self.dtype = dtype
        self.max_seqs = max_seqs
        self.max_seq_len = max_seq_len
        self._plan_n = 0

    def close(self) -> None:
        if self.h:
            _check(_lib.kvp_destroy(self.h), "kvp_destroy")
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- pool ----
    def reset(self, stream=None) -> None:
        call("kvp_reset", self.h, None if self.device < 0 else _stream(stream))

    def free_blocks(self) -> int:
        n = C.c_int()
        call("kvp_free_blocks", self.h, C.byref(n))
        return n.value

    def storage(self):
        k, v, lb = _vp(), _vp(), C.c_size_t()
        call("kvp_storage", self.h, C.byref(k), C.byref(v), C.byref(lb))
        return k.value, v.value, lb.value

    def launch_info(self):
        a, b = C.c_int(), C.c_int()
        call("kvp_launch_info", self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    # ---- sequences ----
    def seq_alloc(self) -> int:
        s = C.c_int()
        call("kvp_seq_alloc", self.h, C.byref(s))
        return s.value

    def seq_free(self, seq: int) -> None:
        call("kvp_seq_free", self.h, seq)

    def reserve(self, seq: int, n_tokens: int) -> None:
        call("kvp_seq_reserve", self.h, seq, n_tokens)

    def set_blocks(self, seq: int, block_ids) -> None:
        ids = list(block_ids)
        call("kvp_seq_set_blocks", self.h, seq, _ints(ids), len(ids))

    def cur_pos(self, seq: int) -> int:
        n = C.c_int()
        call("kvp_seq_len", self.h, seq, C.byref(n))
        return n.value

    def set_cur_pos(self, seq: int, pos: int) -> None:
        call("kvp_seq_set_len", self.h, seq, pos)

    def blocks(self, seq: int) -> list[int]:
        n = C.c_int()
        call("kvp_seq_blocks", self.h, seq, None, 0, C.byref(n))
        buf = (C.c_int * max(1, n.value))()
        call("kvp_seq_blocks", self.h, seq, buf, n.value, C.byref(n))
        return list(buf[:n.value])

    def capacity(self, seq: int) -> int:
        return len(self.blocks(seq)) * BLOCK_TOKENS

    # ---- data movement (device tensors) ----
    def import_rows(self, layer, seq, pos0, k_rows, v_rows, stream=None) -> None:
        n = k_rows.shape[0]
        assert k_rows.shape == (n, self.kv_dim) and v_rows.shape == (n, self.kv_dim)
        call("kvp_import", self.h, layer, seq, pos0, n, _ptr(k_rows), _ptr(v_rows), _stream(stream))

    def gather(self, layer, seq, stream=None):
        import torch
        n = self.cur_pos(seq)
        dev = torch.device("cuda", self.device)
        k = torch.empty((n, self.kv_dim), dtype=torch.int16, device=dev)
        v = torch.empty((n, self.kv_dim), dtype=torch.int16, device=dev)
        call("kvp_gather", self.h, layer, seq, _ptr(k), _ptr(v), _stream(stream))
        return k, v

    def import_i8(self, layer, seq, pos0, k_codes, v_codes, k_scales, v_scales, stream=None) -> None:
        """INT8 pools: codes [n, kv_dim] int8, scales [n, kv_heads] fp32 (device tensors)."""
        n = k_codes.shape[0]
        call("kvp_import_i8", self.h, layer, seq, pos0, n, _ptr(k_codes), _ptr(v_codes), _ptr(k_scales),
             _ptr(v_scales), _stream(stream))

    def gather_i8(self, layer, seq, stream=None):
        """INT8 pools: (k_codes, v_codes, k_scales, v_scales) of positions [0, len)."""
        import torch
        n = self.cur_pos(seq)
        dev = torch.device("cuda", self.device)
        kc = torch.empty((n, self.kv_dim), dtype=torch.int8, device=dev)
        vc = torch.empty((n, self.kv_dim), dtype=torch.int8, device=dev)
        ks = torch.empty((n, self.kv_dim // HEAD_DIM), dtype=torch.float32, device=dev)
        vs = torch.empty((n, self.kv_dim // HEAD_DIM), dtype=torch.float32, device=dev)
        call("kvp_gather_i8", self.h, layer, seq, _ptr(kc), _ptr(vc), _ptr(ks), _ptr(vs), _stream(stream))
        return kc, vc, ks, vs

    def append_chunk(self, layer, seq, pos0, k, v, stream=None) -> None:
        n = k.shape[0]
        assert k.shape == (n, self.kv_dim) and v.shape == (n, self.kv_dim)
        call("kv_append_chunk", self.h, layer, seq, pos0, n, _ptr(k), _ptr(v), _stream(stream))

    def prefill(self, layer, seq, pos0, q, out, stream=None, kernel="tc") -> None:
        """Causal attention of q [n, hidden] (unrotated) at positions pos0.. over
        the pool (the chunk's K/V appended first); kernel "tc" (tcgen05) or
        "mma" (the mma.sync baseline)."""
        n = q.shape[0]
        fn = "attn_prefill" if kernel == "tc" else "attn_prefill_mma"
        call(fn, self.h, layer, seq, pos0, n, _ptr(q), _ptr(out), _stream(stream))

    def append_chunk_batch(self, layer, seqs, pos0s, k, v, ns=None, stream=None) -> None:
        """Chunks of several sequences in one call: chunk i is ns[i] rows of
        k / v [sum(ns), kv_dim] (in order) at positions pos0s[i].. of seqs[i]."""
        ns = list(ns) if ns is not None else [k.shape[0]]
        assert len(seqs) == len(pos0s) == len(ns) and sum(ns) == k.shape[0]
        call("kv_append_chunk_batch", self.h, layer, len(seqs), _ints(seqs), _ints(pos0s), _ints(ns), _ptr(k),
             _ptr(v), _stream(stream))

    def prefill_batch(self, layer, seqs, pos0s, ns, q, out, stream=None) -> None:
        """Causal attention of several chunks (rows concatenated in q / out, in
        order) in shared tcgen05 launches."""
        assert len(seqs) == len(pos0s) == len(ns) and sum(ns) == q.shape[0]
        call("attn_prefill_batch", self.h, layer, len(seqs), _ints(seqs), _ints(pos0s), _ints(ns), _ptr(q),
             _ptr(out), _stream(stream))

    # ---- decode ----
    def plan(self, seq_ids, rope_pos=None, append=None, stream=None) -> None:
        ids = list(seq_ids)
        st = None if self.device < 0 else _stream(stream)
        if rope_pos is None and append is None:
            call("attn_decode_plan", self.h, len(ids), _ints(ids), st)
        else:
            rp = _ints(rope_pos) if rope_pos is not None else None
            ap = _ints(append) if append is not None else None
            call("attn_decode_plan_ex", self.h, len(ids), _ints(ids), rp, ap, st)
        self._plan_n = len(ids)

    def plan_info(self):
        """The active plan: pieces (slot, kv head, b0, b1), CTA ranges, patches."""
        n, grid, npatch = C.c_int(), C.c_int(), C.c_int()
        call("kvp_plan_info", self.h, C.byref(n), C.byref(grid), C.byref(npatch), None, None, None,
             None, 0)
        cap = max(1, n.value)
        a, b, c, d = [(C.c_int * cap)() for _ in range(4)]
        call("kvp_plan_info", self.h, C.byref(n), C.byref(grid), C.byref(npatch), a, b, c, d, cap)
        cs = (C.c_int * (grid.value + 1))()
        call("kvp_plan_cta_start", self.h, cs, grid.value + 1)
        return {"nitems": n.value, "grid": grid.value, "npatch": npatch.value,
                "items": list(zip(a[:n.value], b[:n.value], c[:n.value], d[:n.value])),
                "cta_start": list(cs)}

    def decode_layer(self, layer, q, k_new, v_new, out, m=None, l=None, stream=None) -> None:
        n = self._plan_n
        assert q.shape[0] >= n and out.shape[0] >= n
        if m is None:
            call("attn_decode_append", self.h, layer, _ptr(q), _ptr(k_new), _ptr(v_new), _ptr(out),
                 _stream(stream))
        else:
            call("attn_decode_append_partial", self.h, layer, _ptr(q), _ptr(k_new), _ptr(v_new),
                 _ptr(out), _ptr(m), _ptr(l), _stream(stream))

    def commit(self) -> None:
        call("attn_decode_commit", self.h)

    def timing(self, enable: bool) -> None:
        call("kvp_timing_enable", self.h, int(enable))

    def set_overlap(self, enable: bool) -> None:
        """kvp_set_overlap: decode launches may copy their first tiles while
        the previous kernel in the stream finishes (that kernel must not
        write this pool, other than as one of this pool's decode launches)."""
        call("kvp_set_overlap", self.h, int(enable))

    def set_merge_mode(self, mode: int) -> None:
        """kvp_set_merge_mode: KVP_MERGE_GRID (a merge launch behind the
        decode launch, the default) or KVP_MERGE_CLUSTER (splits merged inside
        8-CTA clusters when the packing balances)."""
        call("kvp_set_merge_mode", self.h, int(mode))

    def plan_clusters(self):
        """(launches of the active plan merging inside clusters, launches)."""
        a, b = C.c_int(), C.c_int()
        call("kvp_plan_clusters", self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def timing_read(self):
        """(summed decode-launch milliseconds, launches) since timing(True)."""
        ms, n = C.c_double(), C.c_int()
        call("kvp_timing_read", self.h, C.byref(ms), C.byref(n))
        return ms.value, n.value

    def device_status(self, stream=None) -> int:
        s = C.c_int()
        call("kvp_device_status", self.h, _stream(stream), C.byref(s))
        return s.value


def kernel_count() -> int:
    """Kernels the library has launched in this process so far."""
    n = C.c_longlong()
    call("kv_kernel_count", C.byref(n))
    return n.value


def combine_lse(m, l, o, out, stream=None) -> None:
    """out[rows, dim] = LSE merge of G partial states m, l [G, rows], o [G, rows, dim]."""
    G, rows, dim = o.shape
    call("attn_combine_lse", G, rows, dim, _ptr(m), _ptr(l), _ptr(o), _ptr(out), _stream(stream))


def combine_lse_packed(packed, rows, out, stream=None) -> None:
    """The same merge over packed [G, rows*(2+dim)] rows of [m | l | o]."""
    G = packed.shape[0]
    dim = packed.shape[1] // rows - 2
    call("attn_combine_lse_packed", G, rows, dim, _ptr(packed), _ptr(out), _stream(stream))


class Scheduler:
    """Placement of requests onto GPUs by resident KV blocks (kvs_* C ABI).

    Deterministic: ranks that make the same calls in the same order agree
    on every placement without communicating."""

    def __init__(self, blocks_per_gpu, block_tokens: int = BLOCK_TOKENS):
        L = load()
        caps = (C.c_longlong * len(blocks_per_gpu))(*[int(b) for b in blocks_per_gpu])
        h = _vp()
        _check(L.kvs_create(len(blocks_per_gpu), block_tokens, caps, C.byref(h)), "kvs_create")
        self.h = h
        self.n_gpus = len(blocks_per_gpu)

    def close(self) -> None:
        if self.h:
            _check(_lib.kvs_destroy(self.h), "kvs_destroy")
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def place(self, request: int, tokens: int) -> int:
        g = C.c_int()
        call("kvs_place", self.h, request, tokens, C.byref(g))
        return g.value

    def resize(self, request: int, tokens: int) -> None:
        call("kvs_resize", self.h, request, tokens)

    def release(self, request: int) -> None:
        call("kvs_release", self.h, request)

    def gpu_of(self, request: int) -> int:
        g = C.c_int()
        call("kvs_gpu_of", self.h, request, C.byref(g))
        return g.value

    def load(self, gpu: int) -> tuple[int, int]:
        b, n = C.c_longlong(), C.c_int()
        call("kvs_load", self.h, gpu, C.byref(b), C.byref(n))
        return b.value, n.value
