"""Long sequences whose cached positions are split across GPUs.

Every rank of a torch.distributed process group keeps a contiguous slice of
each sequence's positions in its own pool (rank r: positions [lo_r, hi_r) of
the initial context; new tokens are appended on the last rank).  One decode
step per layer:

  1. each rank attends over its slice, the last rank also appending the new
     token: per (sequence, query head) a partial state (m, l, o) -- max of
     the scaled scores, sum of exp, normalised o;
  2. one all-gather of the packed states;
  3. their log-sum-exp merge into the output.

transport="nccl" (the default): all three in one library call per layer,
attn_decode_append_nccl -- the local decode, ncclAllGather over NVLink on the
library's NCCL communicator (kvn_create; the unique id passed through
torch.distributed), and the merge kernel, all on the caller's stream.

transport="p2p": attn_decode_append_xgpu -- right behind the local decode, an
exchange kernel pushes the states into every peer's area over NVLink (CUDA
IPC mappings set up once, the handles passed through torch.distributed),
waits for the peers' states of the same call and merges.

transport="collective": attn_decode_append_partial, then torch.distributed's
all-gather and attn_combine_lse_packed -- for process groups whose backend is
not NCCL (two ranks sharing one GPU over gloo in the tests).

The reference has no split-KV; the merge restates the log-sum-exp identity
the oracle checks (oracle/kvattn_oracle.c: orc_lse_combine).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

import ctypes as C

from . import Pool, call, _ptr, _stream, _vp, HEAD_DIM, KVX_HANDLE_BYTES, KVN_UNIQUE_ID_BYTES


def slice_bounds(length: int, rank: int, world: int) -> tuple[int, int]:
    """Positions [lo, hi) of a `length`-token context held by `rank`."""
    return length * rank // world, length * (rank + 1) // world


class SplitKV:
    """A batch of sequences split across `world` ranks (this process is `rank`).

    pool      the rank's Pool (its device)
    lengths   initial global context length of each sequence
    """

    def __init__(self, pool: Pool, lengths, rank: int, world: int, group=None,
                 transport: str = "nccl"):
        assert transport in ("nccl", "p2p", "collective")
        self.pool, self.rank, self.world, self.group = pool, rank, world, group
        self.transport = transport
        self._x = None
        self._n = None
        self.lengths = [int(x) for x in lengths]
        self.initial = list(self.lengths)
        self.ids = []
        self.bounds = []
        for L in self.lengths:
            lo, hi = slice_bounds(L, rank, world)
            s = pool.seq_alloc()
            self.ids.append(s)
            self.bounds.append((lo, hi))
        self.rows = len(self.ids) * pool.q_heads
        self._buf = None
        if transport == "p2p" and world > 1 and pool.device >= 0:
            self._open_exchange()
        if transport == "nccl" and world > 1 and pool.device >= 0:
            self._open_nccl()

    def _open_nccl(self) -> None:
        """The library's NCCL communicator (a collective: every rank joins)."""
        uid = (C.c_char * KVN_UNIQUE_ID_BYTES)()
        if self.rank == 0:
            call("kvn_unique_id", uid)
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0, group=self.group)
        c = _vp()
        call("kvn_create", self.pool.device, self.rank, self.world,
             C.create_string_buffer(obj[0], KVN_UNIQUE_ID_BYTES), self.rows, C.byref(c))
        self._n = c

    def _open_exchange(self) -> None:
        x = _vp()
        call("kvx_create", self.pool.device, self.rank, self.world, self.rows, C.byref(x))
        self._x = x
        h = (C.c_char * KVX_HANDLE_BYTES)()
        call("kvx_handle", x, h)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=self.group)
        for g, hb in enumerate(handles):
            if g != self.rank:
                call("kvx_open", x, g, C.create_string_buffer(hb, KVX_HANDLE_BYTES))
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Release the exchange / communicator (every rank, after its last
        layer call)."""
        if self._x is not None:
            torch.cuda.synchronize(self.pool.device)
            dist.barrier(group=self.group)
            call("kvx_destroy", self._x)
            self._x = None
        if self._n is not None:
            torch.cuda.synchronize(self.pool.device)
            dist.barrier(group=self.group)
            call("kvn_destroy", self._n)
            self._n = None

    @property
    def is_last(self) -> bool:
        return self.rank == self.world - 1

    def reserve(self, extra_tokens: int) -> None:
        """Blocks for the slice (and, on the last rank, `extra_tokens` appends)."""
        for s, (lo, hi) in zip(self.ids, self.bounds):
            self.pool.reserve(s, hi - lo + (extra_tokens if self.is_last else 0))

    def load_slice(self, layer: int, i: int, k_rows, v_rows, stream=None) -> None:
        """Import encoded rows [hi-lo, kv_dim] of sequence i's slice."""
        lo, hi = self.bounds[i]
        assert k_rows.shape[0] == hi - lo
        if hi > lo:
            self.pool.import_rows(layer, self.ids[i], 0, k_rows, v_rows, stream)
        if layer == self.pool.num_layers - 1:
            self.pool.set_cur_pos(self.ids[i], hi - lo)

    def begin_step(self, stream=None) -> None:
        """Plan one step: q and the new k rotate at the global position; only
        the last rank appends."""
        rope = list(self.lengths)
        append = [1 if self.is_last else 0] * len(self.ids)
        self.pool.plan(self.ids, rope_pos=rope, append=append, stream=stream)
        if self._buf is None and self.pool.device >= 0 and self.transport == "collective":  # host-only pools never run
            dev = torch.device("cuda", self.pool.device)
            n = self.rows * (2 + HEAD_DIM)
            self._buf = torch.empty(n, device=dev)
            self._all = torch.empty((self.world, n), device=dev)

    def layer(self, layer: int, q, k_new, v_new, out, stream=None) -> None:
        """One layer of the step.  q [B, q_heads*128], k/v [B, kv_heads*128]
        fp32 (the same on every rank), out [B, q_heads*128] fp32."""
        if self.world == 1:  # the whole context is here: no partials
            self.pool.decode_layer(layer, q, k_new, v_new, out, stream=stream)
            return
        if self._x is not None:
            call("attn_decode_append_xgpu", self.pool.h, layer, _ptr(q), _ptr(k_new), _ptr(v_new),
                 _ptr(out), self._x, _stream(stream))
            return
        if self._n is not None:
            call("attn_decode_append_nccl", self.pool.h, layer, _ptr(q), _ptr(k_new), _ptr(v_new),
                 _ptr(out), self._n, _stream(stream))
            return
        R = self.rows
        buf = self._buf
        m, l, o = buf[:R], buf[R:2 * R], buf[2 * R:]
        self.pool.decode_layer(layer, q, k_new, v_new, o.view(len(self.ids), -1), m, l, stream)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(self._all, buf, group=self.group)
        else:  # gloo (tests on one GPU): list form
            dist.all_gather(list(self._all.unbind(0)), buf, group=self.group)
        # rank g's [m | l | o] at row g of the gathered buffer
        call("attn_combine_lse_packed", self.world, R, HEAD_DIM, _ptr(self._all), _ptr(out),
             _stream(stream))

    def end_step(self) -> None:
        self.pool.commit()
        self.lengths = [L + 1 for L in self.lengths]

    def rewind(self) -> None:
        """Back to the initial contexts (drops the tokens appended since;
        their blocks stay reserved)."""
        self.lengths = list(self.initial)
        for s, (lo, hi) in zip(self.ids, self.bounds):
            self.pool.set_cur_pos(s, hi - lo)
