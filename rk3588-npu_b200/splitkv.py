"""Long sequences whose cached positions are split across GPUs.

Every rank of a torch.distributed process group keeps a contiguous slice of
each sequence's positions in its own pool (rank r: positions [lo_r, hi_r) of
the initial context; new tokens are appended on the last rank).  One decode
step per layer:

  1. each rank attends over its slice (attn_decode_append_partial), the last
     rank also appending the new token: per (sequence, query head) a partial
     state (m, l, o) -- max of the scaled scores, sum of exp, normalised o;
  2. one all-gather of the packed states (NCCL over NVLink on GPUs);
  3. attn_combine_lse merges the gathered states into the full output.

The reference has no split-KV; the merge restates the log-sum-exp identity
the oracle checks (oracle/kvattn_oracle.c: orc_lse_combine).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import Pool, call, _ptr, _stream, HEAD_DIM


def slice_bounds(length: int, rank: int, world: int) -> tuple[int, int]:
    """Positions [lo, hi) of a `length`-token context held by `rank`."""
    return length * rank // world, length * (rank + 1) // world


class SplitKV:
    """A batch of sequences split across `world` ranks (this process is `rank`).

    pool      the rank's Pool (its device)
    lengths   initial global context length of each sequence
    """

    def __init__(self, pool: Pool, lengths, rank: int, world: int, group=None):
        self.pool, self.rank, self.world, self.group = pool, rank, world, group
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
        if self._buf is None and self.pool.device >= 0:  # host-only pools plan but never run
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
