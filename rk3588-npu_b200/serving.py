"""Continuous batching over the paged pool, one process per GPU.

The reference engine serves one sequence at a time: LLMEngine::generate
(worker/src/engine/llm_engine.cpp:68-98) prefills the prompt, then runs one
forward per generated token, and the position advances after the last layer
(worker/src/model/qwen2_model.cpp:268).  Serving many sequences on a multi-GPU
box keeps that per-sequence contract and adds three things:

  placement   a request is placed whole on the GPU with the fewest resident KV
              blocks that has room for its prompt + generation budget
              (Scheduler, the kvs_* C ABI);
  prefill     up to `prefill_slots` admitted requests append one chunk of
              their prompt per step (kv_append_chunk: RoPE + encode + store,
              every layer) and, when the caller passes the chunk's queries,
              attend it causally over the cache (attn_prefill, tcgen05), the
              length advancing after the last layer;
  decode      every request whose prompt is in the cache advances one token
              per step (one plan, one fused append + attention launch per
              layer, one commit); a request that generated its budget frees
              its blocks and its placement.

Every rank runs the same Server over the same request stream.  The request
lifecycle and the placement are deterministic host state, so the ranks agree
on them without communicating; each rank executes only the requests placed
on its own GPU (no collective on the data path).
"""
from __future__ import annotations

from dataclasses import dataclass

from . import KVError, KV_ERR_OOM, Pool, Scheduler


@dataclass
class Request:
    rid: int
    prompt: int          # prompt tokens (appended in chunks)
    gen: int             # tokens to generate
    filled: int = 0      # prompt tokens in the cache
    generated: int = 0
    gpu: int = -1
    seq: int = -1        # pool sequence id, on the owning rank only
    state: str = "queued"

    @property
    def length(self) -> int:
        return self.filled + self.generated


class Server:
    """Request lifecycle on `world` GPUs; this process owns GPU `rank`."""

    def __init__(self, pool: Pool, sched: Scheduler, rank: int, world: int, chunk: int = 512,
                 prefill_slots: int = 8):
        assert sched.n_gpus == world
        self.pool, self.sched, self.rank, self.world = pool, sched, rank, world
        self.chunk, self.prefill_slots = chunk, prefill_slots
        self.queue: list[Request] = []
        self.prefilling: list[Request] = []
        self.decoding: list[Request] = []
        self.finished: list[Request] = []
        self.placements: list[tuple[int, int]] = []  # (rid, gpu) in placement order
        self.run_device = pool.device >= 0

    # ---------------------------------------------------------------- intake
    def submit(self, req: Request) -> None:
        self.queue.append(req)

    def add_resident(self, req: Request, load=None) -> None:
        """A request whose prompt is already cached (e.g. restored state):
        placed now, decoding from the next step.  `load(req)` imports its
        rows on the owning rank."""
        req.gpu = self.sched.place(req.rid, req.prompt + req.gen)
        self.placements.append((req.rid, req.gpu))
        req.filled = req.prompt
        req.state = "decode"
        if req.gpu == self.rank:
            req.seq = self.pool.seq_alloc()
            self.pool.reserve(req.seq, req.prompt)
            if load is not None:
                load(req)
            self.pool.set_cur_pos(req.seq, req.prompt)
        self.decoding.append(req)

    def admit(self) -> None:
        """Fill the prefill slots from the queue, first come first served; a
        request that fits on no GPU waits (and holds the queue) until
        completions free room."""
        while self.queue and len(self.prefilling) < self.prefill_slots:
            req = self.queue[0]
            try:
                req.gpu = self.sched.place(req.rid, req.prompt + req.gen)
            except KVError as e:
                if e.status == KV_ERR_OOM:
                    break
                raise
            self.queue.pop(0)
            self.placements.append((req.rid, req.gpu))
            req.state = "prefill"
            if req.gpu == self.rank:
                req.seq = self.pool.seq_alloc()
            self.prefilling.append(req)

    # ------------------------------------------------------------------ step
    def local_decode(self) -> list[Request]:
        return [r for r in self.decoding if r.gpu == self.rank]

    def step(self, decode_io=None, prefill_kv=None, prefill_batch_io=None) -> dict:
        """One engine step on this rank.

        decode_io(layer, reqs) -> (q [n, hidden], k [n, kv_dim], v [n, kv_dim],
            out [n, hidden]) device fp32 for this rank's decoding requests
            (in the order given);
        prefill_kv(layer, req, pos0, n) -> (k [n, kv_dim], v [n, kv_dim]) device
            fp32 for one prompt chunk, or (k, v, q [n, hidden], out [n, hidden])
            to also run the chunk's causal attention (attn_prefill) after its
            append;
        prefill_batch_io(layer, chunks) -> the same for all of this rank's
            chunks [(req, pos0, n), ...] at once, rows concatenated in that
            order: appended (and attended) with kv_append_chunk_batch /
            attn_prefill_batch in shared launches.  Used instead of prefill_kv
            when given.
        Returns the step's global counts (every rank returns the same)."""
        self.admit()
        dec = self.local_decode()
        chunks = [(r, min(self.chunk, r.prompt - r.filled)) for r in self.prefilling]
        local_chunks = [(r, c) for r, c in chunks if r.gpu == self.rank]
        for r, c in local_chunks:
            self.pool.reserve(r.seq, r.filled + c)
        if dec:
            self.pool.plan([r.seq for r in dec])
        if self.run_device:
            for layer in range(self.pool.num_layers):
                if dec:
                    q, k, v, out = decode_io(layer, dec)
                    self.pool.decode_layer(layer, q, k, v, out)
                if prefill_batch_io is not None and local_chunks:
                    seqs = [r.seq for r, _ in local_chunks]
                    pos0 = [r.filled for r, _ in local_chunks]
                    ns = [c for _, c in local_chunks]
                    io = prefill_batch_io(layer, [(r, r.filled, c) for r, c in local_chunks])
                    self.pool.append_chunk_batch(layer, seqs, pos0, io[0], io[1], ns=ns)
                    if len(io) == 4:
                        self.pool.prefill_batch(layer, seqs, pos0, ns, io[2], io[3])
                    continue
                for r, c in local_chunks:
                    io = prefill_kv(layer, r, r.filled, c)
                    self.pool.append_chunk(layer, r.seq, r.filled, io[0], io[1])
                    if len(io) == 4:
                        self.pool.prefill(layer, r.seq, r.filled, io[2], io[3])
        if dec:
            self.pool.commit()
        # ---- bookkeeping, identical on every rank ----
        n_decode = len(self.decoding)
        prefill_tokens = sum(c for _, c in chunks)
        for r, c in chunks:
            r.filled += c
            if r.gpu == self.rank:
                self.pool.set_cur_pos(r.seq, r.filled)
        done = []
        still = []
        for r in self.decoding:
            r.generated += 1
            if r.generated >= r.gen:
                done.append(r)
            else:
                still.append(r)
        for r in done:
            self.sched.release(r.rid)
            if r.gpu == self.rank:
                self.pool.seq_free(r.seq)
                r.seq = -1
            r.state = "done"
            self.finished.append(r)
        ready = [r for r in self.prefilling if r.filled >= r.prompt]
        self.prefilling = [r for r in self.prefilling if r.filled < r.prompt]
        for r in ready:
            r.state = "decode"
        self.decoding = still + ready
        return {"decode_tokens": n_decode, "prefill_tokens": prefill_tokens,
                "local_decode": len(dec), "completed": len(done)}
