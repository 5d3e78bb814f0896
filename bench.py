"""Decode hot-path benchmark: KV append + GQA decode attention on B200.

Default workload (the one the headline metric is quoted on, one GPU): batch
32, per-sequence context lengths uniform in [256, 4096] (seed 1), fp16 KV
cache with values N(0,1), Q [32,12,128] / new K,V [32,2,128] per step, one
layer, Qwen2-1.5B head shapes (12 query heads share 2 KV heads, head_dim
128), softmax scale 1/sqrt(128).  A step appends one token to every sequence
and attends over its whole context.  Synthetic seeded data; the 72 MB working
set fits in the 126 MB L2, so L2 is flushed (256 MiB write) before every
timed step and the flush is kept out of the step's events.

--workload paged28: 256 sequences, lengths lognormal (median 2048, sigma 0.8)
capped at 32768 (seed 2), block tables a random permutation (seed 2) of a
pool sized to 1.1x the blocks the contexts need, bf16 KV N(0,1), all 28
layers per step (one plan, 28 decode launches, one commit).  The ~20 GB read
per step is far larger than L2, so no flush is needed.  --workload paged1 is
the same sequences with one layer (the size of one of those launches), for
profiling.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload batch32|paged28|paged1]

N > 1 is launched by torchrun, one process per GPU; every rank owns its own
sequences (placement by request, no collective on the data path: weak
scaling); timing is the max over ranks of device-event time.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "rk3588-npu_b200")

METRIC = "decode attention tokens/s and achieved HBM GB/s vs B200 peak at 1/2/4/8 GPUs"
NQ, NKV, HD = 12, 2, 128
KVD = NKV * HD
HID = NQ * HD
FLUSH_BYTES = 256 << 20


class Workload:
    """One bench workload: the sequences a GPU holds and how a step runs."""

    def __init__(self, name, batch, layers, dtype, lens, perm_seed, flush, desc, data, profile):
        self.name, self.batch, self.layers, self.dtype = name, batch, layers, dtype
        self.lens, self.perm_seed, self.flush = lens, perm_seed, flush
        self.desc, self.data, self.profile = desc, data, profile

    @property
    def dtype_name(self) -> str:
        return ("f16", "bf16", "int8")[self.dtype]


def uniform_lengths(n=32, seed=1) -> list[int]:
    return [int(x) for x in np.random.default_rng(seed).integers(256, 4097, n)]


def lognormal_lengths(n=256, seed=2) -> list[int]:
    """Lognormal context lengths, median 2048, sigma 0.8, capped at 32768."""
    x = np.random.default_rng(seed).lognormal(np.log(2048.0), 0.8, n)
    return [int(min(32768, max(1, round(v)))) for v in x]


def serve_stream(seed=4, resident=128, new=4096):
    """Resident (context, budget) pairs, then the stream of new requests
    (prompt, budget): contexts and prompts U[512,8192], budgets U[16,256]."""
    rng = np.random.default_rng(seed)
    pairs = [(int(rng.integers(512, 8193)), int(rng.integers(16, 257))) for _ in range(resident + new)]
    return pairs[:resident], pairs[resident:]


def make_workload(name: str) -> Workload:
    if name == "batch32":
        return Workload(
            "batch32", 32, 1, 0, uniform_lengths(), None, True,
            "decode step: KV append + GQA decode attention, batch 32 per GPU, context U[256,4096], "
            "12 q / 2 kv heads x 128, fp16 KV, 1 layer",
            "synthetic (seeded N(0,1) K/V/q; context lengths U[256,4096] seed 1)",
            "decode_kernel_b32_ncu.txt")
    if name in ("paged28", "paged1"):
        layers = 28 if name == "paged28" else 1
        return Workload(
            name, 256, layers, 1, lognormal_lengths(), 2, False,
            f"paged decode step: block gather + KV append + GQA decode attention over {layers} "
            "layer(s), 256 sequences per GPU, context lognormal(median 2048, sigma 0.8) capped at "
            "32768, block tables a random permutation of a pool of 1.1x the needed blocks, "
            "12 q / 2 kv heads x 128, bf16 KV",
            "synthetic (seeded N(0,1) K/V/q; lognormal context lengths and block permutation seed 2)",
            "decode_kernel_paged256_ncu.txt")
    if name in ("long1", "long4"):
        b = 1 if name == "long1" else 4
        return Workload(
            name, b, 28, 1, [131072] * b, None, False,
            f"long-context decode step: batch {b}, context 131072 per sequence split along the "
            "sequence across the GPUs (contiguous slices), 28 layers, bf16 KV; per layer partial "
            "(m, l, o) per GPU, NCCL all-gather, log-sum-exp combine",
            "synthetic (seeded N(0,1) K/V/q, seed 3)",
            "decode_kernel_long_ncu.txt")
    if name == "prefill":
        return Workload(
            "prefill", 8, 28, 1, None, None, False,
            "chunked prefill: 8 requests (prompts U[512,8192], seed 4) each appending and attending "
            "one 512-token chunk (the middle chunk of its prompt, causal over all earlier "
            "positions) in every one of 28 layers, bf16 KV",
            "synthetic (seeded N(0,1) K/V/q; prompts seed 4)",
            None)
    if name == "model1":
        return Workload(
            "model1", 1, 28, 0, None, None, False,
            "Qwen2-1.5B greedy decode on one GPU: 28 layers, hidden 1536, 12 q / 2 kv heads x 128, "
            "SwiGLU 8960, vocab 151936 (tied lm_head), fp16 weights and KV cache; prompt of 128 ids "
            "uniform in [0,151936) (seed 0), then one greedy token per step",
            "synthetic (random-init N(0,0.02) weights from seed 0, RMSNorm weights 1; prompt seed 0)",
            None)
    if name == "serve":
        return Workload(
            "serve", 128, 28, 1, [L for L, _ in serve_stream()[0]], None, False,
            "continuous batching: 128 resident decode sequences (context U[512,8192], generation "
            "budget U[16,256]) plus 8 requests at a time in chunked prefill (prompt U[512,8192], "
            "512-token chunks appended into the paged pool), completed sequences free their blocks, "
            "requests placed by resident KV blocks across the GPUs, 28 layers, bf16 KV",
            "synthetic (seeded N(0,1) K/V/q; request stream seed 4)",
            "decode_kernel_paged256_ncu.txt")
    raise ValueError(f"unknown workload {name}")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload",
                    choices=["batch32", "paged28", "paged1", "long1", "long4", "serve", "prefill", "model1",
                             "model_batch"],
                    default="batch32")
    ap.add_argument("--transport", choices=["nccl", "p2p"], default="p2p",
                    help="long workloads: merge of the per-GPU states by the fused peer-memory exchange "
                         "kernel (p2p), or by NCCL all-gather + merge launch (nccl)")
    ap.add_argument("--prefill-kernel", choices=["tc", "tc1", "mma"], default="tc",
                    help="prefill workload: the tcgen05 kernel over all requests per launch "
                         "(kv_append_chunk_batch + attn_prefill_batch), the tcgen05 kernel one request per "
                         "call (tc1), or the mma.sync baseline (one request per call)")
    ap.add_argument("--kv-dtype", choices=["native", "int8"], default="native",
                    help="batch32 / paged28 / paged1: keep the workload's cache type, or an INT8 cache "
                         "(per-row scales) with the same contexts")
    ap.add_argument("--merge", choices=["grid", "cluster"], default="grid",
                    help="batch32 / paged28 / paged1: split heads merged by a merge launch behind the decode "
                         "launch (grid), or inside 8-CTA clusters when the plan balances that way (cluster)")
    ap.add_argument("--sessions", type=int, default=8,
                    help="model_batch workload: concurrent sessions decoding together")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--settle", type=float, default=1.0,
                    help="seconds of untimed load before the timed steps (clock samples)")
    return ap.parse_args()


def load_pkg():
    name = "rk3588_npu_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def step_bytes(kv_lens, dtype: int = 0) -> float:
    """Algorithmic HBM bytes of one decode launch.  Per sequence attending T
    tokens: the K and V rows of the T-1 cached tokens (2 KV heads x 128 dims
    x 2 B x 2 = 1024 B per token; INT8: 2 x (128 codes + a 4-byte scale) x 2
    = 528 B), the appended row, fp32 q/k/v in and fp32 out
    (4 x (1536 + 256 + 256 + 1536) B), and 4 B per block-table entry."""
    row = 528.0 if dtype == 2 else 1024.0
    tot = 0.0
    for T in kv_lens:
        tot += row * (T - 1) + row + 4.0 * -(-T // 16) + 4.0 * (HID + 2 * KVD + HID)
    return tot


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(gpu_indices)
        self.proc = None
        self.path = None

    def start(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx not in self.gpus:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        busy = [s for s, p in zip(sm, power) if p > 0] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


def encode_device(x, dtype: int):
    """fp32 -> 16-bit codes with the reference's truncating encoders
    (half.h:17-20 bf16, half.h:24-32 fp16), on the device: input preparation."""
    import torch
    u = x.contiguous().view(torch.int32)
    if dtype == 1:
        return (u >> 16).to(torch.int16)
    sign = (u >> 16) & 0x8000
    e = ((u >> 23) & 0xFF) - 112
    mant = u & 0x7FFFFF
    h = sign | (e.clamp(0, 31) << 10) | (mant >> 13)
    h = torch.where(e <= 0, sign, h)
    h = torch.where(e >= 31, sign | 0x7C00, h)
    return torch.where(h >= 32768, h - 65536, h).to(torch.int16)

def peak_hbm():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def ncu_traffic(profile: str):
    """Per-launch DRAM bytes of the decode kernel from the committed ncu
    summary of the workload (line `traffic_bytes_per_launch:`)."""
    if not profile:
        return None
    path = os.path.join(ROOT, "profiles", profile)
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


L2_BYTES = 126 << 20


def rotation_groups(wl: Workload) -> int:
    """Independent copies of the workload's sequences that the timed steps
    cycle through.  A step whose K/V would fit in L2 (batch32: 72 MB of the
    126 MB L2) would otherwise be served from L2 on the next step; with G
    groups each step reads a group whose K/V was last touched G-1 steps (more
    than 300 MB of other traffic) before, so every step reads HBM and the
    steps run back to back without an L2 flush between them."""
    per_step = step_bytes(wl.lens, wl.dtype) * wl.layers
    if per_step > 2 * L2_BYTES:
        return 1
    return max(2, -(-int(400e6) // int(per_step)))


def setup_pool(kv, torch, dev, wl: Workload, steps_total: int, seed: int, groups: int = 1):
    """A pool holding `groups` copies of the workload's contexts (distinct
    blocks, independent seeded data) in every layer.  Permuted workloads take
    a pool of 1.1x the blocks the contexts need and hand each sequence
    consecutive runs of a seeded random permutation of its block ids; the
    rest stay free for the blocks appended tokens open.  Returns the pool and
    the sequence ids of every group."""
    lens = wl.lens * groups
    need = [-(-L // 16) for L in lens]
    grow = [-(-(L + steps_total + 1) // 16) - n for L, n in zip(lens, need)]
    if wl.perm_seed is None:
        nb = sum(need) + sum(grow) + 64
    else:
        nb = max(-(-sum(need) * 11 // 10), sum(need) + sum(grow) + 64)
    P = kv.Pool(dev, wl.layers, nb, num_q_heads=NQ, num_kv_heads=NKV, dtype=wl.dtype,
                max_seqs=len(lens), max_seq_len=max(lens) + steps_total + 32)
    ids = [P.seq_alloc() for _ in lens]
    if wl.perm_seed is None:
        for s, L in zip(ids, lens):
            P.reserve(s, L)
    else:
        perm = np.random.default_rng(wl.perm_seed).permutation(nb)
        o = 0
        for s, n in zip(ids, need):
            P.set_blocks(s, perm[o:o + n].tolist())
            o += n
    g = torch.Generator(device="cuda").manual_seed(seed)
    total = sum(lens)
    for layer in range(wl.layers):
        if wl.dtype == 2:  # INT8: seeded codes and per-row scales
            kc = torch.randint(-127, 128, (total, KVD), generator=g, device="cuda", dtype=torch.int8)
            vc = torch.randint(-127, 128, (total, KVD), generator=g, device="cuda", dtype=torch.int8)
            ks = torch.rand((total, NKV), generator=g, device="cuda") * 0.03 + 0.001
            vs = torch.rand((total, NKV), generator=g, device="cuda") * 0.03 + 0.001
            o = 0
            for s, L in zip(ids, lens):
                if L:
                    P.import_i8(layer, s, 0, kc[o:o + L], vc[o:o + L], ks[o:o + L], vs[o:o + L])
                o += L
            del kc, vc, ks, vs
            continue
        k_all = encode_device(torch.randn((total, KVD), generator=g, device="cuda"), wl.dtype)
        v_all = encode_device(torch.randn((total, KVD), generator=g, device="cuda"), wl.dtype)
        o = 0
        for s, L in zip(ids, lens):
            P.import_rows(layer, s, 0, k_all[o:o + L], v_all[o:o + L])
            o += L
        del k_all, v_all
    for s, L in zip(ids, lens):
        P.set_cur_pos(s, L)
    torch.cuda.synchronize()
    B = len(wl.lens)
    return P, [ids[i * B:(i + 1) * B] for i in range(groups)]


class CudaRt:
    """The few CUDA runtime calls the e2e loops make, through ctypes (the
    runtime torch ships).  Streams and events are shared with torch."""

    def __init__(self):
        import ctypes as C
        import glob
        lib = None
        try:
            import nvidia
            for d in nvidia.__path__:
                for f in sorted(glob.glob(os.path.join(d, "cuda_runtime", "lib", "libcudart.so*"))):
                    lib = C.CDLL(f)
                    break
        except ImportError:
            pass
        self.C, self.lib = C, lib or C.CDLL("libcudart.so")
        v, i = C.c_void_p, C.c_int
        for name, args in (("cudaMemcpyAsync", [v, v, C.c_size_t, i, v]), ("cudaEventRecord", [v, v]),
                           ("cudaStreamWaitEvent", [v, v, C.c_uint]), ("cudaEventSynchronize", [v]),
                           ("cudaEventCreateWithFlags", [C.POINTER(v), C.c_uint]), ("cudaEventDestroy", [v]),
                           ("cudaEventElapsedTime", [C.POINTER(C.c_float), v, v])):
            fn = getattr(self.lib, name)
            fn.argtypes, fn.restype = args, i

    def _ok(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{what} failed with CUDA error {rc}")

    def event(self, timing=False):
        e = self.C.c_void_p()
        self._ok(self.lib.cudaEventCreateWithFlags(self.C.byref(e), 0 if timing else 2), "cudaEventCreate")
        return e

    def destroy(self, e):
        self.lib.cudaEventDestroy(e)

    def record(self, e, stream):
        self._ok(self.lib.cudaEventRecord(e, stream), "cudaEventRecord")

    def wait(self, stream, e):
        self._ok(self.lib.cudaStreamWaitEvent(stream, e, 0), "cudaStreamWaitEvent")

    def sync(self, e):
        self._ok(self.lib.cudaEventSynchronize(e), "cudaEventSynchronize")

    def h2d(self, dst, src, n, stream):
        self._ok(self.lib.cudaMemcpyAsync(dst, src, n, 1, stream), "cudaMemcpyAsync")

    def d2h(self, dst, src, n, stream):
        self._ok(self.lib.cudaMemcpyAsync(dst, src, n, 2, stream), "cudaMemcpyAsync")

    def elapsed(self, a, b) -> float:
        ms = self.C.c_float()
        self._ok(self.lib.cudaEventElapsedTime(self.C.byref(ms), a, b), "cudaEventElapsedTime")
        return ms.value



def run_ours(args, rank, world, local):
    import torch
    kv = load_pkg()
    kv.load()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    wl = make_workload(args.workload)
    if args.kv_dtype == "int8":
        wl.dtype = 2
        wl.desc += "; INT8 KV cache (per (token, KV head) row fp32 scale, codes in [-127, 127])"
        wl.data = wl.data.replace("K/V", "INT8 K/V codes and scales")
        wl.profile = None
    B, NL, lens = wl.batch, wl.layers, wl.lens
    K, W = args.steps, args.warmup
    NG = rotation_groups(wl)
    P, gids = setup_pool(kv, torch, local, wl, K + W + 10, seed=1 + rank, groups=NG)
    # The previous kernel before every decode launch is a decode (or merge)
    # launch of another group, or a copy: let each launch start its first
    # tile copies while that kernel finishes (the pool's overlap contract).
    P.set_overlap(True)
    P.set_merge_mode(kv.KVP_MERGE_CLUSTER if args.merge == "cluster" else kv.KVP_MERGE_GRID)
    P.plan(gids[0], append=[0] * len(gids[0]))  # the plan's shape only: appends nothing
    merge = "8-CTA clusters" if P.plan_clusters()[0] else "merge launch"
    P.commit()
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    nsteps = W + K
    q = torch.randn((nsteps, NL, B, HID), generator=g, device="cuda")
    kn = torch.randn((nsteps, NL, B, KVD), generator=g, device="cuda")
    vn = torch.randn((nsteps, NL, B, KVD), generator=g, device="cuda")
    out = torch.empty((NG, NL, B, HID), device="cuda")
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.int32, device="cuda")
    L = kv._lib
    h = P.h
    ids_c = [kv._ints(ids) for ids in gids]
    # One created stream for the library calls and every torch op from here
    # on (decode launches chain as programmatic dependents only on created
    # streams, not on the legacy default stream).
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.Stream())
    st = torch.cuda.current_stream().cuda_stream

    def chk(rc, fn):
        if rc != 0:
            raise kv.KVError(rc, fn, L.kv_last_error().decode())

    # device pointers of every (input row, layer) and (group, layer), built
    # once so the timed loops make nothing but C ABI calls
    in_ptr = [[(q[j, y].data_ptr(), kn[j, y].data_ptr(), vn[j, y].data_ptr()) for y in range(NL)]
              for j in range(nsteps)]
    out_ptr = [[out[gi, y].data_ptr() for y in range(NL)] for gi in range(NG)]

    def step(i, j=None):
        """Step i of the run (inputs row j): one plan, NL layer launches, one
        commit, for group i % NG, through the C ABI."""
        j = i if j is None else j
        gi = i % NG
        chk(L.attn_decode_plan(h, B, ids_c[gi], st), "attn_decode_plan")
        for y in range(NL):
            qa, ka, va = in_ptr[j][y]
            chk(L.attn_decode_append(h, y, qa, ka, va, out_ptr[gi][y], st), "attn_decode_append")
        chk(L.attn_decode_commit(h), "attn_decode_commit")

    def reset_lens():
        torch.cuda.synchronize()
        for ids in gids:
            for s, Ln in zip(ids, lens):
                P.set_cur_pos(s, Ln)

    sampler = ClockSampler(range(local, local + 1)) if rank == 0 else None
    if sampler:
        sampler.start()
    for i in range(W):
        step(i)
    # Keep the GPU loaded ~1 s so the clock samples reflect load; lengths
    # are put back afterwards so the timed steps see the stated contexts.
    t_end = time.time() + args.settle
    while time.time() < t_end:
        for i in range(4 * NG):
            step(i, i % nsteps)
        reset_lens()
    reset_lens()

    # ---- value: inputs resident in HBM, steps back to back ----
    # K steps (group i % NG each) between one pair of events on the launching
    # stream: tokens/s = B * K / elapsed, and the average launch duration is
    # elapsed / (K * NL) -- nothing else runs on the stream in between.
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    kc0 = kv.kernel_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t0 = time.perf_counter()
    for i in range(K):
        step(i, W + i)
    host_ms = (time.perf_counter() - t0) * 1e3
    e1.record()
    torch.cuda.synchronize()
    kernels = kv.kernel_count() - kc0
    step_ms = e0.elapsed_time(e1)
    if dist:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    assert P.device_status() == 0, "device-side check failed: " + L.kv_last_error().decode()
    kv_lens_per_step = [[Ln + 1 + i // NG for Ln in lens] for i in range(K)]

    # ---- isolated launches: L2 flushed before every step, the library's
    # events around every decode launch (each launch pays the event-to-event
    # floor of an otherwise idle stream) ----
    reset_lens()
    KI = min(K, 16)
    P.timing(True)
    for i in range(KI):
        flush.zero_()
        step(i, W + i)
    iso_ms, iso_launches = P.timing_read()
    P.timing(False)
    assert iso_launches == KI * NL

    # ---- e2e: host buffers, copies inside the timed region ----
    # Every step copies its inputs for all layers from pinned host memory --
    # per layer q [B][1536] | k [B][256] | v [B][256], the layout a fused QKV
    # projection writes -- on an upload stream, runs on the compute stream,
    # and reads all layers' outputs back to pinned memory on a download
    # stream, so copies overlap other groups' launches.  A group's next step
    # is issued only once its previous result is on the host.  Copies and
    # events go straight to the CUDA runtime (one call each).
    reset_lens()
    rt = CudaRt()
    R = min(K, 8)
    per = B * (HID + 2 * KVD)
    inh = torch.cat([q[W:W + R].reshape(R, NL, -1), kn[W:W + R].reshape(R, NL, -1),
                     vn[W:W + R].reshape(R, NL, -1)], dim=2).cpu().pin_memory()
    oh = torch.empty((NG, NL, B, HID)).pin_memory()
    ind = torch.empty((NG, NL, per), device="cuda")
    dptr = [[(ind[gi, y].data_ptr(), ind[gi, y].data_ptr() + 4 * B * HID,
              ind[gi, y].data_ptr() + 4 * B * (HID + KVD), out[gi, y].data_ptr()) for y in range(NL)]
            for gi in range(NG)]
    in_bytes, out_bytes = 4 * NL * per, 4 * NL * B * HID
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    ups, downs = up.cuda_stream, down.cuda_stream
    h2d = [rt.event() for _ in range(K)]
    kdone = [rt.event() for _ in range(K)]
    d2h = [rt.event() for _ in range(K)]
    a0, a1 = rt.event(timing=True), rt.event(timing=True)
    inh_p = [inh[r].data_ptr() for r in range(R)]
    ind_p = [ind[gi].data_ptr() for gi in range(NG)]
    oh_p = [oh[gi].data_ptr() for gi in range(NG)]
    out_p = [out[gi].data_ptr() for gi in range(NG)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    rt.record(a0, ups)
    for i in range(K):
        gi = i % NG
        if i >= NG:
            rt.sync(d2h[i - NG])  # the group's previous result is on the host
        rt.h2d(ind_p[gi], inh_p[i % R], in_bytes, ups)
        rt.record(h2d[i], ups)
        rt.wait(st, h2d[i])
        chk(L.attn_decode_plan(h, B, ids_c[gi], st), "attn_decode_plan")
        for y, (qa, ka, va, oa) in enumerate(dptr[gi]):
            chk(L.attn_decode_append(h, y, qa, ka, va, oa, st), "attn_decode_append")
        chk(L.attn_decode_commit(h), "attn_decode_commit")
        rt.record(kdone[i], st)
        rt.wait(downs, kdone[i])
        rt.d2h(oh_p[gi], out_p[gi], out_bytes, downs)
        rt.record(d2h[i], downs)
    rt.record(a1, downs)
    rt.sync(a1)
    e2e_ms = rt.elapsed(a0, a1)
    for e in h2d + kdone + d2h + [a0, a1]:
        rt.destroy(e)
    if dist:
        dist.barrier()

    times = torch.tensor([step_ms, iso_ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    step_ms, iso_ms, e2e_ms = times.tolist()
    if rank == 0:
        alg = sum(step_bytes(kl, wl.dtype) for kl in kv_lens_per_step) / K  # per launch
        peak, peak_kind = peak_hbm()
        launch_ms = step_ms / (K * NL)
        achieved = alg / (launch_ms * 1e-3) / 1e9
        iso_launch_ms = iso_ms / (KI * NL)
        line = {
            "metric": METRIC,
            "value": round(world * B * K / (step_ms * 1e-3), 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": K,
            "warmup": W,
            "ms_per_step": round(step_ms / K, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": wl.dtype_name,
            "data": wl.data,
            "config": {"workload": wl.desc, "name": wl.name,
                       "batch_per_gpu": B, "layers": NL, "kv_dtype": wl.dtype_name, "block_tokens": 16,
                       "parallelism": f"request placement x{world} (no data-path collective)",
                       "l2": (f"inputs larger than L2: {NG} independent groups of the {B} sequences "
                              f"({NG * step_bytes(lens, wl.dtype) * NL / 1e6:.0f} MB of K/V) stepped in "
                              "turn, so every step reads HBM; no flush" if NG > 1
                              else "inputs larger than L2 (no flush)")},
            "hbm_gbs_step": round(alg * NL / (step_ms / K * 1e-3) / 1e9, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": ncu_traffic(wl.profile), "peak_source": peak_kind,
                         "kernel_ms": round(launch_ms, 5), "algorithmic_bytes": round(alg),
                         "timing": "events around the K back-to-back steps; average launch = elapsed / launches",
                         "split_merge": merge,
                         "isolated": {"kernel_ms": round(iso_launch_ms, 5),
                                      "frac": round(alg / (iso_launch_ms * 1e-3) / 1e9 / peak, 4),
                                      "how": "L2 flushed before each step, events around each decode launch"}},
            "e2e": {"value": round(world * B * K / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * NL * B * (HID + 2 * KVD),
                    "d2h_bytes_per_step": 4 * NL * B * HID},
            "gpu_launches": int(kernels),
            "host_ms_per_step": round(host_ms / K, 5),
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    P.close()
    if dist:
        dist.destroy_process_group()


def run_long(args, rank, world, local):
    """A few long sequences split along the sequence across the GPUs: every
    rank holds a contiguous 1/world of each context in its own pool; per layer
    partial states, an NCCL all-gather and a log-sum-exp combine (strong
    scaling: the total work is fixed as the GPU count grows)."""
    import torch
    kv = load_pkg()
    kv.load()
    from importlib import import_module
    splitkv = import_module("rk3588_npu_b200.splitkv")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    wl = make_workload(args.workload)
    B, NL = wl.batch, wl.layers
    K, W = args.steps, args.warmup
    extra = K + W + 16
    lo, hi = splitkv.slice_bounds(wl.lens[0], rank, world)
    n_loc = hi - lo
    nb = B * (-(-(n_loc + extra) // 16)) + 16
    P = kv.Pool(local, NL, nb, num_q_heads=NQ, num_kv_heads=NKV, dtype=wl.dtype, max_seqs=B,
                max_seq_len=wl.lens[0] + extra + 32)
    S = splitkv.SplitKV(P, wl.lens, rank, world, transport=args.transport)
    S.reserve(extra)
    g = torch.Generator(device="cuda").manual_seed(3 + 1000 * rank)
    for layer in range(NL):
        for i in range(B):
            k = encode_device(torch.randn((n_loc, KVD), generator=g, device="cuda"), wl.dtype)
            v = encode_device(torch.randn((n_loc, KVD), generator=g, device="cuda"), wl.dtype)
            S.load_slice(layer, i, k, v)
    torch.cuda.synchronize()
    # q / k / v of a step are the same on every rank (seeded alike)
    gq = torch.Generator(device="cuda").manual_seed(103)
    R = min(K + W, 16)
    q = torch.randn((R, NL, B, HID), generator=gq, device="cuda")
    kn = torch.randn((R, NL, B, KVD), generator=gq, device="cuda")
    vn = torch.randn((R, NL, B, KVD), generator=gq, device="cuda")
    out = torch.empty((NL, B, HID), device="cuda")
    # a created stream for every call from here on, and decode launches that
    # start while the previous layer's merge / exchange finishes (the kernel
    # before each decode launch writes none of the pool's blocks)
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.Stream())
    P.set_overlap(True)

    # The step through the C ABI with pointers built once (what a C++ worker
    # does; the SplitKV methods cost more host time per layer than a layer
    # of a 1/8 slice takes on the GPU).  Same calls as S.begin_step /
    # S.layer / S.end_step.
    L = kv._lib
    h = P.h
    st = torch.cuda.current_stream().cuda_stream
    ids_c = kv._ints(S.ids)
    app_c = kv._ints([1 if S.is_last else 0] * B)

    def chk(rc, fn):
        if rc != 0:
            raise kv.KVError(rc, fn, L.kv_last_error().decode())

    in_ptr = [[(q[j, y].data_ptr(), kn[j, y].data_ptr(), vn[j, y].data_ptr()) for y in range(NL)]
              for j in range(R)]
    out_ptr = [out[y].data_ptr() for y in range(NL)]
    if world == 1:
        def layer_call(y, qa, ka, va):
            chk(L.attn_decode_append(h, y, qa, ka, va, out_ptr[y], st), "attn_decode_append")
    elif S._x is not None:
        def layer_call(y, qa, ka, va):
            chk(L.attn_decode_append_xgpu(h, y, qa, ka, va, out_ptr[y], S._x, st), "attn_decode_append_xgpu")
    else:
        def layer_call(y, qa, ka, va):
            chk(L.attn_decode_append_nccl(h, y, qa, ka, va, out_ptr[y], S._n, st), "attn_decode_append_nccl")

    def step(i, qs=None, ks=None, vs=None):
        if qs is not None:  # e2e: this step's inputs were just copied in
            ptrs = [(qs[y].data_ptr(), ks[y].data_ptr(), vs[y].data_ptr()) for y in range(NL)]
        else:
            ptrs = in_ptr[i % R]
        chk(L.attn_decode_plan_ex(h, B, ids_c, kv._ints(S.lengths), app_c, st), "attn_decode_plan_ex")
        for y in range(NL):
            qa, ka, va = ptrs[y]
            layer_call(y, qa, ka, va)
        chk(L.attn_decode_commit(h), "attn_decode_commit")
        S.lengths = [n + 1 for n in S.lengths]

    sampler = ClockSampler(range(local, local + 1)) if rank == 0 else None
    if sampler:
        sampler.start()
    for i in range(W):
        step(i)
    # ~settle seconds of load (the same number of steps on every rank)
    torch.cuda.synchronize()
    t0 = time.time()
    step(0)
    torch.cuda.synchronize()
    n_settle = int(args.settle / max(time.time() - t0, 1e-4))
    n_settle = torch.tensor([n_settle], device="cuda")
    if dist:
        dist.all_reduce(n_settle, op=dist.ReduceOp.MIN)
    for i in range(int(n_settle.item())):
        step(i)
        if (i + 1) % 8 == 0:
            torch.cuda.synchronize()
            S.rewind()
    torch.cuda.synchronize()
    S.rewind()

    # ---- value: K steps back to back between one pair of events ----
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    kc0 = kv.kernel_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        step(W + i)
    e1.record()
    torch.cuda.synchronize()
    kernels = kv.kernel_count() - kc0
    if dist:
        dist.barrier()
    step_ms = e0.elapsed_time(e1)
    # ---- the decode launches alone: the library's events around each one
    # (ordinary launches while timing), the same steps again ----
    S.rewind()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    P.timing(True)
    for i in range(K):
        step(W + i)
    torch.cuda.synchronize()
    kern_ms, launches = P.timing_read()
    P.timing(False)
    clocks = sampler.stop() if sampler else None
    assert launches == K * NL
    assert P.device_status() == 0, "device-side check failed: " + kv._lib.kv_last_error().decode()

    # ---- e2e: host inputs per step, outputs read back ----
    S.rewind()
    qh = q[:1].cpu().pin_memory()
    kh = kn[:1].cpu().pin_memory()
    vh = vn[:1].cpu().pin_memory()
    oh = torch.empty((NL, B, HID)).pin_memory()
    qd, kd, vd = torch.empty_like(q[0]), torch.empty_like(kn[0]), torch.empty_like(vn[0])
    e2e_ms = 0.0
    if dist:
        dist.barrier()
    for i in range(K):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        qd.copy_(qh[0], non_blocking=True)
        kd.copy_(kh[0], non_blocking=True)
        vd.copy_(vh[0], non_blocking=True)
        step(i, qd, kd, vd)
        oh.copy_(out, non_blocking=True)
        b.record()
        b.synchronize()
        e2e_ms += a.elapsed_time(b)
    if dist:
        dist.barrier()

    times = torch.tensor([step_ms, kern_ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    step_ms, kern_ms, e2e_ms = times.tolist()
    if rank == 0:
        # per-GPU bytes of one decode launch (rank 0's slice; the last rank's
        # differs by one appended token per sequence)
        alg = step_bytes([n_loc] * B)
        peak, peak_kind = peak_hbm()
        achieved = alg / (kern_ms / (K * NL) * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": round(B * K / (step_ms * 1e-3), 2),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": K,
            "warmup": W,
            "ms_per_step": round(step_ms / K, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": wl.dtype_name,
            "data": wl.data,
            "config": {"workload": wl.desc, "name": wl.name, "batch": B, "context": wl.lens[0],
                       "layers": NL, "kv_dtype": wl.dtype_name, "block_tokens": 16,
                       "parallelism": f"sequence split x{world} (" + (
                           "NCCL all-gather of partial states + combine launch" if args.transport == "nccl"
                           else "fused peer-memory exchange of partial states") + ")",
                       "l2": "inputs larger than L2 (no flush)"},
            "hbm_gbs_step": round(world * alg * NL / (step_ms / K * 1e-3) / 1e9, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": ncu_traffic(wl.profile), "peak_source": peak_kind,
                         "kernel_ms": round(kern_ms / (K * NL), 5), "algorithmic_bytes": round(alg),
                         "per": "GPU (its slice)"},
            "e2e": {"value": round(B * K / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * NL * B * (HID + 2 * KVD),
                    "d2h_bytes_per_step": 4 * NL * B * HID},
            "gpu_launches": int(kernels),
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    S.close()
    P.close()
    if dist:
        dist.destroy_process_group()


def run_serve(args, rank, world, local):
    """Continuous batching through serving.Server on every rank (placement
    replicated, each rank executes its own requests; no collective on the
    data path).  Strong scaling: the request stream is fixed."""
    import torch
    kv = load_pkg()
    kv.load()
    from importlib import import_module
    serving = import_module("rk3588_npu_b200.serving")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    wl = make_workload("serve")
    NL = wl.layers
    K, W = args.steps, args.warmup
    residents, stream = serve_stream()
    foot = sum(-(-(L + g) // 16) for L, g in residents) + 8 * (-(-(8192 + 256) // 16))
    nb = int(foot * 1.3 / world) + 2048
    P = kv.Pool(local, NL, nb, num_q_heads=NQ, num_kv_heads=NKV, dtype=wl.dtype, max_seqs=512,
                max_seq_len=8192 + 256 + 64)
    S = kv.Scheduler([nb] * world)
    srv = serving.Server(P, S, rank, world, chunk=512, prefill_slots=8)
    g = torch.Generator(device="cuda").manual_seed(4 + 1000 * rank)
    local_res = []
    for i, (L, gen) in enumerate(residents):
        srv.add_resident(serving.Request(i, L, gen))
        if srv.decoding[-1].gpu == rank:
            local_res.append(srv.decoding[-1])
    total = sum(r.prompt for r in local_res)
    for layer in range(NL):
        k_all = encode_device(torch.randn((max(total, 1), KVD), generator=g, device="cuda"), wl.dtype)
        v_all = encode_device(torch.randn((max(total, 1), KVD), generator=g, device="cuda"), wl.dtype)
        o = 0
        for r in local_res:
            P.import_rows(layer, r.seq, 0, k_all[o:o + r.prompt], v_all[o:o + r.prompt])
            o += r.prompt
        del k_all, v_all
    for i, (L, gen) in enumerate(stream):
        srv.submit(serving.Request(len(residents) + i, L, gen))
    maxrows = 512
    gq = torch.Generator(device="cuda").manual_seed(104 + rank)
    qb = torch.randn((NL, maxrows, HID), generator=gq, device="cuda")
    kb = torch.randn((NL, maxrows, KVD), generator=gq, device="cuda")
    vb = torch.randn((NL, maxrows, KVD), generator=gq, device="cuda")
    ob = torch.empty((NL, maxrows, HID), device="cuda")
    # prompt-chunk rows of all prefilling requests (8 slots x 512), concatenated
    kp = torch.randn((NL, 8 * 512, KVD), generator=gq, device="cuda")
    vp = torch.randn((NL, 8 * 512, KVD), generator=gq, device="cuda")

    def decode_io(layer, reqs):
        n = len(reqs)
        return qb[layer, :n], kb[layer, :n], vb[layer, :n], ob[layer, :n]

    def prefill_kv(layer, chunks):  # every local chunk at once (kv_append_chunk_batch)
        n = sum(c for _, _, c in chunks)
        return kp[layer, :n], vp[layer, :n]

    torch.cuda.synchronize()
    sampler = ClockSampler(range(local, local + 1)) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(W):
        srv.step(decode_io, prefill_batch_io=prefill_kv)
    # ~settle seconds more of untimed steps (the same count on every rank)
    torch.cuda.synchronize()
    t0 = time.time()
    srv.step(decode_io, prefill_batch_io=prefill_kv)
    torch.cuda.synchronize()
    n_settle = torch.tensor([int(args.settle / max(time.time() - t0, 1e-4))], device="cuda")
    if dist:
        dist.all_reduce(n_settle, op=dist.ReduceOp.MIN)
    for _ in range(int(n_settle.item())):
        srv.step(decode_io, prefill_batch_io=prefill_kv)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    alg = 0.0
    dec_tokens = pre_tokens = completed = 0
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    P.timing(True)
    kc0 = kv.kernel_count()
    for i in range(K):
        mine = srv.local_decode()
        alg += NL * step_bytes([r.length + 1 for r in mine]) if mine else 0.0
        e0, e1 = ev[i]
        e0.record()
        c = srv.step(decode_io, prefill_batch_io=prefill_kv)
        e1.record()
        dec_tokens += c["decode_tokens"]
        pre_tokens += c["prefill_tokens"]
        completed += c["completed"]
    torch.cuda.synchronize()
    kernels = kv.kernel_count() - kc0
    if dist:
        dist.barrier()
    step_ms = sum(a.elapsed_time(b) for a, b in ev)
    kern_ms, launches = P.timing_read()
    P.timing(False)
    clocks = sampler.stop() if sampler else None
    assert P.device_status() == 0, "device-side check failed: " + kv._lib.kv_last_error().decode()
    times = torch.tensor([step_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    step_ms = times.item()
    if rank == 0:
        peak, peak_kind = peak_hbm()
        achieved = alg / (kern_ms * 1e-3) / 1e9 if kern_ms > 0 else 0.0
        line = {
            "metric": METRIC,
            "value": round(dec_tokens / (step_ms * 1e-3), 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": K,
            "warmup": W,
            "ms_per_step": round(step_ms / K, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": wl.dtype_name,
            "data": wl.data,
            "config": {"workload": wl.desc, "name": wl.name, "layers": NL, "kv_dtype": wl.dtype_name,
                       "block_tokens": 16, "chunk": 512, "prefill_slots": 8,
                       "parallelism": f"request placement x{world} (no data-path collective)",
                       "l2": "inputs larger than L2 (no flush)"},
            "prefill_tokens_per_s": round(pre_tokens / (step_ms * 1e-3), 1),
            "decode_tokens_per_step": round(dec_tokens / K, 2),
            "completed": completed,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": None, "peak_source": peak_kind,
                         "kernel_ms": round(kern_ms / max(launches, 1), 5),
                         "per": "GPU 0, decode launches (prefill appends excluded)"},
            "gpu_launches": int(kernels),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    P.close()
    if dist:
        dist.destroy_process_group()


def run_prefill(args, rank, world, local):
    """Chunked-prefill attention (attn_prefill after kv_append_chunk) for 8
    requests per step; tensor-core bound.  One process per GPU, each its own
    requests (weak scaling)."""
    import torch
    kv = load_pkg()
    kv.load()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    wl = make_workload("prefill")
    NL, CH = wl.layers, 512
    K, W = args.steps, args.warmup
    _, stream = serve_stream()
    prompts = [L for L, _ in stream[:wl.batch]]
    pos0 = [max(0, (L // CH // 2) * CH) for L in prompts]
    need = sum(-(-(p + CH) // 16) for p in pos0) + 16
    P = kv.Pool(local, NL, need, num_q_heads=NQ, num_kv_heads=NKV, dtype=wl.dtype, max_seqs=wl.batch,
                max_seq_len=max(pos0) + CH + 32)
    g = torch.Generator(device="cuda").manual_seed(4 + 1000 * rank)
    ids = []
    for p0 in pos0:
        s = P.seq_alloc()
        P.reserve(s, p0 + CH)
        ids.append(s)
    for y in range(NL):
        for s, p0 in zip(ids, pos0):
            if p0:
                k = encode_device(torch.randn((p0, KVD), generator=g, device="cuda"), wl.dtype)
                v = encode_device(torch.randn((p0, KVD), generator=g, device="cuda"), wl.dtype)
                P.import_rows(y, s, 0, k, v)
    for s, p0 in zip(ids, pos0):
        P.set_cur_pos(s, p0)
    # every request's chunk rows, concatenated (as a batched projection writes them)
    R = wl.batch * CH
    qb = torch.randn((NL, R, HID), generator=g, device="cuda")
    kb = torch.randn((NL, R, KVD), generator=g, device="cuda")
    vb = torch.randn((NL, R, KVD), generator=g, device="cuda")
    ob = torch.empty((R, HID), device="cuda")
    L = kv._lib
    st = torch.cuda.current_stream().cuda_stream
    prefill_fn = L.attn_prefill_mma if args.prefill_kernel == "mma" else L.attn_prefill
    ids_c, pos_c, ns_c = kv._ints(ids), kv._ints(pos0), kv._ints([CH] * len(ids))

    def chk(rc, fn):
        if rc != 0:
            raise kv.KVError(rc, fn, L.kv_last_error().decode())

    def step():
        for y in range(NL):
            if args.prefill_kernel == "tc":  # all requests' chunks in shared launches
                chk(L.kv_append_chunk_batch(P.h, y, len(ids), ids_c, pos_c, ns_c, kb[y].data_ptr(),
                                            vb[y].data_ptr(), st), "kv_append_chunk_batch")
                chk(L.attn_prefill_batch(P.h, y, len(ids), ids_c, pos_c, ns_c, qb[y].data_ptr(), ob.data_ptr(),
                                         st), "attn_prefill_batch")
                continue
            for i, (s, p0) in enumerate(zip(ids, pos0)):  # one call per request
                r = i * CH
                chk(L.kv_append_chunk(P.h, y, s, p0, CH, kb[y, r].data_ptr(), vb[y, r].data_ptr(), st),
                    "kv_append_chunk")
                chk(prefill_fn(P.h, y, s, p0, CH, qb[y, r].data_ptr(), ob[r].data_ptr(), st), "attn_prefill")

    # real (not doubled by the hi/lo split) FLOPs: QK^T and PV, 2 * 128 each per (query, key, head)
    flops = NL * sum(sum(4.0 * HD * NQ * (p0 + i + 1) for i in range(CH)) for p0 in pos0)
    sampler = ClockSampler(range(local, local + 1)) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(W):
        step()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    kc0 = kv.kernel_count()
    for i in range(K):
        ev[i][0].record()
        step()
        ev[i][1].record()
    torch.cuda.synchronize()
    kernels = kv.kernel_count() - kc0
    if dist:
        dist.barrier()
    step_ms = sum(a.elapsed_time(b) for a, b in ev)
    clocks = sampler.stop() if sampler else None
    assert P.device_status() == 0, "device-side check failed: " + L.kv_last_error().decode()
    times = torch.tensor([step_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    step_ms = times.item()
    if rank == 0:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
            os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
        peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
        achieved = flops / (step_ms / K * 1e-3) / 1e12
        line = {
            "metric": "chunked-prefill attention tokens/s and achieved TFLOP/s vs B200 bf16 peak",
            "value": round(world * wl.batch * CH * K / (step_ms * 1e-3), 1),
            "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(step_ms / K, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": wl.dtype_name, "data": wl.data,
            "config": {"workload": wl.desc, "name": wl.name, "chunk": CH, "layers": NL,
                       "kernel": {"tc": "tcgen05, all requests per launch", "tc1": "tcgen05, one launch per request",
                                  "mma": "mma.sync, one launch per request"}[args.prefill_kernel],
                       "contexts_before_chunk": pos0, "l2": "inputs larger than L2 (no flush)"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_source": "measured (bf16 sustained)",
                         "note": "whole step (append + attention launches); the hi/lo operand "
                                 "splits issue 2x these FLOPs on the tensor cores"},
            "gpu_launches": int(kernels),
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_prefill(pos0, CH, NL, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    P.close()
    if dist:
        dist.destroy_process_group()


def cpu_baseline_prefill(pos0, ch, layers, seconds):
    """The reference's own RoPE + append + op_attention for one 512-token
    chunk (one request, one layer, 1 thread), scaled by attention FLOPs to
    the workload's 8 requests x 28 layers."""
    orc = _oracle()
    if not orc.have_ref():
        return {"value": None, "unit": "tokens/s", "cores": 1, "kind": "unavailable",
                "sample": "the reference functions were not built"}
    rng = np.random.default_rng(4)
    p0 = pos0[0]
    kc = np.zeros((p0 + ch, KVD), np.uint16)
    vc = np.zeros((p0 + ch, KVD), np.uint16)
    kc[:p0] = orc.encode(rng.standard_normal((p0, KVD), dtype=np.float32))
    vc[:p0] = orc.encode(rng.standard_normal((p0, KVD), dtype=np.float32))
    work = lambda p: sum(p + i + 1 for i in range(ch))
    t0 = time.perf_counter()
    reps = 0
    while reps == 0 or (time.perf_counter() - t0 < seconds and reps < 4):
        q = rng.standard_normal((ch, HID), dtype=np.float32)
        k = rng.standard_normal((ch, KVD), dtype=np.float32)
        v = rng.standard_normal((ch, KVD), dtype=np.float32)
        orc.ref_layer_step(q, k, v, kc, vc, p0)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    full = dt * layers * sum(work(p) for p in pos0) / work(p0)
    return {"value": round(len(pos0) * ch / full, 3), "unit": "tokens/s", "cores": 1, "kind": "reference",
            "sample": f"{reps} x one 512-token chunk at position {p0}, 1 layer, 1 host thread "
                      f"({dt:.2f} s each), scaled by attention work to {len(pos0)} chunks x {layers} "
                      f"layers; fp16 caches (the reference's only cache type)"}


def _qwen2():
    load_pkg()
    import importlib
    return importlib.import_module("rk3588_npu_b200.qwen2")


def run_model(args, rank, world, local):
    """Qwen2-1.5B greedy decode through the device model (qw2_forward, one
    token per step).  Every GPU runs its own replica of the model and its own
    request (replicas only: no collective).  value: device time (CUDA events
    on the model's stream around each step); e2e: the same calls timed on the
    host clock (host token id in, host argmax out, the call's one sync)."""
    import torch
    kv = load_pkg()
    kv.load()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    q2 = _qwen2()
    wl = make_workload("model1")
    K, W = args.steps, args.warmup
    M = q2.Model(local)
    t0 = time.perf_counter()
    M.load_synthetic(seed=0)
    load_s = time.perf_counter() - t0
    stream = torch.cuda.current_stream()
    kv.call("qw2_set_stream", M.h, stream.cuda_stream)
    prompt = q2.synth_prompt(128, q2.QWEN2_1_5B["vocab"], seed=0).tolist()
    assert len(prompt) + K + W <= q2.QWEN2_1_5B["max_position"], "steps + warmup must fit 512 positions"
    _, nxt = M.forward(prompt)
    for _ in range(W):
        _, nxt = M.forward([nxt])
    sampler = ClockSampler(range(local, local + 1)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(args.settle)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    kc0 = kv.kernel_count()
    pos0 = M.cur_pos()
    t_host = time.perf_counter()
    for i in range(K):
        ev[i][0].record(stream)
        _, nxt = M.forward([nxt])
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    host_s = time.perf_counter() - t_host
    kernels = kv.kernel_count() - kc0
    step_ms = sum(a.elapsed_time(b) for a, b in ev)
    clocks = sampler.stop() if sampler else None
    times = torch.tensor([step_ms, host_s], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.barrier()
    step_ms, host_s = times[0].item(), times[1].item()
    if rank == 0:
        wbytes = M.weight_bytes()
        # KV read of every layer at this step's length + the appended row
        kv_bytes = 28 * 2 * 2 * 128 * 2 * (pos0 + K / 2 + 1)
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
            os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
        peak = float(peaks.get("hbm_gbs", 6650.0))
        achieved = (wbytes + kv_bytes) / (step_ms / K * 1e-3) / 1e9
        line = {
            "metric": "Qwen2-1.5B greedy decode tokens/s and achieved HBM GB/s (weights + KV per token)",
            "value": round(world * K / (step_ms * 1e-3), 2), "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(step_ms / K, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": wl.data,
            "config": {"workload": wl.desc, "name": wl.name, "prompt": 128, "positions_timed": [pos0, pos0 + K],
                       "parallelism": "replicas only (one model and one request per GPU)",
                       "l2": "inputs larger than L2 (3.09 GB of weights per step, no flush)",
                       "weights_load_s": round(load_s, 1)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                         "note": "whole decode step (all launches); algorithmic bytes = fp16 weights "
                                 f"({wbytes} B: 28 layers of projections + the tied lm_head) + KV rows read"},
            "e2e": {"value": round(world * K / host_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4 + 4 * 32,
                    "note": "qw2_forward from a host token id to the host argmax (and the pool's status "
                            "words), host clock"},
            "gpu_launches": int(kernels),
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_model(q2, max(1, int(args.cpu_seconds // 3)))
        print(json.dumps(line), flush=True)
    M.close()
    if dist:
        dist.destroy_process_group()


def run_model_batch(args, rank, world, local):
    """Qwen2-1.5B greedy decode of `--sessions` concurrent sessions through
    the batching engine (qw2_generate_batch): every engine step is one
    forward over all sessions (one weight pass of the projections for up to
    8 rows, one planned decode-attention launch).  Each session first
    prefills its own 128-id prompt; the timed call then generates K ids per
    session (K + 1 forwards).  value: device events around that call; e2e:
    the host clock around it (host ids in and out)."""
    import torch
    kv = load_pkg()
    kv.load()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    q2 = _qwen2()
    B, K, W = args.sessions, args.steps, args.warmup
    M = q2.Model(local, max_sessions=B)
    M.load_synthetic(seed=0)
    stream = torch.cuda.current_stream()
    kv.call("qw2_set_stream", M.h, stream.cuda_stream)
    sessions = [0] + [M.create_session() for _ in range(B - 1)]
    prompts = [q2.synth_prompt(128, q2.QWEN2_1_5B["vocab"], seed=s).tolist() for s in range(B)]
    assert 128 + W + K + 2 <= q2.QWEN2_1_5B["max_position"], "steps + warmup must fit 512 positions"
    M.generate_batch([dict(session=s, input_ids=p, max_new_tokens=0) for s, p in zip(sessions, prompts)])
    last = [p[-1] for p in prompts]
    if W:
        out = M.generate_batch([dict(session=s, input_ids=[t], max_new_tokens=W) for s, t in zip(sessions, last)])
        last = [ids[-1] for ids, _ in out]
    sampler = ClockSampler(range(local, local + 1)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(args.settle)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    kc0 = kv.kernel_count()
    pos0 = M.session_len(0)
    t0 = time.perf_counter()
    e0.record(stream)
    out = M.generate_batch([dict(session=s, input_ids=[t], max_new_tokens=K) for s, t in zip(sessions, last)])
    e1.record(stream)
    torch.cuda.synchronize()
    host_s = time.perf_counter() - t0
    kernels = kv.kernel_count() - kc0
    dev_ms = e0.elapsed_time(e1)
    clocks = sampler.stop() if sampler else None
    tokens = sum(len(ids) for ids, _ in out)
    assert tokens == B * K and all(r["status"] == 0 for _, r in out)
    times = torch.tensor([dev_ms, host_s], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.barrier()
    dev_ms, host_s = times[0].item(), times[1].item()
    if rank == 0:
        wbytes = M.weight_bytes()
        steps = K + 1
        passes = -(-B // 8)  # the projections read their weights once per 8 rows
        kv_bytes = B * 28 * 2 * 2 * 128 * 2 * (pos0 + K / 2 + 1)
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
            os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
        peak = float(peaks.get("hbm_gbs", 6650.0))
        achieved = (passes * wbytes + kv_bytes) / (dev_ms / steps * 1e-3) / 1e9
        line = {
            "metric": "Qwen2-1.5B greedy decode tokens/s, concurrent sessions through the batching engine",
            "value": round(world * tokens / (dev_ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(dev_ms / steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (random-init N(0,0.02) weights from seed 0, RMSNorm weights 1; prompts seeds 0..B-1)",
            "config": {"workload": f"Qwen2-1.5B greedy decode of {B} sessions at once on one GPU (each after its "
                                   "own 128-id prompt), one engine step = one forward over all sessions",
                       "name": "model_batch", "sessions": B, "positions_timed": [pos0, pos0 + K + 1],
                       "parallelism": "replicas only (one model per GPU)",
                       "l2": "inputs larger than L2 (3.09 GB of weights per pass, no flush)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                         "note": f"whole engine step; algorithmic bytes = {passes} pass(es) over the fp16 "
                                 f"weights ({wbytes} B each) + the KV rows of {B} sessions"},
            "e2e": {"value": round(world * tokens / host_s, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 8 * B + 4 * 32,
                    "note": "qw2_generate_batch from host ids to host ids, host clock"},
            "gpu_launches": int(kernels),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    M.close()
    if dist:
        dist.destroy_process_group()


def _ref_model(q2, tmpdir):
    """The reference's Qwen2Model compiled from its sources (oracle/_ref),
    loaded from an F16 safetensors file of the same seeded weights."""
    import ctypes as C
    so = os.path.join(ROOT, "oracle", "_ref", "libqwen2ref.so")
    if not os.path.exists(so):
        return None, None
    R = C.CDLL(so)
    R.ref_qwen2_load.restype = C.c_void_p
    R.ref_qwen2_load.argtypes = [C.c_char_p]
    R.ref_qwen2_forward.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.c_int, C.c_void_p, C.c_int]
    R.ref_greedy_sample.argtypes = [C.c_void_p, C.c_int]
    R.ref_qwen2_free.argtypes = [C.c_void_p]
    os.makedirs(tmpdir, exist_ok=True)
    path = os.path.join(tmpdir, "model.safetensors")
    cfg = q2.QWEN2_1_5B
    q2.write_safetensors(path, q2.tensor_specs(cfg), q2.synth_weights(cfg, seed=0), dtype="F16")
    R.ref_set_threads(os.cpu_count() or 1)
    # the reference's loader reports progress on stdout (qwen2_model.cpp:53-117):
    # send it to stderr so this process's stdout stays one JSON line
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        m = R.ref_qwen2_load(tmpdir.encode())
    finally:
        os.dup2(saved, 1)
        os.close(saved)
    return R, m


def _ref_decode(R, m, q2, ids):
    import ctypes as C
    V = q2.QWEN2_1_5B["vocab"]
    logits = np.empty(V, np.float32)
    a = (C.c_int * len(ids))(*ids)
    R.ref_qwen2_forward(m, a, len(ids), logits.ctypes.data_as(C.c_void_p), V)
    return R.ref_greedy_sample(logits.ctypes.data_as(C.c_void_p), V)


def cpu_baseline_model(q2, tokens):
    """The reference's own model (Qwen2Model::forward, CPU stand-in linears on
    every host thread) decoding `tokens` greedy tokens from position 0."""
    import shutil
    tmp = "/tmp/qwen2_bench_ref"
    R, m = _ref_model(q2, tmp)
    if not m:
        shutil.rmtree(tmp, ignore_errors=True)
        return {"value": None, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "unavailable",
                "sample": "oracle/_ref/libqwen2ref.so was not built"}
    nxt = 0
    t0 = time.perf_counter()
    for _ in range(tokens):
        nxt = _ref_decode(R, m, q2, [nxt])
    dt = time.perf_counter() - t0
    R.ref_qwen2_free(m)
    shutil.rmtree(tmp, ignore_errors=True)
    return {"value": round(tokens / dt, 3), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "reference",
            "sample": f"{tokens} greedy decode tokens at positions 0..{tokens - 1} of the same seeded model "
                      f"({dt:.1f} s), Qwen2Model::forward compiled from the reference sources with a CPU "
                      f"fp16 linear stand-in on {os.cpu_count()} host threads"}


def run_reference_model(args, world):
    """Reference arm of the model workload: Qwen2Model::forward of the
    reference (oracle/_ref), one greedy token per step, all host threads."""
    q2 = _qwen2()
    import shutil
    tmp = "/tmp/qwen2_bench_ref"
    R, m = _ref_model(q2, tmp)
    wl = make_workload("model1")
    if not m:
        shutil.rmtree(tmp, ignore_errors=True)
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libqwen2ref.so was not built"}))
        return
    K, W = args.steps, args.warmup
    nxt = 0
    total = 0.0
    for i in range(W + K):
        t0 = time.perf_counter()
        nxt = _ref_decode(R, m, q2, [nxt])
        if i >= W:
            total += time.perf_counter() - t0
    R.ref_qwen2_free(m)
    shutil.rmtree(tmp, ignore_errors=True)
    value = round(K / total, 3)
    cores = os.cpu_count()
    sample = (f"{K} greedy decode tokens after {W} untimed, positions 0..{K + W - 1}, Qwen2Model::forward "
              f"compiled from the reference sources with a CPU fp16 linear stand-in on {cores} host threads")
    print(json.dumps({
        "impl": "reference", "metric": "Qwen2-1.5B greedy decode tokens/s and achieved HBM GB/s (weights + KV per token)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(total / K * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": wl.data,
        "config": {"workload": wl.desc, "name": wl.name},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
        flush=True)


# ------------------------------------------------------- CPU (reference) path
def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    return oracle


def cpu_workload(orc, lens, extra, seed=1):
    rng = np.random.default_rng(seed)
    kcs, vcs = [], []
    for L in lens:
        kc = np.zeros((L + extra, KVD), np.uint16)
        vc = np.zeros((L + extra, KVD), np.uint16)
        kc[:L] = orc.encode(rng.standard_normal((L, KVD), dtype=np.float32))
        vc[:L] = orc.encode(rng.standard_normal((L, KVD), dtype=np.float32))
        kcs.append(kc)
        vcs.append(vc)
    return kcs, vcs, rng


def cpu_step_fn(orc, threads):
    """One decode step of all sequences on the host: the reference's own
    functions (oracle/_ref) when built, else the C restatement."""
    if orc.have_ref():
        return "reference", lambda q, k, v, kc, vc, pos: orc.ref_batch_step(q, k, v, kc, vc, pos, threads)
    from concurrent.futures import ThreadPoolExecutor
    ex = ThreadPoolExecutor(threads)

    def port(q, k, v, kc, vc, pos):
        def one(i):
            o, _, _ = orc.layer_step(q[i:i + 1], k[i:i + 1], v[i:i + 1], kc[i], vc[i], int(pos[i]))
            return o[0]
        return np.stack(list(ex.map(one, range(len(kc)))))
    return "port", port


def cpu_sample(wl: Workload, nseq: int):
    """The first `nseq` sequences of the workload, one layer, and the factor
    that scales a step over them to a full step of the workload (all its
    sequences' tokens, all its layers)."""
    lens = wl.lens[:nseq]
    return lens, wl.layers * sum(wl.lens) / sum(lens)


CPU_DTYPE_NOTE = ("the reference CPU path keeps fp16 caches (its only cache type); "
                  "bf16 workloads are timed on it at the same sizes in fp16")


def cpu_baseline(wl: Workload, seconds):
    """Single-thread CPU sample of the same workload (rank 0, N=1 only)."""
    orc = _oracle()
    kind, fn = cpu_step_fn(orc, 1)
    max_steps = 64
    lens, scale = cpu_sample(wl, 32)
    n = len(lens)
    kcs, vcs, rng = cpu_workload(orc, lens, max_steps + 1)
    pos = list(lens)
    t0 = time.perf_counter()
    steps = 0
    while steps < max_steps and (steps == 0 or time.perf_counter() - t0 < seconds):
        q = rng.standard_normal((n, HID), dtype=np.float32)
        k = rng.standard_normal((n, KVD), dtype=np.float32)
        v = rng.standard_normal((n, KVD), dtype=np.float32)
        fn(q, k, v, kcs, vcs, pos)
        pos = [p + 1 for p in pos]
        steps += 1
    dt = time.perf_counter() - t0
    full_step = dt / steps * scale
    sample = (f"{steps} decode steps of {n} of the workload's {wl.batch} sequences, 1 layer, "
              f"1 host thread ({dt:.1f} s), scaled x{scale:.2f} to a full step")
    if wl.dtype != 0:
        sample += "; " + CPU_DTYPE_NOTE
    return {"value": round(wl.batch / full_step, 3), "unit": "tokens/s", "cores": 1, "kind": kind,
            "sample": sample}


def run_reference_prefill(args, world):
    """Reference arm of the prefill workload: the reference's RoPE + append +
    op_attention, one host thread per request; each step a bounded sample
    (the first 64 queries of every request's chunk, one layer), scaled by
    attention work to the full step."""
    from concurrent.futures import ThreadPoolExecutor
    orc = _oracle()
    wl = make_workload("prefill")
    CH, SUB, NL = 512, 64, wl.layers
    _, stream = serve_stream()
    pos0 = [max(0, (L // CH // 2) * CH) for L, _ in stream[:wl.batch]]
    rng = np.random.default_rng(4)
    caches = []
    for p0 in pos0:
        kc = np.zeros((p0 + CH, KVD), np.uint16)
        vc = np.zeros((p0 + CH, KVD), np.uint16)
        kc[:p0] = orc.encode(rng.standard_normal((p0, KVD), dtype=np.float32))
        vc[:p0] = orc.encode(rng.standard_normal((p0, KVD), dtype=np.float32))
        caches.append((kc, vc))
    threads = max(1, min(os.cpu_count() or 1, wl.batch))
    ex = ThreadPoolExecutor(threads)
    work_full = NL * sum(sum(p + i + 1 for i in range(CH)) for p in pos0)
    work_sub = sum(sum(p + i + 1 for i in range(SUB)) for p in pos0)
    K, W = args.steps, args.warmup
    total = 0.0
    for it in range(W + K):
        qs = [rng.standard_normal((SUB, HID), dtype=np.float32) for _ in pos0]
        ks = [rng.standard_normal((SUB, KVD), dtype=np.float32) for _ in pos0]
        vs = [rng.standard_normal((SUB, KVD), dtype=np.float32) for _ in pos0]
        t0 = time.perf_counter()
        list(ex.map(lambda j: orc.ref_layer_step(qs[j], ks[j], vs[j], caches[j][0], caches[j][1], pos0[j]),
                    range(len(pos0))))
        dt = time.perf_counter() - t0
        if it >= W:
            total += dt * work_full / work_sub
    value = round(wl.batch * CH * K / total, 3)
    sample = (f"{K} steps of the first {SUB} queries of each of the {wl.batch} chunks, 1 layer, {threads} "
              f"host threads (one per request), reference functions compiled from source, scaled by "
              f"attention work to {wl.batch} x {CH}-token chunks x {NL} layers; fp16 caches")
    line = {"impl": "reference", "metric": "chunked-prefill attention tokens/s and achieved TFLOP/s vs B200 bf16 peak",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(total / K * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": wl.dtype_name, "data": wl.data,
            "config": {"workload": wl.desc, "name": wl.name, "chunk": CH, "layers": NL},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference(args, rank, world):
    if rank != 0:
        return
    orc = _oracle()
    if args.workload == "prefill":
        run_reference_prefill(args, world)
        return
    if args.workload in ("model1", "model_batch"):
        run_reference_model(args, world)
        return
    wl = make_workload(args.workload)
    threads = max(1, min(os.cpu_count() or 1, wl.batch))
    kind, fn = cpu_step_fn(orc, threads)
    lens, scale = cpu_sample(wl, min(wl.batch, max(32, threads)))
    n = len(lens)
    K, W = args.steps, args.warmup
    kcs, vcs, rng = cpu_workload(orc, lens, K + W + 1)
    pos = list(lens)
    total = 0.0
    for i in range(W + K):
        q = rng.standard_normal((n, HID), dtype=np.float32)
        k = rng.standard_normal((n, KVD), dtype=np.float32)
        v = rng.standard_normal((n, KVD), dtype=np.float32)
        t0 = time.perf_counter()
        fn(q, k, v, kcs, vcs, pos)
        dt = time.perf_counter() - t0
        if i >= W:
            total += dt * scale
        pos = [p + 1 for p in pos]
    value = round(wl.batch * K / total, 3)
    sample = (f"{K} timed decode steps over {n} of the workload's {wl.batch} sequences, 1 layer, "
              f"{threads} host threads taking whole sequences, scaled x{scale:.2f} to a full step, "
              f"{'reference functions compiled from source' if kind == 'reference' else 'C restatement'}")
    if wl.dtype != 0:
        sample += "; " + CPU_DTYPE_NOTE
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(total / K * 1e3, 3),
            "higher_is_better": True,
            "scaling": "strong" if wl.name.startswith("long") or wl.name == "serve" else "weak",
            "vs_baseline": None,
            "dtype": wl.dtype_name, "data": wl.data,
            "config": {"workload": wl.desc, "name": wl.name, "batch_per_gpu": wl.batch,
                       "layers": wl.layers, "kv_dtype": wl.dtype_name},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.workload.startswith("long"):
        run_long(args, rank, world, local)
    elif args.workload == "serve":
        run_serve(args, rank, world, local)
    elif args.workload == "prefill":
        run_prefill(args, rank, world, local)
    elif args.workload == "model1":
        run_model(args, rank, world, local)
    elif args.workload == "model_batch":
        run_model_batch(args, rank, world, local)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
