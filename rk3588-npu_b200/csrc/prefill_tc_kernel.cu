// prefill_tc_kernel.cu -- chunked-prefill attention on the 5th-generation
// tensor cores (tcgen05 MMA, accumulators in tensor memory).
//
// Same semantics as prefill_kernel.cu (op_attention with seq = n > 1,
// worker/src/ops/op_attention.cpp:9-56, causal, GQA; q rotated here at
// pos0 + s): query s attends to positions [0, pos0 + s] of the pool.
//
// One launch covers the prompt chunks of up to kMaxChunkBatch sequences (their
// rows concatenated in q and out); the host lists each chunk's CTAs, longest
// first.  One CTA = one chunk, one KV head h, Tc = 128 / G query tokens x the
// G query heads of the group = up to 128 rows (row r = token r / G, head
// r % G), one key split.
//   warps 0-7  rows: warps w and w+4 own tensor-memory lanes 32(w%4).. (rows),
//              each half of the row's columns.  They rotate,
//              scale and split their q row into 16-bit hi + lo halves in shared
//              memory (K-major, 128-byte swizzle), then per key stage of 128
//              keys read the row's scores from tensor memory, apply the causal
//              mask, run the online softmax, rescale the output row in tensor
//              memory when the row maximum moved, and write P (hi + lo) back
//              over the stage's score columns in tensor memory, where the
//              P*V MMA reads it as its A operand;
//   warp 8     producer: bulk async copies (TMA engine, into this CTA only) of
//              the stage's eight (block, head) tiles -- each K tile as two
//              2 KiB halves into two 64-row K-major regions, each V tile whole;
//   warp 9     allocates 512 tensor-memory columns (two 128-column score
//              buffers, a 128-column output, 128 columns of Q hi + lo) and one
//              elected lane issues the MMAs:
//                     S = Qhi K^T + Qlo K^T  (M 128, N 128, K 16 x 8 x 2; Q from
//              tensor memory, K from shared memory),
//                     O += Phi V + Plo V    (M 128, N 128, K 16 x 8 x 2; P from
//              tensor memory, the pool's V tile an MN-major operand as it
//              lies), committing
//              each group to an mbarrier.  The next stage's S is computed while
//              the rows run the softmax of this one (double-buffered S); the
//              issuing lane polls both conditions and issues whichever group is
//              ready, so a P*V never waits for the next stage's copies.
// Every wait is bounded; a timeout is recorded in the pool's status words and
// the CTA still drains its copies, retires its MMAs and frees its tensor memory.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kvattn.h"
#include "kvattn_internal.h"

namespace kvattn {

namespace {

constexpr int kTcRows = 128;                 // MMA M: rows per CTA
constexpr int kTcStageKeys = 128;            // keys per stage = 8 tiles
constexpr int kTcStageTiles = kTcStageKeys / kBlockTokens;
constexpr int kTcRowWarps = 8;               // two softmax warps per row quarter
constexpr int kTcThreads = (kTcRowWarps + 2) * 32;
constexpr int kTcKvStages = 2;               // K/V stages in flight (64 KB each)
constexpr uint32_t kTmemCols = 512;          // S0 [0,128) S1 [128,256) O [256,384) Qhi [384,448) Qlo [448,512)
constexpr uint32_t kTmemO = 256;             // first column of the output accumulator
constexpr uint32_t kTmemQ = 384;             // first column of Q (hi, then lo)
constexpr long long kTcWaitLimit = 4000000000LL;
constexpr int kTcPartFloats = kHeadDim + 4;  // 16-byte aligned rows
constexpr float kTcRescale = 8.f;            // lazy-rescale threshold (log2 units)

// Shared memory: all regions 1024-byte aligned (128-byte swizzle atoms).
struct TcSmem {
    uint8_t q[2][2][kTcRows * 128];         // [hi/lo][dims 0-63 / 64-127][row][128 B]
    uint8_t k[kTcKvStages][2][kTcStageKeys * 128];  // [stage][dims half][key][128 B]
    uint8_t v[kTcKvStages][kTcStageTiles][kTileBytes];  // [stage][tile] pool tile layout
    uint64_t full[kTcKvStages], empty[kTcKvStages], s_full[2], p_ready, o_done, q_ready, mma_done;
    float xmax[2][2][kTcRows];  // [stage parity][column half][row]: the pair's row maxima
    float xsum[2][kTcRows];     // [column half][row]: the pair's row sums
    int xbad[2][2][4];          // [stage parity][column half][row quarter]: a wait gave up
    uint32_t tmem_base;
    int failed;
};

// ---- tcgen05 wrappers (PTX ISA, sm_100a) ----
__device__ __forceinline__ void tmem_alloc(uint32_t* holder, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]: A (M rows x K 16-bit values) read from
// tensor memory, lane = row, two K values per 32-bit column.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
    uint32_t* u = reinterpret_cast<uint32_t*>(r);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
          "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]),
          "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]),
          "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]),
          "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&r)[32]) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(r);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]),
        "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15]), "r"(u[16]),
        "r"(u[17]), "r"(u[18]), "r"(u[19]), "r"(u[20]), "r"(u[21]), "r"(u[22]), "r"(u[23]), "r"(u[24]),
        "r"(u[25]), "r"(u[26]), "r"(u[27]), "r"(u[28]), "r"(u[29]), "r"(u[30]), "r"(u[31])
        : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle, version 1 (sm_100):
// start address >> 4 [0,14), leading byte offset >> 4 [16,30), stride byte
// offset >> 4 [32,46), version [46,48), layout type [61,64) = 2 (128B swizzle).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16 with fp32 accumulate: D format [4,6) = 1,
// A/B format [7,10)/[10,13) (0 f16, 1 bf16), B major [16] (1 = MN-major),
// N >> 3 [17,23), M >> 4 [24,29).
__host__ __device__ constexpr uint32_t idesc_f16(int dt, int m, int n, int b_mn) {
    return (1u << 4) | ((uint32_t)dt << 7) | ((uint32_t)dt << 10) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, const PoolView& pv, int code,
                                        int* failed) {
    if (mbar_wait_bounded(bar, parity, kTcWaitLimit)) return true;
    if (atomicCAS(pv.status, 0, KV_ERR_TIMEOUT) == 0) {
        pv.status[1] = blockIdx.x;
        pv.status[2] = code;
    }
    *reinterpret_cast<volatile int*>(failed) = 1;
    return false;
}

// Swizzled byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-row region.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// P split into hi + lo 16-bit halves.  For bf16 with integer ops only: hi =
// the upper 16 bits (truncation, remainder below 2^-7 |p|, exact in fp32),
// lo = the upper 16 bits of that remainder, so |hi + lo - p| < 2^-14 |p|.
// For f16 the rounding converter is used.
template <int DT>
__device__ __forceinline__ void split_p(float a, float b, uint32_t& hi, uint32_t& lo) {
    if (DT == 1) {
        const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
        hi = __byte_perm(ua, ub, 0x7632);
        const float ra = a - __uint_as_float(ua & 0xFFFF0000u);
        const float rb = b - __uint_as_float(ub & 0xFFFF0000u);
        lo = __byte_perm(__float_as_uint(ra), __float_as_uint(rb), 0x7632);
    } else {
        split_pair<DT>(a, b, hi, lo);
    }
}

}  // namespace

// The chunk of CTA `cta` (chunks in cta0 order).
__device__ __forceinline__ int tc_chunk_of(const TcBatch& b, int cta) {
    int i = 0;
    while (i + 1 < b.nreq && cta >= b.r[i + 1].cta0) ++i;
    return i;
}

// A chunk's partial row ((qhead * n + s) * nsplit + sp), kTcPartFloats
// floats from its part0, holds o[128] (normalised), then m (base 2) and l.
template <int DT>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(PoolView pv, int layer, const __grid_constant__ TcBatch b, const float* __restrict__ q,
                      float* __restrict__ out, float* __restrict__ part) {
    extern __shared__ uint8_t smem_raw[];
    TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int G = pv.group, Tc = kTcRows / G;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const TcReq& R = b.r[tc_chunk_of(b, (int)blockIdx.x)];
    const int seq = R.seq, pos0 = R.pos0, n = R.n, nsplit = R.nsplit, tiles_per_split = R.tps;
    const int local = (int)blockIdx.x - R.cta0;
    const int h = (local / R.nq) % pv.kv_heads, sp = local / (R.nq * pv.kv_heads);
    const int s0 = (local % R.nq) * Tc;
    q += (size_t)R.row0 * (pv.q_heads * kHeadDim);
    out += (size_t)R.row0 * (pv.q_heads * kHeadDim);
    part += R.part0;
    const int s_last = min(n, s0 + Tc) - 1;
    const int ntiles = (pos0 + s_last) / kBlockTokens + 1;
    const int t_begin = sp * tiles_per_split;  // a multiple of kTcStageTiles
    const int t_end = min(ntiles, t_begin + tiles_per_split);
    const int nst = t_end > t_begin ? (t_end - t_begin + kTcStageTiles - 1) / kTcStageTiles : 0;
    const int kv_lim = min(t_end * kBlockTokens, pos0 + s_last + 1);  // keys >= kv_lim never count

    if (tid == 0) {
        for (int i = 0; i < kTcKvStages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) mbar_init(&sm.s_full[i], 1);
        mbar_init(&sm.p_ready, kTcRowWarps * 32);
        mbar_init(&sm.o_done, 1);
        mbar_init(&sm.q_ready, kTcRowWarps * 32);
        mbar_init(&sm.mma_done, 1);
        sm.failed = 0;
    }
    fence_mbar_init();
    if (warp == kTcRowWarps + 1) {
        tmem_alloc(&sm.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == kTcRowWarps) {
        // ---------------------------------------------------------- producer
        // Lane 0 waits for the stage and arms its barrier; lanes 0-7 then
        // issue one tile each (its block id, two K halves, the V tile).
        const uint64_t policy = policy_evict_first();
        const int* trow = pv.table + (size_t)seq * pv.max_blocks_per_seq;
        int issued = 0;
        for (int j = 0; j < nst; ++j) {
            const int b = j % kTcKvStages;
            int tiles = 0;
            for (int u = 0; u < kTcStageTiles; ++u) tiles += (t_begin + kTcStageTiles * j + u < t_end);
            int go = 1;
            if (lane == 0) {
                if (j >= kTcKvStages &&
                    !tc_wait(&sm.empty[b], ((j / kTcKvStages) - 1) & 1, pv, 700, &sm.failed))
                    go = 0;
                if (*reinterpret_cast<volatile int*>(&sm.failed)) go = 0;
                if (go) mbar_arrive_expect_tx(&sm.full[b], (uint32_t)tiles * 2u * kTileBytes);
            }
            go = __shfl_sync(0xffffffffu, go, 0);
            if (!go) break;
            if (lane < tiles) {
                const int t = t_begin + kTcStageTiles * j + lane;
                int blk = (t < pv.max_blocks_per_seq) ? trow[t] : -1;
                if (blk < 0 || blk >= pv.num_blocks) {
                    if (atomicCAS(pv.status, 0, 5) == 0) {
                        pv.status[1] = t;
                        pv.status[2] = 701;
                    }
                    blk = 0;  // stay inside the pool; the status voids the outputs
                }
                const size_t off = (size_t)layer * pv.layer_bytes + ((size_t)blk * pv.kv_heads + h) * kTileBytes;
                bulk_g2s_hint(sm.k[b][0] + lane * 2048, pv.k + off, 2048, &sm.full[b], policy);
                bulk_g2s_hint(sm.k[b][1] + lane * 2048, pv.k + off + 2048, 2048, &sm.full[b], policy);
                bulk_g2s_hint(sm.v[b][lane], pv.v + off, kTileBytes, &sm.full[b], policy);
            }
            __syncwarp();
            ++issued;
        }
        // Drain: the stages issued last must land before the CTA exits.
        if (lane == 0)
            for (int j = issued > kTcKvStages ? issued - kTcKvStages : 0; j < issued; ++j)
                mbar_wait_bounded(&sm.full[j % kTcKvStages], (j / kTcKvStages) & 1, kTcWaitLimit);
    } else if (warp == kTcRowWarps + 1) {
        // ------------------------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t id_qk = idesc_f16(DT, kTcRows, kTcStageKeys, 0);
            const uint32_t id_pv = idesc_f16(DT, kTcRows, kHeadDim, 1);
            bool ok = tc_wait(&sm.q_ready, 0, pv, 710, &sm.failed);
            // Q (hi, lo) is read from tensor memory: dims 16kk.. are columns
            // 8kk.. of each 64-column block.
            auto issue_qk = [&](int j) {
                const uint32_t kb = smem_u32(sm.k[j % kTcKvStages][0]);
                const uint32_t d = tmem + (uint32_t)((j & 1) * kTcStageKeys);  // S: one column per key
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t koff = (uint32_t)((kk >> 2) * (kTcStageKeys * 128) + (kk & 3) * 32);
                    const uint64_t bd = sdesc(kb + koff, 16, 1024);
#pragma unroll
                    for (int hl = 0; hl < 2; ++hl)
                        tc_mma_ts(d, tmem + kTmemQ + (uint32_t)(hl * 64 + kk * 8), bd, id_qk, (kk | hl) != 0);
                }
                tc_commit(&sm.s_full[j & 1]);
            };
            auto issue_pv = [&](int j) {
                const int b = j % kTcKvStages;
#pragma unroll
                for (int u = 0; u < kTcStageTiles; ++u) {
                    const uint64_t bd = sdesc(smem_u32(sm.v[b][u]), 2048, 1024);
#pragma unroll
                    for (int hl = 0; hl < 2; ++hl)  // P of stage j sits in its score columns (hi, then lo)
                        tc_mma_ts(tmem + kTmemO,
                                  tmem + (uint32_t)((j & 1) * kTcStageKeys + hl * (kTcStageKeys / 2) + u * 8), bd,
                                  id_pv, (j | u | hl) != 0);
                }
                tc_commit(&sm.o_done);
                tc_commit(&sm.empty[b]);
            };
            // Issue whichever group is ready: S of stage q (its K/V landed and
            // its score buffer was read) or P*V of stage p (its P written).
            int qk = 0, pvn = 0;
            long long since = clock64();
            while (ok && pvn < nst) {
                bool progressed = false;
                if (qk < nst && qk <= pvn + 1 &&
                    mbar_test_wait(&sm.full[qk % kTcKvStages], (qk / kTcKvStages) & 1)) {
                    tc_fence_after();
                    issue_qk(qk);
                    ++qk;
                    progressed = true;
                }
                if (pvn < qk && mbar_test_wait(&sm.p_ready, pvn & 1)) {
                    tc_fence_after();
                    issue_pv(pvn);
                    ++pvn;
                    progressed = true;
                }
                if (progressed) {
                    since = clock64();
                } else {
                    __nanosleep(32);  // leave the issue slots to the row warps
                    if (*reinterpret_cast<volatile int*>(&sm.failed)) {
                        ok = false;
                    } else if (clock64() - since > kTcWaitLimit) {
                        if (atomicCAS(pv.status, 0, KV_ERR_TIMEOUT) == 0) {
                            pv.status[1] = blockIdx.x;
                            pv.status[2] = 711;
                        }
                        *reinterpret_cast<volatile int*>(&sm.failed) = 1;
                        ok = false;
                    }
                }
            }
            // every MMA issued above has completed once this arrives
            tc_commit(&sm.mma_done);
            mbar_wait_bounded(&sm.mma_done, 0, kTcWaitLimit);
        }
    } else {
        // ------------------------------------------------------------ rows
        // Warps w and w + 4 share tensor-memory lanes 32(w%4).. (the CTA rows
        // 32(w%4)..+31): warp w < 4 takes score columns 0-31 and output
        // columns 0-63 of those rows, warp w + 4 the other halves; the pair
        // exchanges its row maxima (and at the end its row sums) through
        // shared memory at its own named barrier.
        const int quarter = warp & 3, ch = warp >> 2;
        const int r = quarter * 32 + lane;  // tensor-memory lane and CTA row
        const int tr = warp * 32 + lane;    // 0..255
        const int tok = r / G, g = r % G;
        const int s = s0 + tok;
        const bool live = tok < Tc && s < n;
        const int qhead = h * G + g;
        const int prow = pos0 + s;  // keys <= prow count for this row
        const int bar_id = 1 + quarter;
        // q rows: warp w prepares rows 16w..16w+15 one row at a time, lane l
        // holding dims 4l..4l+3 (one coalesced 512-byte load per row); the
        // NeoX partner of dim d < 64 is d + 64, i.e. lane l ^ 16.  Rotate
        // (non-fused, host cos/sin), scale, split into hi + lo 16-bit halves
        // and store into the swizzled K-major rows.
        {
            const float qscale = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
            const int half = lane >> 4, c = (lane & 15) >> 1;  // dims 4l..: half, 16-byte chunk
            const int ip = 4 * (lane & 15);                   // rotation pair index of dim 4l
            // 8 rows per batch: all their loads are issued before any is used.
#pragma unroll 1
            for (int i0 = 0; i0 < 16; i0 += 8) {
                float4 xs[8], c0s[8], c1s[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int rr = warp * 16 + i0 + u;
                    const int tk = rr / G, gg = rr % G, ss = s0 + tk;
                    xs[u] = c0s[u] = c1s[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (tk < Tc && ss < n) {  // the same for the whole warp
                        xs[u] = __ldg(reinterpret_cast<const float4*>(q + (size_t)ss * (pv.q_heads * kHeadDim) +
                                                                      (size_t)(h * G + gg) * kHeadDim + 4 * lane));
                        const float* cs = reinterpret_cast<const float*>(pv.rope + (size_t)(pos0 + ss) * (kHeadDim / 2));
                        c0s[u] = __ldg(reinterpret_cast<const float4*>(cs + 2 * ip));      // pairs ip, ip+1
                        c1s[u] = __ldg(reinterpret_cast<const float4*>(cs + 2 * ip + 4));  // pairs ip+2, ip+3
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int rr = warp * 16 + i0 + u;
                    const float4 x = xs[u], c0 = c0s[u], c1 = c1s[u];
                    float y[4];
                    y[0] = __shfl_xor_sync(0xffffffffu, x.x, 16);
                    y[1] = __shfl_xor_sync(0xffffffffu, x.y, 16);
                    y[2] = __shfl_xor_sync(0xffffffffu, x.z, 16);
                    y[3] = __shfl_xor_sync(0xffffffffu, x.w, 16);
                    const float xv[4] = {x.x, x.y, x.z, x.w};
                    const float cc[4] = {c0.x, c0.z, c1.x, c1.z}, sn[4] = {c0.y, c0.w, c1.y, c1.w};
                    float o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float r0, r1;  // (first half, second half) of the rotated pair
                        if (half == 0) rope_pair(xv[e], y[e], cc[e], sn[e], r0, r1);
                        else rope_pair(y[e], xv[e], cc[e], sn[e], r0, r1);
                        o[e] = (half == 0 ? r0 : r1) * qscale;
                    }
                    uint32_t wh[2], wl[2];
                    split_pair<DT>(o[0], o[1], wh[0], wl[0]);
                    split_pair<DT>(o[2], o[3], wh[1], wl[1]);
                    const uint32_t off = swz(rr, c) + (uint32_t)((lane & 1) * 8);
                    *reinterpret_cast<uint2*>(sm.q[0][half] + off) = make_uint2(wh[0], wh[1]);
                    *reinterpret_cast<uint2*>(sm.q[1][half] + off) = make_uint2(wl[0], wl[1]);
                }
            }
        }
        // Each row into its tensor-memory lane, the QK MMA's A operand:
        // warp ch = 0 copies the row's hi half, ch = 1 its lo half (64
        // columns, two dims per column), unswizzling the staged rows.
        named_bar_sync(5, kTcRowWarps * 32);  // every row staged
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
#pragma unroll 1
        for (int c2 = 0; c2 < 2; ++c2) {  // dims 64c2..64c2+63 = columns 32c2..
            float w[32];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                const uint4 v4 = *reinterpret_cast<const uint4*>(sm.q[ch][c2] + swz(r, cc));
                w[4 * cc + 0] = __uint_as_float(v4.x);
                w[4 * cc + 1] = __uint_as_float(v4.y);
                w[4 * cc + 2] = __uint_as_float(v4.z);
                w[4 * cc + 3] = __uint_as_float(v4.w);
            }
            tmem_st32(tmem + lane_base + kTmemQ + (uint32_t)(ch * 64 + c2 * 32), w);
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&sm.q_ready);

        float m = -INFINITY, lh = 0.f;  // lh: this half's share of the row sum
        bool ok = true;
        bool bad = false;  // a bounded wait of this warp gave up (acted on with the partner)
        for (int j = 0; j < nst; ++j) {
            // Both warps of a pair meet at their named barrier exactly once
            // per stage and leave the loop together: a failed wait is
            // published next to the row maxima and acted on after the barrier.
            bad = bad || !__all_sync(0xffffffffu, tc_wait(&sm.s_full[j & 1], (j >> 1) & 1, pv, 720, &sm.failed));
            constexpr int kHalf = kTcStageKeys / 2;  // this warp's keys of the stage
            float sc[kHalf];
            float mx = -INFINITY;
            const int kbase = (t_begin + kTcStageTiles * j) * kBlockTokens + ch * kHalf;
            if (!bad) {
                tc_fence_after();
                const uint32_t scol = tmem + lane_base + (uint32_t)((j & 1) * kTcStageKeys + ch * kHalf);
                tmem_ld32(scol, *reinterpret_cast<float(*)[32]>(sc));
                tmem_ld32(scol + 32u, *reinterpret_cast<float(*)[32]>(sc + 32));
                tc_wait_ld();
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                if (kbase + kHalf - 1 <= prow && kbase + kHalf <= kv_lim) {
                    // every key of this warp's half is visible to the row
#pragma unroll
                    for (int c = 0; c < kHalf; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], sc[c]);
                } else {
#pragma unroll
                    for (int c = 0; c < kHalf; ++c) {
                        const int key = kbase + c;
                        if (key > prow || key >= kv_lim) sc[c] = -INFINITY;
                        mx4[c & 3] = fmaxf(mx4[c & 3], sc[c]);
                    }
                }
                mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            }
            // exchange with the partner warp; the barrier also orders both
            // warps' score reads before either writes P over those columns
            sm.xmax[j & 1][ch][r] = mx;
            if (lane == 0) sm.xbad[j & 1][ch][quarter] = bad ? 1 : 0;
            tc_fence_before();
            named_bar_sync(bar_id, 64);
            tc_fence_after();
            if (bad || sm.xbad[j & 1][ch ^ 1][quarter]) {
                ok = false;
                *reinterpret_cast<volatile int*>(&sm.failed) = 1;
                break;
            }
            mx = fmaxf(mx, sm.xmax[j & 1][ch ^ 1][r]);
            // Lazy rescale: the reference max m moves only when a score
            // exceeds it by more than kTcRescale (base 2), so weights stay
            // <= 2^kTcRescale and the output row in tensor memory is rescaled
            // rarely; the sums and O always share the same reference, so the
            // result is the same softmax.  Both warps of a row decide alike.
            float alpha = 1.f;
            if (mx > m + kTcRescale || m == -INFINITY) {
                const float mn = fmaxf(m, mx);
                const float mu = (mn == -INFINITY) ? 0.f : mn;
                alpha = fast_exp2(m - mu);  // 0 while m is -inf
                m = mn;
            }
            const float mu = (m == -INFINITY) ? 0.f : m;
            float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < kHalf; ++c) {
                sc[c] = fast_exp2(sc[c] - mu);
                sum4[c & 3] += sc[c];
            }
            lh = lh * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
            // The last stage: V rows of keys >= kv_lim may hold anything
            // (stale smem, rows past the sequence); zero them so masked
            // weights (exactly 0) stay 0.
            if (j == nst - 1) {
                const int kb0 = (t_begin + kTcStageTiles * j) * kBlockTokens;
                for (int x = tr; x < kTcStageKeys * 16; x += 256) {  // (key row, 16-byte chunk)
                    const int kr = x >> 4, cq = x & 15;
                    if (kb0 + kr >= kv_lim) {
                        const int u = kr >> 4, t = kr & 15;
                        *reinterpret_cast<uint4*>(sm.v[j % kTcKvStages][u] + ((cq >> 3) * 16 + t) * 128 + (cq & 7) * 16) =
                            make_uint4(0u, 0u, 0u, 0u);
                    }
                }
            }
            // P (hi + lo) over this stage's score columns: the A operand of
            // P*V (hi of the 128 keys in columns 0-63, lo in 64-127, two keys
            // per column; this warp's 64 keys are columns 32ch.. of each).
            {
                float ph[32], pl[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    uint32_t hh, ll;
                    split_p<DT>(sc[2 * e], sc[2 * e + 1], hh, ll);
                    ph[e] = __uint_as_float(hh);
                    pl[e] = __uint_as_float(ll);
                }
                const uint32_t sbuf = tmem + lane_base + (uint32_t)((j & 1) * kTcStageKeys + ch * 32);
                tmem_st32(sbuf, ph);
                tmem_st32(sbuf + (uint32_t)(kTcStageKeys / 2), pl);
            }
            // The output row is rescaled only when its reference max moved
            // (rare after the first stages); then the previous P*V must be done.
            if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f) &&
                !(bad = !__all_sync(0xffffffffu, tc_wait(&sm.o_done, (j - 1) & 1, pv, 721, &sm.failed)))) {
                tc_fence_after();
#pragma unroll 1
                for (int c2 = 0; c2 < 2; ++c2) {
                    float o[32];
                    const uint32_t oc = tmem + lane_base + kTmemO + (uint32_t)(ch * 64 + 32 * c2);
                    tmem_ld32(oc, o);
                    tc_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] *= alpha;
                    tmem_st32(oc, o);
                }
            }
            tc_wait_st();
            if (j == nst - 1) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // zeroed V rows
            tc_fence_before();
            mbar_arrive(&sm.p_ready);
        }
        ok = ok && !bad;
        // ---- the output row: this warp's 64 columns ----
        const bool fin = ok && nst > 0 &&
                         __all_sync(0xffffffffu, tc_wait(&sm.o_done, (nst - 1) & 1, pv, 722, &sm.failed));
        sm.xsum[ch][r] = lh;
        named_bar_sync(bar_id, 64);
        const float l = lh + sm.xsum[ch ^ 1][r];
        if (fin) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            float* dst = nullptr;
            if (live) {
                if (nsplit == 1) {
                    dst = out + (size_t)s * (pv.q_heads * kHeadDim) + (size_t)qhead * kHeadDim + ch * 64;
                } else {
                    float* prow_p = part + (((size_t)qhead * n + s) * nsplit + sp) * kTcPartFloats;
                    if (ch == 0) {
                        prow_p[kHeadDim] = m;
                        prow_p[kHeadDim + 1] = l;
                    }
                    dst = prow_p + ch * 64;
                }
            }
#pragma unroll 1
            for (int c2 = 0; c2 < 2; ++c2) {
                float o[32];
                tmem_ld32(tmem + lane_base + kTmemO + (uint32_t)(ch * 64 + 32 * c2), o);
                tc_wait_ld();
                if (dst) {
#pragma unroll
                    for (int c = 0; c < 32; c += 4)
                        *reinterpret_cast<float4*>(dst + 32 * c2 + c) =
                            make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
                }
            }
        } else if (live && nsplit > 1) {
            // no keys in this split (or a failure): an empty partial
            if (ch == 0) {
                float* prow_p = part + (((size_t)qhead * n + s) * nsplit + sp) * kTcPartFloats;
                prow_p[kHeadDim] = -INFINITY;
                prow_p[kHeadDim + 1] = 0.f;
            }
        } else if (live && nst == 0) {
            float* dst = out + (size_t)s * (pv.q_heads * kHeadDim) + (size_t)qhead * kHeadDim + ch * 64;
            for (int c = 0; c < 64; ++c) dst[c] = 0.f;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcRowWarps + 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Merge of the key splits: one CTA per (query of a split chunk, 4 query
// heads), one thread per (head, dim).  Merge row x belongs to the last chunk
// whose mrow0 <= x (chunks without splits add no rows).
__global__ void __launch_bounds__(4 * kHeadDim)
    prefill_tc_merge_kernel(int q_heads, const __grid_constant__ TcBatch b, const float* __restrict__ part,
                            float* __restrict__ out) {
    const int x = blockIdx.x, qhead = blockIdx.y * 4 + threadIdx.y, d = threadIdx.x;
    if (qhead >= q_heads) return;
    int i = 0;
    while (i + 1 < b.nreq && x >= b.r[i + 1].mrow0) ++i;
    const TcReq& R = b.r[i];
    const int n = R.n, nsplit = R.nsplit, s = x - R.mrow0;
    part += R.part0;
    out += (size_t)R.row0 * q_heads * kHeadDim;
    float M = -INFINITY, L = 0.f, A = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
        const float* pr = part + (((size_t)qhead * n + s) * nsplit + sp) * kTcPartFloats;
        const float lc = __ldcg(pr + kHeadDim + 1);
        if (!(lc > 0.f)) continue;
        const float mc = __ldcg(pr + kHeadDim);
        const float Mn = fmaxf(M, mc);
        const float a = fast_exp2(M - Mn), e = lc * fast_exp2(mc - Mn);
        A = A * a + e * __ldcg(pr + d);
        L = L * a + e;
        M = Mn;
    }
    out[(size_t)s * q_heads * kHeadDim + (size_t)qhead * kHeadDim + d] = L > 0.f ? A / L : 0.f;
}

size_t prefill_tc_smem_bytes() { return sizeof(TcSmem) + 1024; }

int prefill_tc_tokens_per_cta(int group) { return kTcRows / group; }
int prefill_tc_stage_tiles() { return kTcStageTiles; }
size_t prefill_tc_part_floats(int q_heads, int n, int nsplit) {
    return (size_t)q_heads * n * nsplit * kTcPartFloats;
}

cudaError_t launch_prefill_tc(const PoolView& pv, int layer, const TcBatch& b, int total_ctas, int merge_rows,
                              const float* q, float* out, float* part, cudaStream_t st) {
    if (total_ctas <= 0) return cudaSuccess;
    const int smem = (int)prefill_tc_smem_bytes();
    cudaError_t e;
    if (pv.dtype == 0) {
        e = cudaFuncSetAttribute(prefill_tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        prefill_tc_kernel<0><<<total_ctas, kTcThreads, smem, st>>>(pv, layer, b, q, out, part);
    } else {
        e = cudaFuncSetAttribute(prefill_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        prefill_tc_kernel<1><<<total_ctas, kTcThreads, smem, st>>>(pv, layer, b, q, out, part);
    }
    e = counted(cudaGetLastError());
    if (e != cudaSuccess || merge_rows == 0) return e;
    prefill_tc_merge_kernel<<<dim3((unsigned)merge_rows, (unsigned)((pv.q_heads + 3) / 4)), dim3(kHeadDim, 4), 0,
                              st>>>(pv.q_heads, b, part, out);
    return counted(cudaGetLastError());
}

}  // namespace kvattn
