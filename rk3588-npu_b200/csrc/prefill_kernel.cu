// prefill_kernel.cu -- causal attention of a prompt chunk over the paged pool.
//
// op_attention (worker/src/ops/op_attention.cpp:9-56, with op_softmax,
// op_softmax.cpp:6-16) for seq = n > 1: query s of the chunk sits at absolute
// position pos0 + s and attends to positions [0, pos0 + s].  The chunk's own
// K/V rows are already in the pool (kv_append_chunk); q comes straight from
// the projections and is rotated here at pos0 + s with the same arithmetic as
// the append (op_rope.cpp:17-18, non-fused, host-built cos/sin table).
//
// Grid (query block of 16 tokens, KV head, key split).  Per CTA one consumer
// warp per query head of the KV group (G <= 8 warps) and one producer warp.
// The producer streams the (block, head) tiles of the key range -- 4 KiB of K
// and 4 KiB of V each, contiguous in HBM -- into a ring of shared-memory
// stages with 1-D bulk async copies (TMA engine, into this CTA only); every
// consumer warp reads every stage, so all G query heads share one load.
// Consumer warp g (query head h*G+g, 16 query tokens = the MMA's M):
//   S = Q K^T     mma.sync m16n8k16, q split into hi + lo 16-bit halves
//                 (products keep ~22 bits), K tile as the B operand (ldmatrix);
//   online softmax per query row in fp32 (base 2), causal mask;
//   O += P V      P as the A operand straight from S's accumulator layout
//                 (split hi + lo), V tile as the B operand (ldmatrix.trans).
// A split of the key range writes partial (m, l, o) per (query, head); a
// merge kernel combines the splits.  Tensor-core bound for long contexts;
// this mma.sync version is the baseline for a tcgen05 one.
//
// INT8 caches (DT 2): the producer copies the two compact tiles (codes +
// per-row scales); the consumer warps expand them together into one 16-bit
// tile pair per ring stage (codes are exact in fp16), each warp its share,
// and meet at a named barrier.  Scores are multiplied by the key's K scale
// and the softmax weights by the key's V scale on their way into P*V (the
// row sums keep the unscaled weights): attention over code * scale, as the
// decode kernel computes it.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kvattn.h"
#include "kvattn_internal.h"

namespace kvattn {

namespace {

constexpr int kPStages = 4;                   // ring stages (K + V tile each)
constexpr int kPStageBytes = 2 * kTileBytes;
constexpr long long kPWaitLimit = 4000000000LL;  // SM clocks before a wait gives up

template <int DT>
struct PrefillSmem {
    static constexpr int kWide = DT == 2 ? kPStages : 1;  // expanded stages (INT8 only)
    alignas(1024) uint8_t stage[kPStages][kPStageBytes];
    alignas(1024) uint8_t wide[kWide][DT == 2 ? kPStageBytes : 16];
    float scales[kWide][2][kBlockTokens];  // INT8: K and V scales of the stage's 16 keys
    uint64_t full[kPStages];
    uint64_t empty[kPStages];
};

// Thread (r = lane/4, c = lane%4) of a 16x16 A fragment holds rows r, r+8 and
// columns 2c, 2c+1 (regs 0, 1) and 8+2c, 9+2c (regs 2, 3).  For k-step kk the
// columns are dims kk*16 + ...; dims i < 64 pair with i + 64 in NeoX RoPE and
// kk + 4 holds the partners of kk, so each thread rotates its own pairs.
template <int DT>
__device__ __forceinline__ void load_q_rows(const PoolView& pv, const float* q, int s0, int n,
                                            int pos0, int qhead, float qscale, int lane,
                                            uint32_t (&qh)[8][4], uint32_t (&ql)[8][4]) {
    const int r = lane >> 2, c = lane & 3;
    const int hid = pv.q_heads * kHeadDim;
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // rows r (regs 0, 2) and r + 8 (regs 1, 3)
        const int s = s0 + r + 8 * half;
        const bool live = s < n;
        const float* qr = q + (size_t)(live ? s : 0) * hid + (size_t)qhead * kHeadDim;
        const float* cs = reinterpret_cast<const float*>(pv.rope + (size_t)(pos0 + (live ? s : 0)) * (kHeadDim / 2));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int w = 0; w < 2; ++w) {  // columns 2c.. (w = 0) and 8 + 2c.. (w = 1)
                const int i = kk * 16 + w * 8 + 2 * c;  // even, < 64
                float lo0 = 0.f, hi0 = 0.f, lo1 = 0.f, hi1 = 0.f;
                if (live) {
                    const float2 a = *reinterpret_cast<const float2*>(qr + i);
                    const float2 b = *reinterpret_cast<const float2*>(qr + i + 64);
                    const float4 t = *reinterpret_cast<const float4*>(cs + 2 * i);
                    rope_pair(a.x, b.x, t.x, t.y, lo0, hi0);
                    rope_pair(a.y, b.y, t.z, t.w, lo1, hi1);
                }
                const int reg = half + 2 * w;
                split_pair<DT>(lo0 * qscale, lo1 * qscale, qh[kk][reg], ql[kk][reg]);
                split_pair<DT>(hi0 * qscale, hi1 * qscale, qh[kk + 4][reg], ql[kk + 4][reg]);
            }
        }
    }
}

// D += A(16x16, row) * B(16x8, col) with A given as 4 registers.
template <int DT>
__device__ __forceinline__ void mma_a4(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    mma16816<DT>(d, a[0], a[1], a[2], a[3], b0, b1);
}

}  // namespace

// part layout: row (((h * nqb + qb) * nsplit + sp) * G + g) * 16 + r holds
// [m (base-2 units), l, o[128]].
template <int DT>
__global__ void __launch_bounds__(9 * 32, 1)
    prefill_kernel(PoolView pv, int layer, int seq, int pos0, int n, const float* __restrict__ q,
                   float* __restrict__ out, float* __restrict__ part, int nsplit, int tiles_per_split) {
    constexpr int MT = DT == 1 ? 1 : 0;  // operand type: bf16 for bf16 caches, else fp16
    constexpr int TB = DT == 2 ? kTileBytesI8 : kTileBytes;  // bytes of one K or V tile in HBM
    extern __shared__ uint8_t smem_raw[];
    PrefillSmem<DT>& sm =
        *reinterpret_cast<PrefillSmem<DT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int G = pv.group;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qb = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
    const int nqb = gridDim.x;
    const int s0 = qb * 16;
    const int s_last = min(n, s0 + 16) - 1;             // last query of the block
    const int ntiles = (pos0 + s_last) / kBlockTokens + 1;  // tiles holding keys [0, pos0 + s_last]
    const int t_begin = sp * tiles_per_split;
    const int t_end = min(ntiles, t_begin + tiles_per_split);
    const int* trow = pv.table + (size_t)seq * pv.max_blocks_per_seq;

    if (tid < kPStages) {
        mbar_init(&sm.full[tid], 1);
        mbar_init(&sm.empty[tid], G);
    }
    fence_mbar_init();
    __syncthreads();

    if (warp == G) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            uint32_t issued = 0;
            for (int t = t_begin; t < t_end; ++t) {
                const int k = t - t_begin, s = k % kPStages;
                if (k >= kPStages && !mbar_wait_bounded(&sm.empty[s], ((k / kPStages) - 1) & 1, kPWaitLimit)) {
                    if (atomicCAS(pv.status, 0, KV_ERR_TIMEOUT) == 0) {
                        pv.status[1] = qb;
                        pv.status[2] = 600;
                    }
                    break;
                }
                const int blk = (t < pv.max_blocks_per_seq) ? trow[t] : -1;
                if (blk < 0 || blk >= pv.num_blocks) {
                    if (atomicCAS(pv.status, 0, 5) == 0) {
                        pv.status[1] = t;
                        pv.status[2] = 601;
                    }
                    mbar_arrive(&sm.full[s]);  // nothing loaded: the outputs are void, the status says so
                } else {
                    const size_t off = (size_t)layer * pv.layer_bytes + ((size_t)blk * pv.kv_heads + h) * TB;
                    mbar_arrive_expect_tx(&sm.full[s], 2 * TB);
                    bulk_g2s_hint(sm.stage[s], pv.k + off, TB, &sm.full[s], policy);
                    bulk_g2s_hint(sm.stage[s] + TB, pv.v + off, TB, &sm.full[s], policy);
                }
                ++issued;
            }
            // Drain: every issued stage lands before the CTA exits.
            for (uint32_t k = issued > kPStages ? issued - kPStages : 0; k < issued; ++k)
                mbar_wait_bounded(&sm.full[k % kPStages], (k / kPStages) & 1, kPWaitLimit);
        }
        return;
    }
    if (warp > G) return;

    // -------------------------------------------------------------- consumer
    const int g = warp, qhead = h * G + g;
    const int r = lane >> 2, c = lane & 3;
    const float qscale = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
    uint32_t qh[8][4], ql[8][4];
    load_q_rows<MT>(pv, q, s0, n, pos0, qhead, qscale, lane, qh, ql);
    const int p0 = pos0 + s0 + r, p1 = p0 + 8;                // absolute positions of rows r, r+8
    float m2[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f};
    float o[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    const int mi = lane >> 3, rr = lane & 7;

    bool dead = false;  // INT8: a wait gave up; the warp keeps meeting the others at the barrier
    for (int t = t_begin; t < t_end; ++t) {
        const int k = t - t_begin, s = k % kPStages;
        if (!dead && !mbar_wait_bounded(&sm.full[s], (k / kPStages) & 1, kPWaitLimit)) {
            if (atomicCAS(pv.status, 0, KV_ERR_TIMEOUT) == 0) {
                pv.status[1] = qb;
                pv.status[2] = 602;
            }
            if (DT != 2) break;
            dead = true;
        }
        uint32_t sK = smem_u32(sm.stage[s]);
        uint32_t sV = sK + kTileBytes;
        float ksc[2][2] = {{1.f, 1.f}, {1.f, 1.f}}, vsc[2][2] = {{1.f, 1.f}, {1.f, 1.f}};  // keys 8j + 2c + e
        if constexpr (DT == 2) {
            // this warp's share of the two compact tiles into the stage's 16-bit pair
            const uint8_t* cK = sm.stage[s];
            uint8_t* wK = sm.wide[s];
            if (!dead) {
                for (int x = g * 32 + lane; x < 2 * kBlockTokens * 16; x += G * 32) {
                    const int which = x >> 8, y = x & 255, tt = y >> 4, ch = y & 15;
                    const uint2 raw = *reinterpret_cast<const uint2*>(cK + which * TB + i8_offset(tt, ch * 8));
                    const int8_t* cc = reinterpret_cast<const int8_t*>(&raw);
                    *reinterpret_cast<uint4*>(wK + which * kTileBytes + tile_offset(tt, ch * 8)) =
                        make_uint4(codes_to_half2(cc[0], cc[1]), codes_to_half2(cc[2], cc[3]),
                                   codes_to_half2(cc[4], cc[5]), codes_to_half2(cc[6], cc[7]));
                }
                if (g == 0)  // lanes 0-15 the K scales, 16-31 the V scales
                    sm.scales[s][lane >> 4][lane & 15] =
                        reinterpret_cast<const float*>(cK + (lane >> 4) * TB + kBlockTokens * kHeadDim)[lane & 15];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[s]);  // the compact stage is no longer read
            named_bar_sync(1, G * 32);                  // every share expanded
            if (dead) continue;
            sK = smem_u32(wK);
            sV = sK + kTileBytes;
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    ksc[j][e] = sm.scales[s][0][8 * j + 2 * c + e];
                    vsc[j][e] = sm.scales[s][1][8 * j + 2 * c + e];
                }
        }
        // ---- S[16 q][16 keys] = Q K^T ----
        float sc[2][4] = {};
        {
            const int key = (mi >> 1) * 8 + rr;
            const uint32_t rowb = sK + (uint32_t)key * 128u;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const int cidx = 2 * kk + (mi & 1);
                const uint32_t addr = rowb + (uint32_t)(cidx >> 3) * 2048u + (uint32_t)(((cidx & 7) ^ rr) << 4);
                uint32_t b00, b01, b10, b11;
                ldsm_x4(addr, b00, b01, b10, b11);
                mma_a4<MT>(sc[0], qh[kk], b00, b01);
                mma_a4<MT>(sc[1], qh[kk], b10, b11);
                mma_a4<MT>(sc[0], ql[kk], b00, b01);
                mma_a4<MT>(sc[1], ql[kk], b10, b11);
            }
        }
        if constexpr (DT == 2) {  // scores of codes times the key's K scale
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                sc[j][0] *= ksc[j][0];
                sc[j][1] *= ksc[j][1];
                sc[j][2] *= ksc[j][0];
                sc[j][3] *= ksc[j][1];
            }
        }
        // causal mask (and keys past the context of the last query)
        const int kb = t * kBlockTokens;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int k0 = kb + 8 * j + 2 * c;
            if (k0 > p0) sc[j][0] = -INFINITY;
            if (k0 + 1 > p0) sc[j][1] = -INFINITY;
            if (k0 > p1) sc[j][2] = -INFINITY;
            if (k0 + 1 > p1) sc[j][3] = -INFINITY;
        }
        // ---- online softmax, rows r (values 0, 1) and r + 8 (values 2, 3) ----
        float bm0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
        float bm1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 1));
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 2));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 1));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 2));
        const float mn0 = fmaxf(m2[0], bm0), mn1 = fmaxf(m2[1], bm1);
        const float mu0 = (mn0 == -INFINITY) ? 0.f : mn0;
        const float mu1 = (mn1 == -INFINITY) ? 0.f : mn1;
        const float al0 = fast_exp2(m2[0] - mu0), al1 = fast_exp2(m2[1] - mu1);
        m2[0] = mn0;
        m2[1] = mn1;
        float pv_[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            pv_[j][0] = fast_exp2(sc[j][0] - mu0);
            pv_[j][1] = fast_exp2(sc[j][1] - mu0);
            pv_[j][2] = fast_exp2(sc[j][2] - mu1);
            pv_[j][3] = fast_exp2(sc[j][3] - mu1);
        }
        lsum[0] = lsum[0] * al0 + (pv_[0][0] + pv_[0][1]) + (pv_[1][0] + pv_[1][1]);
        lsum[1] = lsum[1] * al1 + (pv_[0][2] + pv_[0][3]) + (pv_[1][2] + pv_[1][3]);
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
            o[nt][0] *= al0;
            o[nt][1] *= al0;
            o[nt][2] *= al1;
            o[nt][3] *= al1;
        }
        // P as the A operand: regs (row r, keys 2c..), (row r+8, keys 2c..),
        // (row r, keys 8+2c..), (row r+8, keys 8+2c..)
        if constexpr (DT == 2) {  // weights times the key's V scale (masked keys stay exactly 0)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                pv_[j][0] = pv_[j][0] > 0.f ? pv_[j][0] * vsc[j][0] : 0.f;
                pv_[j][1] = pv_[j][1] > 0.f ? pv_[j][1] * vsc[j][1] : 0.f;
                pv_[j][2] = pv_[j][2] > 0.f ? pv_[j][2] * vsc[j][0] : 0.f;
                pv_[j][3] = pv_[j][3] > 0.f ? pv_[j][3] * vsc[j][1] : 0.f;
            }
        }
        uint32_t ph[4], pl[4];
        split_pair<MT>(pv_[0][0], pv_[0][1], ph[0], pl[0]);
        split_pair<MT>(pv_[0][2], pv_[0][3], ph[1], pl[1]);
        split_pair<MT>(pv_[1][0], pv_[1][1], ph[2], pl[2]);
        split_pair<MT>(pv_[1][2], pv_[1][3], ph[3], pl[3]);
        // ---- O[16 q][128] += P V ----
        {
            const int key = (mi & 1) * 8 + rr;
            const uint32_t rowb = sV + (uint32_t)key * 128u;
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int cidx = 2 * m + (mi >> 1);
                const uint32_t addr = rowb + (uint32_t)(cidx >> 3) * 2048u + (uint32_t)(((cidx & 7) ^ rr) << 4);
                uint32_t b0a, b1a, b0b, b1b;  // dims 16m..16m+7 (a) and 16m+8.. (b)
                ldsm_x4_t(addr, b0a, b1a, b0b, b1b);
                mma_a4<MT>(o[2 * m], ph, b0a, b1a);
                mma_a4<MT>(o[2 * m + 1], ph, b0b, b1b);
                mma_a4<MT>(o[2 * m], pl, b0a, b1a);
                mma_a4<MT>(o[2 * m + 1], pl, b0b, b1b);
            }
        }
        __syncwarp();
        if (DT != 2 && lane == 0) mbar_arrive(&sm.empty[s]);
    }

    // ---- row sums across the quad, then outputs or partials ----
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        lsum[0] += __shfl_xor_sync(0xffffffffu, lsum[0], off);
        lsum[1] += __shfl_xor_sync(0xffffffffu, lsum[1], off);
    }
    const int hid = pv.q_heads * kHeadDim;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int s = s0 + r + 8 * half;
        if (s >= n) continue;
        const float L = lsum[half];
        const float inv = L > 0.f ? 1.f / L : 0.f;
        if (nsplit == 1) {
            float* orow = out + (size_t)s * hid + (size_t)qhead * kHeadDim;
#pragma unroll
            for (int nt = 0; nt < 16; ++nt)
                *reinterpret_cast<float2*>(orow + nt * 8 + 2 * c) =
                    make_float2(o[nt][2 * half] * inv, o[nt][2 * half + 1] * inv);
        } else {
            float* prow = part + ((((size_t)h * nqb + qb) * nsplit + sp) * G + g) * 16 * (2 + kHeadDim) +
                          (size_t)(r + 8 * half) * (2 + kHeadDim);
            if (c == 0) {
                prow[0] = m2[half];
                prow[1] = L;
            }
#pragma unroll
            for (int nt = 0; nt < 16; ++nt)
                *reinterpret_cast<float2*>(prow + 2 + nt * 8 + 2 * c) =
                    make_float2(o[nt][2 * half] * inv, o[nt][2 * half + 1] * inv);
        }
    }
}

// Merge of the key splits: one CTA per (query, query head), one thread per dim.
__global__ void __launch_bounds__(kHeadDim)
    prefill_merge_kernel(PoolView pv, int n, const float* __restrict__ part, float* __restrict__ out,
                         int nqb, int nsplit) {
    const int s = blockIdx.x, qhead = blockIdx.y, d = threadIdx.x;
    if (s >= n) return;
    const int G = pv.group, h = qhead / G, g = qhead % G, qb = s / 16, r = s % 16;
    float M = -INFINITY, L = 0.f, A = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
        const float* prow = part + ((((size_t)h * nqb + qb) * nsplit + sp) * G + g) * 16 * (2 + kHeadDim) +
                            (size_t)r * (2 + kHeadDim);
        const float lc = __ldcg(prow + 1);
        if (!(lc > 0.f)) continue;  // a split with no unmasked key
        const float mc = __ldcg(prow);
        const float Mn = fmaxf(M, mc);
        const float a = fast_exp2(M - Mn), e = lc * fast_exp2(mc - Mn);
        A = A * a + e * __ldcg(prow + 2 + d);
        L = L * a + e;
        M = Mn;
    }
    out[(size_t)s * pv.q_heads * kHeadDim + (size_t)qhead * kHeadDim + d] = L > 0.f ? A / L : 0.f;
}


cudaError_t launch_prefill(const PoolView& pv, int layer, int seq, int pos0, int n, const float* q,
                           float* out, float* part, int nsplit, int tiles_per_split, cudaStream_t st) {
    const int nqb = (n + 15) / 16;
    const dim3 grid((unsigned)nqb, (unsigned)pv.kv_heads, (unsigned)nsplit);
    const int threads = (pv.group + 1) * 32;
    if (pv.dtype == 0) {
        const int smem = (int)sizeof(PrefillSmem<0>) + 1024;
        cudaFuncSetAttribute(prefill_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        prefill_kernel<0><<<grid, threads, smem, st>>>(pv, layer, seq, pos0, n, q, out, part, nsplit,
                                                       tiles_per_split);
    } else if (pv.dtype == 1) {
        const int smem = (int)sizeof(PrefillSmem<1>) + 1024;
        cudaFuncSetAttribute(prefill_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        prefill_kernel<1><<<grid, threads, smem, st>>>(pv, layer, seq, pos0, n, q, out, part, nsplit,
                                                       tiles_per_split);
    } else {
        const int smem = (int)sizeof(PrefillSmem<2>) + 1024;
        cudaFuncSetAttribute(prefill_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        prefill_kernel<2><<<grid, threads, smem, st>>>(pv, layer, seq, pos0, n, q, out, part, nsplit,
                                                       tiles_per_split);
    }
    cudaError_t e = counted(cudaGetLastError());
    if (e != cudaSuccess || nsplit == 1) return e;
    prefill_merge_kernel<<<dim3((unsigned)n, (unsigned)pv.q_heads), kHeadDim, 0, st>>>(pv, n, part, out,
                                                                                      nqb, nsplit);
    return counted(cudaGetLastError());
}

}  // namespace kvattn
