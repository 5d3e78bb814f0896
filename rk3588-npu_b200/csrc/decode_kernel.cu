// decode_kernel.cu -- fused RoPE + KV append + grouped-query split-KV decode
// attention over the paged pool, one launch per layer.
//
// Replaces, for seq = 1, steps 3-5 of Qwen2Model::forward
// (worker/src/model/qwen2_model.cpp:180-206): op_rope (op_rope.cpp:8-30),
// the append loop (qwen2_model.cpp:188-200) and op_attention with op_softmax
// (op_attention.cpp:9-56, op_softmax.cpp:6-16).
//
// Work: the host planner flattens the step into segments (one per batch slot
// and KV head, all its 16-token blocks) and gives every CTA one contiguous,
// equal run of that flat block sequence; a segment crossing a CTA boundary
// becomes several pieces.  Per CTA:
//   warp 4     producer: lane l < 8 owns ring stage l and issues 1-D bulk
//              async copies (TMA engine, into this CTA only) of the K and V tiles
//              (4 KiB each, contiguous in HBM) of flat blocks l, l+8, ...; the
//              eight lanes run in step, so one instruction issues up to eight
//              stages, and each lane fetches its next block id a round ahead;
//   warps 0-3  consumers: flat block f goes to warp f % 4 (two ring stages
//              per warp).  Per block: S^T = K * Q^T with mma.sync m16n8k16
//              (16 tokens x 8 query heads, fp32 q split into hi + lo 16-bit
//              halves so the products keep ~22 bits), online softmax in fp32
//              (base 2), P^T transposed in registers with movmatrix,
//              O^T += V^T * P^T (P split hi + lo).
// At the end of a piece the four warps' states are merged in shared memory.
// A segment cut into pieces keeps per-piece partial (m, l, o) states, merged
// in one of two ways the plan chooses:
//  * a small combine kernel, launched behind the decode grid with
//    programmatic dependent launch (resident early, released when the grid
//    completes), merges each split segment's pieces (written to HBM) with
//    one round of loads;
//  * when the plan keeps every segment inside a cluster of kClusterCtas
//    CTAs, the states stay in shared memory: after a cluster barrier the CTA
//    holding a segment's first block reads the other pieces' states over
//    distributed shared memory (ld.shared::cluster), writes the merged rows
//    and releases the cluster with a second barrier, so the step is one
//    launch.
//
// INT8 caches: the ring has 16 stages of compact tiles (codes + row scales,
// half the bytes of a 16-bit block) and the consumers read the codes in
// place: ldmatrix on pairs of codes, each pair converted to an exact f16x2 in
// registers, the scores scaled by the key's K scale and the weights by its V
// scale (consume_block_i8).
//
// The new token: the consumer that owns the block holding position kv_len-1
// rotates k (non-fused fp32, cos/sin from the host-built table), encodes k
// and v with the truncating encoders, stores the row to HBM (the append) and
// into the staged tile, so attention sees exactly what the cache holds.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kvattn_internal.h"

namespace kvattn {

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;

// Shared-memory ring per cache type: a stage holds one block's K and V tiles
// as they lie in HBM -- 16-bit caches the swizzled mma layout (8 KB a
// stage), INT8 caches the compact tiles (codes in the swizzled i8_offset
// layout + row scales, 4.1 KB a stage), which the consumers read in place.
// INT8 stages are half the size, so the ring has twice as many: the bytes
// in flight per CTA, which bound its streaming rate, stay the same.
// Stage k of the ring is consumed by warp k % kConsumerWarps.  With the
// stage count a multiple of kConsumerWarps every stage belongs to ONE warp,
// which consumes its rounds in order; so no waiter is ever more than one
// phase ahead of a barrier, the condition under which a parity wait is
// unambiguous.  (With 6 stages and 4 warps a warp could wait on round r+1 of
// a stage whose round r, owned by another warp, had not landed; the parity
// test then passed early.)
template <int DT>
struct StageCfg {
    static constexpr int tile = kTileBytes;
    static constexpr int stage = 2 * kTileBytes;
    static constexpr int stages = 8;
};
template <>
struct StageCfg<2> {
    static constexpr int tile = kTileBytesI8;
    static constexpr int stage = 2 * kTileBytesI8;
    static constexpr int stages = 16;
};
static_assert(StageCfg<0>::stages % kConsumerWarps == 0 && StageCfg<2>::stages % kConsumerWarps == 0,
              "each ring stage must belong to one consumer warp");
static_assert(StageCfg<2>::stages <= 32, "one producer lane per stage");
// The tensor-core operand type: fp16 for fp16 and int8 caches (int8 codes are
// exact in fp16), bf16 for bf16 caches.
template <int DT>
__host__ __device__ constexpr int mma_type() { return DT == 1 ? 1 : 0; }
constexpr int kMergeStride = 132;            // floats per (warp, head) row, padded
constexpr long long kWaitLimit = 4000000000LL;  // SM clocks (~2 s) before a wait gives up
constexpr int kQPre = 4;                     // pieces whose q fragments are prepared up front

// One piece of a CTA's range: blocks [b0, b1) of segment (slot, head).  A
// split piece (its segment has blocks in other CTAs too) writes its partial
// state to partials[part]; any other piece writes the output rows directly.
struct Piece {
    int slot;
    int head;
    int b0;
    int b1;
    int split;  // 0 whole segment, 1 merged by the combine kernel, 2 merged in the cluster
    int part;   // split 1: partials row; split 2: cpart slot (0 first piece, 1 last)
    int span;   // split 2, first piece of its segment: CTAs after this one holding the rest
    int pad;
};

template <int DT>
struct Smem {
    static constexpr int kS = StageCfg<DT>::stages;
    alignas(1024) uint8_t stage[kS][StageCfg<DT>::stage];
    float merge_o[kConsumerWarps][kMaxGroup][kMergeStride];
    float merge_m[kConsumerWarps][kMaxGroup];
    float merge_l[kConsumerWarps][kMaxGroup];
    float merge_w[kMaxGroup][kConsumerWarps];  // weight 2^(m_w - M) of warp w's state, per head
    float merge_inv[kMaxGroup];                // 1 / L per head (0 for an empty head)
    float merge_M[kMaxGroup];
    float merge_L[kMaxGroup];
    // States of the first and last piece when they are split inside a
    // cluster: m[8], l[8], o[8][128] (the layout of a partials row).
    alignas(16) float cpart[2][kPartialFloats];
    Piece items[kMaxCtaItems];        // this CTA's pieces
    int cum[kMaxCtaItems + 1];        // flat block offset of each piece
    int ok[kMaxCtaItems];             // piece's slot passed the checks
    // q fragments (hi, lo) of the first kQPre pieces, as each lane holds them
    // q fragments (hi, lo) of the pieces in flight, slot j % kQPre for piece
    // j: [hi/lo][k-step][lane] = the lane's two registers of that k-step.
    // The consumers read them per block from here rather than holding 32
    // registers across the block loop.
    uint2 qfrag[kQPre][2][8][32];
    uint64_t full[kS];
    uint64_t empty[kS];
    int nitems;
    int last_flag;
    int failed;
    int prod_issued;                  // stages issued by the producer (progress record)
    int cons_done[kConsumerWarps];    // stages released by each consumer warp
};

// Record the first device-side error: status[0] = code, [1] = item, [2] = detail.
__device__ __forceinline__ void report(const PoolView& pv, int code, int item, int detail) {
    if (atomicCAS(pv.status, 0, code) == 0) {
        pv.status[1] = item;
        pv.status[2] = detail;
    }
}

// A bounded wait gave up: record where (status[3..16]) for the host to read.
template <class SmemT>
__device__ __forceinline__ void flag_timeout(const PoolView& pv, SmemT& sm, int item, int role,
                                             uint32_t k) {
    if (atomicCAS(pv.status, 0, 7 /* KV_ERR_TIMEOUT */) == 0) {
        const int s = k % SmemT::kS;
        const uint64_t f = *reinterpret_cast<volatile uint64_t*>(&sm.full[s]);
        const uint64_t e = *reinterpret_cast<volatile uint64_t*>(&sm.empty[s]);
        pv.status[1] = item;
        pv.status[2] = role;
        pv.status[3] = blockIdx.x;
        pv.status[4] = threadIdx.x >> 5;
        pv.status[5] = (int)k;
        pv.status[6] = (int)(k / SmemT::kS);
        pv.status[7] = (int)(uint32_t)f;
        pv.status[8] = (int)(uint32_t)(f >> 32);
        pv.status[9] = (int)(uint32_t)e;
        pv.status[10] = (int)(uint32_t)(e >> 32);
        pv.status[11] = *reinterpret_cast<volatile int*>(&sm.prod_issued);
        for (int w = 0; w < kConsumerWarps; ++w)
            pv.status[12 + w] = *reinterpret_cast<volatile int*>(&sm.cons_done[w]);
    }
    sm.failed = 1;
}

// Slot fields checked before any access they lead to (the plan comes from the
// host planner; a slot that fails is reported and its pieces are skipped).
__device__ __forceinline__ int slot_check(const PoolView& pv, const DecodeSlot& s) {
    if (s.seq < 0 || s.seq >= pv.max_seqs) return 3;
    if (s.kv_len < 0 || s.kv_len > pv.max_blocks_per_seq * kBlockTokens) return 4;
    if (s.rope_pos < 0 || s.rope_pos >= pv.max_seq_len) return 5;
    if (s.new_block >= 0 && (s.kv_len < 1 || s.new_block >= pv.num_blocks)) return 6;
    return 0;
}

__host__ __device__ __forceinline__ int nblocks_of(int kv_len) { return (kv_len + kBlockTokens - 1) / kBlockTokens; }

// Position of flat block f (< a.total) of a launch: segment k (slot i, KV
// head h), block b of its nb.  seg_f0 is increasing (segments have blocks).
template <int S>
__device__ __forceinline__ void locate(const DecodeArgs<S>& a, int f, int& k, int& i, int& h, int& b, int& nb) {
    int lo = 0, hi = a.nsegs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.seg_f0[mid] <= f) lo = mid;
        else hi = mid - 1;
    }
    k = lo;
    i = a.seg[k] & 0xffff;
    h = a.seg[k] >> 16;
    b = f - a.seg_f0[k];
    nb = a.seg_f0[k + 1] - a.seg_f0[k];
}

// Step a position `n` flat blocks forward (never past the launch's segments).
template <int S>
__device__ __forceinline__ void advance(const DecodeArgs<S>& a, int n, int& k, int& i, int& h, int& b, int& nb) {
    b += n;
    while (b >= nb && k < a.nsegs) {
        b -= nb;
        if (++k < a.nsegs) {
            i = a.seg[k] & 0xffff;
            h = a.seg[k] >> 16;
            nb = a.seg_f0[k + 1] - a.seg_f0[k];
        } else {
            nb = 1;
        }
    }
}

// Segment (slot i, head h, nb blocks) is usable: it names a slot of the
// launch (checked before that slot is read) whose fields pass slot_check,
// a KV head of the pool, and the slot's block count.
template <int S>
__device__ __forceinline__ bool seg_ok(const DecodeArgs<S>& a, const PoolView& pv, int i, int h, int nb) {
    return i < a.nslots && h >= 0 && h < pv.kv_heads && slot_check(pv, a.slot[i]) == 0 && nb == nblocks_of(a.slot[i].kv_len) &&
           nb > 0;
}

// Tile id (block * kv_heads + head) of block b of a slot's segment, or -1
// for a block that holds only the new token (nothing to load).  The new
// token's block comes from the plan, every other from the block table.
__device__ __forceinline__ int tile_of(const PoolView& pv, const DecodeSlot& s, int h, int b) {
    int blk;
    if (s.new_block >= 0 && b == (s.kv_len - 1) / kBlockTokens) {
        if (s.kv_len - b * kBlockTokens == 1) return -1;
        blk = s.new_block;
    } else {
        blk = __ldcg(pv.table + (size_t)s.seq * pv.max_blocks_per_seq + b);
    }
    return blk * pv.kv_heads + h;
}

// Rotated, pre-scaled q of query head (head*group + g) as mma B fragments.
// Thread (g = lane/4, c = lane%4) holds, for k-step kk, dims kk*16 + 2c + {0,1}
// (reg 0) and kk*16 + 8 + 2c + {0,1} (reg 1).  Dims i < 64 pair with i + 64
// in NeoX RoPE, and kk + 4 covers exactly the partners of kk, so each thread
// rotates its own 16 pairs.
template <int DT>
__device__ __forceinline__ void load_q_frags(const PoolView& pv, const float* q, int row,
                                             int head, int rope_pos, float qscale, int lane,
                                             uint32_t (&qh)[8][2], uint32_t (&ql)[8][2]) {
    const int g = lane >> 2, c = lane & 3;
    if (g >= pv.group) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) qh[kk][0] = qh[kk][1] = ql[kk][0] = ql[kk][1] = 0u;
        return;
    }
    const float* qr = q + (size_t)row * (pv.q_heads * kHeadDim) + (size_t)(head * pv.group + g) * kHeadDim;
    const float* cs = reinterpret_cast<const float*>(pv.rope + (size_t)rope_pos * (kHeadDim / 2));
    if constexpr (DT == 2) {
        // INT8 keys are read in place by ldmatrix as pairs of codes: k-step
        // kk's slots 2c, 2c+1 / 2c+8, 2c+9 hold dims kk*16 + 4c + {0, 1} /
        // {2, 3} (a permutation of the dot product's terms, the same for
        // every key row), so this thread's q dims are kk*16 + 4c .. + 3.
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const int i = kk * 16 + 4 * c;  // < 64; partners i + 64 are k-step kk + 4
            const float2 a01 = *reinterpret_cast<const float2*>(qr + i);  // q rows are 8-byte aligned
            const float2 a23 = *reinterpret_cast<const float2*>(qr + i + 2);
            const float2 b01 = *reinterpret_cast<const float2*>(qr + i + 64);
            const float2 b23 = *reinterpret_cast<const float2*>(qr + i + 66);
            const float4 a = make_float4(a01.x, a01.y, a23.x, a23.y);
            const float4 b = make_float4(b01.x, b01.y, b23.x, b23.y);
            const float4 t0 = *reinterpret_cast<const float4*>(cs + 2 * i);      // c_i, s_i, c_i+1, s_i+1
            const float4 t1 = *reinterpret_cast<const float4*>(cs + 2 * i + 4);  // c_i+2, s_i+2, ...
            float lo[4], hi[4];
            rope_pair(a.x, b.x, t0.x, t0.y, lo[0], hi[0]);
            rope_pair(a.y, b.y, t0.z, t0.w, lo[1], hi[1]);
            rope_pair(a.z, b.z, t1.x, t1.y, lo[2], hi[2]);
            rope_pair(a.w, b.w, t1.z, t1.w, lo[3], hi[3]);
            split_pair<0>(lo[0] * qscale, lo[1] * qscale, qh[kk][0], ql[kk][0]);
            split_pair<0>(lo[2] * qscale, lo[3] * qscale, qh[kk][1], ql[kk][1]);
            split_pair<0>(hi[0] * qscale, hi[1] * qscale, qh[kk + 4][0], ql[kk + 4][0]);
            split_pair<0>(hi[2] * qscale, hi[3] * qscale, qh[kk + 4][1], ql[kk + 4][1]);
        }
    } else {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int i = kk * 16 + r * 8 + 2 * c;  // even, < 64
                float2 a = *reinterpret_cast<const float2*>(qr + i);
                float2 b = *reinterpret_cast<const float2*>(qr + i + 64);
                float4 t = *reinterpret_cast<const float4*>(cs + 2 * i);  // c_i, s_i, c_i+1, s_i+1
                float lo0, hi0, lo1, hi1;
                rope_pair(a.x, b.x, t.x, t.y, lo0, hi0);
                rope_pair(a.y, b.y, t.z, t.w, lo1, hi1);
                split_pair<mma_type<DT>()>(lo0 * qscale, lo1 * qscale, qh[kk][r], ql[kk][r]);
                split_pair<mma_type<DT>()>(hi0 * qscale, hi1 * qscale, qh[kk + 4][r], ql[kk + 4][r]);
            }
        }
    }
}

// Write the new token's encoded K and V rows for `head` into the staged tiles
// (row `t`) and into the pool block `blk` of `layer` (the append).
template <int DT>
__device__ __forceinline__ void write_new_row(const PoolView& pv, int layer, int blk, int head,
                                              int t, const float* k_new, const float* v_new,
                                              int row, int rope_pos, uint8_t* sK, uint8_t* sV,
                                              int lane) {
    const size_t kvw = (size_t)pv.kv_heads * kHeadDim;
    const float* kr = k_new + (size_t)row * kvw + (size_t)head * kHeadDim;
    const float* vr = v_new + (size_t)row * kvw + (size_t)head * kHeadDim;
    const float* cs = reinterpret_cast<const float*>(pv.rope + (size_t)rope_pos * (kHeadDim / 2));
    const int i = 2 * lane;  // dims i, i+1 and their partners i+64, i+65
    float2 a = *reinterpret_cast<const float2*>(kr + i);
    float2 b = *reinterpret_cast<const float2*>(kr + i + 64);
    float4 cc = *reinterpret_cast<const float4*>(cs + 2 * i);
    float lo0, hi0, lo1, hi1;
    rope_pair(a.x, b.x, cc.x, cc.y, lo0, hi0);
    rope_pair(a.y, b.y, cc.z, cc.w, lo1, hi1);
    const uint32_t klo = (uint32_t)enc_trunc<DT>(lo0) | ((uint32_t)enc_trunc<DT>(lo1) << 16);
    const uint32_t khi = (uint32_t)enc_trunc<DT>(hi0) | ((uint32_t)enc_trunc<DT>(hi1) << 16);
    float2 va = *reinterpret_cast<const float2*>(vr + i);
    float2 vb = *reinterpret_cast<const float2*>(vr + i + 64);
    const uint32_t vlo = (uint32_t)enc_trunc<DT>(va.x) | ((uint32_t)enc_trunc<DT>(va.y) << 16);
    const uint32_t vhi = (uint32_t)enc_trunc<DT>(vb.x) | ((uint32_t)enc_trunc<DT>(vb.y) << 16);
    const uint32_t o_lo = tile_offset(t, i), o_hi = tile_offset(t, i + 64);
    const size_t tile = (size_t)layer * pv.layer_bytes + ((size_t)blk * pv.kv_heads + head) * kTileBytes;
    *reinterpret_cast<uint32_t*>(pv.k + tile + o_lo) = klo;
    *reinterpret_cast<uint32_t*>(pv.k + tile + o_hi) = khi;
    *reinterpret_cast<uint32_t*>(pv.v + tile + o_lo) = vlo;
    *reinterpret_cast<uint32_t*>(pv.v + tile + o_hi) = vhi;
    *reinterpret_cast<uint32_t*>(sK + o_lo) = klo;
    *reinterpret_cast<uint32_t*>(sK + o_hi) = khi;
    *reinterpret_cast<uint32_t*>(sV + o_lo) = vlo;
    *reinterpret_cast<uint32_t*>(sV + o_hi) = vhi;
}

// INT8 cache: the new token's k (rotated) and v rows quantised by the warp
// (quant_row_warp), codes and scales stored to the pool tile (the append)
// and the codes into the staged compact tiles; ks / vs receive the row's
// scales.
__device__ __forceinline__ void write_new_row_i8(const PoolView& pv, int layer, int blk, int head, int t,
                                                 const float* k_new, const float* v_new, int row, int rope_pos,
                                                 uint8_t* sK, uint8_t* sV, int lane, float& ks, float& vs) {
    const size_t kvw = (size_t)pv.kv_heads * kHeadDim;
    const float* kr = k_new + (size_t)row * kvw + (size_t)head * kHeadDim;
    const float* vr = v_new + (size_t)row * kvw + (size_t)head * kHeadDim;
    const float* cs = reinterpret_cast<const float*>(pv.rope + (size_t)rope_pos * (kHeadDim / 2));
    const int i = 2 * lane;  // dims i, i+1 and their partners i+64, i+65
    const float2 a = *reinterpret_cast<const float2*>(kr + i);
    const float2 b = *reinterpret_cast<const float2*>(kr + i + 64);
    const float4 cc = *reinterpret_cast<const float4*>(cs + 2 * i);
    float kx[4], vx[4];
    rope_pair(a.x, b.x, cc.x, cc.y, kx[0], kx[2]);
    rope_pair(a.y, b.y, cc.z, cc.w, kx[1], kx[3]);
    const float2 va = *reinterpret_cast<const float2*>(vr + i);
    const float2 vb = *reinterpret_cast<const float2*>(vr + i + 64);
    vx[0] = va.x;
    vx[1] = va.y;
    vx[2] = vb.x;
    vx[3] = vb.y;
    int8_t kc[4], vc[4];
    ks = quant_row_warp(kx, kc);
    vs = quant_row_warp(vx, vc);
    const size_t tile = (size_t)layer * pv.layer_bytes + ((size_t)blk * pv.kv_heads + head) * kTileBytesI8;
    uint8_t* kt = pv.k + tile;
    uint8_t* vt = pv.v + tile;
    const uint32_t o_lo = i8_offset(t, i), o_hi = i8_offset(t, i + 64);
    *reinterpret_cast<char2*>(kt + o_lo) = make_char2(kc[0], kc[1]);
    *reinterpret_cast<char2*>(kt + o_hi) = make_char2(kc[2], kc[3]);
    *reinterpret_cast<char2*>(vt + o_lo) = make_char2(vc[0], vc[1]);
    *reinterpret_cast<char2*>(vt + o_hi) = make_char2(vc[2], vc[3]);
    if (lane == 0) {
        reinterpret_cast<float*>(kt + kBlockTokens * kHeadDim)[t] = ks;
        reinterpret_cast<float*>(vt + kBlockTokens * kHeadDim)[t] = vs;
    }
    *reinterpret_cast<char2*>(sK + o_lo) = make_char2(kc[0], kc[1]);
    *reinterpret_cast<char2*>(sK + o_hi) = make_char2(kc[2], kc[3]);
    *reinterpret_cast<char2*>(sV + o_lo) = make_char2(vc[0], vc[1]);
    *reinterpret_cast<char2*>(sV + o_hi) = make_char2(vc[2], vc[3]);
}

// Two int8 codes of a 32-bit word, chosen by the byte selector `sel`
// (0x4140: bytes 0 and 1, 0x4342: 2 and 3, 0x4240: 0 and 2, 0x4341: 1 and 3),
// as an exact f16x2.  `xf` is the word with every byte's sign bit flipped
// (code + 128 as an unsigned byte); under the exponent bits 0x64 that byte
// is the half 1024 + code + 128, and subtracting 1152 (0x6480) leaves code.
__device__ __forceinline__ uint32_t i8pair_h2(uint32_t xf, uint32_t sel) {
    const uint32_t w = __byte_perm(xf, 0x64646464u, sel);
    uint32_t h;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(h) : "r"(w), "r"(0x64806480u));
    return h;
}

// One 16-token block: scores, online softmax update, P*V accumulate.
// `valid` tokens (rows 0..valid-1) take part; the rest are masked.
// For an INT8 cache (DT 2) the staged tiles hold the codes; ks / vs are the
// K / V scales of token rows g and g + 8: the scores are scaled by ks and the
// softmax weights by vs on their way into P*V (the sums keep the unscaled
// weights), which is attention over code * scale exactly up to fp32 rounding.
template <int DT>
__device__ __forceinline__ void consume_block(uint32_t sK, uint32_t sV, int valid, int lane,
                                              const uint2* qf, float (&m2)[2],
                                              float (&lsum)[2], float (&o)[8][4], const float (&ks)[2],
                                              const float (&vs_in)[2]) {
    const float vs[2] = {DT == 2 ? vs_in[0] : 1.f, DT == 2 ? vs_in[1] : 1.f};
    const int g = lane >> 2;
    const int mi = lane >> 3, r = lane & 7;
    // ---- S^T[16 tokens][8 heads] = K[16][128] * Qs^T ----
    // Four independent accumulator chains (hi/lo x even/odd k-steps).
    float sa[2][4] = {}, sb[2][4] = {};
    {
        const int t = (mi & 1) * 8 + r;
        const uint32_t rowb = sK + (uint32_t)t * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int cidx = 2 * kk + (mi >> 1);
            const uint32_t addr = rowb + (uint32_t)(cidx >> 3) * 2048u + (uint32_t)(((cidx & 7) ^ r) << 4);
            uint32_t a0, a1, a2, a3;
            ldsm_x4(addr, a0, a1, a2, a3);
            const uint2 qh = qf[kk * 32], ql = qf[256 + kk * 32];
            mma16816<mma_type<DT>()>(sa[kk & 1], a0, a1, a2, a3, qh.x, qh.y);
            mma16816<mma_type<DT>()>(sb[kk & 1], a0, a1, a2, a3, ql.x, ql.y);
        }
    }
    float s[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) s[e] = (sa[0][e] + sa[1][e]) + (sb[0][e] + sb[1][e]);
    if (DT == 2) {
        s[0] *= ks[0];
        s[1] *= ks[0];
        s[2] *= ks[1];
        s[3] *= ks[1];
    }
    if (g >= valid) s[0] = s[1] = -INFINITY;
    if (g + 8 >= valid) s[2] = s[3] = -INFINITY;
    // ---- online softmax, per head column (2c, 2c+1) ----
    float bm0 = fmaxf(s[0], s[2]), bm1 = fmaxf(s[1], s[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
    }
    const float mn0 = fmaxf(m2[0], bm0), mn1 = fmaxf(m2[1], bm1);
    const float mu0 = (mn0 == -INFINITY) ? 0.f : mn0;
    const float mu1 = (mn1 == -INFINITY) ? 0.f : mn1;
    const float al0 = fast_exp2(m2[0] - mu0), al1 = fast_exp2(m2[1] - mu1);
    m2[0] = mn0;
    m2[1] = mn1;
    const float p0 = fast_exp2(s[0] - mu0), p1 = fast_exp2(s[1] - mu1);
    const float p2 = fast_exp2(s[2] - mu0), p3 = fast_exp2(s[3] - mu1);
    lsum[0] = lsum[0] * al0 + p0 + p2;
    lsum[1] = lsum[1] * al1 + p1 + p3;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
    }
    // ---- P^T as B fragments (k = tokens, n = heads) ----
    uint32_t h01, l01, h23, l23;
    split_pair<mma_type<DT>()>(p0 * vs[0], p1 * vs[0], h01, l01);
    split_pair<mma_type<DT>()>(p2 * vs[1], p3 * vs[1], h23, l23);
    const uint32_t bh0 = movmatrix_t(h01), bh1 = movmatrix_t(h23);
    const uint32_t bl0 = movmatrix_t(l01), bl1 = movmatrix_t(l23);
    // ---- O^T[128 dims][8 heads] += V^T * P^T ----
    {
        const int t = (mi >> 1) * 8 + r;
        const uint32_t rowb = sV + (uint32_t)t * 128u;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            const int cidx = 2 * mt + (mi & 1);
            const uint32_t addr = rowb + (uint32_t)(cidx >> 3) * 2048u + (uint32_t)(((cidx & 7) ^ r) << 4);
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(addr, a0, a1, a2, a3);
            mma16816<mma_type<DT>()>(o[mt], a0, a1, a2, a3, bh0, bh1);
            mma16816<mma_type<DT>()>(o[mt], a0, a1, a2, a3, bl0, bl1);
        }
    }
}

// The same for an INT8 block, read in place from the staged compact tiles
// (codes at i8_offset, ldmatrix on pairs of codes, converted to exact fp16
// in registers).  Keys: ldmatrix gives thread (g, c) codes 4c..4c+3 of a
// 16-dim chunk of key rows g and g + 8, the A fragment of one k-step under
// the dim permutation load_q_frags applies to q.  Values: ldmatrix .trans
// gives it dims 2g, 2g+1 of keys 2c, 2c+1 (and 2c+8, 2c+9), the V^T A
// fragment of one 16-dim output tile with rows g -> dim 2g, g + 8 -> dim
// 2g + 1; o[mt] holds dims mt*16 + 2g (regs 0, 1) and mt*16 + 2g + 1 (regs
// 2, 3).  Rows past `valid` are masked (their scores -inf, their V scale 0;
// codes are finite, so their weight 0 contributes exactly 0).
template <int QS, int QLO>
__device__ __forceinline__ void consume_block_i8(uint32_t sK, uint32_t sV, int valid, int lane,
                                                 const uint2* qf,
                                                 float (&m2)[2], float (&lsum)[2], float (&o)[8][4],
                                                 const float (&ks)[2], const float (&vs)[2]) {
    const int g = lane >> 2;
    const int mi = lane >> 3, r = lane & 7;
    const int t = (mi & 1) * 8 + r;  // key row this lane addresses for ldmatrix
    // ---- S^T[16 keys][8 heads] = K[16][128] * Qs^T ----
    float sa[2][4] = {}, sb[2][4] = {};
    {
        const uint32_t rowb = sK + (uint32_t)t * 128u;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int chunk = 2 * p + (mi >> 1);
            uint32_t r0, r1, r2, r3;  // keys g / g+8 of chunk 2p, then of chunk 2p+1
            ldsm_x4(rowb + (uint32_t)(((chunk ^ t) & 7) << 4), r0, r1, r2, r3);
            r0 ^= 0x80808080u;
            r1 ^= 0x80808080u;
            r2 ^= 0x80808080u;
            r3 ^= 0x80808080u;
            {
                const uint32_t a0 = i8pair_h2(r0, 0x4140), a1 = i8pair_h2(r1, 0x4140);
                const uint32_t a2 = i8pair_h2(r0, 0x4342), a3 = i8pair_h2(r1, 0x4342);
                const uint2 qh = qf[(2 * p) * QS], ql = qf[QLO + (2 * p) * QS];
                mma16816<0>(sa[0], a0, a1, a2, a3, qh.x, qh.y);
                mma16816<0>(sb[0], a0, a1, a2, a3, ql.x, ql.y);
            }
            {
                const uint32_t a0 = i8pair_h2(r2, 0x4140), a1 = i8pair_h2(r3, 0x4140);
                const uint32_t a2 = i8pair_h2(r2, 0x4342), a3 = i8pair_h2(r3, 0x4342);
                const uint2 qh = qf[(2 * p + 1) * QS], ql = qf[QLO + (2 * p + 1) * QS];
                mma16816<0>(sa[1], a0, a1, a2, a3, qh.x, qh.y);
                mma16816<0>(sb[1], a0, a1, a2, a3, ql.x, ql.y);
            }
        }
    }
    float s[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) s[e] = (sa[0][e] + sa[1][e]) + (sb[0][e] + sb[1][e]);
    s[0] *= ks[0];
    s[1] *= ks[0];
    s[2] *= ks[1];
    s[3] *= ks[1];
    if (g >= valid) s[0] = s[1] = -INFINITY;
    if (g + 8 >= valid) s[2] = s[3] = -INFINITY;
    // ---- online softmax, per head column (2c, 2c+1) ----
    float bm0 = fmaxf(s[0], s[2]), bm1 = fmaxf(s[1], s[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
    }
    const float mn0 = fmaxf(m2[0], bm0), mn1 = fmaxf(m2[1], bm1);
    const float mu0 = (mn0 == -INFINITY) ? 0.f : mn0;
    const float mu1 = (mn1 == -INFINITY) ? 0.f : mn1;
    const float al0 = fast_exp2(m2[0] - mu0), al1 = fast_exp2(m2[1] - mu1);
    m2[0] = mn0;
    m2[1] = mn1;
    const float p0 = fast_exp2(s[0] - mu0), p1 = fast_exp2(s[1] - mu1);
    const float p2 = fast_exp2(s[2] - mu0), p3 = fast_exp2(s[3] - mu1);
    lsum[0] = lsum[0] * al0 + p0 + p2;
    lsum[1] = lsum[1] * al1 + p1 + p3;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
    }
    // ---- P^T as B fragments (weights times the keys' V scales) ----
    uint32_t h01, l01, h23, l23;
    split_pair<0>(p0 * vs[0], p1 * vs[0], h01, l01);
    split_pair<0>(p2 * vs[1], p3 * vs[1], h23, l23);
    const uint32_t bh0 = movmatrix_t(h01), bh1 = movmatrix_t(h23);
    const uint32_t bl0 = movmatrix_t(l01), bl1 = movmatrix_t(l23);
    // ---- O^T[128 dims][8 heads] += V^T * P^T ----
    {
        const uint32_t rowb = sV + (uint32_t)t * 128u;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int chunk = 2 * p + (mi >> 1);
            uint32_t r0, r1, r2, r3;  // keys 2c.. / 8+2c.. of chunk 2p, then of chunk 2p+1
            ldsm_x4_t(rowb + (uint32_t)(((chunk ^ t) & 7) << 4), r0, r1, r2, r3);
            r0 ^= 0x80808080u;
            r1 ^= 0x80808080u;
            r2 ^= 0x80808080u;
            r3 ^= 0x80808080u;
            {
                const uint32_t a0 = i8pair_h2(r0, 0x4240), a1 = i8pair_h2(r0, 0x4341);
                const uint32_t a2 = i8pair_h2(r1, 0x4240), a3 = i8pair_h2(r1, 0x4341);
                mma16816<0>(o[2 * p], a0, a1, a2, a3, bh0, bh1);
                mma16816<0>(o[2 * p], a0, a1, a2, a3, bl0, bl1);
            }
            {
                const uint32_t a0 = i8pair_h2(r2, 0x4240), a1 = i8pair_h2(r2, 0x4341);
                const uint32_t a2 = i8pair_h2(r3, 0x4240), a3 = i8pair_h2(r3, 0x4341);
                mma16816<0>(o[2 * p + 1], a0, a1, a2, a3, bh0, bh1);
                mma16816<0>(o[2 * p + 1], a0, a1, a2, a3, bl0, bl1);
            }
        }
    }
}

}  // namespace


template <int DT, int S>
__global__ void __launch_bounds__(kThreads, 2)
    decode_kernel(PoolView pv, const __grid_constant__ DecodeArgs<S> a, const float* __restrict__ q,
                  const float* __restrict__ k_new, const float* __restrict__ v_new, float* __restrict__ out,
                  float* __restrict__ m_out, float* __restrict__ l_out) {
    extern __shared__ uint8_t smem_raw[];
    Smem<DT>& sm = *reinterpret_cast<Smem<DT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int TB = StageCfg<DT>::tile;  // bytes of one K or V tile in HBM and in a stage
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int layer = a.layer;
    const int kvh = pv.kv_heads;
    const bool early = (a.flags & kDecEarly) != 0;
    // Merge inside clusters of `C` CTAs (every CTA takes the same branch:
    // the cluster barriers below are reached by all threads of a cluster).
    const int C = a.cluster;
    const bool cmode = C > 1;
    const int cbase = (int)blockIdx.x - (int)cluster_rank();
    const bool cluster_ok = !cmode || ((int)cluster_size() == C && a.grid % C == 0);
    // This CTA's flat range, from the kernel parameters (checked; a bad range
    // is reported once the previous kernel has finished, and no work runs).
    int f0 = 0, f1 = 0;
    const bool range_ok = a.nslots >= 0 && a.nslots <= S && a.nsegs >= 0 && a.nsegs <= kSegsPerSlot * S &&
                          a.grid <= kMaxGrid && (int)blockIdx.x < a.grid && a.total >= 0 &&
                          (a.nsegs > 0 || a.total == 0) && a.seg_f0[0] == 0 && a.seg_f0[a.nsegs] == a.total &&
                          cluster_ok;
    if (range_ok) {
        f0 = a.cta_f0[blockIdx.x];
        f1 = a.cta_f0[blockIdx.x + 1];
        if (f0 < 0 || f1 < f0 || f1 > a.total) f0 = f1 = 0;
    }
    constexpr int kStages = StageCfg<DT>::stages;  // ring stages (one producer lane each)
    constexpr unsigned kLaneMask = kStages >= 32 ? 0xffffffffu : ((1u << kStages) - 1u);
    const bool prod_lane = warp == kConsumerWarps && lane < kStages;
    const uint64_t policy = policy_evict_first();
    const long ntile_ids = (long)pv.num_blocks * kvh;
    // One ring round of producer lane `s` for flat block f with tile id `tile`.
    auto issue = [&](int s, int f, int tile) {
        if (tile == -1) {
            mbar_arrive(&sm.full[s]);  // only the new token: nothing to load
        } else if (tile < 0 || tile >= ntile_ids) {
            report(pv, 5, blockIdx.x, 200 + f);  // never read outside the pool
            mbar_arrive(&sm.full[s]);
        } else {
            const size_t off = (size_t)layer * pv.layer_bytes + (size_t)tile * TB;
            mbar_arrive_expect_tx(&sm.full[s], 2 * TB);
            bulk_g2s_hint(sm.stage[s], pv.k + off, TB, &sm.full[s], policy);
            bulk_g2s_hint(sm.stage[s] + TB, pv.v + off, TB, &sm.full[s], policy);
        }
    };
    // Producer lane l owns ring stage l and flat blocks f0 + l, f0 + l + 8, ...
    int pf = f0 + (prod_lane ? lane : 0);
    int pk = 0, pi = 0, ph = 0, pb = 0, pnb = 1;
    bool issued0 = false;
    if (prod_lane) {
        mbar_init(&sm.full[lane], 1);
        mbar_init(&sm.empty[lane], 1);
        fence_mbar_init();
        if (pf < f1) {
            locate(a, pf, pk, pi, ph, pb, pnb);
            // Round 0 before the previous kernel has finished (kDecEarly): a
            // block that kernel may still write (the row the previous decode
            // launch appended) is read only after it.
            if (early && seg_ok(a, pv, pi, ph, pnb) && a.defer_blk[pi] != pb) {
                issue(lane, pf, tile_of(pv, a.slot[pi], ph, pb));
                issued0 = true;
            }
        }
    }
    if (tid == 0) {
        // This CTA's pieces (kernel parameters only).
        int n = 0, f = f0;
        if (f < f1) {
            int k, i, h, b, nb;
            locate(a, f, k, i, h, b, nb);
            while (f < f1 && n < kMaxCtaItems && k < a.nsegs) {
                const int seg_end = a.seg_f0[k + 1];
                const int e = min(seg_end, f1);
                Piece& pc = sm.items[n];
                pc.slot = i;
                pc.head = h;
                pc.b0 = b;
                pc.b1 = b + (e - f);
                pc.split = (b > 0 || e < seg_end) ? (cmode ? 2 : 1) : 0;
                pc.part = cmode ? (n == 0 ? 0 : 1) : 2 * (int)blockIdx.x + (n == 0 ? 0 : 1);
                pc.span = 0;
                if (cmode && b == 0 && e < seg_end) {
                    // The segment continues in the next CTAs of the cluster
                    // (each holds it as its first piece); the plan never lets
                    // it leave the cluster.
                    int g = (int)blockIdx.x + 1;
                    while (g < cbase + C && a.cta_f0[g] < seg_end) ++g;
                    pc.span = g - (int)blockIdx.x - 1;
                    if (g == cbase + C && a.cta_f0[g] < seg_end) {
                        n = -2;
                        break;
                    }
                }
                sm.ok[n] = seg_ok(a, pv, i, h, nb);
                ++n;
                advance(a, e - f, k, i, h, b, nb);
                f = e;
            }
            if (n >= 0 && f < f1) n = -1;  // more pieces than a CTA holds: reported below, nothing runs
        }
        sm.nitems = n;
        for (int x = 0; x < 2 * kMaxGroup; ++x) {
            sm.cpart[x / kMaxGroup][x % kMaxGroup] = -INFINITY;
            sm.cpart[x / kMaxGroup][kMaxGroup + x % kMaxGroup] = 0.f;  // no weight until written
        }
        sm.failed = 0;
        sm.prod_issued = 0;
        for (int w = 0; w < kConsumerWarps; ++w) sm.cons_done[w] = 0;
    }
    __syncthreads();
    int n = sm.nitems;
    if (n < 0) n = 0;
    if (tid == 0) {
        sm.cum[0] = 0;
        for (int j = 0; j < n; ++j) sm.cum[j + 1] = sm.cum[j] + (sm.items[j].b1 - sm.items[j].b0);
    }
    __syncthreads();
    const int total = sm.cum[n];
    const int nf = (total == f1 - f0) ? total : 0;  // blocks the producer streams

    // Cluster merge, reached by every thread of the CTA (producer lanes too)
    // after its own work: the CTA holding the first block of a segment split
    // across the cluster (its last piece, first block 0) merges the states of
    // the span CTAs after it (their first pieces, cpart[0]) with its own;
    // the second barrier keeps every CTA's shared memory alive until then.
    auto cluster_merge = [&]() {
        if (!cmode) return;
        cluster_sync();
        if (warp < kConsumerWarps && n > 0 && nf > 0) {
            const Piece w = sm.items[n - 1];
            if (w.split == 2 && w.b0 == 0 && sm.ok[n - 1]) {
                const uint32_t me = cluster_rank();
                const int qrow = (a.row0 + w.slot) * pv.q_heads + w.head * pv.group;
                const float* own = sm.cpart[w.part];
                const uint32_t peer0 = smem_u32(sm.cpart[0]);
                for (int x = tid; x < pv.group * 32; x += kConsumerWarps * 32) {
                    const int h = x >> 5, c4 = x & 31;  // query head h, dims 4 c4 .. 4 c4 + 3
                    float pm[kClusterCtas], pl[kClusterCtas];
                    float4 po[kClusterCtas];
                    pm[0] = own[h];
                    pl[0] = own[kMaxGroup + h];
                    po[0] = *reinterpret_cast<const float4*>(own + 2 * kMaxGroup + h * kHeadDim + 4 * c4);
#pragma unroll
                    for (int r = 1; r < kClusterCtas; ++r) {
                        if (r <= w.span) {
                            const uint32_t base = cluster_map(peer0, me + (uint32_t)r);
                            pm[r] = ld_cluster_f32(base + 4u * h);
                            pl[r] = ld_cluster_f32(base + 4u * (kMaxGroup + h));
                            po[r] = ld_cluster_v4(base + 4u * (2 * kMaxGroup + h * kHeadDim + 4 * c4));
                        } else {
                            pm[r] = -INFINITY;
                            pl[r] = 0.f;
                            po[r] = make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
                    float M = -INFINITY, L = 0.f;
                    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int r = 0; r < kClusterCtas; ++r) {
                        if (!(pl[r] > 0.f)) continue;  // empty piece: no weight
                        const float Mn = fmaxf(M, pm[r]);
                        const float al = fast_exp2(M - Mn);  // 0 while M is -inf
                        const float e = pl[r] * fast_exp2(pm[r] - Mn);
                        A.x = A.x * al + e * po[r].x;
                        A.y = A.y * al + e * po[r].y;
                        A.z = A.z * al + e * po[r].z;
                        A.w = A.w * al + e * po[r].w;
                        L = L * al + e;
                        M = Mn;
                    }
                    float* orow = out + (size_t)(qrow + h) * kHeadDim + 4 * c4;
                    orow[0] = L > 0.f ? A.x / L : 0.f;
                    orow[1] = L > 0.f ? A.y / L : 0.f;
                    orow[2] = L > 0.f ? A.z / L : 0.f;
                    orow[3] = L > 0.f ? A.w / L : 0.f;
                    if (m_out != nullptr && c4 == 0) {
                        m_out[qrow + h] = M * 0.6931471805599453f;
                        l_out[qrow + h] = L;
                    }
                }
            }
        }
        cluster_sync();
    };

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer
        // Everything below reads state the previous kernel may write (the
        // block table, deferred blocks): wait for it, then let the next
        // kernel launch (it can overlap only this one).
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        if (lane < kStages) {
            const int s = lane;
            const bool live0 = pf < f1 && pf - f0 < nf;
            uint32_t rounds = issued0 ? 1u : 0u;  // rounds issued (all drained before the exit)
            if (live0 && !issued0) {
                issue(s, pf, seg_ok(a, pv, pi, ph, pnb) ? tile_of(pv, a.slot[pi], ph, pb) : -2);
                rounds = 1;
            }
            // Lane s refills its stage as soon as the consumer releases it,
            // polling without blocking; the next round's tile id is fetched
            // one round ahead.
            int f = pf + kStages;
            if (live0) advance(a, kStages, pk, pi, ph, pb, pnb);
            auto next_tile = [&]() -> int {
                return seg_ok(a, pv, pi, ph, pnb) ? tile_of(pv, a.slot[pi], ph, pb) : -2;
            };
            int cur = (live0 && f - f0 < nf) ? next_tile() : -1;
            bool stopped = false;
            long long since = clock64();
            for (;;) {
                const bool has = live0 && !stopped && f - f0 < nf;
                if (!__any_sync(kLaneMask, has)) break;
                const bool ready = has && mbar_test_wait(&sm.empty[s], (rounds & 1) ^ 1);
                if (ready) {
                    issue(s, f, cur);
                    ++rounds;
                    atomicMax(&sm.prod_issued, f - f0 + 1);
                    f += kStages;
                    if (f - f0 < nf) {
                        advance(a, kStages, pk, pi, ph, pb, pnb);
                        cur = next_tile();  // in flight while the stage drains
                    }
                    since = clock64();
                } else if (has && clock64() - since > kWaitLimit) {
                    flag_timeout(pv, sm, blockIdx.x, 0, (uint32_t)(f - f0));
                    stopped = true;
                }
                if (!__any_sync(kLaneMask, ready)) __nanosleep(32);
            }
            // Drain, on every path (also after a timeout or a rejected plan):
            // this lane's last issued stage must land before the CTA exits.
            if (rounds > 0 && !mbar_wait_bounded(&sm.full[s], (rounds - 1) & 1, kWaitLimit))
                flag_timeout(pv, sm, -2, 2, (uint32_t)(lane + (rounds - 1) * kStages));
        }
        cluster_merge();
        return;
    }

    // ---------------------------------------------------------- consumers
    // q / k_new / v_new come from the previous kernel and every write below
    // may race with it: wait for it to finish first.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0) {
        if (!range_ok) report(pv, 5, blockIdx.x, cluster_ok ? 300 : 305);
        else if (sm.nitems == -2) report(pv, 5, blockIdx.x, 304);
        else if (sm.nitems < 0) report(pv, 5, blockIdx.x, 302);
        else if (nf != f1 - f0) report(pv, 5, blockIdx.x, 301);
    }
    if (blockIdx.x == 0 && range_ok) {
        // Rows of slots with nothing to attend are zero (m = -inf, l = 0),
        // and the first launch of a plan enters its new blocks in the table.
        for (int i = tid; i < a.nslots; i += kConsumerWarps * 32) {
            const DecodeSlot sl = a.slot[i];
            if (slot_check(pv, sl) != 0) {
                report(pv, 5, i, 303);
                continue;
            }
            if ((a.flags & kDecPatch) && sl.new_block >= 0)
                pv.table[(size_t)sl.seq * pv.max_blocks_per_seq + (sl.kv_len - 1) / kBlockTokens] = sl.new_block;
            if (sl.kv_len == 0) {
                const int row = (a.row0 + i) * pv.q_heads;
                for (int x = 0; x < pv.q_heads * kHeadDim; ++x) out[(size_t)row * kHeadDim + x] = 0.f;
                if (m_out != nullptr)
                    for (int hq = 0; hq < pv.q_heads; ++hq) {
                        m_out[row + hq] = -INFINITY;
                        l_out[row + hq] = 0.f;
                    }
            }
        }
    }
    if (nf == 0) n = 0;
    const float qscale = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
    const int g = lane >> 2, c = lane & 3;
    // Warp w prepares the q fragments of piece w (w < kQPre) while the first
    // copies are in flight, so piece switches read them from shared memory.
    if (warp < n && warp < kQPre && sm.ok[warp]) {
        const Piece& w = sm.items[warp];
        uint32_t qh[8][2], ql[8][2];
        load_q_frags<DT>(pv, q, a.row0 + w.slot, w.head, a.slot[w.slot].rope_pos, qscale, lane, qh, ql);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            sm.qfrag[warp][0][kk][lane] = make_uint2(qh[kk][0], qh[kk][1]);
            sm.qfrag[warp][1][kk][lane] = make_uint2(ql[kk][0], ql[kk][1]);
        }
    }
    named_bar_sync(1, kConsumerWarps * 32);
    bool dead = false;
    for (int j = 0; j < n; ++j) {
        const Piece wi = sm.items[j];
        const int nb = wi.b1 - wi.b0;
        const int fbase = sm.cum[j];
        if (!sm.ok[j]) {
            // A rejected slot: still release the stages its blocks occupy so
            // the producer's ring keeps moving (it loaded nothing for them).
            for (int b = (warp - fbase % kConsumerWarps + kConsumerWarps) % kConsumerWarps; b < nb;
                 b += kConsumerWarps) {
                const uint32_t k = (uint32_t)(fbase + b);
                const int s = k % kStages;
                if (!dead && !mbar_wait_bounded(&sm.full[s], (k / kStages) & 1, kWaitLimit)) {
                    flag_timeout(pv, sm, blockIdx.x, 1, k);
                    dead = true;
                }
                if (dead) continue;
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&sm.empty[s]);
                    *reinterpret_cast<volatile int*>(&sm.cons_done[warp]) = (int)k + 1;
                }
            }
            continue;
        }
        const DecodeSlot sl = a.slot[wi.slot];
        const int row = a.row0 + wi.slot;
        const bool append = sl.new_block >= 0;
        const int last_blk = (sl.kv_len - 1) / kBlockTokens;

        // Piece j's q fragments: prepared up front for j < kQPre, else now
        // into slot j % kQPre (piece j - kQPre has been merged by every warp:
        // the merge barriers of the pieces in between have passed).  Every
        // warp writes the same values and reads back only its own lanes'.
        const int qslot = j % kQPre;
        if (j >= kQPre) {
            uint32_t qh[8][2], ql[8][2];
            load_q_frags<DT>(pv, q, row, wi.head, sl.rope_pos, qscale, lane, qh, ql);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                sm.qfrag[qslot][0][kk][lane] = make_uint2(qh[kk][0], qh[kk][1]);
                sm.qfrag[qslot][1][kk][lane] = make_uint2(ql[kk][0], ql[kk][1]);
            }
            __syncwarp();
        }
        const uint2* qf = &sm.qfrag[qslot][0][0][lane];
        // INT8 blocks keep the fragments in registers: their consumers are
        // bound by instructions, not registers (16 shared loads per block
        // cost more there than the registers they free).
        uint2 qreg[16];
        if (DT == 2) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                qreg[kk] = qf[kk * 32];
                qreg[8 + kk] = qf[256 + kk * 32];
            }
        }
        float m2[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f};
        float o[8][4];
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

        for (int b = (warp - fbase % kConsumerWarps + kConsumerWarps) % kConsumerWarps; b < nb;
             b += kConsumerWarps) {
            const uint32_t k = (uint32_t)(fbase + b);  // k % kConsumerWarps == warp
            const int s = k % kStages;
            if (!dead && !mbar_wait_bounded(&sm.full[s], (k / kStages) & 1, kWaitLimit)) {
                flag_timeout(pv, sm, blockIdx.x, 1, k);
                dead = true;
            }
            if (dead) continue;
            const int idx = wi.b0 + b;
            const int valid = min(kBlockTokens, sl.kv_len - idx * kBlockTokens);
            const bool newblk = append && idx == last_blk;
            uint8_t* sK;
            uint8_t* sV;
            float ks[2] = {1.f, 1.f}, vs[2] = {1.f, 1.f};  // INT8: scales of token rows g, g + 8
            sK = sm.stage[s];
            sV = sm.stage[s] + TB;
            if (DT == 2) {
                const float* kss = reinterpret_cast<const float*>(sK + kBlockTokens * kHeadDim);
                const float* vss = reinterpret_cast<const float*>(sV + kBlockTokens * kHeadDim);
                ks[0] = kss[g];
                ks[1] = kss[g + 8];
                vs[0] = vss[g];
                vs[1] = vss[g + 8];
            }
            if (newblk) {
                if (DT == 2) {
                    float nks, nvs;
                    write_new_row_i8(pv, layer, sl.new_block, wi.head, valid - 1, k_new, v_new, row, sl.rope_pos,
                                     sK, sV, lane, nks, nvs);
                    if (g == valid - 1) {
                        ks[0] = nks;
                        vs[0] = nvs;
                    }
                    if (g + 8 == valid - 1) {
                        ks[1] = nks;
                        vs[1] = nvs;
                    }
                } else {
                    write_new_row<DT>(pv, layer, sl.new_block, wi.head, valid - 1, k_new, v_new, row, sl.rope_pos,
                                      sK, sV, lane);
                }
            }
            const bool zeroed = DT != 2 && valid < kBlockTokens;
            if (zeroed) {
                // Rows past the end may hold anything (stale tiles, inf):
                // zero them in V so masked weights (exactly 0) stay 0.
                for (int x = lane; x < (kBlockTokens - valid) * 16; x += 32) {
                    const int t = valid + (x >> 4), ch = x & 15;
                    *reinterpret_cast<uint4*>(sV + ((ch >> 3) * 16 + t) * 128 + (ch & 7) * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
            }
            if (DT == 2) {
                // INT8 codes are finite: rows past the end only need a zero
                // V scale (their stale scale words may be inf or NaN).
                if (g >= valid) vs[0] = 0.f;
                if (g + 8 >= valid) vs[1] = 0.f;
            }
            __syncwarp();
            if constexpr (DT == 2)
                consume_block_i8<1, 8>(smem_u32(sK), smem_u32(sV), valid, lane, qreg, m2, lsum, o, ks, vs);
            else
                consume_block<DT>(smem_u32(sK), smem_u32(sV), valid, lane, qf, m2, lsum, o, ks, vs);
            // Generic-proxy writes to the tile must be ordered before the
            // next bulk copy (async proxy) overwrites it.
            if (zeroed || newblk) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&sm.empty[s]);
                *reinterpret_cast<volatile int*>(&sm.cons_done[warp]) = (int)k + 1;
            }
        }

        // ---- merge the four warps' states for this piece ----
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            lsum[0] += __shfl_xor_sync(0xffffffffu, lsum[0], off);
            lsum[1] += __shfl_xor_sync(0xffffffffu, lsum[1], off);
        }
        named_bar_sync(1, kConsumerWarps * 32);  // previous piece's readers are done
        if (g == 0) {
            sm.merge_m[warp][2 * c] = m2[0];
            sm.merge_m[warp][2 * c + 1] = m2[1];
            sm.merge_l[warp][2 * c] = lsum[0];
            sm.merge_l[warp][2 * c + 1] = lsum[1];
        }
        // Output dims of o[mt]'s rows g and g + 8: mt*16 + g and + 8 (16-bit
        // caches), mt*16 + 2g and + 1 (INT8, consume_block_i8).
        const int dr0 = DT == 2 ? 2 * g : g, dr1 = DT == 2 ? 2 * g + 1 : g + 8;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            sm.merge_o[warp][2 * c][mt * 16 + dr0] = o[mt][0];
            sm.merge_o[warp][2 * c + 1][mt * 16 + dr0] = o[mt][1];
            sm.merge_o[warp][2 * c][mt * 16 + dr1] = o[mt][2];
            sm.merge_o[warp][2 * c + 1][mt * 16 + dr1] = o[mt][3];
        }
        named_bar_sync(1, kConsumerWarps * 32);
        // The merge weights once per (head, warp) -- thread 4h + w of warp 0
        // -- instead of by every output dim: M, 2^(m_w - M), L and 1 / L.
        static_assert(kConsumerWarps == 4 && kMaxGroup * kConsumerWarps <= 32, "one warp computes the weights");
        if (tid < pv.group * kConsumerWarps) {
            const int h = tid >> 2, w = tid & 3;
            const unsigned mask = pv.group * kConsumerWarps >= 32 ? 0xffffffffu
                                                                  : ((1u << (pv.group * kConsumerWarps)) - 1u);
            float M = -INFINITY;
#pragma unroll
            for (int x = 0; x < kConsumerWarps; ++x) M = fmaxf(M, sm.merge_m[x][h]);
            const float Mu = (M == -INFINITY) ? 0.f : M;
            const float e = fast_exp2(sm.merge_m[w][h] - Mu);
            sm.merge_w[h][w] = e;
            float L = sm.merge_l[w][h] * e;
            L += __shfl_xor_sync(mask, L, 1);
            L += __shfl_xor_sync(mask, L, 2);
            if (w == 0) {
                sm.merge_inv[h] = L > 0.f ? __frcp_rn(L) : 0.f;
                sm.merge_M[h] = M;
                sm.merge_L[h] = L;
            }
        }
        named_bar_sync(1, kConsumerWarps * 32);

        const int d = tid;  // 0..127: one output dim per thread
        const int qrow = row * pv.q_heads + wi.head * pv.group;
        float* part = wi.split == 2 ? sm.cpart[wi.part] : pv.partials + (size_t)wi.part * kPartialFloats;
        for (int h = 0; h < pv.group; ++h) {
            float O = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) O += sm.merge_o[w][h][d] * sm.merge_w[h][w];
            const float on = O * sm.merge_inv[h];
            const float M = sm.merge_M[h], L = sm.merge_L[h];
            if (!wi.split) {
                out[(size_t)(qrow + h) * kHeadDim + d] = on;
                if (m_out != nullptr && d == 0) {
                    m_out[qrow + h] = M * 0.6931471805599453f;
                    l_out[qrow + h] = L;
                }
            } else {
                part[2 * kMaxGroup + h * kHeadDim + d] = on;
                if (d == 0) {
                    part[h] = M;
                    part[kMaxGroup + h] = L;
                }
            }
        }
    }
    cluster_merge();
}

// Merge of the pieces of every split segment, one CTA per (segment, query
// head).  Launched right behind the decode grid with programmatic dependent
// launch: its CTAs become resident while the decode grid runs, read their
// segment from the kernel parameters and block in griddepcontrol.wait until
// the decode grid has completed and its partial stores are visible.  Warp w
// takes pieces w, w+W, ... eight at a time (all their loads issued together;
// lane l holds dims 4l..4l+3), merging with an online log-sum-exp; the W
// warps' states are then merged in shared memory.  A segment of P pieces
// costs ceil(P / 8W) load rounds: W = 4 normally, 16 when a segment has
// more than 64 pieces (a few very long contexts over the whole GPU).
template <int kCombineWarps>
__global__ void __launch_bounds__(kCombineWarps * 32)
    combine_kernel(PoolView pv, const __grid_constant__ CombineArgs cargs, float* __restrict__ out,
                   float* __restrict__ m_out, float* __restrict__ l_out) {
    static_assert(kCombineWarps * 32 >= kHeadDim, "the final merge maps one thread to each dim");
    __shared__ float s_m[kCombineWarps], s_l[kCombineWarps];
    __shared__ __align__(16) float s_o[kCombineWarps][kHeadDim];
    const int G = pv.group;
    const int si = blockIdx.x / G, h = blockIdx.x % G;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bool ok = si < cargs.nsegs && si < kMaxGrid;
    int slot = 0, head = 0, first = 0, np = 0;
    if (ok) {
        const int2 sg = cargs.seg[si];
        slot = sg.x & 0xffff;
        head = sg.x >> 16;
        first = sg.y & 0xffff;
        np = sg.y >> 16;
        if (head >= pv.kv_heads || np < 1 || (first >> 1) + np > kMaxGrid) {
            if (threadIdx.x == 0) report(pv, 5, si, 400);
            ok = false;
        }
    }
    // The next decode launch may start now: it overlaps this merge and the
    // end of the decode grid (which completes before this kernel can), and
    // it waits for this kernel before it reads or writes anything shared.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (!ok) return;
    const int g0 = first >> 1;
    float M = -INFINITY, L = 0.f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = warp; c0 < np; c0 += 8 * kCombineWarps) {
        float mm[8], ll[8];
        float4 oo[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int pc = c0 + u * kCombineWarps;
            const bool live = pc < np;
            const int pidx = pc == 0 ? first : 2 * (g0 + pc);
            const float* pp = pv.partials + (size_t)(live ? pidx : 0) * kPartialFloats;
            mm[u] = live ? __ldcg(pp + h) : 0.f;
            ll[u] = live ? __ldcg(pp + kMaxGroup + h) : 0.f;
            oo[u] = live ? __ldcg(reinterpret_cast<const float4*>(pp + 2 * kMaxGroup + h * kHeadDim) + lane)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (!(ll[u] > 0.f)) continue;  // empty piece (or past the end): no weight
            const float Mn = fmaxf(M, mm[u]);
            const float a = fast_exp2(M - Mn);  // 0 while M is -inf
            const float e = ll[u] * fast_exp2(mm[u] - Mn);
            A.x = A.x * a + e * oo[u].x;
            A.y = A.y * a + e * oo[u].y;
            A.z = A.z * a + e * oo[u].z;
            A.w = A.w * a + e * oo[u].w;
            L = L * a + e;
            M = Mn;
        }
    }
    if (lane == 0) {
        s_m[warp] = M;
        s_l[warp] = L;
    }
    reinterpret_cast<float4*>(s_o[warp])[lane] = A;
    __syncthreads();
    const int d = threadIdx.x;  // 0..127: one output dim per thread
    if (d >= kHeadDim) return;
    float Mt = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w)
        if (s_l[w] > 0.f) Mt = fmaxf(Mt, s_m[w]);
    float Lt = 0.f, At = 0.f;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) {
        if (!(s_l[w] > 0.f)) continue;
        const float f = fast_exp2(s_m[w] - Mt);
        Lt += s_l[w] * f;
        At += s_o[w][d] * f;
    }
    const int row = (cargs.row0 + slot) * pv.q_heads + head * G + h;
    out[(size_t)row * kHeadDim + d] = Lt > 0.f ? At / Lt : 0.f;
    if (m_out != nullptr && d == 0) {
        m_out[row] = Mt * 0.6931471805599453f;
        l_out[row] = Lt;
    }
}

// Two CTAs per SM: 228 KB of shared memory per SM, 1 KB of it reserved per CTA.
static_assert(sizeof(Smem<0>) + 1024 <= 228 * 1024 / 2 - 1024, "two decode CTAs must fit an SM");
static_assert(sizeof(Smem<1>) + 1024 <= 228 * 1024 / 2 - 1024, "two decode CTAs must fit an SM");
static_assert(sizeof(Smem<2>) + 1024 <= 228 * 1024 / 2 - 1024, "two decode CTAs must fit an SM");

template <int DT>
static cudaError_t decode_occupancy_t(int* ctas_per_sm, int* clusters) {
    const int smem = (int)sizeof(Smem<DT>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<DT, kSlotsSmall>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(decode_kernel<DT, kSlotsLarge>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, decode_kernel<DT, kSlotsSmall>, kThreads, smem);
    if (e != cudaSuccess) return e;
    // Merge clusters that fit the device at once (GPC boundaries can leave
    // some CTA slots unused).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kClusterCtas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kClusterCtas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    *clusters = 0;
    e = cudaOccupancyMaxActiveClusters(clusters, decode_kernel<DT, kSlotsSmall>, &cfg);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();  // no clusters: grid-wide merges only
        *clusters = 0;
    }
    return cudaSuccess;
}

cudaError_t decode_occupancy(int dtype, int* ctas_per_sm, int* clusters) {
    // The combine kernel runs beside two decode CTAs on an SM (resident
    // while the decode grid streams): give it the decode kernel's
    // shared-memory carveout, or the SM could not host both.
    cudaError_t e = cudaFuncSetAttribute(combine_kernel<4>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(combine_kernel<16>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    return dtype == 0   ? decode_occupancy_t<0>(ctas_per_sm, clusters)
           : dtype == 1 ? decode_occupancy_t<1>(ctas_per_sm, clusters)
                        : decode_occupancy_t<2>(ctas_per_sm, clusters);
}

template <int S>
cudaError_t launch_decode(const PoolView& pv, const DecodeArgs<S>& a, const CombineArgs& c, int max_pieces,
                          const float* q, const float* k_new, const float* v_new, float* out, float* m_out,
                          float* l_out, bool pdl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.grid < 1 ? 1 : a.grid));
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)(a.cluster > 1 ? a.cluster : 1);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchAttribute dattr[2];
    int nd = 0;
    if (pdl) dattr[nd++] = attr[0];
    if (a.cluster > 1) dattr[nd++] = attr[1];
    cfg.attrs = dattr;
    cfg.numAttrs = nd;
    cudaError_t e;
    if (pv.dtype == 0) {
        cfg.dynamicSmemBytes = sizeof(Smem<0>) + 1024;
        e = cudaLaunchKernelEx(&cfg, decode_kernel<0, S>, pv, a, q, k_new, v_new, out, m_out, l_out);
    } else if (pv.dtype == 1) {
        cfg.dynamicSmemBytes = sizeof(Smem<1>) + 1024;
        e = cudaLaunchKernelEx(&cfg, decode_kernel<1, S>, pv, a, q, k_new, v_new, out, m_out, l_out);
    } else {
        cfg.dynamicSmemBytes = sizeof(Smem<2>) + 1024;
        e = cudaLaunchKernelEx(&cfg, decode_kernel<2, S>, pv, a, q, k_new, v_new, out, m_out, l_out);
    }
    e = counted(e);
    if (e != cudaSuccess || c.nsegs == 0) return e;
    const int warps = max_pieces > 64 ? 16 : 4;
    cudaLaunchConfig_t ccfg = {};
    ccfg.gridDim = dim3((unsigned)(c.nsegs * pv.group));
    ccfg.blockDim = dim3(warps * 32);
    ccfg.dynamicSmemBytes = 0;
    ccfg.stream = st;
    ccfg.attrs = attr;  // programmatic dependent of the decode grid
    ccfg.numAttrs = 1;
    if (warps == 16) return counted(cudaLaunchKernelEx(&ccfg, combine_kernel<16>, pv, c, out, m_out, l_out));
    return counted(cudaLaunchKernelEx(&ccfg, combine_kernel<4>, pv, c, out, m_out, l_out));
}

template cudaError_t launch_decode<kSlotsSmall>(const PoolView&, const DecodeArgs<kSlotsSmall>&, const CombineArgs&,
                                                int, const float*, const float*, const float*, float*, float*,
                                                float*, bool, cudaStream_t);
template cudaError_t launch_decode<kSlotsLarge>(const PoolView&, const DecodeArgs<kSlotsLarge>&, const CombineArgs&,
                                                int, const float*, const float*, const float*, float*, float*,
                                                float*, bool, cudaStream_t);

}  // namespace kvattn
