// model_kernels.cu -- the non-attention kernels of the Qwen2 forward
// (qwen2_model.cpp:131-274) on sm_100a: embedding lookup, RMSNorm, the
// projections as HBM-streaming GEMVs with fused epilogues, greedy argmax, and
// the load-time weight conversion.
//
// Projection contract (the reference's ILinearOp, op_linear.h, as the device
// model computes it): input rows are fp16 values (the truncating f32_to_f16 of
// half.h), weights fp16 [N][K] (the file's [out][in] layout), products exact
// in fp32 (11-bit x 11-bit significands), fp32 accumulation, result truncated
// to fp16 and widened back, then the fp32 epilogue of the call site.
//
// An RMSNorm feeding a projection is fused into it: every CTA first computes
// 1/rms of its input rows (a few KB read from L2) and applies the norm while
// loading the input.
//
// GEMV layout: `ks` warps share one output row, each summing every ks-th
// 16-byte chunk (8 weights) of it, 8 chunks per lane in flight; 8 warps per
// CTA, so 8/ks rows per row group; a grid of (SMs x resident CTAs) walks the
// row groups.  A CTA processes up to MR input rows at once, reading each
// weight chunk once for all of them.  Weights stream through with no L1
// allocation; the input rows are staged once per CTA in shared memory as
// fp16 codes (the norm and the rounding applied there, not per weight).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <math.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "device_common.cuh"
#include "kvattn.h"
#include "kvattn_internal.h"

namespace kvattn {

namespace {

constexpr int kGemvWarps = 8;

// fp16 -> fp32 exactly as worker/include/core/half.h:34-43 (its exponent-0
// branch included).
__device__ __forceinline__ float dec_f16_ref(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    uint32_t x;
    if (e == 0) x = sign | (mant << 13);
    else if (e == 31) x = sign | 0x7F800000u | (mant << 13);
    else x = sign | ((e + 112u) << 23) | (mant << 13);
    return __uint_as_float(x);
}

// Round an fp32 value through the reference's fp16 (f16_to_f32(f32_to_f16(x))).
__device__ __forceinline__ float f16_round(float x) { return dec_f16_ref(enc_f16_trunc(x)); }

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// 8 fp16 weights against 8 fp16 inputs (both as 16-byte chunks), fp32 FMAs;
// every product is exact in fp32.
__device__ __forceinline__ float dot8h(const uint4& w, const uint4& x, float acc) {
    const __half2* wh = reinterpret_cast<const __half2*>(&w);
    const __half2* xh = reinterpret_cast<const __half2*>(&x);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 fw = __half22float2(wh[j]), fx = __half22float2(xh[j]);
        acc = fmaf(fw.x, fx.x, acc);
        acc = fmaf(fw.y, fx.y, acc);
    }
    return acc;
}

constexpr int kStageU = 2;  // 16-byte fp32 input chunks per thread in flight while staging

// 1 / rms of an fp32 row of H values (op_rmsnorm.cpp:12-15) by a 256-thread
// block: thread t sums the rounded squares of its float4 chunks t, t + 256,
// ... (components in order), then a warp tree, then the 8 warps in order.
// Every caller (the standalone kernel and the fused projections) runs this
// same order, so all of them get the same value.  All loads of a thread are
// issued before any is used.
__device__ __forceinline__ float sum_sq4(float s, const float4& v) {
    s = __fadd_rn(s, __fmul_rn(v.x, v.x));
    s = __fadd_rn(s, __fmul_rn(v.y, v.y));
    s = __fadd_rn(s, __fmul_rn(v.z, v.z));
    return __fadd_rn(s, __fmul_rn(v.w, v.w));
}

// Finish 1/rms from each thread's partial sum (warp tree, then the 8 warps in
// order; every thread of the 256 gets the value).
__device__ __forceinline__ float block_inv_rms_from(float s, int H, float eps, float* part) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += part[i];
    __syncthreads();  // part is reused by the next row
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)H), eps));
    return __fdiv_rn(1.0f, rms);
}

__device__ __forceinline__ float block_inv_rms(const float* __restrict__ xr, int H, float eps, float* part) {
    const float4* src = reinterpret_cast<const float4*>(xr);
    const int n4 = H >> 2;
    float s = 0.f;
    for (int base = threadIdx.x; base < n4; base += kStageU * 256) {
        float4 v[kStageU];
#pragma unroll
        for (int u = 0; u < kStageU; ++u)
            if (base + u * 256 < n4) v[u] = __ldg(src + base + u * 256);
#pragma unroll
        for (int u = 0; u < kStageU; ++u)
            if (base + u * 256 < n4) s = sum_sq4(s, v[u]);
    }
    return block_inv_rms_from(s, H, eps, part);
}

// Stage input row `row` of a projection into shared memory as the fp16 codes
// the projection multiplies (IN: 0 fp16 codes as given; 1 fp32 rounded
// through fp16; 2 RMSNorm of an fp32 row, (x * inv) * w (op_rmsnorm.cpp:
// 17-18), rounded through fp16), by the reference's truncating f32_to_f16.
// These codes are never fp16 subnormals, so the hardware conversion back to
// fp32 is the reference's f16_to_f32.  16-byte loads, several in flight per
// thread.
template <int IN>
__device__ __forceinline__ void stage_row(const GemvArgs& a, int row, uint16_t* xs_row, float* part) {
    const int K = a.K;
    if (IN == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) + (size_t)row * K);
        uint4* dst = reinterpret_cast<uint4*>(xs_row);
        const int n8 = K >> 3;
        // 5 chunks per thread: a row of up to 10240 values in one round of loads
        for (int base = threadIdx.x; base < n8; base += 5 * 256) {
            uint4 v[5];
#pragma unroll
            for (int u = 0; u < 5; ++u)
                if (base + u * 256 < n8) v[u] = __ldg(src + base + u * 256);
#pragma unroll
            for (int u = 0; u < 5; ++u)
                if (base + u * 256 < n8) dst[base + u * 256] = v[u];
        }
        return;
    }
    const float* xr = static_cast<const float*>(a.x) + (size_t)row * K;
    const float4* src = reinterpret_cast<const float4*>(xr);
    const float4* wsrc = reinterpret_cast<const float4*>(a.norm_w);
    uint2* dst = reinterpret_cast<uint2*>(xs_row);
    const int n4 = K >> 2;
    auto encode = [&](const float4& v, const float4& w, float inv, int i) {
        float e[4] = {v.x, v.y, v.z, v.w};
        if (IN == 2) {
            const float f[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) e[j] = __fmul_rn(__fmul_rn(e[j], inv), f[j]);
        }
        dst[i] = make_uint2((uint32_t)enc_f16_trunc(e[0]) | ((uint32_t)enc_f16_trunc(e[1]) << 16),
                            (uint32_t)enc_f16_trunc(e[2]) | ((uint32_t)enc_f16_trunc(e[3]) << 16));
    };
    if (n4 <= kStageU * 256) {
        // the whole row in registers: one round of loads (row and norm
        // weights together), the sum of squares from registers, then the codes
        float4 v[kStageU], w[kStageU];
        float sq = 0.f;
#pragma unroll
        for (int u = 0; u < kStageU; ++u) {
            const int i = threadIdx.x + u * 256;
            if (i < n4) {
                v[u] = __ldg(src + i);
                if (IN == 2) w[u] = __ldg(wsrc + i);
            }
        }
        float inv = 1.f;
        if (IN == 2) {
#pragma unroll
            for (int u = 0; u < kStageU; ++u)
                if (threadIdx.x + u * 256 < n4) sq = sum_sq4(sq, v[u]);
            inv = block_inv_rms_from(sq, K, a.eps, part);
        }
#pragma unroll
        for (int u = 0; u < kStageU; ++u) {
            const int i = threadIdx.x + u * 256;
            if (i < n4) encode(v[u], w[u], inv, i);
        }
        return;
    }
    const float inv = IN == 2 ? block_inv_rms(xr, K, a.eps, part) : 1.f;
    for (int base = threadIdx.x; base < n4; base += kStageU * 256) {
        float4 v[kStageU], w[kStageU];
#pragma unroll
        for (int u = 0; u < kStageU; ++u)
            if (base + u * 256 < n4) {
                v[u] = __ldg(src + base + u * 256);
                if (IN == 2) w[u] = __ldg(wsrc + base + u * 256);
            }
#pragma unroll
        for (int u = 0; u < kStageU; ++u)
            if (base + u * 256 < n4) encode(v[u], w[u], inv, base + u * 256);
    }
}

// The same codes as stage_row, one row staged by one warp (used when a CTA
// stages several rows): lane l takes the 16-byte chunks l, l + 32, ...; the
// RMSNorm sum is lane-sequential then a warp tree, with no CTA barrier.
template <int IN>
__device__ __forceinline__ void stage_row_warp(const GemvArgs& a, int row, uint16_t* xs_row) {
    const int K = a.K, lane = threadIdx.x & 31;
    if (IN == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) + (size_t)row * K);
        uint4* dst = reinterpret_cast<uint4*>(xs_row);
        const int n8 = K >> 3;
        for (int base = lane; base < n8; base += 8 * 32) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (base + u * 32 < n8) v[u] = __ldg(src + base + u * 32);
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (base + u * 32 < n8) dst[base + u * 32] = v[u];
        }
        return;
    }
    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + (size_t)row * K);
    const float4* wsrc = reinterpret_cast<const float4*>(a.norm_w);
    uint2* dst = reinterpret_cast<uint2*>(xs_row);
    const int n4 = K >> 2;
    float inv = 1.f;
    if (IN == 2) {
        float s = 0.f;
        for (int base = lane; base < n4; base += 8 * 32) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (base + u * 32 < n4) v[u] = __ldg(src + base + u * 32);
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (base + u * 32 < n4) s = sum_sq4(s, v[u]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)K), a.eps));
        inv = __fdiv_rn(1.0f, rms);
    }
    for (int base = lane; base < n4; base += 4 * 32) {
        float4 v[4], w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (base + u * 32 < n4) {
                v[u] = __ldg(src + base + u * 32);
                if (IN == 2) w[u] = __ldg(wsrc + base + u * 32);
            }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (base + u * 32 < n4) {
                float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                if (IN == 2) {
                    const float f[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) e[j] = __fmul_rn(__fmul_rn(e[j], inv), f[j]);
                }
                dst[base + u * 32] = make_uint2((uint32_t)enc_f16_trunc(e[0]) | ((uint32_t)enc_f16_trunc(e[1]) << 16),
                                                (uint32_t)enc_f16_trunc(e[2]) | ((uint32_t)enc_f16_trunc(e[3]) << 16));
            }
    }
}

}  // namespace

constexpr int kGemvUnroll = 8;  // 16-byte weight chunks in flight per lane

// The call site's fp32 epilogue of output n of input row `row`, from the fp32
// sums of its weight row (acc) and, for gate/up, of its up row (acc2).
template <int MODE>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int row, int n, float acc, float acc2) {
    const float r = f16_round(acc);
    if (MODE == 0) {
        const float v = __fadd_rn(r, a.bias[n]);  // op_vec_add_bias (op_elementwise.cpp:8-11)
        if (n < a.n0) a.out0[(size_t)row * a.n0 + n] = v;
        else if (n < a.n0 + a.n1) a.out1[(size_t)row * a.n1 + (n - a.n0)] = v;
        else a.out2[(size_t)row * (a.N - a.n0 - a.n1) + (n - a.n0 - a.n1)] = v;
    } else if (MODE == 1) {
        float* h = a.resid + (size_t)row * a.N + n;  // op_vec_add (op_elementwise.cpp:3-5)
        *h = __fadd_rn(*h, r);
    } else if (MODE == 2) {
        // op_silu (op_silu.cpp:4-7), then gate *= up, then f32_to_f16
        const float u = f16_round(acc2);
        const float sg = __fdiv_rn(r, __fadd_rn(1.0f, expf(-r)));
        a.out16[(size_t)row * a.N + n] = enc_f16_trunc(__fmul_rn(sg, u));
    } else {
        a.logits[(size_t)row * a.N + n] = r;
    }
}

// MODE: 0 QKV (+bias, split into q / k / v), 1 residual add, 2 gate/up +
// SiLU product (fp16 out), 3 logits.  NW = 2 for gate/up (two weight rows per
// output), else 1.  Dynamic shared memory: the MR input rows as fp16 codes
// [MR][K].  The CTA walks row groups blockIdx.x, +gridDim.x, ...; its first
// weight loads are issued before it waits for the previous kernel (every
// access before that wait reads only weights, which no kernel writes).
// U: 16-byte weight chunks in flight per lane (kGemvUnroll, or more when one
// batch of that depth would not cover a warp's share of the row).
template <int MODE, int IN, int MR, int U>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_kernel(GemvArgs a) {
    constexpr int NW = MODE == 2 ? 2 : 1;
    extern __shared__ uint4 gemv_smem[];
    uint16_t* xs = reinterpret_cast<uint16_t*>(gemv_smem);
    __shared__ float red[kGemvWarps][NW * MR];
    __shared__ float s_part[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = a.ks, rows_per_cta = kGemvWarps / ks, sub = warp / ks, part = warp % ks;
    const int m0 = blockIdx.y * MR;
    const int K = a.K, nch = K >> 3, step = 32 * ks;
    const int ngroups = (a.N + rows_per_cta - 1) / rows_per_cta;
    const uint16_t* w2 = NW == 2 ? a.w2 : a.w;

    uint4 wv[NW][U];
    auto load_batch = [&](int n, int base) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = base + u * step;
            if (n < a.N && c < nch) {
                wv[0][u] = ld_stream16(reinterpret_cast<const uint4*>(a.w + (size_t)n * K) + c);
                if (NW == 2) wv[NW - 1][u] = ld_stream16(reinterpret_cast<const uint4*>(w2 + (size_t)n * K) + c);
            }
        }
    };
    // Launched as a programmatic dependent of the previous kernel: let the
    // next one launch, stream the first (read-only) weights, and only then
    // wait for the previous kernel's results (the input rows) to be visible.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    int rg = blockIdx.x;
    bool loaded = false;
    if (rg < ngroups) {
        load_batch(rg * rows_per_cta + sub, part * 32 + lane);
        loaded = true;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // stage the input rows (RMSNorm and fp16 rounding applied once per CTA):
    // one row with the whole CTA, several rows one per warp, all at once
    if (MR == 1) {
        if (m0 < a.M) stage_row<IN>(a, m0, xs, s_part);
    } else {
        for (int m = warp; m < MR; m += kGemvWarps)
            if (m0 + m < a.M) stage_row_warp<IN>(a, m0 + m, xs + m * K);
    }
    __syncthreads();

#pragma unroll 1
    for (; rg < ngroups; rg += gridDim.x) {
        const int n = rg * rows_per_cta + sub;
        float acc[NW][MR];
#pragma unroll
        for (int t = 0; t < NW; ++t)
#pragma unroll
            for (int m = 0; m < MR; ++m) acc[t][m] = 0.f;
#pragma unroll 1
        for (int base = part * 32 + lane; base < nch; base += U * step) {
            if (!loaded) load_batch(n, base);
            loaded = false;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + u * step;
                if (n < a.N && c < nch) {
#pragma unroll
                    for (int m = 0; m < MR; ++m) {
                        if (m0 + m < a.M) {
                            const uint4 x8 = *reinterpret_cast<const uint4*>(xs + m * K + c * 8);
#pragma unroll
                            for (int t = 0; t < NW; ++t) acc[t][m] = dot8h(wv[t][u], x8, acc[t][m]);
                        }
                    }
                }
            }
        }
        loaded = false;
#pragma unroll
        for (int t = 0; t < NW; ++t)
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                float v = acc[t][m];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                acc[t][m] = v;
            }
        if (ks > 1) {
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < NW; ++t)
#pragma unroll
                    for (int m = 0; m < MR; ++m) red[warp][t * MR + m] = acc[t][m];
            }
            __syncthreads();
            if (part == 0) {
#pragma unroll
                for (int t = 0; t < NW; ++t)
#pragma unroll
                    for (int m = 0; m < MR; ++m) {
                        float v = red[warp][t * MR + m];
                        for (int p = 1; p < ks; ++p) v += red[warp + p][t * MR + m];
                        acc[t][m] = v;
                    }
            }
        }
        if (part == 0 && n < a.N) {
            // lane m finishes input row m0 + m
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                const int row = m0 + m;
                if (lane != m || row >= a.M) continue;
                gemv_epilogue<MODE>(a, row, n, acc[0][m], acc[NW - 1][m]);
            }
        }
        if (ks > 1) __syncthreads();  // red is reused by the next row group
    }
}

// ---------------------------------------------------------------------------
// Several input rows (2..32: a decode step of several sessions) on the tensor
// cores: y^T = W x^T as mma.sync m16n8k16 tiles, W the A operand (16 weight
// rows x 16 k), the staged input rows the B operand (16 k x 8 rows), fp32
// accumulators.  Products of fp16 values are exact, sums fp32: the contract
// of the one-row kernel, in another order.
//
// The k order inside each 32-wide span is permuted consistently for A and B
// so that both operands come from plain 16-byte loads: lane (g, c) loads
// weights [row g][8c, 8c+8) and [row g+8][8c, 8c+8) of the span and input
// [row g][8c, 8c+8) from shared memory; step 0 of the span multiplies the
// pairs (8c, 8c+1) and (8c+2, 8c+3) (in the fragment slots of logical k
// 2c.. and 2c+8..), step 1 the pairs (8c+4, 8c+5) and (8c+6, 8c+7).  Every
// physical k of the span is used exactly once.
//
// Warp w: weight rows tile w / kMmaKs (16 rows), k spans w % kMmaKs, +kMmaKs,
// ...; 8 warps = 16 * 8 / kMmaKs rows per row group.  Input rows are staged
// with a padded stride (K + 8 halves) so that the 8 rows of a B load sit in
// different banks.
constexpr int kMmaKs = 8;      // warps per 16-row tile (k split)
constexpr int kMmaPad = 8;     // halves of padding per staged row
constexpr int kMmaU = 8;       // k spans per warp in flight

template <int MODE, int IN, int NT>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_mma_kernel(GemvArgs a) {
    constexpr int NW = MODE == 2 ? 2 : 1;
    constexpr int MR = NT * 8;
    extern __shared__ uint4 gemv_smem[];
    uint16_t* xs = reinterpret_cast<uint16_t*>(gemv_smem);  // [MR][K + kMmaPad]
    __shared__ float red[kGemvWarps][NW * NT * 4][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int tiles_per_cta = kGemvWarps / kMmaKs, sub = warp / kMmaKs, part = warp % kMmaKs;
    const int m0 = blockIdx.y * MR;
    const int K = a.K, spans = K >> 5, ldx = K + kMmaPad;
    const int ngroups = (a.N + 16 * tiles_per_cta - 1) / (16 * tiles_per_cta);
    const uint16_t* wmat[2] = {a.w, NW == 2 ? a.w2 : a.w};

    uint4 wa[NW][kMmaU], wb[NW][kMmaU];
    auto load_batch = [&](int n0, int base) {
#pragma unroll
        for (int u = 0; u < kMmaU; ++u) {
            const int sp = base + u * kMmaKs;
#pragma unroll
            for (int q = 0; q < NW; ++q) {
                wa[q][u] = make_uint4(0u, 0u, 0u, 0u);
                wb[q][u] = make_uint4(0u, 0u, 0u, 0u);
                if (sp < spans) {
                    const uint16_t* base_q = wmat[q] + (size_t)sp * 32 + 8 * c;
                    if (n0 + g < a.N) wa[q][u] = ld_stream16(base_q + (size_t)(n0 + g) * K);
                    if (n0 + g + 8 < a.N) wb[q][u] = ld_stream16(base_q + (size_t)(n0 + g + 8) * K);
                }
            }
        }
    };
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    int rg = blockIdx.x;
    bool loaded = false;
    if (rg < ngroups) {
        load_batch((rg * tiles_per_cta + sub) * 16, part);
        loaded = true;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // stage the input rows, one per warp (rows past M as zeros)
    for (int m = warp; m < MR; m += kGemvWarps) {
        if (m0 + m < a.M) {
            stage_row_warp<IN>(a, m0 + m, xs + (size_t)m * ldx);
        } else {
            uint4* z = reinterpret_cast<uint4*>(xs + (size_t)m * ldx);
            for (int i = lane; i < (K >> 3); i += 32) z[i] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    __syncthreads();

#pragma unroll 1
    for (; rg < ngroups; rg += gridDim.x) {
        const int n0 = (rg * tiles_per_cta + sub) * 16;
        float d[NW][NT][4];
#pragma unroll
        for (int q = 0; q < NW; ++q)
#pragma unroll
            for (int t = 0; t < NT; ++t) d[q][t][0] = d[q][t][1] = d[q][t][2] = d[q][t][3] = 0.f;
#pragma unroll 1
        for (int base = part; base < spans; base += kMmaU * kMmaKs) {
            if (!loaded) load_batch(n0, base);
            loaded = false;
#pragma unroll
            for (int u = 0; u < kMmaU; ++u) {
                const int sp = base + u * kMmaKs;
                if (sp < spans) {
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const uint4 xb = *reinterpret_cast<const uint4*>(xs + (size_t)(t * 8 + g) * ldx + sp * 32 + 8 * c);
#pragma unroll
                        for (int q = 0; q < NW; ++q) {
                            mma16816<0>(d[q][t], wa[q][u].x, wb[q][u].x, wa[q][u].y, wb[q][u].y, xb.x, xb.y);
                            mma16816<0>(d[q][t], wa[q][u].z, wb[q][u].z, wa[q][u].w, wb[q][u].w, xb.z, xb.w);
                        }
                    }
                }
            }
        }
        loaded = false;
        // the kMmaKs partial tiles of the same 16 rows, summed in order
        if (part != 0) {
#pragma unroll
            for (int q = 0; q < NW; ++q)
#pragma unroll
                for (int t = 0; t < NT; ++t)
#pragma unroll
                    for (int i = 0; i < 4; ++i) red[warp][(q * NT + t) * 4 + i][lane] = d[q][t][i];
        }
        __syncthreads();
        if (part == 0) {
#pragma unroll
            for (int q = 0; q < NW; ++q)
#pragma unroll
                for (int t = 0; t < NT; ++t)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float v = d[q][t][i];
                        for (int p2 = 1; p2 < kMmaKs; ++p2) v += red[warp + p2][(q * NT + t) * 4 + i][lane];
                        d[q][t][i] = v;
                    }
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int n = n0 + g + (i >= 2 ? 8 : 0), row = m0 + t * 8 + 2 * c + (i & 1);
                    if (n < a.N && row < a.M) gemv_epilogue<MODE>(a, row, n, d[0][t][i], d[NW - 1][t][i]);
                }
        }
        __syncthreads();  // red is reused by the next row group
    }
}

// RMSNorm (op_rmsnorm.cpp:4-20) of row blockIdx.x, output rounded to fp16 (the
// f32_to_f16 before every projection).  Per-term products rounded like the
// reference's loop; the sum is a tree.
__global__ void __launch_bounds__(256)
    rmsnorm_f16_kernel(const float* __restrict__ x, const float* __restrict__ w, uint16_t* __restrict__ y, int H,
                       float eps) {
    __shared__ float part[8];
    const float* xr = x + (size_t)blockIdx.x * H;
    uint16_t* yr = y + (size_t)blockIdx.x * H;
    const float inv = block_inv_rms(xr, H, eps, part);
    for (int i = threadIdx.x; i < H; i += blockDim.x) yr[i] = enc_f16_trunc(__fmul_rn(__fmul_rn(xr[i], inv), w[i]));
}

// op_embedding_lookup (op_embedding.cpp:4-12): row ids[blockIdx.x] of the table.
__global__ void __launch_bounds__(256)
    embed_kernel(const int* __restrict__ ids, const uint16_t* __restrict__ table, float* __restrict__ hidden,
                 int H) {
    const size_t id = (size_t)ids[blockIdx.x];
    for (int d = threadIdx.x; d < H; d += blockDim.x)
        hidden[(size_t)blockIdx.x * H + d] = dec_f16_ref(table[id * H + d]);
}

// op_greedy_sample (op_sampling.cpp:4-11) of each row: the first index of
// the largest value above -FLT_MAX (index 0 if none).  Packed key: order-preserving bits
// of the value, then the complement of the index, so the maximum key is the
// largest value at its lowest index; NaN never counts.
__global__ void __launch_bounds__(256)
    argmax_kernel(const float* __restrict__ v, int n, unsigned long long* __restrict__ best) {
    v += (size_t)blockIdx.y * n;  // row blockIdx.y
    best += blockIdx.y;
    unsigned long long k = 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float f = v[i];
        if (f > -FLT_MAX) {
            const uint32_t u = __float_as_uint(f);
            const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            const unsigned long long key = ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)i);
            k = key > k ? key : k;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, k, o);
        k = t > k ? t : k;
    }
    if ((threadIdx.x & 31) == 0 && k) atomicMax(best, k);
}

// Load-time conversion of a matrix to the stored fp16 (weight_loader.cpp:184-194):
// F16 as is (subnormals to signed zero), BF16 via f32 to fp16 (bf16_to_f16),
// F32 by the truncating f32_to_f16.
__global__ void __launch_bounds__(256)
    weight_to_f16_kernel(const void* __restrict__ src, int dtype, uint16_t* __restrict__ dst, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        uint16_t h;
        if (dtype == 0) {
            h = static_cast<const uint16_t*>(src)[i];
            if ((h & 0x7C00u) == 0) h &= 0x8000u;
        } else if (dtype == 1) {
            h = enc_f16_trunc(__uint_as_float((uint32_t)static_cast<const uint16_t*>(src)[i] << 16));
        } else {
            h = enc_f16_trunc(static_cast<const float*>(src)[i]);
        }
        dst[i] = h;
    }
}

int gemv_split(int K) {
    int ks = 1;
    while (ks < kGemvWarps && K / (ks * 2) >= 1536) ks *= 2;
    return ks;
}

// Launch facts of one kernel, per device (a process may drive several GPUs,
// from several threads): the dynamic shared memory granted so far, the SM
// count, and the resident CTAs per SM by 4 KiB shared-memory bucket.  The
// shared-memory attribute is raised under a per-device lock, so it only
// grows and never falls below the recorded grant (two first calls with
// different sizes cannot leave the smaller one set).  Concurrent first
// calls may query the occupancy twice; every value written is the same.
struct LaunchCache {
    static constexpr int kDevices = 64;
    std::atomic<int> smem_set[kDevices];
    std::atomic<int> sms[kDevices];
    std::atomic<int> ctas[kDevices][64];
    std::mutex mu[kDevices];

    cudaError_t get(const void* fn, int smem, int* sms_out, int* ctas_out) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kDevices) return cudaErrorInvalidDevice;
        if (smem > smem_set[dev].load()) {
            std::lock_guard<std::mutex> lk(mu[dev]);
            if (smem > smem_set[dev].load()) {
                e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
                if (e != cudaSuccess) return e;
                smem_set[dev].store(smem);
            }
        }
        if (!sms[dev].load()) {
            int n = 0;
            if ((e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
            sms[dev].store(n);
        }
        const int bucket = smem >> 12 < 64 ? smem >> 12 : 63;
        if (!ctas[dev][bucket].load()) {
            int n = 0;
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kGemvWarps * 32, (size_t)smem);
            if (e != cudaSuccess) return e;
            ctas[dev][bucket].store(n > 0 ? n : 1);
        }
        *sms_out = sms[dev].load();
        *ctas_out = ctas[dev][bucket].load();
        return cudaSuccess;
    }
};

template <int MODE, int IN, int MR, int U>
static cudaError_t launch_gemv_mr(const GemvArgs& a, cudaStream_t st) {
    static LaunchCache cache;
    const int smem = MR * a.K * 2;
    int sms = 0, ctas = 0;
    cudaError_t e = cache.get(reinterpret_cast<const void*>(gemv_kernel<MODE, IN, MR, U>), smem, &sms, &ctas);
    if (e != cudaSuccess) return e;
    const int rows_per_cta = kGemvWarps / a.ks;
    const int groups = (a.N + rows_per_cta - 1) / rows_per_cta;
    const int ylen = (a.M + MR - 1) / MR;
    int cap = sms * ctas / ylen;
    cap = cap < 1 ? 1 : cap;
    // as many CTAs as fit, but every CTA the same number of row groups (the
    // next kernel waits for the last CTA)
    const int rounds = (groups + cap - 1) / cap;
    const int gx = (groups + rounds - 1) / rounds;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)gx, (unsigned)ylen);
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return counted(cudaLaunchKernelEx(&cfg, gemv_kernel<MODE, IN, MR, U>, a));
}

template <int MODE, int IN, int NT>
static cudaError_t launch_gemv_mma_nt(const GemvArgs& a, cudaStream_t st) {
    static LaunchCache cache;  // static (the reduction buffer) + dynamic may pass 48 KB at any size
    const int smem = NT * 8 * (a.K + kMmaPad) * 2;
    int sms = 0, ctas = 0;
    cudaError_t e = cache.get(reinterpret_cast<const void*>(gemv_mma_kernel<MODE, IN, NT>), smem, &sms, &ctas);
    if (e != cudaSuccess) return e;
    const int rows_per_group = 16 * (kGemvWarps / kMmaKs);
    const int groups = (a.N + rows_per_group - 1) / rows_per_group;
    const int ylen = (a.M + NT * 8 - 1) / (NT * 8);
    int cap = sms * ctas / ylen;
    cap = cap < 1 ? 1 : cap;
    const int rounds = (groups + cap - 1) / cap;
    const int gx = (groups + rounds - 1) / rounds;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)gx, (unsigned)ylen);
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return counted(cudaLaunchKernelEx(&cfg, gemv_mma_kernel<MODE, IN, NT>, a));
}

// Rows of one pass: up to 32 while their staged copies fit beside the rest
// (K = 1536: 32 rows, 98 KB; K = 8960: 8 rows, 143 KB); more rows take more
// passes over the weights.
template <int MODE, int IN>
static cudaError_t launch_gemv_mma(const GemvArgs& a, cudaStream_t st) {
    const int fit = (200 * 1024) / (8 * (a.K + kMmaPad) * 2);  // n8 tiles whose rows fit
    const int need = (a.M + 7) / 8;
    const int nt = need < fit ? need : fit;
    if (nt >= 4) return launch_gemv_mma_nt<MODE, IN, 4>(a, st);
    if (nt >= 2) return launch_gemv_mma_nt<MODE, IN, 2>(a, st);
    return launch_gemv_mma_nt<MODE, IN, 1>(a, st);
}

// One row: the CUDA-core kernel (HBM-bound at 2 B per weight).  Several rows
// (sessions decoding together, prompt chunks): the tensor-core kernel, in
// passes of up to 32 rows.
template <int MODE, int IN>
static cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t st) {
    if (a.M == 1) {
        // one batch of loads per row part when 9 chunks per lane cover it
        // (the 8960-wide down projection: 1120 chunks over 4 x 32 lanes;
        // 9 keeps three CTAs per SM resident, 12 would leave two)
        const int per_lane = ((a.K >> 3) + 32 * a.ks - 1) / (32 * a.ks);
        if (per_lane == kGemvUnroll + 1) return launch_gemv_mr<MODE, IN, 1, kGemvUnroll + 1>(a, st);
        return launch_gemv_mr<MODE, IN, 1, kGemvUnroll>(a, st);
    }
    return launch_gemv_mma<MODE, IN>(a, st);
}

cudaError_t launch_gemv(int mode, int in, GemvArgs a, cudaStream_t st) {
    if (a.K % 8 != 0 || a.N <= 0 || a.M <= 0) return cudaErrorInvalidValue;
    if (a.M > 1 && a.K % 32 != 0) return cudaErrorInvalidValue;  // the tensor-core path walks 32-wide k spans
    a.ks = gemv_split(a.K);
    switch (mode * 4 + in) {
        case 0 * 4 + 2: return launch_gemv_t<0, 2>(a, st);  // RMSNorm -> QKV
        case 1 * 4 + 0: return launch_gemv_t<1, 0>(a, st);  // down + residual
        case 1 * 4 + 1: return launch_gemv_t<1, 1>(a, st);  // O (fp32 attention) + residual
        case 2 * 4 + 2: return launch_gemv_t<2, 2>(a, st);  // RMSNorm -> gate/up
        case 3 * 4 + 2: return launch_gemv_t<3, 2>(a, st);  // final RMSNorm -> lm_head
        case 0 * 4 + 0: return launch_gemv_t<0, 0>(a, st);
        case 2 * 4 + 0: return launch_gemv_t<2, 0>(a, st);
        case 3 * 4 + 0: return launch_gemv_t<3, 0>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_rmsnorm_f16(const float* x, const float* w, uint16_t* y, int rows, int H, float eps,
                               cudaStream_t st) {
    rmsnorm_f16_kernel<<<rows, 256, 0, st>>>(x, w, y, H, eps);
    return counted(cudaGetLastError());
}

cudaError_t launch_embed(const int* ids, int n, const uint16_t* table, float* hidden, int H, cudaStream_t st) {
    embed_kernel<<<n, 256, 0, st>>>(ids, table, hidden, H);
    return counted(cudaGetLastError());
}

cudaError_t launch_argmax(const float* v, int n, int rows, unsigned long long* best, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(best, 0, sizeof(unsigned long long) * rows, st);
    if (e != cudaSuccess) return e;
    const int gx = rows >= 296 ? 1 : 296 / rows;
    argmax_kernel<<<dim3((unsigned)gx, (unsigned)rows), 256, 0, st>>>(v, n, best);
    return counted(cudaGetLastError());
}

// dst[i] = src row idx[i] (H floats), one CTA per row.
__global__ void __launch_bounds__(256)
    gather_rows_kernel(const float* __restrict__ src, const int* __restrict__ idx, float* __restrict__ dst, int H) {
    const float* s = src + (size_t)idx[blockIdx.x] * H;
    float* d = dst + (size_t)blockIdx.x * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) d[i] = s[i];
}

cudaError_t launch_gather_rows(const float* src, const int* idx, int rows, float* dst, int H, cudaStream_t st) {
    gather_rows_kernel<<<rows, 256, 0, st>>>(src, idx, dst, H);
    return counted(cudaGetLastError());
}

cudaError_t launch_weight_to_f16(const void* src, int dtype, uint16_t* dst, size_t n, cudaStream_t st) {
    weight_to_f16_kernel<<<592, 256, 0, st>>>(src, dtype, dst, n);
    return counted(cudaGetLastError());
}

}  // namespace kvattn
