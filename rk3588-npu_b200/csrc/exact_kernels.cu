// exact_kernels.cu -- the Qwen2 forward in the reference's operation order.
//
// The fast device model (model_kernels.cu, the kvattn attention kernels)
// keeps the reference's arithmetic contract but sums in parallel orders, so
// its fp32 results differ from the reference's sequential loops in the last
// bits, and a greedy choice between two logits closer than that noise can
// differ.  These kernels repeat every float operation of
// Qwen2Model::forward (worker/src/model/qwen2_model.cpp:131-274) in the
// reference's order, with its rounding:
//   RMSNorm        op_rmsnorm.cpp:6-20     sum of squares in index order,
//                                          sqrt, 1/rms, (x * inv) * w
//   projections    the linear contract      fp16 inputs (truncating
//                                          f32_to_f16), fp16 weights, fp32
//                                          sum in k order, truncated fp16 out
//   bias, residual op_elementwise.cpp       fp32 adds
//   attention      op_attention.cpp:9-56   dot in d order, * 1/sqrt(128),
//                  op_softmax.cpp:6-16     max, exp, sum in key order, 1/sum,
//                                          weighted V sum in key order
//   SiLU           op_silu.cpp:4-7         x / (1 + exp(-x)), then * up
// RoPE and the KV append are the pool's (already bit-exact: kv_append_chunk
// and the host-built cos/sin table).  No fused multiply-add is used except
// where the product is exact (fp16 x fp16 in fp32), where it equals the
// separately rounded multiply and add.
//
// exp: the reference calls the C library's expf.  Here exp is evaluated in
// double precision and rounded to float once -- the correctly rounded float
// exponential -- which is what the C library returns for all but a small
// set of inputs (0.004 % of the floats on x86-64 glibc 2.39, spread over the
// whole finite range, each one unit in the last place away).  Those inputs
// and the library's results come in a table (ExpTab) that the host builds
// from its own expf; with it, every exp here equals the host's.
#include <cuda_runtime.h>
#include <float.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kvattn_internal.h"

namespace kvattn {
namespace {

// fp16 -> fp32 exactly as worker/include/core/half.h:34-43 (a subnormal code
// decodes to sign | mant << 13, as there).
__device__ __forceinline__ float ref_f16(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    uint32_t x;
    if (e == 0) x = sign | (mant << 13);
    else if (e == 31) x = sign | 0x7F800000u | (mant << 13);
    else x = sign | ((e + 112u) << 23) | (mant << 13);
    return __uint_as_float(x);
}

// exp as the host C library's expf: the correctly rounded value, or the
// library's own result on the inputs listed in the table.
__device__ __forceinline__ float exp_ref(float x, const ExpTab& t) {
    float r = __double2float_rn(exp((double)x));
    if (t.keys != nullptr) {
        const uint32_t b = __float_as_uint(x), hb = b >> 16;
        uint32_t lo = t.bucket[hb];
        const uint32_t end = t.bucket[hb + 1];
        uint32_t hi = end;
        while (lo < hi) {
            const uint32_t mid = (lo + hi) >> 1;
            if (t.keys[mid] < b) lo = mid + 1;
            else hi = mid;
        }
        if (lo < end && t.keys[lo] == b) r = __uint_as_float(t.vals[lo]);
    }
    return r;
}

constexpr int kThreadsE = 128;

// op_rmsnorm of row blockIdx.x, written as the fp16 codes the projection
// after it takes (op_f32_to_f16).  The row is staged in shared memory; one
// thread sums the squares in index order.
__global__ void __launch_bounds__(kThreadsE)
    rmsnorm_exact_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps, int H,
                         uint16_t* __restrict__ y16) {
    extern __shared__ float xs[];
    __shared__ float s_inv;
    const float* xr = x + (size_t)blockIdx.x * H;
    for (int i = threadIdx.x; i < H; i += kThreadsE) xs[i] = xr[i];
    __syncthreads();
    if (threadIdx.x == 0) {
        float sum = 0.f;
        for (int i = 0; i < H; ++i) sum = __fadd_rn(sum, __fmul_rn(xs[i], xs[i]));
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)H), eps));
        s_inv = __fdiv_rn(1.0f, rms);
    }
    __syncthreads();
    const float inv = s_inv;
    uint16_t* yr = y16 + (size_t)blockIdx.x * H;
    for (int i = threadIdx.x; i < H; i += kThreadsE) yr[i] = enc_f16_trunc(__fmul_rn(__fmul_rn(xs[i], inv), w[i]));
}

// y16[m][n] = f32_to_f16( sum_{k = 0..K-1} x16[m][k] * W[n][k] ) with the
// fp32 sum taken in k order (one thread per output column; every product of
// two fp16 values is exact in fp32, so a fused multiply-add rounds exactly
// like the separate add).  CTA: 128 columns x kRowsE rows; W tiles of 128
// rows x 64 k staged in shared memory with 16-byte loads (row pitch 66
// halves, so column n's reads hit distinct banks).  K % 8 == 0.
constexpr int kRowsE = 8;
constexpr int kChunkE = 64;
constexpr int kPitchE = kChunkE + 2;

__global__ void __launch_bounds__(kThreadsE)
    gemv_exact_kernel(const uint16_t* __restrict__ x16, int M, int K, const uint16_t* __restrict__ W, int N,
                      uint16_t* __restrict__ y16) {
    __shared__ __align__(16) uint16_t sw[kThreadsE][kPitchE];
    __shared__ uint16_t sx[kRowsE][kChunkE];
    const int tid = threadIdx.x;
    const int n0 = blockIdx.x * kThreadsE, n = n0 + tid;
    const int m0 = blockIdx.y * kRowsE;
    float acc[kRowsE];
#pragma unroll
    for (int r = 0; r < kRowsE; ++r) acc[r] = 0.f;
    for (int k0 = 0; k0 < K; k0 += kChunkE) {
        const int kc = min(kChunkE, K - k0);
        for (int v = tid; v < kThreadsE * (kChunkE / 8); v += kThreadsE) {
            const int r = v >> 3, c = v & 7;
            uint4 val = make_uint4(0u, 0u, 0u, 0u);
            if (n0 + r < N && c * 8 < kc)
                val = __ldg(reinterpret_cast<const uint4*>(W + (size_t)(n0 + r) * K + k0 + c * 8));
            uint32_t* d = reinterpret_cast<uint32_t*>(&sw[r][c * 8]);
            d[0] = val.x;
            d[1] = val.y;
            d[2] = val.z;
            d[3] = val.w;
        }
        for (int v = tid; v < kRowsE * kChunkE; v += kThreadsE) {
            const int r = v / kChunkE, kk = v % kChunkE;
            sx[r][kk] = (m0 + r < M && kk < kc) ? x16[(size_t)(m0 + r) * K + k0 + kk] : (uint16_t)0;
        }
        __syncthreads();
        for (int kk = 0; kk < kc; ++kk) {
            const float wv = ref_f16(sw[tid][kk]);
#pragma unroll
            for (int r = 0; r < kRowsE; ++r) acc[r] = fmaf(ref_f16(sx[r][kk]), wv, acc[r]);
        }
        __syncthreads();
    }
    if (n < N)
#pragma unroll
        for (int r = 0; r < kRowsE; ++r)
            if (m0 + r < M) y16[(size_t)(m0 + r) * N + n] = enc_f16_trunc(acc[r]);
}

// q / k / v of the stacked projection: f16_to_f32 then + bias (one fp32 add).
__global__ void __launch_bounds__(256)
    qkv_bias_exact_kernel(const uint16_t* __restrict__ qkv16, const float* __restrict__ bias, int rows, int H, int kvd,
                          float* __restrict__ q, float* __restrict__ k, float* __restrict__ v) {
    const int W = H + 2 * kvd;
    for (long i = blockIdx.x * 256L + threadIdx.x; i < (long)rows * W; i += gridDim.x * 256L) {
        const int r = (int)(i / W), c = (int)(i % W);
        const float x = __fadd_rn(ref_f16(qkv16[i]), bias[c]);
        if (c < H) q[(size_t)r * H + c] = x;
        else if (c < H + kvd) k[(size_t)r * kvd + c - H] = x;
        else v[(size_t)r * kvd + c - H - kvd] = x;
    }
}

// op_rope of q (op_rope.cpp:4-16): row r at position pos0 + r, pairs (i,
// i + 64) of every head, cos/sin from the pool's table, non-fused.
__global__ void __launch_bounds__(256)
    rope_q_exact_kernel(float* __restrict__ q, int rows, int heads, int pos0, const float2* __restrict__ rope) {
    const long pairs = (long)rows * heads * (kHeadDim / 2);
    for (long i = blockIdx.x * 256L + threadIdx.x; i < pairs; i += gridDim.x * 256L) {
        const int j = (int)(i % (kHeadDim / 2));
        const long rh = i / (kHeadDim / 2);
        const int r = (int)(rh / heads);
        float* h = q + rh * kHeadDim;
        const float2 cs = rope[(size_t)(pos0 + r) * (kHeadDim / 2) + j];
        float a, b;
        rope_pair(h[j], h[j + 64], cs.x, cs.y, a, b);
        h[j] = a;
        h[j + 64] = b;
    }
}

// op_attention + op_softmax for query row blockIdx.y, head blockIdx.x over
// contiguous caches [total_len][kv_dim] (the reference layout): scores in d
// order, masked keys -1e9, softmax over all total_len keys with the sums in
// key order, output sums in key order (masked keys add 0 * v).
__global__ void __launch_bounds__(kThreadsE)
    attn_exact_kernel(const float* __restrict__ q, const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc,
                      float* __restrict__ out, int total_len, int n_heads, int n_kv_heads, int pos_base, float scale,
                      ExpTab et) {
    extern __shared__ float sc[];  // [total_len] scores, then weights
    __shared__ float qs[kHeadDim];
    __shared__ float red[kThreadsE / 32];
    __shared__ float s_inv;
    const int h = blockIdx.x, sq = blockIdx.y, tid = threadIdx.x;
    const int kvh = h / (n_heads / n_kv_heads);
    const int hidden = n_heads * kHeadDim, kv_dim = n_kv_heads * kHeadDim;
    const int abs_sq = pos_base + sq;
    qs[tid] = q[(size_t)sq * hidden + (size_t)h * kHeadDim + tid];
    __syncthreads();
    for (int sk = tid; sk < total_len; sk += kThreadsE) {
        if (sk > abs_sq) {
            sc[sk] = -1e9f;
            continue;
        }
        const uint16_t* kr = kc + (size_t)sk * kv_dim + (size_t)kvh * kHeadDim;
        float dot = 0.f;
        for (int d = 0; d < kHeadDim; ++d) dot = __fadd_rn(dot, __fmul_rn(qs[d], ref_f16(kr[d])));
        sc[sk] = __fmul_rn(dot, scale);
    }
    __syncthreads();
    float mx = -FLT_MAX;
    for (int i = tid; i < total_len; i += kThreadsE) mx = fmaxf(mx, sc[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < kThreadsE / 32; ++w) mx = fmaxf(mx, red[w]);
    for (int i = tid; i < total_len; i += kThreadsE) sc[i] = exp_ref(__fsub_rn(sc[i], mx), et);
    __syncthreads();
    if (tid == 0) {
        float sum = 0.f;
        for (int i = 0; i < total_len; ++i) sum = __fadd_rn(sum, sc[i]);
        s_inv = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = tid; i < total_len; i += kThreadsE) sc[i] = __fmul_rn(sc[i], inv);
    __syncthreads();
    const uint16_t* vr = vc + (size_t)kvh * kHeadDim + tid;
    float acc = 0.f;
    for (int sk = 0; sk < total_len; ++sk) acc = __fadd_rn(acc, __fmul_rn(sc[sk], ref_f16(vr[(size_t)sk * kv_dim])));
    out[(size_t)sq * hidden + (size_t)h * kHeadDim + tid] = acc;
}

// op_f32_to_f16 (truncating) of n floats.
__global__ void __launch_bounds__(256) to_f16_exact_kernel(const float* __restrict__ x, long n, uint16_t* __restrict__ y) {
    for (long i = blockIdx.x * 256L + threadIdx.x; i < n; i += gridDim.x * 256L) y[i] = enc_f16_trunc(x[i]);
}

// hidden += f16_to_f32(codes) (op_vec_add after a projection).
__global__ void __launch_bounds__(256)
    resid_exact_kernel(float* __restrict__ hidden, const uint16_t* __restrict__ y16, long n) {
    for (long i = blockIdx.x * 256L + threadIdx.x; i < n; i += gridDim.x * 256L)
        hidden[i] = __fadd_rn(hidden[i], ref_f16(y16[i]));
}

// gate = silu(gate) * up, then f32_to_f16 (qwen2_model.cpp:232-246):
// silu(x) = x / (1 + exp(-x)).
__global__ void __launch_bounds__(256)
    silu_mul_exact_kernel(const uint16_t* __restrict__ g16, const uint16_t* __restrict__ u16, long n,
                          uint16_t* __restrict__ h16, ExpTab et) {
    for (long i = blockIdx.x * 256L + threadIdx.x; i < n; i += gridDim.x * 256L) {
        const float g = ref_f16(g16[i]);
        const float s = __fdiv_rn(g, __fadd_rn(1.0f, exp_ref(-g, et)));
        h16[i] = enc_f16_trunc(__fmul_rn(s, ref_f16(u16[i])));
    }
}

// logits f32 from the lm_head's fp16 codes (op_f16_to_f32).
__global__ void __launch_bounds__(256) f16_to_f32_exact_kernel(const uint16_t* __restrict__ y16, long n, float* __restrict__ y) {
    for (long i = blockIdx.x * 256L + threadIdx.x; i < n; i += gridDim.x * 256L) y[i] = ref_f16(y16[i]);
}

unsigned grid_for_e(long n) {
    long g = (n + 255) / 256;
    return (unsigned)(g < 1 ? 1 : g > 4096 ? 4096 : g);
}

}  // namespace

cudaError_t launch_rmsnorm_exact(const float* x, const float* w, float eps, int rows, int H, uint16_t* y16,
                                 cudaStream_t st) {
    if ((size_t)H * sizeof(float) > 48 * 1024) return cudaErrorInvalidValue;
    rmsnorm_exact_kernel<<<rows, kThreadsE, (size_t)H * sizeof(float), st>>>(x, w, eps, H, y16);
    return counted(cudaGetLastError());
}

cudaError_t launch_gemv_exact(const uint16_t* x16, int M, int K, const uint16_t* W, int N, uint16_t* y16,
                              cudaStream_t st) {
    if (K % 8) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((N + kThreadsE - 1) / kThreadsE), (unsigned)((M + kRowsE - 1) / kRowsE));
    gemv_exact_kernel<<<grid, kThreadsE, 0, st>>>(x16, M, K, W, N, y16);
    return counted(cudaGetLastError());
}

cudaError_t launch_qkv_bias_exact(const uint16_t* qkv16, const float* bias, int rows, int H, int kvd, float* q, float* k,
                                  float* v, cudaStream_t st) {
    qkv_bias_exact_kernel<<<grid_for_e((long)rows * (H + 2 * kvd)), 256, 0, st>>>(qkv16, bias, rows, H, kvd, q, k, v);
    return counted(cudaGetLastError());
}

cudaError_t launch_rope_q_exact(float* q, int rows, int heads, int pos0, const float2* rope, cudaStream_t st) {
    rope_q_exact_kernel<<<grid_for_e((long)rows * heads * (kHeadDim / 2)), 256, 0, st>>>(q, rows, heads, pos0, rope);
    return counted(cudaGetLastError());
}

cudaError_t launch_attn_exact(const float* q, const uint16_t* kc, const uint16_t* vc, float* out, int seq, int total_len,
                              int n_heads, int n_kv_heads, int pos_base, float scale, ExpTab et, cudaStream_t st) {
    const size_t smem = (size_t)total_len * sizeof(float);
    if (smem > 48 * 1024) return cudaErrorInvalidValue;  // up to 12288 keys
    attn_exact_kernel<<<dim3((unsigned)n_heads, (unsigned)seq), kThreadsE, smem, st>>>(q, kc, vc, out, total_len, n_heads,
                                                                                       n_kv_heads, pos_base, scale, et);
    return counted(cudaGetLastError());
}

cudaError_t launch_to_f16_exact(const float* x, long n, uint16_t* y, cudaStream_t st) {
    to_f16_exact_kernel<<<grid_for_e(n), 256, 0, st>>>(x, n, y);
    return counted(cudaGetLastError());
}

cudaError_t launch_resid_exact(float* hidden, const uint16_t* y16, long n, cudaStream_t st) {
    resid_exact_kernel<<<grid_for_e(n), 256, 0, st>>>(hidden, y16, n);
    return counted(cudaGetLastError());
}

cudaError_t launch_silu_mul_exact(const uint16_t* g16, const uint16_t* u16, long n, uint16_t* h16, ExpTab et,
                                  cudaStream_t st) {
    silu_mul_exact_kernel<<<grid_for_e(n), 256, 0, st>>>(g16, u16, n, h16, et);
    return counted(cudaGetLastError());
}

cudaError_t launch_f16_to_f32_exact(const uint16_t* y16, long n, float* y, cudaStream_t st) {
    f16_to_f32_exact_kernel<<<grid_for_e(n), 256, 0, st>>>(y16, n, y);
    return counted(cudaGetLastError());
}

}  // namespace kvattn
