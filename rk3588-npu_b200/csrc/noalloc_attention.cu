// noalloc_attention.cu -- grouped-query attention over contiguous caches that
// allocates nothing.
//
// Some callers cannot allocate device memory at the point where they need
// attention: an inference host that owns every byte of GPU memory through
// its own arena and forbids plugins from calling cudaMalloc, a real-time
// decode loop that may not block on the allocator, or code that must not
// create pool objects.  attn_contig_noalloc serves them: the caller passes
// inputs and outputs only, and the split-KV partial results live in a
// file-scope __device__ array of fixed size (kScratchFloats floats, 4 MiB),
// which every GPU that loads this library holds until the process exits.
//
// The math: for query row s (at absolute position pos_base + s) and query
// head h of KV group g, out = softmax(q_s,h . K_g^T / sqrt(128)) V_g over keys
// 0 .. pos_base + s (causal), with q [seq][n_heads*128] fp32 (already
// rotated), caches [total_len][n_kv_heads*128] 16-bit (fp16 or bf16) and out
// [seq][n_heads*128] fp32, all device pointers (q and the caches 16-byte
// aligned).  Two launches: partials per (query row, KV head, split) into the
// scratch array, then their merge.
//
// The device address of the array is looked up once per device and kept
// for the life of the process; it belongs to that device's primary
// context, so the entry point is not for use across cudaDeviceReset.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "device_common.cuh"
#include "kvattn.h"
#include "kvattn_internal.h"

namespace kvattn {
namespace {

constexpr long kScratchFloats = 1L << 20;  // 4 MiB of partial states
constexpr int kSplitTokens = 256;          // keys per split, at least
constexpr int kMaxSplits = 64;
constexpr int kWarps = 4;

// The scratch array.  In host code its name is only a host-side stand-in;
// kernels get its device address from cudaGetSymbolAddress (see below).
static __device__ __align__(256) float g_scratch[kScratchFloats];

// One partial: m[8], l[8], o[8][128] (kPartialFloats floats), base-2 logits.

// Eight 16-bit cache values (one 16-byte load) as floats.
__device__ __forceinline__ void load8(const uint16_t* p, int dt, float (&f)[8]) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (dt == 0) {
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        } else {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
}

// grid (nsplit, n_kv_heads, seq), 128 threads.  Each half-warp is a key
// stream: warp w takes key pairs t0 + 2w + 8j, its halves one key each, and
// lane i of a half holds dims 8i..8i+7, so a key's K and V rows arrive as
// one 16-byte load per lane; the eight streams' states are merged in shared
// memory.
__global__ void __launch_bounds__(kWarps * 32)
    contig_partial_kernel(const float* __restrict__ q, const uint16_t* __restrict__ kc,
                          const uint16_t* __restrict__ vc, float* __restrict__ scratch, int seq,
                          int total_len, int n_heads, int n_kv_heads, int pos_base, int nsplit,
                          int split_tokens, int dt) {
    constexpr int kStreams = kWarps * 2;
    const int split = blockIdx.x, kvh = blockIdx.y, sq = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stream = warp * 2 + (lane >> 4), li = lane & 15;
    const int group = n_heads / n_kv_heads;
    const int kv_dim = n_kv_heads * kHeadDim;
    const int lim = min(total_len, pos_base + sq + 1);  // keys 0..abs position (causal)
    const int t0 = split * split_tokens, t1 = min(lim, t0 + split_tokens);
    const float scale = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
    __shared__ float sm_o[kStreams][kMaxGroup][kHeadDim];
    __shared__ float sm_m[kStreams][kMaxGroup], sm_l[kStreams][kMaxGroup];

    float qv[kMaxGroup][8], o[kMaxGroup][8], m[kMaxGroup], l[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
        const float4* qr = reinterpret_cast<const float4*>(q + (size_t)sq * n_heads * kHeadDim +
                                                           (size_t)(kvh * group + h) * kHeadDim + 8 * li);
        const float4 a = h < group ? qr[0] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 b = h < group ? qr[1] : make_float4(0.f, 0.f, 0.f, 0.f);
        qv[h][0] = a.x * scale;
        qv[h][1] = a.y * scale;
        qv[h][2] = a.z * scale;
        qv[h][3] = a.w * scale;
        qv[h][4] = b.x * scale;
        qv[h][5] = b.y * scale;
        qv[h][6] = b.z * scale;
        qv[h][7] = b.w * scale;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[h][e] = 0.f;
    }
    // Both halves of a warp run the same iterations (the half-warp sums
    // shuffle with the whole warp's mask); a half whose key is past the
    // split's end loads nothing and keeps its state.
    for (int tp = t0 + 2 * warp; tp < t1; tp += kStreams) {
        const int t = tp + (lane >> 4);
        const bool valid = t < t1;
        float kf[8], vf[8];
        if (valid) {
            const size_t off = (size_t)t * kv_dim + (size_t)kvh * kHeadDim + 8 * li;
            load8(kc + off, dt, kf);
            load8(vc + off, dt, vf);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) kf[e] = vf[e] = 0.f;
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            if (h >= group) break;
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) s += qv[h][e] * kf[e];
#pragma unroll
            for (int off2 = 8; off2; off2 >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off2);  // within the half-warp
            if (!valid) continue;
            const float mn = fmaxf(m[h], s);
            const float a = fast_exp2(m[h] - mn);  // 0 while m is -inf
            const float p = fast_exp2(s - mn);
            l[h] = l[h] * a + p;
#pragma unroll
            for (int e = 0; e < 8; ++e) o[h][e] = o[h][e] * a + p * vf[e];
            m[h] = mn;
        }
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
#pragma unroll
        for (int e = 0; e < 8; ++e) sm_o[stream][h][8 * li + e] = o[h][e];
        if (li == 0) {
            sm_m[stream][h] = m[h];
            sm_l[stream][h] = l[h];
        }
    }
    __syncthreads();
    const int d = threadIdx.x;
    float* part = scratch + ((size_t)(sq * n_kv_heads + kvh) * nsplit + split) * kPartialFloats;
    for (int h = 0; h < group; ++h) {
        float M = -INFINITY;
        for (int w = 0; w < kStreams; ++w) M = fmaxf(M, sm_m[w][h]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
        for (int w = 0; w < kStreams; ++w) {
            const float e = fast_exp2(sm_m[w][h] - Mu);
            L += sm_l[w][h] * e;
            O += sm_o[w][h][d] * e;
        }
        part[2 * kMaxGroup + h * kHeadDim + d] = L > 0.f ? O / L : 0.f;
        if (d == 0) {
            part[h] = M;
            part[kMaxGroup + h] = L;
        }
    }
}

// grid (n_heads, seq), 128 threads: merge the splits of one query row.
__global__ void __launch_bounds__(kHeadDim)
    contig_merge_kernel(const float* __restrict__ scratch, float* __restrict__ out, int n_heads,
                        int n_kv_heads, int nsplit) {
    const int qh = blockIdx.x, sq = blockIdx.y, d = threadIdx.x;
    const int group = n_heads / n_kv_heads, kvh = qh / group, h = qh % group;
    const float* p0 = scratch + (size_t)(sq * n_kv_heads + kvh) * nsplit * kPartialFloats;
    float M = -INFINITY, L = 0.f, A = 0.f;
    for (int c = 0; c < nsplit; ++c) {
        const float* pc = p0 + (size_t)c * kPartialFloats;
        const float lc = pc[kMaxGroup + h];
        if (!(lc > 0.f)) continue;  // split with no keys
        const float mc = pc[h];
        const float Mn = fmaxf(M, mc);
        const float a = fast_exp2(M - Mn), e = lc * fast_exp2(mc - Mn);
        A = A * a + e * pc[2 * kMaxGroup + h * kHeadDim + d];
        L = L * a + e;
        M = Mn;
    }
    out[((size_t)sq * n_heads + qh) * kHeadDim + d] = L > 0.f ? A / L : 0.f;
}

// Device address of g_scratch, looked up once per device with that device
// current (a host reference to g_scratch is not a device address).
std::mutex g_mu;
float* g_addr[64] = {};

}  // namespace
}  // namespace kvattn

using namespace kvattn;

extern "C" int attn_contig_noalloc(const float* q, const void* k_cache, const void* v_cache,
                                   float* out, int seq, int total_len, int n_heads, int n_kv_heads,
                                   int head_dim, int pos_base, int dtype, void* stream) {
    if (!q || !k_cache || !v_cache || !out) return KV_ERR_INVAL;
    if (((uintptr_t)q | (uintptr_t)k_cache | (uintptr_t)v_cache) & 15) return KV_ERR_INVAL;
    if (head_dim != kHeadDim || seq < 1 || total_len < 1 || pos_base < 0 || n_kv_heads < 1 ||
        n_heads < n_kv_heads || n_heads % n_kv_heads != 0 || n_heads / n_kv_heads > kMaxGroup ||
        (dtype != KV_F16 && dtype != KV_BF16))
        return KV_ERR_INVAL;
    // Splits: up to kMaxSplits of at least kSplitTokens keys each, fewer if
    // their partial states would not fit the scratch array.  A problem whose
    // partials do not fit even with one split per (row, KV head) is rejected.
    const long per_split = (long)seq * n_kv_heads * kPartialFloats;
    if (per_split > kScratchFloats) return KV_ERR_RANGE;
    int nsplit = (total_len + kSplitTokens - 1) / kSplitTokens;
    if (nsplit > kMaxSplits) nsplit = kMaxSplits;
    if ((long)nsplit * per_split > kScratchFloats) nsplit = (int)(kScratchFloats / per_split);
    const int split_tokens = (total_len + nsplit - 1) / nsplit;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KV_ERR_CUDA;
    float* scratch;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_addr[dev]) {
            void* ptr = nullptr;
            if (cudaGetSymbolAddress(&ptr, g_scratch) != cudaSuccess || !ptr) return KV_ERR_CUDA;
            g_addr[dev] = static_cast<float*>(ptr);
        }
        scratch = g_addr[dev];
    }
    cudaStream_t st = (cudaStream_t)stream;
    contig_partial_kernel<<<dim3(nsplit, n_kv_heads, seq), kWarps * 32, 0, st>>>(
        q, (const uint16_t*)k_cache, (const uint16_t*)v_cache, scratch, seq, total_len, n_heads,
        n_kv_heads, pos_base, nsplit, split_tokens, dtype);
    if (counted(cudaGetLastError()) != cudaSuccess) return KV_ERR_CUDA;
    contig_merge_kernel<<<dim3(n_heads, seq), kHeadDim, 0, st>>>(scratch, out, n_heads, n_kv_heads, nsplit);
    if (counted(cudaGetLastError()) != cudaSuccess) return KV_ERR_CUDA;
    return KV_OK;
}
