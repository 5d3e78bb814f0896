// pool_kernels.cu -- data movement on the paged pool: import/gather between the
// reference row layout and swizzled tiles, prefill append with RoPE, block-table
// patches, and the cross-GPU log-sum-exp combine.
//
// All of these are HBM-bound byte work: one 16-byte vector per thread where
// the data allows it, grid-stride loops sized to the SM count.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kvattn_internal.h"

namespace kvattn {

namespace {

__device__ __forceinline__ size_t tile_base(const PoolView& pv, int layer, int blk, int head) {
    return (size_t)layer * pv.layer_bytes + ((size_t)blk * pv.kv_heads + head) * pv.tile_bytes;
}

// Chunk `ch` (0..15, 8 dims each) of token row t inside a tile.
__device__ __forceinline__ uint32_t chunk_offset(int t, int ch) {
    return (uint32_t)(((ch >> 3) * 16 + t) * 128 + (((ch & 7) ^ (t & 7)) << 4));
}

// One thread per 16-byte chunk: (row, kv head, chunk, K|V).
__global__ void import_kernel(PoolView pv, int layer, int seq, int pos0, int n,
                              const uint4* __restrict__ k_rows, const uint4* __restrict__ v_rows) {
    const long total = (long)n * pv.kv_heads * 16 * 2;
    const int* trow = pv.table + (size_t)seq * pv.max_blocks_per_seq;
    for (long x = blockIdx.x * (long)blockDim.x + threadIdx.x; x < total; x += (long)gridDim.x * blockDim.x) {
        const int ch = (int)(x & 15);
        long rest = x >> 4;
        const int h = (int)(rest % pv.kv_heads);
        rest /= pv.kv_heads;
        const int isv = (int)(rest & 1);
        const int r = (int)(rest >> 1);
        const int p = pos0 + r;
        const int blk = trow[p / kBlockTokens];
        const int t = p % kBlockTokens;
        const uint4 val = (isv ? v_rows : k_rows)[((size_t)r * pv.kv_heads + h) * 16 + ch];
        uint8_t* base = isv ? pv.v : pv.k;
        *reinterpret_cast<uint4*>(base + tile_base(pv, layer, blk, h) + chunk_offset(t, ch)) = val;
    }
}

__global__ void gather_kernel(PoolView pv, int layer, int seq, int len, uint4* __restrict__ k_rows,
                              uint4* __restrict__ v_rows) {
    const long total = (long)len * pv.kv_heads * 16 * 2;
    const int* trow = pv.table + (size_t)seq * pv.max_blocks_per_seq;
    for (long x = blockIdx.x * (long)blockDim.x + threadIdx.x; x < total; x += (long)gridDim.x * blockDim.x) {
        const int ch = (int)(x & 15);
        long rest = x >> 4;
        const int h = (int)(rest % pv.kv_heads);
        rest /= pv.kv_heads;
        const int isv = (int)(rest & 1);
        const int p = (int)(rest >> 1);
        const int blk = trow[p / kBlockTokens];
        const int t = p % kBlockTokens;
        const uint8_t* base = isv ? pv.v : pv.k;
        const uint4 val = *reinterpret_cast<const uint4*>(base + tile_base(pv, layer, blk, h) + chunk_offset(t, ch));
        (isv ? v_rows : k_rows)[((size_t)p * pv.kv_heads + h) * 16 + ch] = val;
    }
}

// Chunk of concatenated row r and its position.
__device__ __forceinline__ int chunk_of(const ChunkBatch& cb, int r, int& p) {
    int i = 0;
    while (i + 1 < cb.nreq && r >= cb.row0[i + 1]) ++i;
    p = cb.pos0[i] + (r - cb.row0[i]);
    return i;
}

// Prefill append (qwen2_model.cpp:180-200 for seq = n) of every chunk of the
// batch: one warp per (row, kv head); lane l rotates dims 2l, 2l+1 with
// partners +64.
template <int DT>
__global__ void append_chunk_kernel(PoolView pv, int layer, const __grid_constant__ ChunkBatch cb,
                                    const float* __restrict__ k, const float* __restrict__ v) {
    const int lane = threadIdx.x & 31;
    const long nwarps = (long)cb.row0[cb.nreq] * pv.kv_heads;
    const size_t kvw = (size_t)pv.kv_heads * kHeadDim;
    for (long w = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; w < nwarps;
         w += ((long)gridDim.x * blockDim.x) >> 5) {
        const int h = (int)(w % pv.kv_heads);
        const int r = (int)(w / pv.kv_heads);
        int p;
        const int* trow = pv.table + (size_t)cb.seq[chunk_of(cb, r, p)] * pv.max_blocks_per_seq;
        const float* kr = k + (size_t)r * kvw + (size_t)h * kHeadDim;
        const float* vr = v + (size_t)r * kvw + (size_t)h * kHeadDim;
        const float* cs = reinterpret_cast<const float*>(pv.rope + (size_t)p * (kHeadDim / 2));
        const int i = 2 * lane;
        float2 a = *reinterpret_cast<const float2*>(kr + i);
        float2 b = *reinterpret_cast<const float2*>(kr + i + 64);
        float4 cc = *reinterpret_cast<const float4*>(cs + 2 * i);
        float lo0, hi0, lo1, hi1;
        rope_pair(a.x, b.x, cc.x, cc.y, lo0, hi0);
        rope_pair(a.y, b.y, cc.z, cc.w, lo1, hi1);
        float2 va = *reinterpret_cast<const float2*>(vr + i);
        float2 vb = *reinterpret_cast<const float2*>(vr + i + 64);
        const int blk = trow[p / kBlockTokens];
        const int t = p % kBlockTokens;
        const size_t tb = tile_base(pv, layer, blk, h);
        const uint32_t o_lo = tile_offset(t, i), o_hi = tile_offset(t, i + 64);
        *reinterpret_cast<uint32_t*>(pv.k + tb + o_lo) = (uint32_t)enc_trunc<DT>(lo0) | ((uint32_t)enc_trunc<DT>(lo1) << 16);
        *reinterpret_cast<uint32_t*>(pv.k + tb + o_hi) = (uint32_t)enc_trunc<DT>(hi0) | ((uint32_t)enc_trunc<DT>(hi1) << 16);
        *reinterpret_cast<uint32_t*>(pv.v + tb + o_lo) = (uint32_t)enc_trunc<DT>(va.x) | ((uint32_t)enc_trunc<DT>(va.y) << 16);
        *reinterpret_cast<uint32_t*>(pv.v + tb + o_hi) = (uint32_t)enc_trunc<DT>(vb.x) | ((uint32_t)enc_trunc<DT>(vb.y) << 16);
    }
}

// The same append into an INT8 pool: the rotated k row and the v row of each
// (token, kv head) quantised by its warp (quant_row_warp), codes and scale
// written to the tile.
__global__ void append_chunk_i8_kernel(PoolView pv, int layer, const __grid_constant__ ChunkBatch cb,
                                       const float* __restrict__ k, const float* __restrict__ v) {
    const int lane = threadIdx.x & 31;
    const long nwarps = (long)cb.row0[cb.nreq] * pv.kv_heads;
    const size_t kvw = (size_t)pv.kv_heads * kHeadDim;
    for (long w = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; w < nwarps;
         w += ((long)gridDim.x * blockDim.x) >> 5) {
        const int h = (int)(w % pv.kv_heads);
        const int r = (int)(w / pv.kv_heads);
        int p;
        const int* trow = pv.table + (size_t)cb.seq[chunk_of(cb, r, p)] * pv.max_blocks_per_seq;
        const float* kr = k + (size_t)r * kvw + (size_t)h * kHeadDim;
        const float* vr = v + (size_t)r * kvw + (size_t)h * kHeadDim;
        const float* cs = reinterpret_cast<const float*>(pv.rope + (size_t)p * (kHeadDim / 2));
        const int i = 2 * lane;
        float2 a = *reinterpret_cast<const float2*>(kr + i);
        float2 b = *reinterpret_cast<const float2*>(kr + i + 64);
        float4 cc = *reinterpret_cast<const float4*>(cs + 2 * i);
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
        const float ks = quant_row_warp(kx, kc), vs = quant_row_warp(vx, vc);
        const int blk = trow[p / kBlockTokens];
        const int t = p % kBlockTokens;
        const size_t tb = tile_base(pv, layer, blk, h);
        uint8_t* kt = pv.k + tb;
        uint8_t* vt = pv.v + tb;
        *reinterpret_cast<char2*>(kt + i8_offset(t, i)) = make_char2(kc[0], kc[1]);
        *reinterpret_cast<char2*>(kt + i8_offset(t, i + 64)) = make_char2(kc[2], kc[3]);
        *reinterpret_cast<char2*>(vt + i8_offset(t, i)) = make_char2(vc[0], vc[1]);
        *reinterpret_cast<char2*>(vt + i8_offset(t, i + 64)) = make_char2(vc[2], vc[3]);
        if (lane == 0) {
            reinterpret_cast<float*>(kt + kBlockTokens * kHeadDim)[t] = ks;
            reinterpret_cast<float*>(vt + kBlockTokens * kHeadDim)[t] = vs;
        }
    }
}

// INT8 rows <-> tiles: codes [n][kv_heads * 128], scales [n][kv_heads]; one
// thread per (row, kv head, K|V, 16-byte chunk of 8 chunks) plus the scale.
__global__ void import_i8_kernel(PoolView pv, int layer, int seq, int pos0, int n, const uint4* __restrict__ kc,
                                 const uint4* __restrict__ vc, const float* __restrict__ ks,
                                 const float* __restrict__ vs) {
    const long total = (long)n * pv.kv_heads * 9 * 2;
    const int* trow = pv.table + (size_t)seq * pv.max_blocks_per_seq;
    for (long x = blockIdx.x * (long)blockDim.x + threadIdx.x; x < total; x += (long)gridDim.x * blockDim.x) {
        const int ch = (int)(x % 9);
        long rest = x / 9;
        const int h = (int)(rest % pv.kv_heads);
        rest /= pv.kv_heads;
        const int isv = (int)(rest & 1);
        const int r = (int)(rest >> 1);
        const int p = pos0 + r;
        const int blk = trow[p / kBlockTokens];
        const int t = p % kBlockTokens;
        uint8_t* tile = (isv ? pv.v : pv.k) + tile_base(pv, layer, blk, h);
        if (ch < 8) {
            *reinterpret_cast<uint4*>(tile + i8_offset(t, ch * 16)) = (isv ? vc : kc)[((size_t)r * pv.kv_heads + h) * 8 + ch];
        } else {
            reinterpret_cast<float*>(tile + kBlockTokens * kHeadDim)[t] = (isv ? vs : ks)[(size_t)r * pv.kv_heads + h];
        }
    }
}

__global__ void gather_i8_kernel(PoolView pv, int layer, int seq, int len, uint4* __restrict__ kc,
                                 uint4* __restrict__ vc, float* __restrict__ ks, float* __restrict__ vs) {
    const long total = (long)len * pv.kv_heads * 9 * 2;
    const int* trow = pv.table + (size_t)seq * pv.max_blocks_per_seq;
    for (long x = blockIdx.x * (long)blockDim.x + threadIdx.x; x < total; x += (long)gridDim.x * blockDim.x) {
        const int ch = (int)(x % 9);
        long rest = x / 9;
        const int h = (int)(rest % pv.kv_heads);
        rest /= pv.kv_heads;
        const int isv = (int)(rest & 1);
        const int p = (int)(rest >> 1);
        const int blk = trow[p / kBlockTokens];
        const int t = p % kBlockTokens;
        const uint8_t* tile = (isv ? pv.v : pv.k) + tile_base(pv, layer, blk, h);
        if (ch < 8) {
            (isv ? vc : kc)[((size_t)p * pv.kv_heads + h) * 8 + ch] = *reinterpret_cast<const uint4*>(tile + i8_offset(t, ch * 16));
        } else {
            (isv ? vs : ks)[(size_t)p * pv.kv_heads + h] = reinterpret_cast<const float*>(tile + kBlockTokens * kHeadDim)[t];
        }
    }
}

__global__ void patch_kernel(PoolView pv, const TablePatch* __restrict__ patches, int npatch) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < npatch; i += gridDim.x * blockDim.x) {
        const TablePatch p = patches[i];
        pv.table[(size_t)p.seq * pv.max_blocks_per_seq + p.idx] = p.block;
    }
}

// out[r][d] = sum_g l_g e^(m_g - M) o_g[r][d] / sum_g l_g e^(m_g - M); states
// with l == 0 (nothing attended) carry no weight.
// Rank g's m, l and o start `gstride` floats after rank g-1's.
__global__ void combine_kernel(int G, int rows, int dim, const float* __restrict__ m,
                               const float* __restrict__ l, const float* __restrict__ o,
                               size_t gstride_ml, size_t gstride_o, float* __restrict__ out) {
    // A decode launch behind this merge may start now: it writes nothing
    // before this kernel completes.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const long total = (long)rows * dim;
    for (long x = blockIdx.x * (long)blockDim.x + threadIdx.x; x < total; x += (long)gridDim.x * blockDim.x) {
        const int r = (int)(x / dim);
        float M = -INFINITY;
        for (int g = 0; g < G; ++g)
            if (l[(size_t)g * gstride_ml + r] > 0.f) M = fmaxf(M, m[(size_t)g * gstride_ml + r]);
        float L = 0.f, acc = 0.f;
        for (int g = 0; g < G; ++g) {
            const float lg = l[(size_t)g * gstride_ml + r];
            if (lg > 0.f) {
                const float w = lg * expf(m[(size_t)g * gstride_ml + r] - M);
                L += w;
                acc += w * o[(size_t)g * gstride_o + x];
            }
        }
        out[x] = L > 0.f ? acc / L : 0.f;
    }
}

int grid_for(long work, int threads) {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
            sms = 132;
    }
    long g = (work + threads - 1) / threads;
    const long cap = (long)sms * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace

cudaError_t launch_import(const PoolView& pv, int layer, int seq, int pos0, int n,
                          const uint16_t* k_rows, const uint16_t* v_rows, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const long work = (long)n * pv.kv_heads * 32;
    import_kernel<<<grid_for(work, 256), 256, 0, st>>>(pv, layer, seq, pos0, n,
                                                       reinterpret_cast<const uint4*>(k_rows),
                                                       reinterpret_cast<const uint4*>(v_rows));
    return counted(cudaGetLastError());
}

cudaError_t launch_gather(const PoolView& pv, int layer, int seq, int len, uint16_t* k_rows,
                          uint16_t* v_rows, cudaStream_t st) {
    if (len <= 0) return cudaSuccess;
    const long work = (long)len * pv.kv_heads * 32;
    gather_kernel<<<grid_for(work, 256), 256, 0, st>>>(pv, layer, seq, len, reinterpret_cast<uint4*>(k_rows),
                                                       reinterpret_cast<uint4*>(v_rows));
    return counted(cudaGetLastError());
}

cudaError_t launch_append_batch(const PoolView& pv, int layer, const ChunkBatch& cb, const float* k,
                                const float* v, cudaStream_t st) {
    const long rows = cb.nreq > 0 ? cb.row0[cb.nreq] : 0;
    if (rows <= 0) return cudaSuccess;
    const long work = rows * pv.kv_heads * 32;
    const int grid = grid_for(work, 256);
    if (pv.dtype == 0)
        append_chunk_kernel<0><<<grid, 256, 0, st>>>(pv, layer, cb, k, v);
    else if (pv.dtype == 1)
        append_chunk_kernel<1><<<grid, 256, 0, st>>>(pv, layer, cb, k, v);
    else
        append_chunk_i8_kernel<<<grid, 256, 0, st>>>(pv, layer, cb, k, v);
    return counted(cudaGetLastError());
}

cudaError_t launch_import_i8(const PoolView& pv, int layer, int seq, int pos0, int n, const int8_t* k_codes,
                             const int8_t* v_codes, const float* k_scales, const float* v_scales, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const long work = (long)n * pv.kv_heads * 18;
    import_i8_kernel<<<grid_for(work, 256), 256, 0, st>>>(pv, layer, seq, pos0, n,
                                                          reinterpret_cast<const uint4*>(k_codes),
                                                          reinterpret_cast<const uint4*>(v_codes), k_scales, v_scales);
    return counted(cudaGetLastError());
}

cudaError_t launch_gather_i8(const PoolView& pv, int layer, int seq, int len, int8_t* k_codes, int8_t* v_codes,
                             float* k_scales, float* v_scales, cudaStream_t st) {
    if (len <= 0) return cudaSuccess;
    const long work = (long)len * pv.kv_heads * 18;
    gather_i8_kernel<<<grid_for(work, 256), 256, 0, st>>>(pv, layer, seq, len, reinterpret_cast<uint4*>(k_codes),
                                                          reinterpret_cast<uint4*>(v_codes), k_scales, v_scales);
    return counted(cudaGetLastError());
}

cudaError_t launch_patch(const PoolView& pv, const TablePatch* patches, int npatch, cudaStream_t st) {
    if (npatch <= 0) return cudaSuccess;
    patch_kernel<<<grid_for(npatch, 256), 256, 0, st>>>(pv, patches, npatch);
    return counted(cudaGetLastError());
}

cudaError_t launch_combine(int G, int rows, int dim, const float* m, const float* l, const float* o,
                           size_t gstride_ml, size_t gstride_o, float* out, cudaStream_t st) {
    const long total = (long)rows * dim;
    if (total <= 0) return cudaSuccess;
    combine_kernel<<<grid_for(total, 256), 256, 0, st>>>(G, rows, dim, m, l, o, gstride_ml, gstride_o, out);
    return counted(cudaGetLastError());
}

}  // namespace kvattn
