// xgpu_exchange.cu -- split-KV across GPUs, merged over peer memory.
//
// A long sequence is split along its positions across the GPUs of a node
// (one process per GPU).  Per layer every rank attends over its slice; the
// partial states (m, l, o) of every (sequence, query head) row must then be
// merged across ranks.  The reference has no split-KV (it runs one sequence
// on one device); the merge is the log-sum-exp identity
//   out = sum_g l_g e^(m_g - M) o_g / sum_g l_g e^(m_g - M),  M = max_g m_g.
//
// Instead of an all-gather followed by a separate merge launch, the exchange
// kernel runs right behind the local decode (programmatic dependent launch).
// Per row, thread d (one per dim) writes this rank's value of dim d into
// every peer's inbox as one 64-bit word {value, epoch of this layer call}
// with one store over NVLink (the areas are mapped with CUDA IPC); two
// more words carry m and l.  Readers poll the words of their own inbox (all
// peers' words loaded together in each sweep) until every word carries the
// current epoch -- a scalar 64-bit access is seen
// whole, so the value beside a current epoch is current -- and merge.  No fence, flag
// or barrier sits on the path (the low-latency protocol NCCL calls LL).  No
// multicast and no bulk copies touch peer memory.
//
// Two inbox buffers alternate by layer call, so a rank that runs ahead never
// overwrites words a peer has not read yet: it cannot write call e+2's words
// before it has read every peer's call-(e+1) words, which a peer writes only
// after its call-e kernel completed.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "kvattn.h"
#include "kvattn_internal.h"

struct kvx_exch {
    int device = 0, rank = 0, world = 1, max_rows = 0;
    float* base[kvattn::kMaxRanks] = {};  // [rank] is the local allocation
    bool opened[kvattn::kMaxRanks] = {};
    unsigned epoch = 0;                   // layer calls made
    std::mutex mu;
};

namespace kvattn {
namespace {

constexpr long long kXchgWaitLimit = 2000000000LL;  // SM clocks (~1 s) before a wait gives up

// An inbox word is one scalar 64-bit access (value bits low, epoch high):
// relaxed at system scope, so a reader observes it whole.
__device__ __forceinline__ void st_word(uint2* p, float v, unsigned epoch) {
    const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint2 ld_word(const uint2* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return make_uint2((unsigned)w, (unsigned)(w >> 32));
}

constexpr int kXchgWarps = 16;  // warps of a row's CTA (the first 4 run the exchange)

// One CTA per (sequence, query head) row.  Its local state is either this
// rank's slot (written by the decode launch) or, for a row of a split
// segment (nsplit > 0), the merge of the segment's pieces: warp w takes
// pieces w, w + 16, ... eight at a time (lane l holds dims 4l..4l+3), online
// log-sum-exp in base 2 as the decode kernel keeps it, then the 16 warps
// merge in shared memory.  Then thread d < 128 (one per dim) exchanges and
// merges across ranks.
__global__ void __launch_bounds__(kXchgWarps * 32) xchg_kernel(const __grid_constant__ XchgArgs a) {
    __shared__ float s_m[kXchgWarps], s_l[kXchgWarps];
    __shared__ __align__(16) float s_o[kXchgWarps][kHeadDim];
    // The next layer's decode launch may start now (it writes nothing before
    // this kernel completes, and its early tile copies read another layer):
    // it overlaps the wait for the peers.  The local states come from the
    // decode grid (and its split merge): wait until they are complete and
    // visible.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int r = blockIdx.x, d = threadIdx.x;
    if (r >= a.rows) return;
    const int W = a.world, R = a.max_rows;
    const float* mine = a.base[a.me];
    // ---- this rank's state of row r ----
    int first = 0, np = 0;
    if (a.nsplit > 0 && a.q_heads > 0 && a.group > 0) {
        const int key = (r / a.q_heads) | (((r % a.q_heads) / a.group) << 16);
        for (int k = 0; k < a.nsplit && k < kMaxXchgSplit; ++k)
            if (a.seg[k].x == key) {
                first = a.seg[k].y & 0xffff;
                np = a.seg[k].y >> 16;
                break;
            }
        if (np > 0 && (first >> 1) + np > kMaxGrid) {  // never read past the partials
            if (d == 0 && atomicCAS(a.status, 0, 5 /* KV_ERR_RANGE */) == 0) {
                a.status[1] = r;
                a.status[2] = 510;
            }
            np = 0;
        }
    }
    float m0, l0, o0;
    if (np > 0) {
        const int warp = d >> 5, lane = d & 31, h = r % a.group, g0 = first >> 1;
        float M = -INFINITY, L = 0.f;
        float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c0 = warp; c0 < np; c0 += 8 * kXchgWarps) {
            float mm[8], ll[8];
            float4 oo[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int pc = c0 + u * kXchgWarps;
                const bool live = pc < np;
                const int pidx = pc == 0 ? first : 2 * (g0 + pc);
                const float* pp = a.partials + (size_t)(live ? pidx : 0) * kPartialFloats;
                mm[u] = live ? __ldcg(pp + h) : 0.f;
                ll[u] = live ? __ldcg(pp + kMaxGroup + h) : 0.f;
                oo[u] = live ? __ldcg(reinterpret_cast<const float4*>(pp + 2 * kMaxGroup + h * kHeadDim) + lane)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (!(ll[u] > 0.f)) continue;  // empty piece (or past the end): no weight
                const float Mn = fmaxf(M, mm[u]);
                const float sa = exp2f(M - Mn);  // 0 while M is -inf
                const float e = ll[u] * exp2f(mm[u] - Mn);
                A.x = A.x * sa + e * oo[u].x;
                A.y = A.y * sa + e * oo[u].y;
                A.z = A.z * sa + e * oo[u].z;
                A.w = A.w * sa + e * oo[u].w;
                L = L * sa + e;
                M = Mn;
            }
        }
        if (lane == 0) {
            s_m[warp] = M;
            s_l[warp] = L;
        }
        reinterpret_cast<float4*>(s_o[warp])[lane] = A;
        __syncthreads();
        if (d >= kHeadDim) return;
        float Mt = -INFINITY;
#pragma unroll
        for (int w = 0; w < kXchgWarps; ++w)
            if (s_l[w] > 0.f) Mt = fmaxf(Mt, s_m[w]);
        float Lt = 0.f, At = 0.f;
#pragma unroll
        for (int w = 0; w < kXchgWarps; ++w) {
            if (!(s_l[w] > 0.f)) continue;
            const float f = exp2f(s_m[w] - Mt);
            Lt += s_l[w] * f;
            At += s_o[w][d] * f;
        }
        m0 = Mt * 0.6931471805599453f;  // natural-log units, as the decode writes the slot
        l0 = Lt;
        o0 = Lt > 0.f ? At / Lt : 0.f;
    } else {
        if (d >= kHeadDim) return;
        m0 = __ldcg(mine + r);
        l0 = __ldcg(mine + R + r);
        o0 = __ldcg(mine + 2 * R + (size_t)r * kHeadDim + d);
    }
    const int buf = (int)(a.epoch & 1u);
    for (int g = 0; g < W; ++g) {
        if (g == a.me) continue;
        uint2* w = xchg_inbox(a.base[g], W, R, buf, a.me) + (size_t)r * (2 + kHeadDim);
        st_word(w + 2 + d, o0, a.epoch);
        if (d == 0) st_word(w, m0, a.epoch);
        if (d == 1) st_word(w + 1, l0, a.epoch);
    }
    // Collect every peer's state: each sweep issues the loads of all words
    // still missing (one round trip for all peers, not one per peer and
    // word), then keeps those that carry this call's epoch; bounded.
    float mg[kMaxRanks], lg[kMaxRanks], og[kMaxRanks];
    unsigned need = 0;
    for (int g = 0; g < W; ++g)
        if (g != a.me) need |= 1u << g;
    bool ok = true;
    const long long t0 = clock64();
    while (need) {
        uint2 wm[kMaxRanks], wl[kMaxRanks], wo[kMaxRanks];
#pragma unroll
        for (int g = 0; g < kMaxRanks; ++g) {
            if (!((need >> g) & 1u)) continue;
            const uint2* w = xchg_inbox(a.base[a.me], W, R, buf, g) + (size_t)r * (2 + kHeadDim);
            wm[g] = ld_word(w);
            wl[g] = ld_word(w + 1);
            wo[g] = ld_word(w + 2 + d);
        }
#pragma unroll
        for (int g = 0; g < kMaxRanks; ++g) {
            if (!((need >> g) & 1u)) continue;
            if (wm[g].y == a.epoch && wl[g].y == a.epoch && wo[g].y == a.epoch) {
                mg[g] = __uint_as_float(wm[g].x);
                lg[g] = __uint_as_float(wl[g].x);
                og[g] = __uint_as_float(wo[g].x);
                need &= ~(1u << g);
            }
        }
        if (need && clock64() - t0 > kXchgWaitLimit) {
            ok = false;
            if (atomicCAS(a.status, 0, KV_ERR_TIMEOUT) == 0) {
                a.status[1] = r;
                a.status[2] = 500 + (__ffs(need) - 1);
                a.status[3] = (int)a.epoch;
            }
            break;
        }
    }
    // Merge in rank order (the same arithmetic on every rank); this rank's
    // own state comes from its local area.
    float M = -INFINITY, L = 0.f, A = 0.f;
#pragma unroll
    for (int g = 0; g < kMaxRanks; ++g) {
        if (!ok || g >= W) continue;
        const float m = g == a.me ? m0 : mg[g], l = g == a.me ? l0 : lg[g], o = g == a.me ? o0 : og[g];
        if (!(l > 0.f)) continue;  // an empty slice: no weight
        const float Mn = fmaxf(M, m);
        const float sa = expf(M - Mn);  // 0 while M is -inf
        const float e = l * expf(m - Mn);
        A = A * sa + e * o;
        L = L * sa + e;
        M = Mn;
    }
    a.out[(size_t)r * kHeadDim + d] = (ok && L > 0.f) ? A / L : 0.f;
}

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(dev);
    }
    ~DevGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int cuda_err(cudaError_t e, const char* what) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
    return set_error(KV_ERR_CUDA, buf);
}

}  // namespace

cudaError_t launch_xchg(const XchgArgs& a, cudaStream_t st) {
    if (a.rows <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.rows);
    cfg.blockDim = dim3(a.nsplit > 0 ? kXchgWarps * 32 : kHeadDim);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return counted(cudaLaunchKernelEx(&cfg, xchg_kernel, a));
}

int xchg_prepare(kvx_exch* x, int device, int rows, int* status, float* out, XchgArgs* a,
                 float** m, float** l, float** o) {
    if (!x) return set_error(KV_ERR_INVAL, "exchange is NULL");
    if (x->device != device) return set_error(KV_ERR_INVAL, "exchange and pool are on different devices");
    if (rows > x->max_rows) return set_error(KV_ERR_RANGE, "more rows than the exchange holds");
    for (int g = 0; g < x->world; ++g)
        if (!x->base[g]) return set_error(KV_ERR_STATE, "a peer's area is not open (kvx_open)");
    *a = XchgArgs{};
    for (int g = 0; g < x->world; ++g) a->base[g] = x->base[g];
    a->world = x->world;
    a->me = x->rank;
    a->rows = rows;
    a->max_rows = x->max_rows;
    a->epoch = x->epoch + 1;
    a->out = out;
    a->status = status;
    float* slot = x->base[x->rank];  // the local states
    *m = slot;
    *l = slot + x->max_rows;
    *o = slot + 2 * (size_t)x->max_rows;
    return KV_OK;
}

void xchg_commit(kvx_exch* x) { x->epoch += 1; }

}  // namespace kvattn

using namespace kvattn;

extern "C" {

int kvx_create(int device, int rank, int world, int max_rows, kvx_exch** out) {
    if (!out) return set_error(KV_ERR_INVAL, "out is NULL");
    *out = nullptr;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || max_rows < 1)
        return set_error(KV_ERR_INVAL, "need 1 <= world <= 8, 0 <= rank < world, max_rows >= 1");
    DevGuard dg(device);
    kvx_exch* x = new kvx_exch;
    x->device = device;
    x->rank = rank;
    x->world = world;
    x->max_rows = (max_rows + 3) & ~3;
    const size_t bytes = xchg_bytes(world, x->max_rows);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);  // inbox words start at epoch 0
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        delete x;
        return cuda_err(e, "kvx_create");
    }
    x->base[rank] = static_cast<float*>(p);
    *out = x;
    return KV_OK;
}

int kvx_handle(const kvx_exch* x, void* handle) {
    if (!x || !handle) return set_error(KV_ERR_INVAL, "NULL argument");
    DevGuard dg(x->device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, x->base[x->rank]);
    if (e != cudaSuccess) return cuda_err(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == KVX_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof h);
    return KV_OK;
}

int kvx_open(kvx_exch* x, int peer, const void* handle) {
    if (!x || !handle) return set_error(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(x->mu);
    if (peer < 0 || peer >= x->world || peer == x->rank) return set_error(KV_ERR_INVAL, "bad peer rank");
    if (x->opened[peer]) return set_error(KV_ERR_STATE, "peer already open");
    DevGuard dg(x->device);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_err(e, "cudaIpcOpenMemHandle");
    x->base[peer] = static_cast<float*>(p);
    x->opened[peer] = true;
    return KV_OK;
}

int kvx_destroy(kvx_exch* x) {
    if (!x) return KV_OK;
    {
        DevGuard dg(x->device);
        cudaDeviceSynchronize();
        for (int g = 0; g < x->world; ++g)
            if (x->opened[g]) cudaIpcCloseMemHandle(x->base[g]);
        if (x->base[x->rank]) cudaFree(x->base[x->rank]);
    }
    delete x;
    return KV_OK;
}

}  // extern "C"
