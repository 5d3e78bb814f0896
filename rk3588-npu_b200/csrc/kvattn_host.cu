// kvattn_host.cu -- host runtime behind include/kvattn.h: the paged pool,
// its block allocator and block tables, the decode planner, and the C ABI.
//
// Replaces KVCache (worker/include/model/kv_cache.h:19-41,
// worker/src/model/kv_cache.cpp:4-16) with a pool of fixed-size blocks shared
// by many sequences, and the inline KV write + op_attention call of
// Qwen2Model::forward (worker/src/model/qwen2_model.cpp:180-206) with a
// planned, batched device step.
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "kvattn.h"
#include "kvattn_internal.h"

using namespace kvattn;

// ------------------------------------------------------------------ errors
namespace {

thread_local std::string g_err;

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return status;
}

}  // namespace

int kvattn::set_error(int status, const char* msg) { return fail(status, "%s", msg); }

namespace {
std::atomic<long long> g_kernel_launches{0};
}  // namespace

void kvattn::count_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }

int kv_kernel_count(long long* n) {
    if (!n) return fail(KV_ERR_INVAL, "NULL argument");
    *n = g_kernel_launches.load(std::memory_order_relaxed);
    return KV_OK;
}

namespace {

int cuda_fail(cudaError_t e, const char* what) {
    return fail(KV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define KV_CUDA(call)                                   \
    do {                                                \
        cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

constexpr int kRing = 4;  // plan upload buffers in flight

struct Seq {
    bool live = false;
    int len = 0;
    std::vector<int> blocks;
};

}  // namespace

// ------------------------------------------------------------------- pool
struct kvp_pool {
    std::mutex mu;
    int device = 0;
    bool host_only = false;  // device == KVP_HOST_ONLY: allocator/planner only
    int layers = 0, q_heads = 0, kv_heads = 0, head_dim = 0, block_tokens = 0;
    int num_blocks = 0, dtype = 0, max_seqs = 0, max_seq_len = 0, mbps = 0;
    float theta = 0.f;
    int num_sms = 0, occupancy = 0;
    bool overlap = false;  // decode launches as programmatic dependents (kvp_set_overlap)
    long max_items = 0;
    long max_tiles = 0;  // bound on flat blocks in one plan
    PoolView pv{};

    // device allocations
    void* d_k = nullptr;
    void* d_v = nullptr;
    float2* d_rope = nullptr;
    int* d_table = nullptr;
    int* d_counters = nullptr;
    float* d_partials = nullptr;
    int* d_status = nullptr;
    float* d_prefill_part = nullptr;  // key-split partials of attn_prefill (grown on demand)
    size_t prefill_part_floats = 0;

    // allocator: LIFO stack of free block ids + position index
    std::vector<int> free_;
    std::vector<int> where_;
    std::vector<Seq> seqs;

    // block-table entries not yet on the device
    std::vector<TablePatch> pending;
    TablePatch* h_pending = nullptr;  // pinned
    TablePatch* d_pending = nullptr;
    size_t pending_cap = 0;
    cudaEvent_t pending_evt = nullptr;

    // plan ring
    size_t plan_bytes = 0;
    uint8_t* h_plan[kRing] = {};
    uint8_t* d_plan[kRing] = {};
    cudaEvent_t copy_done[kRing] = {};  // upload of ring slot r finished (copy stream)
    cudaEvent_t slot_free[kRing] = {};  // last launch reading ring slot r finished
    cudaStream_t copy_stream = nullptr; // non-blocking: plan uploads overlap running kernels
    int ring_next = 0;

    // active plan
    bool plan_active = false;
    bool plan_patched = false;
    int plan_slot_ring = 0;
    int plan_nslots = 0, plan_nitems = 0, plan_npatch = 0, plan_grid = 0, plan_nsplits = 0;
    int plan_max_pieces = 0;  // most pieces of one split segment
    PlanView plan_view{};
    std::vector<int> plan_seqs;
    std::vector<int> plan_append;
    cudaStream_t plan_stream = nullptr;

    // launch timing (kvp_timing_enable)
    bool timing = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> tev;
    size_t tev_used = 0;

    void reset_free_list() {
        free_.resize(num_blocks);
        where_.assign(num_blocks, -1);
        for (int i = 0; i < num_blocks; ++i) {
            free_[i] = num_blocks - 1 - i;  // back() == 0: blocks are handed out 0, 1, 2, ...
            where_[num_blocks - 1 - i] = i;
        }
    }
    int pop_block() {
        int b = free_.back();
        free_.pop_back();
        where_[b] = -1;
        return b;
    }
    void push_block(int b) {
        where_[b] = (int)free_.size();
        free_.push_back(b);
    }
    void remove_block(int b) {  // b must be free
        int i = where_[b];
        int last = free_.back();
        free_[i] = last;
        where_[last] = i;
        free_.pop_back();
        where_[b] = -1;
    }
};

namespace {

// cos/sin for every (position, pair) with the float libm calls and operation
// order of rope_one_head (worker/src/ops/op_rope.cpp:11-14): freq =
// 1/powf(theta, 2i/head_dim), angle = (float)pos * freq.  Built once on the
// host so the device rotation uses bit-identical factors.
void build_rope_table(std::vector<float2>& tab, int max_pos, int head_dim, float theta) {
    const int half = head_dim / 2;
    std::vector<float> freq(half);
    for (int i = 0; i < half; ++i)
        freq[i] = 1.0f / std::pow(theta, (float)(2 * i) / (float)head_dim);
    tab.resize((size_t)max_pos * half);
    for (int p = 0; p < max_pos; ++p)
        for (int i = 0; i < half; ++i) {
            const float angle = (float)p * freq[i];
            tab[(size_t)p * half + i] = make_float2(std::cos(angle), std::sin(angle));
        }
}

// Upload and apply block-table entries queued by reserve/set_blocks.
int flush_pending(kvp_pool* p, cudaStream_t st) {
    if (p->pending.empty()) return KV_OK;
    if (p->host_only) {
        p->pending.clear();
        return KV_OK;
    }
    const size_t n = p->pending.size();
    if (n > p->pending_cap) {
        if (p->h_pending) {
            cudaEventSynchronize(p->pending_evt);
            cudaFreeHost(p->h_pending);
            cudaFree(p->d_pending);
            p->h_pending = nullptr;
            p->d_pending = nullptr;
        }
        size_t cap = std::max<size_t>(n, 1024);
        KV_CUDA(cudaMallocHost((void**)&p->h_pending, cap * sizeof(TablePatch)));
        KV_CUDA(cudaMalloc((void**)&p->d_pending, cap * sizeof(TablePatch)));
        p->pending_cap = cap;
    } else {
        KV_CUDA(cudaEventSynchronize(p->pending_evt));  // previous upload has read the buffer
    }
    memcpy(p->h_pending, p->pending.data(), n * sizeof(TablePatch));
    KV_CUDA(cudaMemcpyAsync(p->d_pending, p->h_pending, n * sizeof(TablePatch), cudaMemcpyHostToDevice, st));
    KV_CUDA(cudaEventRecord(p->pending_evt, st));
    KV_CUDA(launch_patch(p->pv, p->d_pending, (int)n, st));
    p->pending.clear();
    return KV_OK;
}

// Make the device block table current: queued patches and, if no layer call
// applied them yet, the active plan's new-block patches.
int sync_table(kvp_pool* p, cudaStream_t st) {
    int rc = flush_pending(p, st);
    if (rc != KV_OK) return rc;
    if (p->plan_active && !p->plan_patched && p->plan_npatch > 0) {
        const int r = p->plan_slot_ring;
        KV_CUDA(cudaStreamWaitEvent(st, p->copy_done[r], 0));
        KV_CUDA(launch_patch(p->pv, p->plan_view.patches, p->plan_npatch, st));
        KV_CUDA(cudaEventRecord(p->slot_free[r], st));
        p->plan_patched = true;
    }
    return KV_OK;
}

int require_device(const kvp_pool* p) {
    if (p->host_only) return fail(KV_ERR_STATE, "host-only pool has no device storage");
    return KV_OK;
}

int check_seq(const kvp_pool* p, int seq) {
    if (seq < 0 || seq >= p->max_seqs || !p->seqs[seq].live)
        return fail(KV_ERR_BADSEQ, "sequence %d is not live", seq);
    return KV_OK;
}

// Byte layout of one packed plan: header, slots, items, patches, CTA
// descriptors, tile list.
struct PlanLayout {
    size_t slots, items, patches, cta, tiles, splits, bytes;
};

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

PlanLayout plan_layout(int nslots, long nitems, int npatch, long grid, long ntiles, long nsplits) {
    PlanLayout L;
    L.slots = align16(sizeof(PlanHeader));
    L.items = align16(L.slots + (size_t)nslots * sizeof(DecodeSlot));
    L.patches = align16(L.items + (size_t)nitems * sizeof(WorkItem));
    L.cta = align16(L.patches + (size_t)npatch * sizeof(TablePatch));
    L.tiles = align16(L.cta + (size_t)grid * sizeof(CtaDesc));
    L.splits = align16(L.tiles + (size_t)ntiles * sizeof(int));
    L.bytes = align16(L.splits + (size_t)nsplits * sizeof(SplitSeg));
    return L;
}

void free_device(kvp_pool* p) {
    cudaFree(p->d_k);
    cudaFree(p->d_v);
    cudaFree(p->d_rope);
    cudaFree(p->d_table);
    cudaFree(p->d_counters);
    cudaFree(p->d_partials);
    cudaFree(p->d_prefill_part);
    cudaFree(p->d_status);
    cudaFree(p->d_pending);
    cudaFreeHost(p->h_pending);
    if (p->pending_evt) cudaEventDestroy(p->pending_evt);
    for (int i = 0; i < kRing; ++i) {
        cudaFree(p->d_plan[i]);
        cudaFreeHost(p->h_plan[i]);
        if (p->copy_done[i]) cudaEventDestroy(p->copy_done[i]);
        if (p->slot_free[i]) cudaEventDestroy(p->slot_free[i]);
    }
    if (p->copy_stream) cudaStreamDestroy(p->copy_stream);
    for (auto& e : p->tev) {
        cudaEventDestroy(e.first);
        cudaEventDestroy(e.second);
    }
}

}  // namespace

// ------------------------------------------------------------------ C ABI
extern "C" {

const char* kv_last_error(void) { return g_err.c_str(); }

const char* kv_status_str(int s) {
    switch (s) {
        case KV_OK: return "KV_OK";
        case KV_ERR_INVAL: return "KV_ERR_INVAL";
        case KV_ERR_OOM: return "KV_ERR_OOM";
        case KV_ERR_BADSEQ: return "KV_ERR_BADSEQ";
        case KV_ERR_CUDA: return "KV_ERR_CUDA";
        case KV_ERR_RANGE: return "KV_ERR_RANGE";
        case KV_ERR_STATE: return "KV_ERR_STATE";
        case KV_ERR_TIMEOUT: return "KV_ERR_TIMEOUT";
        default: return "KV_ERR_UNKNOWN";
    }
}

const char* kv_version(void) { return "0.1.0"; }

int kvp_create(int device, int num_layers, int num_q_heads, int num_kv_heads, int head_dim,
               int block_tokens, int num_blocks, int dtype, int max_seqs, int max_seq_len,
               float rope_theta, kvp_pool** out) {
    if (!out) return fail(KV_ERR_INVAL, "out is NULL");
    *out = nullptr;
    if (head_dim != kHeadDim) return fail(KV_ERR_INVAL, "head_dim must be %d (got %d)", kHeadDim, head_dim);
    if (block_tokens != kBlockTokens)
        return fail(KV_ERR_INVAL, "block_tokens must be %d (got %d)", kBlockTokens, block_tokens);
    if (num_layers < 1 || num_kv_heads < 1 || num_q_heads < 1 || num_blocks < 1 || max_seqs < 1 ||
        max_seq_len < 1)
        return fail(KV_ERR_INVAL, "sizes must be positive");
    if (num_q_heads % num_kv_heads != 0 || num_q_heads / num_kv_heads > kMaxGroup)
        return fail(KV_ERR_INVAL, "num_q_heads/num_kv_heads must be an integer <= %d", kMaxGroup);
    if (dtype != KV_F16 && dtype != KV_BF16 && dtype != KV_I8)
        return fail(KV_ERR_INVAL, "dtype must be KV_F16, KV_BF16 or KV_I8");
    if (!(rope_theta > 0.f)) return fail(KV_ERR_INVAL, "rope_theta must be > 0");
    const bool host_only = (device == KVP_HOST_ONLY);
    if (!host_only) {
        int ndev = 0;
        KV_CUDA(cudaGetDeviceCount(&ndev));
        if (device < 0 || device >= ndev)
            return fail(KV_ERR_INVAL, "device %d out of range (%d devices)", device, ndev);
    }
    DeviceGuard dg(host_only ? -1 : device);
    if (!dg.ok) return fail(KV_ERR_CUDA, "cudaSetDevice(%d) failed", device);

    kvp_pool* p = new kvp_pool();
    p->device = device;
    p->host_only = host_only;
    p->layers = num_layers;
    p->q_heads = num_q_heads;
    p->kv_heads = num_kv_heads;
    p->head_dim = head_dim;
    p->block_tokens = block_tokens;
    p->num_blocks = num_blocks;
    p->dtype = dtype;
    p->max_seqs = max_seqs;
    p->max_seq_len = max_seq_len;
    p->mbps = (max_seq_len + kBlockTokens - 1) / kBlockTokens;
    p->theta = rope_theta;
    p->seqs.resize(max_seqs);
    p->reset_free_list();
    // Pieces: every CTA boundary splits at most one segment, so items <=
    // segments + CTAs; CTAs <= grid + segments / kMaxCtaItems (item cap).
    p->max_items = 2L * max_seqs * num_kv_heads + 148L * 4 + 64;

    auto bail = [&](cudaError_t e, const char* what) {
        free_device(p);
        delete p;
        return cuda_fail(e, what);
    };
#define KV_CUDA_B(call)                         \
    do {                                        \
        cudaError_t e_ = (call);                \
        if (e_ != cudaSuccess) return bail(e_, #call); \
    } while (0)

    if (host_only) {
        // Bookkeeping only: plans are built for a nominal 148-SM part and kept on the host.
        p->num_sms = 148;
        p->occupancy = 3;
        p->max_tiles = ((long)num_blocks + max_seqs) * num_kv_heads;
        p->plan_bytes = plan_layout(max_seqs, p->max_items, max_seqs, p->max_items, p->max_tiles,
                                 (long)max_seqs * num_kv_heads).bytes;
        p->h_plan[0] = (uint8_t*)malloc(p->plan_bytes);
        if (!p->h_plan[0]) {
            delete p;
            return fail(KV_ERR_INVAL, "host allocation of %zu bytes failed", p->plan_bytes);
        }
        p->pv.num_blocks = num_blocks;
        p->pv.kv_heads = num_kv_heads;
        p->pv.q_heads = num_q_heads;
        p->pv.group = num_q_heads / num_kv_heads;
        p->pv.max_blocks_per_seq = p->mbps;
        p->pv.max_seq_len = max_seq_len;
        p->pv.dtype = dtype;
        *out = p;
        return KV_OK;
    }
    KV_CUDA_B(cudaDeviceGetAttribute(&p->num_sms, cudaDevAttrMultiProcessorCount, device));
    KV_CUDA_B(decode_occupancy(dtype, &p->occupancy));
    if (p->occupancy < 1) p->occupancy = 1;
    p->max_items = 2L * max_seqs * num_kv_heads + (long)p->num_sms * p->occupancy + 64;

    const int tile_bytes = dtype == KV_I8 ? kTileBytesI8 : kTileBytes;
    const size_t layer_bytes = (size_t)num_blocks * num_kv_heads * tile_bytes;
    KV_CUDA_B(cudaMalloc(&p->d_k, layer_bytes * num_layers));
    KV_CUDA_B(cudaMalloc(&p->d_v, layer_bytes * num_layers));
    KV_CUDA_B(cudaMemset(p->d_k, 0, layer_bytes * num_layers));
    KV_CUDA_B(cudaMemset(p->d_v, 0, layer_bytes * num_layers));

    std::vector<float2> tab;
    build_rope_table(tab, max_seq_len, head_dim, rope_theta);
    KV_CUDA_B(cudaMalloc((void**)&p->d_rope, tab.size() * sizeof(float2)));
    KV_CUDA_B(cudaMemcpy(p->d_rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));

    KV_CUDA_B(cudaMalloc((void**)&p->d_table, (size_t)max_seqs * p->mbps * sizeof(int)));
    KV_CUDA_B(cudaMemset(p->d_table, 0, (size_t)max_seqs * p->mbps * sizeof(int)));
    KV_CUDA_B(cudaMalloc((void**)&p->d_counters, (size_t)max_seqs * num_kv_heads * sizeof(int)));
    KV_CUDA_B(cudaMemset(p->d_counters, 0, (size_t)max_seqs * num_kv_heads * sizeof(int)));
    KV_CUDA_B(cudaMalloc((void**)&p->d_partials, (size_t)p->max_items * kPartialFloats * sizeof(float)));
    KV_CUDA_B(cudaMalloc((void**)&p->d_status, 32 * sizeof(int)));
    KV_CUDA_B(cudaMemset(p->d_status, 0, 32 * sizeof(int)));
    KV_CUDA_B(cudaEventCreateWithFlags(&p->pending_evt, cudaEventDisableTiming));

    p->max_tiles = ((long)num_blocks + max_seqs) * num_kv_heads;
    p->plan_bytes = plan_layout(max_seqs, p->max_items, max_seqs, p->max_items, p->max_tiles,
                                 (long)max_seqs * num_kv_heads).bytes;
    KV_CUDA_B(cudaStreamCreateWithFlags(&p->copy_stream, cudaStreamNonBlocking));
    for (int i = 0; i < kRing; ++i) {
        KV_CUDA_B(cudaMallocHost((void**)&p->h_plan[i], p->plan_bytes));
        KV_CUDA_B(cudaMalloc((void**)&p->d_plan[i], p->plan_bytes));
        KV_CUDA_B(cudaEventCreateWithFlags(&p->copy_done[i], cudaEventDisableTiming));
        KV_CUDA_B(cudaEventCreateWithFlags(&p->slot_free[i], cudaEventDisableTiming));
    }
#undef KV_CUDA_B

    PoolView& pv = p->pv;
    pv.k = (uint8_t*)p->d_k;
    pv.v = (uint8_t*)p->d_v;
    pv.rope = p->d_rope;
    pv.table = p->d_table;
    pv.counters = p->d_counters;
    pv.partials = p->d_partials;
    pv.status = p->d_status;
    pv.num_blocks = num_blocks;
    pv.kv_heads = num_kv_heads;
    pv.q_heads = num_q_heads;
    pv.group = num_q_heads / num_kv_heads;
    pv.max_blocks_per_seq = p->mbps;
    pv.max_seq_len = max_seq_len;
    pv.max_seqs = max_seqs;
    pv.max_items = (int)p->max_items;
    pv.dtype = dtype;
    pv.layer_bytes = layer_bytes;
    pv.tile_bytes = tile_bytes;
    *out = p;
    return KV_OK;
}

int kvp_destroy(kvp_pool* p) {
    if (!p) return KV_OK;
    if (p->host_only) {
        free(p->h_plan[0]);
        delete p;
        return KV_OK;
    }
    {
        DeviceGuard dg(p->device);
        cudaDeviceSynchronize();
        free_device(p);
    }
    delete p;
    return KV_OK;
}

int kvp_reset(kvp_pool* p, void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    if (!p->host_only) {
        const size_t bytes = p->pv.layer_bytes * p->layers;
        KV_CUDA(cudaMemsetAsync(p->d_k, 0, bytes, st));
        KV_CUDA(cudaMemsetAsync(p->d_v, 0, bytes, st));
    }
    for (auto& s : p->seqs) s = Seq();
    p->reset_free_list();
    p->pending.clear();
    p->plan_active = false;
    return KV_OK;
}

int kvp_free_blocks(const kvp_pool* p, int* n) {
    if (!p || !n) return fail(KV_ERR_INVAL, "NULL argument");
    *n = (int)p->free_.size();
    return KV_OK;
}

int kvp_num_blocks(const kvp_pool* p, int* n) {
    if (!p || !n) return fail(KV_ERR_INVAL, "NULL argument");
    *n = p->num_blocks;
    return KV_OK;
}

int kvp_storage(const kvp_pool* p, void** k, void** v, size_t* layer_bytes) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    if (k) *k = p->d_k;
    if (v) *v = p->d_v;
    if (layer_bytes) *layer_bytes = p->pv.layer_bytes;
    return KV_OK;
}

int kvp_launch_info(const kvp_pool* p, int* num_sms, int* ctas_per_sm) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    if (num_sms) *num_sms = p->num_sms;
    if (ctas_per_sm) *ctas_per_sm = p->occupancy;
    return KV_OK;
}

int kvp_seq_alloc(kvp_pool* p, int* seq_id) {
    if (!p || !seq_id) return fail(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(p->mu);
    for (int i = 0; i < p->max_seqs; ++i)
        if (!p->seqs[i].live) {
            p->seqs[i] = Seq();
            p->seqs[i].live = true;
            *seq_id = i;
            return KV_OK;
        }
    return fail(KV_ERR_OOM, "all %d sequence slots are live", p->max_seqs);
}

int kvp_seq_free(kvp_pool* p, int seq) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = check_seq(p, seq);
    if (rc) return rc;
    if (p->plan_active && std::find(p->plan_seqs.begin(), p->plan_seqs.end(), seq) != p->plan_seqs.end())
        return fail(KV_ERR_STATE, "sequence %d is part of the active decode plan", seq);
    Seq& s = p->seqs[seq];
    for (int j = (int)s.blocks.size() - 1; j >= 0; --j) p->push_block(s.blocks[j]);
    // Drop queued table writes for this sequence: its row is dead.
    p->pending.erase(std::remove_if(p->pending.begin(), p->pending.end(),
                                    [seq](const TablePatch& t) { return t.seq == seq; }),
                     p->pending.end());
    s = Seq();
    return KV_OK;
}

int kvp_seq_reserve(kvp_pool* p, int seq, int n_tokens) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = check_seq(p, seq);
    if (rc) return rc;
    if (n_tokens < 0) return fail(KV_ERR_INVAL, "n_tokens < 0");
    if (n_tokens > p->max_seq_len)
        return fail(KV_ERR_RANGE, "n_tokens %d > max_seq_len %d", n_tokens, p->max_seq_len);
    Seq& s = p->seqs[seq];
    const int need = (n_tokens + kBlockTokens - 1) / kBlockTokens - (int)s.blocks.size();
    if (need <= 0) return KV_OK;
    if (need > (int)p->free_.size())
        return fail(KV_ERR_OOM, "need %d blocks, %zu free", need, p->free_.size());
    for (int i = 0; i < need; ++i) {
        const int b = p->pop_block();
        p->pending.push_back(TablePatch{seq, (int)s.blocks.size(), b, 0});
        s.blocks.push_back(b);
    }
    return KV_OK;
}

int kvp_seq_set_blocks(kvp_pool* p, int seq, const int* ids, int n) {
    if (!p || (n > 0 && !ids)) return fail(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = check_seq(p, seq);
    if (rc) return rc;
    if (n < 0) return fail(KV_ERR_INVAL, "n < 0");
    Seq& s = p->seqs[seq];
    if ((long)s.blocks.size() + n > p->mbps)
        return fail(KV_ERR_RANGE, "table would hold %ld blocks > %d", (long)s.blocks.size() + n, p->mbps);
    std::vector<char> seen;
    for (int i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= p->num_blocks) return fail(KV_ERR_INVAL, "block id %d out of range", ids[i]);
        if (p->where_[ids[i]] < 0) return fail(KV_ERR_INVAL, "block %d is not free", ids[i]);
    }
    seen.assign(p->num_blocks, 0);
    for (int i = 0; i < n; ++i) {
        if (seen[ids[i]]) return fail(KV_ERR_INVAL, "block %d listed twice", ids[i]);
        seen[ids[i]] = 1;
    }
    for (int i = 0; i < n; ++i) {
        p->remove_block(ids[i]);
        p->pending.push_back(TablePatch{seq, (int)s.blocks.size(), ids[i], 0});
        s.blocks.push_back(ids[i]);
    }
    return KV_OK;
}

int kvp_seq_len(const kvp_pool* p, int seq, int* len) {
    if (!p || !len) return fail(KV_ERR_INVAL, "NULL argument");
    int rc = check_seq(p, seq);
    if (rc) return rc;
    *len = p->seqs[seq].len;
    return KV_OK;
}

int kvp_seq_set_len(kvp_pool* p, int seq, int len) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = check_seq(p, seq);
    if (rc) return rc;
    Seq& s = p->seqs[seq];
    if (len < 0 || len > (int)s.blocks.size() * kBlockTokens)
        return fail(KV_ERR_RANGE, "length %d outside [0, %zu] reserved", len, s.blocks.size() * kBlockTokens);
    s.len = len;
    return KV_OK;
}

int kvp_seq_blocks(const kvp_pool* p, int seq, int* ids, int cap, int* n_out) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    int rc = check_seq(p, seq);
    if (rc) return rc;
    const Seq& s = p->seqs[seq];
    if (n_out) *n_out = (int)s.blocks.size();
    if (ids) {
        const int n = std::min(cap, (int)s.blocks.size());
        for (int i = 0; i < n; ++i) ids[i] = s.blocks[i];
    }
    return KV_OK;
}

int kvp_import(kvp_pool* p, int layer, int seq, int pos0, int n, const void* k_rows,
               const void* v_rows, void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = check_seq(p, seq);
    if (rc) return rc;
    rc = require_device(p);
    if (rc) return rc;
    if (layer < 0 || layer >= p->layers) return fail(KV_ERR_INVAL, "layer %d out of range", layer);
    if (n < 0 || pos0 < 0) return fail(KV_ERR_INVAL, "negative position/count");
    if ((long)pos0 + n > (long)p->seqs[seq].blocks.size() * kBlockTokens)
        return fail(KV_ERR_RANGE, "positions [%d, %d) exceed reserved blocks", pos0, pos0 + n);
    if (p->dtype == KV_I8) return fail(KV_ERR_INVAL, "INT8 pool: use kvp_import_i8");
    if (n == 0) return KV_OK;
    if (!k_rows || !v_rows || ((uintptr_t)k_rows & 15) || ((uintptr_t)v_rows & 15))
        return fail(KV_ERR_INVAL, "row pointers must be non-NULL and 16-byte aligned");
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    rc = sync_table(p, st);
    if (rc) return rc;
    KV_CUDA(launch_import(p->pv, layer, seq, pos0, n, (const uint16_t*)k_rows, (const uint16_t*)v_rows, st));
    return KV_OK;
}

int kvp_import_i8(kvp_pool* p, int layer, int seq, int pos0, int n, const void* k_codes, const void* v_codes,
                  const float* k_scales, const float* v_scales, void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = check_seq(p, seq);
    if (rc) return rc;
    rc = require_device(p);
    if (rc) return rc;
    if (p->dtype != KV_I8) return fail(KV_ERR_INVAL, "not an INT8 pool");
    if (layer < 0 || layer >= p->layers) return fail(KV_ERR_INVAL, "layer %d out of range", layer);
    if (n < 0 || pos0 < 0) return fail(KV_ERR_INVAL, "negative position/count");
    if ((long)pos0 + n > (long)p->seqs[seq].blocks.size() * kBlockTokens)
        return fail(KV_ERR_RANGE, "positions [%d, %d) exceed reserved blocks", pos0, pos0 + n);
    if (n == 0) return KV_OK;
    if (!k_codes || !v_codes || !k_scales || !v_scales || ((uintptr_t)k_codes & 15) || ((uintptr_t)v_codes & 15) ||
        ((uintptr_t)k_scales & 3) || ((uintptr_t)v_scales & 3))
        return fail(KV_ERR_INVAL, "code pointers must be 16-byte aligned, scale pointers 4-byte aligned");
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    rc = sync_table(p, st);
    if (rc) return rc;
    KV_CUDA(launch_import_i8(p->pv, layer, seq, pos0, n, (const int8_t*)k_codes, (const int8_t*)v_codes, k_scales,
                             v_scales, st));
    return KV_OK;
}

int kvp_gather(kvp_pool* p, int layer, int seq, void* k_rows, void* v_rows, void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = check_seq(p, seq);
    if (rc) return rc;
    rc = require_device(p);
    if (rc) return rc;
    if (layer < 0 || layer >= p->layers) return fail(KV_ERR_INVAL, "layer %d out of range", layer);
    if (p->dtype == KV_I8) return fail(KV_ERR_INVAL, "INT8 pool: use kvp_gather_i8");
    const int len = p->seqs[seq].len;
    if (len == 0) return KV_OK;
    if (!k_rows || !v_rows || ((uintptr_t)k_rows & 15) || ((uintptr_t)v_rows & 15))
        return fail(KV_ERR_INVAL, "row pointers must be non-NULL and 16-byte aligned");
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    rc = sync_table(p, st);
    if (rc) return rc;
    KV_CUDA(launch_gather(p->pv, layer, seq, len, (uint16_t*)k_rows, (uint16_t*)v_rows, st));
    return KV_OK;
}

int kvp_gather_i8(kvp_pool* p, int layer, int seq, void* k_codes, void* v_codes, float* k_scales, float* v_scales,
                  void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = check_seq(p, seq);
    if (rc) return rc;
    rc = require_device(p);
    if (rc) return rc;
    if (p->dtype != KV_I8) return fail(KV_ERR_INVAL, "not an INT8 pool");
    if (layer < 0 || layer >= p->layers) return fail(KV_ERR_INVAL, "layer %d out of range", layer);
    const int len = p->seqs[seq].len;
    if (len == 0) return KV_OK;
    if (!k_codes || !v_codes || !k_scales || !v_scales || ((uintptr_t)k_codes & 15) || ((uintptr_t)v_codes & 15) ||
        ((uintptr_t)k_scales & 3) || ((uintptr_t)v_scales & 3))
        return fail(KV_ERR_INVAL, "code pointers must be 16-byte aligned, scale pointers 4-byte aligned");
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    rc = sync_table(p, st);
    if (rc) return rc;
    KV_CUDA(launch_gather_i8(p->pv, layer, seq, len, (int8_t*)k_codes, (int8_t*)v_codes, k_scales, v_scales, st));
    return KV_OK;
}

namespace {

// One prompt chunk's checks, shared by the append and attention entry
// points (in the order the single-chunk calls report them).
int chunk_check(kvp_pool* p, int layer, int seq, int pos0, int n, bool first) {
    int rc = check_seq(p, seq);
    if (rc) return rc;
    if (first && (rc = require_device(p))) return rc;
    if (layer < 0 || layer >= p->layers) return fail(KV_ERR_INVAL, "layer %d out of range", layer);
    if (n < 0 || pos0 < 0) return fail(KV_ERR_INVAL, "negative position/count");
    if ((long)pos0 + n > p->max_seq_len)
        return fail(KV_ERR_RANGE, "position %ld beyond max_seq_len %d", (long)pos0 + n - 1, p->max_seq_len);
    if ((long)pos0 + n > (long)p->seqs[seq].blocks.size() * kBlockTokens)
        return fail(KV_ERR_RANGE, "positions [%d, %d) exceed reserved blocks", pos0, pos0 + n);
    return KV_OK;
}

// Every chunk of a batch (distinct sequences); *rows = the rows of all chunks.
int batch_check(kvp_pool* p, int layer, int nreq, const int* seqs, const int* pos0, const int* ns, long* rows) {
    if (nreq < 0 || (nreq > 0 && (!seqs || !pos0 || !ns))) return fail(KV_ERR_INVAL, "bad chunk list");
    if (nreq == 0) {
        int rc = require_device(p);
        if (rc) return rc;
    }
    long total = 0;
    for (int i = 0; i < nreq; ++i) {
        int rc = chunk_check(p, layer, seqs[i], pos0[i], ns[i], i == 0);
        if (rc) return rc;
        for (int j = 0; j < i; ++j)
            if (seqs[j] == seqs[i]) return fail(KV_ERR_INVAL, "sequence %d appears twice in one batch", seqs[i]);
        total += ns[i];
    }
    *rows = total;
    return KV_OK;
}

}  // namespace

int kv_append_chunk_batch(kvp_pool* p, int layer, int nreq, const int* seqs, const int* pos0, const int* ns,
                          const float* k, const float* v, void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    long rows = 0;
    int rc = batch_check(p, layer, nreq, seqs, pos0, ns, &rows);
    if (rc || rows == 0) return rc;
    if (!k || !v || ((uintptr_t)k & 7) || ((uintptr_t)v & 7))
        return fail(KV_ERR_INVAL, "k/v must be non-NULL and 8-byte aligned");
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    rc = sync_table(p, st);
    if (rc) return rc;
    const size_t kvw = (size_t)p->kv_heads * kHeadDim;
    long row = 0;
    for (int b0 = 0; b0 < nreq; b0 += kMaxChunkBatch) {
        ChunkBatch cb{};
        const long base = row;
        for (int i = b0; i < std::min(nreq, b0 + kMaxChunkBatch); ++i) {
            cb.seq[cb.nreq] = seqs[i];
            cb.pos0[cb.nreq] = pos0[i];
            cb.row0[cb.nreq] = (int)(row - base);
            ++cb.nreq;
            row += ns[i];
        }
        cb.row0[cb.nreq] = (int)(row - base);
        KV_CUDA(launch_append_batch(p->pv, layer, cb, k + base * kvw, v + base * kvw, st));
    }
    return KV_OK;
}

int kv_append_chunk(kvp_pool* p, int layer, int seq, int pos0, int n, const float* k,
                    const float* v, void* stream) {
    return kv_append_chunk_batch(p, layer, 1, &seq, &pos0, &n, k, v, stream);
}

namespace {

int prefill_part_reserve(kvp_pool* p, size_t need, cudaStream_t st) {
    if (need <= p->prefill_part_floats) return KV_OK;
    KV_CUDA(cudaStreamSynchronize(st));
    cudaFree(p->d_prefill_part);
    p->d_prefill_part = nullptr;
    p->prefill_part_floats = 0;
    KV_CUDA(cudaMalloc((void**)&p->d_prefill_part, need * sizeof(float)));
    p->prefill_part_floats = need;
    return KV_OK;
}

// Shared checks of the single-chunk mma.sync entry point; on success the
// table is on the device.
int prefill_checks(kvp_pool* p, int layer, int seq, int pos0, int n, const float* q, float* out,
                   cudaStream_t st) {
    int rc = chunk_check(p, layer, seq, pos0, n, true);
    if (rc) return rc;
    if (n == 0) return KV_OK;
    if (!q || !out || ((uintptr_t)q & 15) || ((uintptr_t)out & 15))
        return fail(KV_ERR_INVAL, "q and out must be 16-byte aligned");
    return sync_table(p, st);
}

// One chunk on the mma.sync kernel (checked, table on the device): key
// splits for about two CTAs per SM, at least 16 tiles (256 keys) per split.
int prefill_mma_launch(kvp_pool* p, int layer, int seq, int pos0, int n, const float* q, float* out,
                       cudaStream_t st) {
    if (n == 0) return KV_OK;
    const int nqb = (n + 15) / 16;
    const int max_tiles = (pos0 + n - 1) / kBlockTokens + 1;
    const long ctas = (long)nqb * p->kv_heads;
    int nsplit = (int)std::min<long>((2L * p->num_sms + ctas - 1) / ctas, (max_tiles + 15) / 16);
    nsplit = std::max(nsplit, 1);
    const int tps = (max_tiles + nsplit - 1) / nsplit;
    nsplit = (max_tiles + tps - 1) / tps;
    if (nsplit > 1) {
        int rc = prefill_part_reserve(p, (size_t)p->q_heads * nqb * 16 * nsplit * (2 + kHeadDim), st);
        if (rc) return rc;
    }
    KV_CUDA(launch_prefill(p->pv, layer, seq, pos0, n, q, out, p->d_prefill_part, nsplit, tps, st));
    return KV_OK;
}

// Key splits of the chunks of one tcgen05 launch.  Every CTA is resident
// alone on its SM and costs (its key tiles + kFixedTiles), the fixed part
// being the q setup, the first copies and the epilogue (measured ~7.7 us, ~2
// key stages).  For a target of X tiles per CTA (whole stages) chunk i gets
// nsplit_i = ceil(T_i / X) splits; the X kept minimises the makespan
// estimate max(W / SMs, w_max) (+ half a CTA when the grid exceeds one
// wave) plus the merge cost, W being the summed CTA costs.  CTAs are then
// listed longest first.
constexpr double kFixedTiles = 16.0;

struct ChunkPlan {
    int seq, pos0, n, row0, nq, ctas_per_split, T, nsplit, tps;
};

void plan_splits(std::vector<ChunkPlan>& cs, int num_sms, int q_heads) {
    const int st = prefill_tc_stage_tiles();
    int tmax = 0;
    for (const ChunkPlan& c : cs) tmax = std::max(tmax, c.T);
    double best = 1e300;
    int best_x = tmax;
    for (int x = st; x < tmax + st; x += st) {
        double W = 0.0, wmax = 0.0, merge = 0.0;
        long N = 0;
        for (const ChunkPlan& c : cs) {
            int ns = std::min(64, std::max(1, (c.T + x - 1) / x));
            int tps = ((c.T + ns - 1) / ns + st - 1) / st * st;
            ns = (c.T + tps - 1) / tps;
            const double w = tps + kFixedTiles;
            W += (double)c.ctas_per_split * ns * w;
            N += (long)c.ctas_per_split * ns;
            wmax = std::max(wmax, w);
            // partials written and read back (~2.3 MB per tile-time), plus a launch
            if (ns > 1) merge += 8.0 + 2.0 * (double)c.n * q_heads * ns * 528.0 / 2.3e6;
        }
        const double cost = (N <= num_sms ? wmax : std::max(W / num_sms, wmax) + 0.5 * wmax) + merge;
        if (cost < best - 1e-9) {
            best = cost;
            best_x = x;
        }
    }
    for (ChunkPlan& c : cs) {
        int ns = std::min(64, std::max(1, (c.T + best_x - 1) / best_x));
        c.tps = ((c.T + ns - 1) / ns + st - 1) / st * st;
        c.nsplit = (c.T + c.tps - 1) / c.tps;
    }
}

// One tcgen05 launch (+ merge) over chunks [b0, b1) of a checked batch whose
// rows start at row `base`.
int prefill_tc_launch(kvp_pool* p, int layer, const int* seqs, const int* pos0, const int* ns, int b0, int b1,
                      long base, const float* q, float* out, cudaStream_t st) {
    const int tc = prefill_tc_tokens_per_cta(p->q_heads / p->kv_heads);
    std::vector<ChunkPlan> cs;
    long row = 0;
    for (int i = b0; i < b1; ++i) {
        if (ns[i] > 0) {
            ChunkPlan c{};
            c.seq = seqs[i];
            c.pos0 = pos0[i];
            c.n = ns[i];
            c.row0 = (int)row;
            c.nq = (ns[i] + tc - 1) / tc;
            c.ctas_per_split = c.nq * p->kv_heads;
            c.T = (pos0[i] + ns[i] - 1) / kBlockTokens + 1;
            cs.push_back(c);
        }
        row += ns[i];
    }
    if (cs.empty()) return KV_OK;
    plan_splits(cs, p->num_sms, p->q_heads);
    std::stable_sort(cs.begin(), cs.end(), [](const ChunkPlan& a, const ChunkPlan& b) { return a.tps > b.tps; });
    TcBatch tb{};
    int ctas = 0, mrows = 0;
    long long partf = 0;
    for (const ChunkPlan& c : cs) {
        TcReq& r = tb.r[tb.nreq++];
        r.seq = c.seq;
        r.pos0 = c.pos0;
        r.n = c.n;
        r.row0 = c.row0;
        r.nq = c.nq;
        r.nsplit = c.nsplit;
        r.tps = c.tps;
        r.cta0 = ctas;
        r.mrow0 = mrows;
        r.part0 = partf;
        ctas += c.ctas_per_split * c.nsplit;
        if (c.nsplit > 1) {
            mrows += c.n;
            partf += (long long)prefill_tc_part_floats(p->q_heads, c.n, c.nsplit);
        }
    }
    if (partf > 0) {
        int rc = prefill_part_reserve(p, (size_t)partf, st);
        if (rc) return rc;
    }
    const size_t qw = (size_t)p->q_heads * kHeadDim;
    KV_CUDA(launch_prefill_tc(p->pv, layer, tb, ctas, mrows, q + base * qw, out + base * qw, p->d_prefill_part,
                              st));
    return KV_OK;
}

}  // namespace

// Tensor-core (tcgen05) version over several chunks: one launch (plus one
// merge launch when a chunk is split) per kMaxChunkBatch chunks.  An INT8
// pool runs each chunk on the mma.sync kernel (codes expanded to fp16 in
// shared memory, scales applied to scores and weights).
int attn_prefill_batch(kvp_pool* p, int layer, int nreq, const int* seqs, const int* pos0, const int* ns,
                       const float* q, float* out, void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    long rows = 0;
    int rc = batch_check(p, layer, nreq, seqs, pos0, ns, &rows);
    if (rc) return rc;
    if (rows == 0) return KV_OK;
    if (!q || !out || ((uintptr_t)q & 15) || ((uintptr_t)out & 15))
        return fail(KV_ERR_INVAL, "q and out must be 16-byte aligned");
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    rc = sync_table(p, st);
    if (rc) return rc;
    long base = 0;
    if (p->dtype == KV_I8) {
        const size_t qw = (size_t)p->q_heads * kHeadDim;
        for (int i = 0; i < nreq; ++i) {
            rc = prefill_mma_launch(p, layer, seqs[i], pos0[i], ns[i], q + base * qw, out + base * qw, st);
            if (rc) return rc;
            base += ns[i];
        }
        return KV_OK;
    }
    for (int b0 = 0; b0 < nreq; b0 += kMaxChunkBatch) {
        const int b1 = std::min(nreq, b0 + kMaxChunkBatch);
        rc = prefill_tc_launch(p, layer, seqs, pos0, ns, b0, b1, base, q, out, st);
        if (rc) return rc;
        for (int i = b0; i < b1; ++i) base += ns[i];
    }
    return KV_OK;
}

int attn_prefill(kvp_pool* p, int layer, int seq, int pos0, int n, const float* q, float* out,
                 void* stream) {
    return attn_prefill_batch(p, layer, 1, &seq, &pos0, &n, q, out, stream);
}

// The same on mma.sync (the baseline the tensor-core version is measured against).
int attn_prefill_mma(kvp_pool* p, int layer, int seq, int pos0, int n, const float* q, float* out,
                     void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    int rc = prefill_checks(p, layer, seq, pos0, n, q, out, st);
    if (rc || n == 0) return rc;
    return prefill_mma_launch(p, layer, seq, pos0, n, q, out, st);
}

int attn_decode_plan_ex(kvp_pool* p, int nseq, const int* seq_ids, const int* rope_pos,
                        const int* append, void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (nseq < 1 || nseq > p->max_seqs) return fail(KV_ERR_INVAL, "nseq %d outside [1, %d]", nseq, p->max_seqs);
    if (!seq_ids) return fail(KV_ERR_INVAL, "seq_ids is NULL");
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;

    // ---- validate everything before changing anything ----
    std::vector<char> seen(p->max_seqs, 0);
    int new_blocks = 0;
    for (int i = 0; i < nseq; ++i) {
        const int sid = seq_ids[i];
        int rc = check_seq(p, sid);
        if (rc) return rc;
        if (seen[sid]) return fail(KV_ERR_INVAL, "sequence %d listed twice", sid);
        seen[sid] = 1;
        const Seq& s = p->seqs[sid];
        const int app = append ? (append[i] != 0) : 1;
        const int rp = rope_pos ? rope_pos[i] : s.len;
        if (rp < 0 || rp >= p->max_seq_len)
            return fail(KV_ERR_RANGE, "rope position %d outside [0, %d)", rp, p->max_seq_len);
        const int kv_len = s.len + app;
        if (kv_len > p->mbps * kBlockTokens || kv_len > p->max_seq_len)
            return fail(KV_ERR_RANGE, "sequence %d would reach %d tokens > max_seq_len %d", sid, kv_len, p->max_seq_len);
        if (app && s.len / kBlockTokens >= (int)s.blocks.size()) ++new_blocks;
    }
    if (new_blocks > (int)p->free_.size())
        return fail(KV_ERR_OOM, "decode step needs %d new blocks, %zu free", new_blocks, p->free_.size());

    // A plan that never reached a layer call still owes its table entries.
    if (p->plan_active && !p->plan_patched && p->plan_npatch > 0 && !p->host_only) {
        const int r0 = p->plan_slot_ring;
        KV_CUDA(cudaStreamWaitEvent(st, p->copy_done[r0], 0));
        KV_CUDA(launch_patch(p->pv, p->plan_view.patches, p->plan_npatch, st));
        KV_CUDA(cudaEventRecord(p->slot_free[r0], st));
        p->plan_patched = true;
    }
    int rc = flush_pending(p, st);
    if (rc) return rc;

    // ---- slots (and the blocks new tokens start) ----
    const int r = p->host_only ? 0 : p->ring_next;
    p->ring_next = (r + 1) % kRing;
    if (!p->host_only) KV_CUDA(cudaEventSynchronize(p->copy_done[r]));  // host buffer reusable
    uint8_t* h = p->h_plan[r];
    std::vector<DecodeSlot> slots(nseq);
    std::vector<TablePatch> patches;
    p->plan_seqs.assign(seq_ids, seq_ids + nseq);
    p->plan_append.resize(nseq);
    long total_blocks = 0;
    int nsegments = 0;
    for (int i = 0; i < nseq; ++i) {
        const int sid = seq_ids[i];
        Seq& s = p->seqs[sid];
        const int app = append ? (append[i] != 0) : 1;
        DecodeSlot& sl = slots[i];
        sl = DecodeSlot{};
        sl.seq = sid;
        sl.kv_len = s.len + app;
        sl.rope_pos = rope_pos ? rope_pos[i] : s.len;
        sl.append = app;
        sl.new_block = -1;
        if (app) {
            const int idx = s.len / kBlockTokens;
            if (idx >= (int)s.blocks.size()) {
                const int b = p->pop_block();
                s.blocks.push_back(b);
                patches.push_back(TablePatch{sid, idx, b, 0});
            }
            sl.new_block = s.blocks[idx];
        }
        p->plan_append[i] = app;
        total_blocks += (long)p->kv_heads * ((sl.kv_len + kBlockTokens - 1) / kBlockTokens);
        nsegments += p->kv_heads;
    }

    // ---- pieces: each CTA gets one contiguous, equal run of the flattened
    // (slot, kv head, block) sequence; a segment crossing a CTA boundary is
    // cut into pieces whose partial results are merged on the device ----
    // Cost model: a piece costs its blocks plus kPieceCost block-equivalents
    // (warp merge, q reload, partial write), so CTAs holding two pieces take
    // fewer blocks and every CTA finishes at about the same time.
    constexpr long kPieceCost = 6;
    const long gmax = std::max(1L, (long)p->num_sms * p->occupancy);
    // At least 16 blocks per CTA: below that, a split costs more (a merge
    // launch) than the blocks it moves to another SM.
    const long G = std::min(gmax, std::max(1L, (total_blocks + 15) / 16));
    const long per = std::max(kPieceCost + 1,
                              (total_blocks + kPieceCost * (nsegments + G - 1) + G - 1) / G);
    std::vector<WorkItem> items;
    std::vector<int> cta_start(1, 0);
    long fill = 0;
    int cta_items = 0;
    auto piece = [&](int i, int hd, int b0, int b1, int seg_first) {
        const DecodeSlot& sl = slots[i];
        return WorkItem{i, hd, b0, b1, seg_first, 1, sl.seq, sl.kv_len, sl.rope_pos, sl.append,
                        sl.new_block, 0};
    };
    auto close_cta = [&]() {
        cta_start.push_back((int)items.size());
        fill = 0;
        cta_items = 0;
    };
    for (int i = 0; i < nseq; ++i) {
        const int nblk = (slots[i].kv_len + kBlockTokens - 1) / kBlockTokens;
        for (int hd = 0; hd < p->kv_heads; ++hd) {
            const int seg_first = (int)items.size();
            if (nblk == 0) {  // nothing to attend: one empty piece still writes the (zero) result
                if (fill + kPieceCost > per || cta_items == kMaxCtaItems) close_cta();
                items.push_back(piece(i, hd, 0, 0, seg_first));
                fill += kPieceCost;
                ++cta_items;
                continue;
            }
            int b = 0;
            while (b < nblk) {
                if (fill + kPieceCost >= per || cta_items == kMaxCtaItems) close_cta();
                fill += kPieceCost;
                const int take = (int)std::min<long>(nblk - b, per - fill);
                items.push_back(piece(i, hd, b, b + take, seg_first));
                b += take;
                fill += take;
                ++cta_items;
            }
            const int seg_n = (int)items.size() - seg_first;
            for (int x = seg_first; x < (int)items.size(); ++x) items[x].seg_n = seg_n;
        }
    }
    close_cta();
    const int grid = (int)cta_start.size() - 1;
    if ((long)items.size() > p->max_items || grid > p->max_items)
        return fail(KV_ERR_STATE, "work list overflow (%zu items, %d CTAs)", items.size(), grid);

    // ---- per-CTA descriptors and the flat tile list (the host owns the
    // block tables, so the kernel needs no table reads to start copying) ----
    std::vector<CtaDesc> ctas(grid);
    std::vector<int> tiles;
    tiles.reserve((size_t)total_blocks);
    for (int gi = 0; gi < grid; ++gi) {
        ctas[gi] = CtaDesc{cta_start[gi], cta_start[gi + 1] - cta_start[gi], (int)tiles.size(), 0,
                           {-2, -2, -2, -2, -2, -2, -2, -2}};
        for (int x = cta_start[gi]; x < cta_start[gi + 1]; ++x) {
            const WorkItem& w = items[x];
            const Seq& sq = p->seqs[w.seq];
            const int last = (w.kv_len - 1) / kBlockTokens;
            for (int b = w.b0; b < w.b1; ++b) {
                const bool newblk = w.append && b == last;
                const int valid = std::min(kBlockTokens, w.kv_len - b * kBlockTokens);
                const int blk = newblk ? w.new_block : sq.blocks[b];
                tiles.push_back(newblk && valid == 1 ? -1 : blk * p->kv_heads + w.head);
            }
        }
        ctas[gi].nf = (int)tiles.size() - ctas[gi].f0;
        for (int x = 0; x < 8 && x < ctas[gi].nf; ++x) ctas[gi].first[x] = tiles[ctas[gi].f0 + x];
    }
    if ((long)tiles.size() > p->max_tiles)
        return fail(KV_ERR_STATE, "tile list overflow (%zu > %ld)", tiles.size(), p->max_tiles);
    std::vector<SplitSeg> splits;
    for (size_t x = 0; x < items.size(); ++x)
        if (items[x].seg_n > 1 && (int)x == items[x].seg_first)
            splits.push_back(SplitSeg{items[x].slot, items[x].head, items[x].seg_first, items[x].seg_n});

    // ---- pack and upload once, on the copy stream ----
    const PlanLayout L = plan_layout(nseq, (long)items.size(), (int)patches.size(), grid, (long)tiles.size(),
                                     (long)splits.size());
    PlanHeader* hdr = (PlanHeader*)h;
    hdr->nslots = nseq;
    hdr->nitems = (int)items.size();
    hdr->npatch = (int)patches.size();
    hdr->grid = grid;
    hdr->off_slots = (int)L.slots;
    hdr->off_items = (int)L.items;
    hdr->off_patches = (int)L.patches;
    hdr->off_cta = (int)L.cta;
    hdr->off_tiles = (int)L.tiles;
    hdr->ntiles = (int)tiles.size();
    hdr->off_splits = (int)L.splits;
    hdr->nsplits = (int)splits.size();
    memcpy(h + L.slots, slots.data(), slots.size() * sizeof(DecodeSlot));
    memcpy(h + L.items, items.data(), items.size() * sizeof(WorkItem));
    if (!patches.empty()) memcpy(h + L.patches, patches.data(), patches.size() * sizeof(TablePatch));
    memcpy(h + L.cta, ctas.data(), ctas.size() * sizeof(CtaDesc));
    if (!tiles.empty()) memcpy(h + L.tiles, tiles.data(), tiles.size() * sizeof(int));
    if (!splits.empty()) memcpy(h + L.splits, splits.data(), splits.size() * sizeof(SplitSeg));

    p->plan_active = true;
    p->plan_patched = patches.empty();
    p->plan_slot_ring = r;
    p->plan_nslots = nseq;
    p->plan_nitems = (int)items.size();
    p->plan_npatch = (int)patches.size();
    p->plan_grid = grid;
    const uint8_t* base = p->host_only ? h : p->d_plan[r];
    p->plan_view.hdr = (const PlanHeader*)base;
    p->plan_view.slots = (const DecodeSlot*)(base + L.slots);
    p->plan_view.items = (const WorkItem*)(base + L.items);
    p->plan_view.patches = (const TablePatch*)(base + L.patches);
    p->plan_view.cta = (const CtaDesc*)(base + L.cta);
    p->plan_view.tiles = (const int*)(base + L.tiles);
    p->plan_view.splits = (const SplitSeg*)(base + L.splits);
    p->plan_nsplits = (int)splits.size();
    p->plan_max_pieces = 0;
    for (const SplitSeg& sg : splits) p->plan_max_pieces = std::max(p->plan_max_pieces, sg.seg_n);
    p->plan_stream = st;
    if (p->host_only) {
        p->plan_patched = true;
        return KV_OK;
    }
    // The previous launches that read ring slot r must be done before the
    // copy overwrites it; the copy itself overlaps whatever runs now.
    KV_CUDA(cudaStreamWaitEvent(p->copy_stream, p->slot_free[r], 0));
    KV_CUDA(cudaMemcpyAsync(p->d_plan[r], h, L.bytes, cudaMemcpyHostToDevice, p->copy_stream));
    KV_CUDA(cudaEventRecord(p->copy_done[r], p->copy_stream));
    return KV_OK;
}

int kvp_plan_info(const kvp_pool* p, int* nitems, int* grid, int* npatch, int* item_slot,
                  int* item_head, int* item_b0, int* item_b1, int cap) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    const uint8_t* h = p->h_plan[p->plan_slot_ring];
    const PlanHeader* hdr = (const PlanHeader*)h;
    const WorkItem* items = (const WorkItem*)(h + hdr->off_items);
    if (nitems) *nitems = hdr->nitems;
    if (grid) *grid = hdr->grid;
    if (npatch) *npatch = hdr->npatch;
    const int n = std::min(cap, hdr->nitems);
    for (int i = 0; i < n; ++i) {
        if (item_slot) item_slot[i] = items[i].slot;
        if (item_head) item_head[i] = items[i].head;
        if (item_b0) item_b0[i] = items[i].b0;
        if (item_b1) item_b1[i] = items[i].b1;
    }
    return KV_OK;
}

int kvp_plan_cta_start(const kvp_pool* p, int* cta_start, int cap) {
    if (!p || !cta_start) return fail(KV_ERR_INVAL, "NULL argument");
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    const uint8_t* h = p->h_plan[p->plan_slot_ring];
    const PlanHeader* hdr = (const PlanHeader*)h;
    const CtaDesc* cs = (const CtaDesc*)(h + hdr->off_cta);
    const int n = std::min(cap, hdr->grid + 1);
    for (int i = 0; i < n; ++i) cta_start[i] = i < hdr->grid ? cs[i].i0 : hdr->nitems;
    return KV_OK;
}

int attn_decode_plan(kvp_pool* p, int nseq, const int* seq_ids, void* stream) {
    return attn_decode_plan_ex(p, nseq, seq_ids, nullptr, nullptr, stream);
}

static int decode_call(kvp_pool* p, int layer, const float* q, const float* k_new, const float* v_new,
                       float* out, float* m, float* l, void* stream, kvx_exch* x = nullptr,
                       float* x_out = nullptr) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    if (int rc = require_device(p)) return rc;
    if (layer < 0 || layer >= p->layers) return fail(KV_ERR_INVAL, "layer %d out of range", layer);
    if (!q || !k_new || !v_new || !out) return fail(KV_ERR_INVAL, "NULL tensor");
    if (((uintptr_t)q | (uintptr_t)k_new | (uintptr_t)v_new) & 7)
        return fail(KV_ERR_INVAL, "q/k_new/v_new must be 8-byte aligned");
    XchgArgs xa;
    if (x) {
        // the local states go to this rank's slot of the exchange area
        if (int rc = xchg_prepare(x, p->device, p->plan_nslots * p->q_heads, p->pv.status, x_out, &xa,
                                  &m, &l, &out))
            return rc;
    }
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    const int r = p->plan_slot_ring;
    KV_CUDA(cudaStreamWaitEvent(st, p->copy_done[r], 0));
    std::pair<cudaEvent_t, cudaEvent_t>* te = nullptr;
    if (p->timing) {
        if (p->tev_used == p->tev.size()) {
            cudaEvent_t a, b;
            KV_CUDA(cudaEventCreate(&a));
            KV_CUDA(cudaEventCreate(&b));
            p->tev.emplace_back(a, b);
        }
        te = &p->tev[p->tev_used++];
        KV_CUDA(cudaEventRecord(te->first, st));
    }
    KV_CUDA(launch_decode(p->pv, p->plan_view, p->plan_nsplits, p->plan_max_pieces, layer, q, k_new,
                          v_new, out, m, l, p->plan_grid, p->overlap && !te, st));
    if (x) {
        KV_CUDA(launch_xchg(xa, st));
        xchg_commit(x);
    }
    if (te) KV_CUDA(cudaEventRecord(te->second, st));
    KV_CUDA(cudaEventRecord(p->slot_free[r], st));
    p->plan_patched = true;
    return KV_OK;
}

int kvp_set_overlap(kvp_pool* p, int enable) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (int rc = require_device(p)) return rc;
    p->overlap = enable != 0;
    return KV_OK;
}

int kvp_timing_enable(kvp_pool* p, int enable) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (int rc = require_device(p)) return rc;
    p->timing = enable != 0;
    p->tev_used = 0;
    return KV_OK;
}

int kvp_timing_read(kvp_pool* p, double* total_ms, int* launches) {
    if (!p || !total_ms || !launches) return fail(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(p->mu);
    if (int rc = require_device(p)) return rc;
    DeviceGuard dg(p->device);
    double tot = 0.0;
    for (size_t i = 0; i < p->tev_used; ++i) {
        KV_CUDA(cudaEventSynchronize(p->tev[i].second));
        float ms = 0.f;
        KV_CUDA(cudaEventElapsedTime(&ms, p->tev[i].first, p->tev[i].second));
        tot += ms;
    }
    *total_ms = tot;
    *launches = (int)p->tev_used;
    p->tev_used = 0;
    return KV_OK;
}

int attn_decode_append(kvp_pool* p, int layer, const float* q, const float* k_new,
                       const float* v_new, float* out, void* stream) {
    return decode_call(p, layer, q, k_new, v_new, out, nullptr, nullptr, stream);
}

int attn_decode_append_partial(kvp_pool* p, int layer, const float* q, const float* k_new,
                               const float* v_new, float* out, float* m, float* l, void* stream) {
    if (!m || !l) return fail(KV_ERR_INVAL, "m and l are required");
    return decode_call(p, layer, q, k_new, v_new, out, m, l, stream);
}

int attn_decode_append_xgpu(kvp_pool* p, int layer, const float* q, const float* k_new,
                            const float* v_new, float* out, kvx_exch* x, void* stream) {
    if (!x || !out) return fail(KV_ERR_INVAL, "NULL argument");
    float* dummy = out;  // replaced by the exchange slot inside decode_call
    return decode_call(p, layer, q, k_new, v_new, dummy, dummy, dummy, stream, x, out);
}

int attn_decode_commit(kvp_pool* p) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    if (!p->plan_patched && p->plan_npatch > 0 && !p->host_only) {
        DeviceGuard dg(p->device);
        const int r = p->plan_slot_ring;
        KV_CUDA(cudaStreamWaitEvent(p->plan_stream, p->copy_done[r], 0));
        KV_CUDA(launch_patch(p->pv, p->plan_view.patches, p->plan_npatch, p->plan_stream));
        KV_CUDA(cudaEventRecord(p->slot_free[r], p->plan_stream));
    }
    for (size_t i = 0; i < p->plan_seqs.size(); ++i)
        if (p->plan_append[i]) p->seqs[p->plan_seqs[i]].len += 1;
    p->plan_active = false;
    return KV_OK;
}


int attn_combine_lse(int G, int rows, int dim, const float* m, const float* l, const float* o,
                     float* out, void* stream) {
    if (G < 1 || rows < 0 || dim < 1) return fail(KV_ERR_INVAL, "bad sizes");
    if (rows == 0) return KV_OK;
    if (!m || !l || !o || !out) return fail(KV_ERR_INVAL, "NULL tensor");
    KV_CUDA(launch_combine(G, rows, dim, m, l, o, (size_t)rows, (size_t)rows * dim, out,
                           (cudaStream_t)stream));
    return KV_OK;
}

int attn_combine_lse_packed(int G, int rows, int dim, const float* packed, float* out, void* stream) {
    if (G < 1 || rows < 0 || dim < 1) return fail(KV_ERR_INVAL, "bad sizes");
    if (rows == 0) return KV_OK;
    if (!packed || !out) return fail(KV_ERR_INVAL, "NULL tensor");
    const size_t per = (size_t)rows * (2 + dim);
    KV_CUDA(launch_combine(G, rows, dim, packed, packed + rows, packed + 2 * (size_t)rows, per, per,
                           out, (cudaStream_t)stream));
    return KV_OK;
}

int kvp_device_status(kvp_pool* p, void* stream, int* status) {
    if (!p || !status) return fail(KV_ERR_INVAL, "NULL argument");
    if (int rc = require_device(p)) return rc;
    DeviceGuard dg(p->device);
    int v[32] = {0};
    KV_CUDA(cudaMemcpyAsync(v, p->d_status, sizeof v, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    KV_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    KV_CUDA(cudaMemsetAsync(p->d_status, 0, sizeof v, (cudaStream_t)stream));
    *status = v[0];
    if (v[0] == KV_ERR_TIMEOUT)
        fail(v[0], "device wait gave up: item %d role %d block %d warp %d stage %d round %d "
                   "full=%08x%08x empty=%08x%08x issued=%d released=%d,%d,%d,%d",
             v[1], v[2], v[3], v[4], v[5], v[6], v[8], v[7], v[10], v[9], v[11], v[12], v[13],
             v[14], v[15]);
    else if (v[0] != 0)
        fail(v[0], "device status %d at item %d (detail %d)", v[0], v[1], v[2]);
    return KV_OK;
}

}  // extern "C"
