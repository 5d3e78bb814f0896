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

struct Seq {
    bool live = false;
    int len = 0;
    std::vector<int> blocks;
    long long app_serial = -1;  // decode launch that last appended to this sequence
    int app_pos = -1;           // the position it wrote
};

// One decode launch's share of a plan (at most kSlotsLarge sequences): the
// kernel parameters of its launches.
struct SubPlan {
    int row0 = 0, nslots = 0, grid = 0, total = 0, max_pieces = 0;
    int cluster = 1;                     // 1: grid-wide merge; kClusterCtas: merge inside clusters
    std::vector<DecodeSlot> slots;
    std::vector<int> seg;                // slot | KV head << 16, in flat order
    std::vector<int> seg_nb;             // blocks of each segment
    std::vector<int> seg_f0;             // nsegs + 1
    std::vector<int> cta_f0;             // grid + 1
    std::vector<int2> comb;              // split segments (CombineArgs::seg)
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
    int clusters = 0;      // merge clusters (kClusterCtas decode CTAs) resident at once; 0: none
    int merge_mode = KVP_MERGE_GRID;  // kvp_set_merge_mode
    bool overlap = false;  // decode launches may copy their first tiles early (kvp_set_overlap)
    PoolView pv{};

    // device allocations
    void* d_k = nullptr;
    void* d_v = nullptr;
    float2* d_rope = nullptr;
    int* d_table = nullptr;
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

    // active plan
    bool plan_active = false;
    bool plan_patched = false;           // its new blocks are in the device table (or queued)
    std::vector<SubPlan> subs;
    std::vector<TablePatch> plan_patches;  // the plan's new blocks
    std::vector<int> plan_seqs;
    std::vector<int> plan_append;
    std::vector<DecodeSlot> plan_slots;
    std::vector<unsigned> seen;   // duplicate check of a plan's ids (stamp per plan)
    unsigned seen_stamp = 0;
    cudaStream_t plan_stream = nullptr;

    // What the previous decode launch may still be writing when the next one
    // starts early (see decode_call).
    long long launch_serial = 0;  // decode launches made
    int last_layer = -1;          // layer of the previous decode launch
    bool last_patched = false;    // the previous decode launch wrote table entries
    bool dirty = true;            // another pool-writing kernel ran since the previous decode launch

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

const float2* kvattn::pool_rope_table(const kvp_pool* p) { return p ? p->d_rope : nullptr; }

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
    p->dirty = true;
    return KV_OK;
}

// A plan whose new blocks no decode launch has entered in the device table
// yet (it may never get one): queue them like reserved blocks.
void queue_plan_patches(kvp_pool* p) {
    if (p->plan_active && !p->plan_patched) {
        p->pending.insert(p->pending.end(), p->plan_patches.begin(), p->plan_patches.end());
        p->plan_patched = true;
    }
}

// Make the device block table current: queued patches and, if no layer call
// applied them yet, the active plan's new-block patches.
int sync_table(kvp_pool* p, cudaStream_t st) {
    queue_plan_patches(p);
    return flush_pending(p, st);
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

void free_device(kvp_pool* p) {
    cudaFree(p->d_k);
    cudaFree(p->d_v);
    cudaFree(p->d_rope);
    cudaFree(p->d_table);
    cudaFree(p->d_partials);
    cudaFree(p->d_prefill_part);
    cudaFree(p->d_status);
    cudaFree(p->d_pending);
    cudaFreeHost(p->h_pending);
    if (p->pending_evt) cudaEventDestroy(p->pending_evt);
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
        // Bookkeeping only: plans are built for a nominal 148-SM part (two
        // decode CTAs per SM) and kept on the host.
        p->num_sms = 148;
        p->occupancy = 2;
        p->clusters = 148 * 2 / kClusterCtas;
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
    KV_CUDA_B(decode_occupancy(dtype, &p->occupancy, &p->clusters));
    if (p->occupancy < 1) p->occupancy = 1;

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
    KV_CUDA_B(cudaMalloc((void**)&p->d_partials, (size_t)2 * kMaxGrid * kPartialFloats * sizeof(float)));
    KV_CUDA_B(cudaMalloc((void**)&p->d_status, 32 * sizeof(int)));
    KV_CUDA_B(cudaMemset(p->d_status, 0, 32 * sizeof(int)));
    KV_CUDA_B(cudaEventCreateWithFlags(&p->pending_evt, cudaEventDisableTiming));
#undef KV_CUDA_B

    PoolView& pv = p->pv;
    pv.k = (uint8_t*)p->d_k;
    pv.v = (uint8_t*)p->d_v;
    pv.rope = p->d_rope;
    pv.table = p->d_table;
    pv.partials = p->d_partials;
    pv.status = p->d_status;
    pv.num_blocks = num_blocks;
    pv.kv_heads = num_kv_heads;
    pv.q_heads = num_q_heads;
    pv.group = num_q_heads / num_kv_heads;
    pv.max_blocks_per_seq = p->mbps;
    pv.max_seq_len = max_seq_len;
    pv.max_seqs = max_seqs;
    pv.dtype = dtype;
    pv.layer_bytes = layer_bytes;
    pv.tile_bytes = tile_bytes;
    *out = p;
    return KV_OK;
}

int kvp_destroy(kvp_pool* p) {
    if (!p) return KV_OK;
    if (p->host_only) {
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
    p->dirty = true;
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
    p->dirty = true;
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
    p->dirty = true;
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
    p->dirty = true;
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

}  // extern "C"

namespace {

// Block-equivalents a piece costs beyond its blocks (q fragments, the warp
// merge, the partial write); 8 measured best for 32 sequences of
// U[256,4096] tokens (6: 18.2, 8-10: 18.0, 12: 18.3, 3: 18.9 us per step).
constexpr long kPieceCost = 8;

// Work partition of one sub-plan whose slots are filled.  Segments (slot,
// KV head) with blocks are listed slot-major; every CTA gets one contiguous
// run of the flat block sequence of about equal cost, a piece costing its
// blocks plus kPieceCost block-equivalents (warp merge, q reload, partial
// write), so CTAs holding two pieces take fewer blocks and every CTA
// finishes at about the same time.  A segment crossing a CTA boundary
// becomes pieces merged by the combine kernel.  Returns the cost per CTA.
long partition_grid(const kvp_pool* p, SubPlan& sp) {
    const int nseg = (int)sp.seg.size();
    long T = 0;
    sp.seg_f0.resize(nseg + 1);
    for (int k = 0; k < nseg; ++k) {
        sp.seg_f0[k] = (int)T;
        T += sp.seg_nb[k];
    }
    sp.seg_f0[nseg] = (int)T;
    sp.total = (int)T;
    sp.cluster = 1;
    const long gmax = std::max(1L, std::min<long>(kMaxGrid, (long)p->num_sms * p->occupancy));
    // At least 16 blocks per CTA: below that, a split costs more (a merge)
    // than the blocks it moves to another SM.
    const long G = std::min(gmax, std::max(1L, (T + 15) / 16));
    long per = std::max(kPieceCost + 1, (T + kPieceCost * (nseg + G - 1) + G - 1) / G);
    for (;;) {
        sp.cta_f0.resize(1);
        sp.cta_f0[0] = 0;
        sp.comb.clear();
        sp.max_pieces = 0;
        long fill = 0;
        int cta_items = 0;
        for (int k = 0; k < nseg; ++k) {
            const int nb = sp.seg_nb[k];
            const long F = sp.seg_f0[k];
            int b = 0, pieces = 0, first = 0;
            while (b < nb) {
                if (cta_items > 0 && (fill + kPieceCost >= per || cta_items == kMaxCtaItems)) {
                    sp.cta_f0.push_back((int)(F + b));
                    fill = 0;
                    cta_items = 0;
                }
                // A split segment's first piece is its CTA's first (partial
                // 2g) or last (2g + 1) piece; every later one is a first.
                if (pieces == 0) first = 2 * ((int)sp.cta_f0.size() - 1) + (cta_items == 0 ? 0 : 1);
                fill += kPieceCost;
                const int take = (int)std::min<long>(nb - b, std::max(1L, per - fill));
                b += take;
                fill += take;
                ++cta_items;
                ++pieces;
            }
            if (pieces > 1) {
                sp.comb.push_back(make_int2(sp.seg[k], first | (pieces << 16)));
                sp.max_pieces = std::max(sp.max_pieces, pieces);
            }
        }
        sp.cta_f0.push_back((int)T);
        if ((int)sp.cta_f0.size() - 1 <= kMaxGrid) break;
        per += per / 4 + 1;  // too many CTAs (the piece cap): coarser runs
    }
    sp.grid = (int)sp.cta_f0.size() - 1;
    return per;
}

// The same step with split segments merged inside thread-block clusters:
// segments are packed onto K clusters of kClusterCtas CTAs (longest first,
// each onto the least loaded cluster), so no segment leaves its cluster;
// each cluster's run is then cut into kClusterCtas equal-cost CTA ranges as
// above.  Taken when the most loaded cluster's CTAs carry at most about the
// grid-wide cost per CTA (`per`) plus what the combine launch costs; the plan
// is left unchanged otherwise.
bool partition_clusters(const kvp_pool* p, SubPlan& sp, long per) {
    constexpr int Cn = kClusterCtas;
    const int nseg = (int)sp.seg.size();
    const long T = sp.total;
    const long gmax = std::max(1L, std::min<long>(kMaxGrid, (long)p->num_sms * p->occupancy));
    const long G = std::min(gmax, std::max(1L, (T + 15) / 16));
    const int K = (int)std::min<long>({(long)p->clusters, kMaxGrid / Cn, (G + Cn - 1) / Cn, (long)nseg});
    if (K < 1) return false;
    std::vector<int> order(nseg);
    for (int k = 0; k < nseg; ++k) order[k] = k;
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return sp.seg_nb[x] > sp.seg_nb[y]; });
    std::vector<long> load(K, 0);
    std::vector<int> owner(nseg);
    std::vector<int> count(K, 0);
    for (int k : order) {
        int j = 0;
        for (int c = 1; c < K; ++c)
            if (load[c] < load[j]) j = c;
        owner[k] = j;
        load[j] += sp.seg_nb[k] + kPieceCost;
        ++count[j];
    }
    long worst = 0;
    for (int j = 0; j < K; ++j) worst = std::max(worst, (load[j] + kPieceCost * (Cn - 1) + Cn - 1) / Cn);
    if (worst > per + per / 10 + 4) return false;
    // Flat order: cluster by cluster, slot-major inside a cluster.
    std::vector<int> seg(nseg), nbs(nseg), start(K + 1, 0);
    for (int j = 0; j < K; ++j) start[j + 1] = start[j] + count[j];
    std::vector<int> pos(start.begin(), start.end() - 1);
    for (int k = 0; k < nseg; ++k) {
        const int at = pos[owner[k]]++;
        seg[at] = sp.seg[k];
        nbs[at] = sp.seg_nb[k];
    }
    std::vector<int> f0(nseg + 1), cta(1, 0);
    long F = 0;
    for (int k = 0; k < nseg; ++k) {
        f0[k] = (int)F;
        F += nbs[k];
    }
    f0[nseg] = (int)F;
    for (int j = 0; j < K; ++j) {
        const long len = (long)f0[start[j + 1]] - f0[start[j]];
        const long pj = std::max(kPieceCost + 1, (len + kPieceCost * (count[j] + Cn - 1) + Cn - 1) / Cn);
        int used = 1;  // CTAs of this cluster begun
        long fill = 0;
        int cta_items = 0;
        for (int k = start[j]; k < start[j + 1]; ++k) {
            int b = 0;
            while (b < nbs[k]) {
                if (cta_items > 0 && used < Cn && (fill + kPieceCost >= pj || cta_items == kMaxCtaItems)) {
                    cta.push_back(f0[k] + b);
                    ++used;
                    fill = 0;
                    cta_items = 0;
                }
                if (cta_items == kMaxCtaItems) return false;  // the last CTA would hold too many pieces
                fill += kPieceCost;
                const int take = used < Cn ? (int)std::min<long>(nbs[k] - b, std::max(1L, pj - fill)) : nbs[k] - b;
                b += take;
                fill += take;
                ++cta_items;
            }
        }
        // CTAs of the cluster left without blocks get empty ranges; the
        // cluster's end is the next cluster's first CTA start (or the end).
        for (; used < Cn; ++used) cta.push_back(f0[start[j + 1]]);
        cta.push_back(f0[start[j + 1]]);
    }
    sp.seg.swap(seg);
    sp.seg_nb.swap(nbs);
    sp.seg_f0.swap(f0);
    sp.cta_f0.swap(cta);
    sp.grid = K * Cn;
    sp.cluster = Cn;
    sp.comb.clear();
    sp.max_pieces = 0;
    return true;
}

void partition(const kvp_pool* p, SubPlan& sp) {
    const int kvh = p->kv_heads;
    sp.seg.clear();
    sp.seg_nb.clear();
    for (int i = 0; i < sp.nslots; ++i) {
        const int nb = (sp.slots[i].kv_len + kBlockTokens - 1) / kBlockTokens;
        for (int h = 0; nb > 0 && h < kvh; ++h) {
            sp.seg.push_back(i | (h << 16));
            sp.seg_nb.push_back(nb);
        }
    }
    const long per = partition_grid(p, sp);
    if (!sp.comb.empty() && p->merge_mode == KVP_MERGE_CLUSTER && p->clusters > 0) partition_clusters(p, sp, per);
}

// The pieces of CTA g of a sub-plan, derived from its flat range exactly as
// the kernel derives them: (plan row, head, b0, b1) for each.
template <class F>
void cta_pieces(const kvp_pool* p, const SubPlan& sp, int g, F&& emit) {
    (void)p;
    int f = sp.cta_f0[g];
    const int f1 = sp.cta_f0[g + 1];
    if (f >= f1) return;
    int k = (int)(std::upper_bound(sp.seg_f0.begin(), sp.seg_f0.end() - 1, f) - sp.seg_f0.begin()) - 1;
    while (f < f1) {
        while (k + 1 < (int)sp.seg.size() && sp.seg_f0[k + 1] <= f) ++k;
        const int b = f - sp.seg_f0[k];
        const int e = std::min(sp.seg_f0[k + 1], f1);
        emit(sp.row0 + (sp.seg[k] & 0xffff), sp.seg[k] >> 16, b, b + (e - f));
        f = e;
    }
}

template <int S>
void fill_args(const kvp_pool* p, const SubPlan& sp, int layer, int flags, DecodeArgs<S>& a) {
    a.nslots = sp.nslots;
    a.grid = sp.grid;
    a.layer = layer;
    a.flags = flags;
    a.total = sp.total;
    a.row0 = sp.row0;
    a.nsegs = (int)sp.seg.size();
    a.cluster = sp.cluster;
    for (int k = 0; k < a.nsegs; ++k) {
        a.seg_f0[k] = sp.seg_f0[k];
        a.seg[k] = sp.seg[k];
    }
    a.seg_f0[a.nsegs] = sp.total;
    for (int i = 0; i < sp.nslots; ++i) {
        const DecodeSlot& sl = sp.slots[i];
        a.slot[i] = sl;
        // A row the previous decode launch of this pool appended (to the
        // same layer, or with a table entry it wrote) is read only after
        // that launch finishes.
        const Seq& sq = p->seqs[sl.seq];
        const bool prev = sq.app_serial >= 0 && sq.app_serial == p->launch_serial - 1 &&
                          (p->last_layer == layer || p->last_patched);
        a.defer_blk[i] = prev ? sq.app_pos / kBlockTokens : -1;
    }
    for (int g = 0; g <= sp.grid; ++g) a.cta_f0[g] = sp.cta_f0[g];
}

}  // namespace

extern "C" {

int attn_decode_plan_ex(kvp_pool* p, int nseq, const int* seq_ids, const int* rope_pos,
                        const int* append, void* stream) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (nseq < 1 || nseq > p->max_seqs) return fail(KV_ERR_INVAL, "nseq %d outside [1, %d]", nseq, p->max_seqs);
    if (!seq_ids) return fail(KV_ERR_INVAL, "seq_ids is NULL");
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;

    // ---- validate everything before changing anything ----
    if (p->seen.size() != (size_t)p->max_seqs || ++p->seen_stamp == 0) {
        p->seen.assign(p->max_seqs, 0u);
        p->seen_stamp = 1;
    }
    int new_blocks = 0;
    for (int i = 0; i < nseq; ++i) {
        const int sid = seq_ids[i];
        int rc = check_seq(p, sid);
        if (rc) return rc;
        if (p->seen[sid] == p->seen_stamp) return fail(KV_ERR_INVAL, "sequence %d listed twice", sid);
        p->seen[sid] = p->seen_stamp;
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
    queue_plan_patches(p);
    int rc = flush_pending(p, st);
    if (rc) return rc;

    // ---- slots (and the blocks new tokens start) ----
    std::vector<DecodeSlot>& slots = p->plan_slots;
    slots.resize(nseq);
    p->plan_patches.clear();
    p->plan_seqs.assign(seq_ids, seq_ids + nseq);
    p->plan_append.resize(nseq);
    for (int i = 0; i < nseq; ++i) {
        const int sid = seq_ids[i];
        Seq& s = p->seqs[sid];
        const int app = append ? (append[i] != 0) : 1;
        DecodeSlot& sl = slots[i];
        sl.seq = sid;
        sl.kv_len = s.len + app;
        sl.rope_pos = rope_pos ? rope_pos[i] : s.len;
        sl.new_block = -1;
        if (app) {
            const int idx = s.len / kBlockTokens;
            if (idx >= (int)s.blocks.size()) {
                const int b = p->pop_block();
                s.blocks.push_back(b);
                p->plan_patches.push_back(TablePatch{sid, idx, b, 0});
            }
            sl.new_block = s.blocks[idx];
        }
        p->plan_append[i] = app;
    }
    // ---- one launch per kSlotsLarge sequences (fewer with more than
    // kSegsPerSlot KV heads), each partitioned on its own ----
    // (the sub-plans' buffers are reused from plan to plan)
    const int per_launch = std::min(kSlotsLarge, kSegsPerSlot * kSlotsLarge / p->kv_heads);
    p->subs.resize((nseq + per_launch - 1) / per_launch);
    for (size_t k = 0; k < p->subs.size(); ++k) {
        SubPlan& sp = p->subs[k];
        sp.row0 = (int)k * per_launch;
        sp.nslots = std::min(per_launch, nseq - sp.row0);
        sp.slots.assign(slots.begin() + sp.row0, slots.begin() + sp.row0 + sp.nslots);
        partition(p, sp);
    }
    p->plan_active = true;
    p->plan_patched = p->plan_patches.empty() || p->host_only;
    p->plan_stream = st;
    return KV_OK;
}

int kvp_plan_info(const kvp_pool* p, int* nitems, int* grid, int* npatch, int* item_slot,
                  int* item_head, int* item_b0, int* item_b1, int cap) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    int n = 0, gtot = 0;
    for (const SubPlan& sp : p->subs) {
        for (int g = 0; g < sp.grid; ++g)
            cta_pieces(p, sp, g, [&](int slot, int h, int b0, int b1) {
                if (n < cap) {
                    if (item_slot) item_slot[n] = slot;
                    if (item_head) item_head[n] = h;
                    if (item_b0) item_b0[n] = b0;
                    if (item_b1) item_b1[n] = b1;
                }
                ++n;
            });
        gtot += sp.grid;
    }
    if (nitems) *nitems = n;
    if (grid) *grid = gtot;
    if (npatch) *npatch = (int)p->plan_patches.size();
    return KV_OK;
}

int kvp_plan_cta_start(const kvp_pool* p, int* cta_start, int cap) {
    if (!p || !cta_start) return fail(KV_ERR_INVAL, "NULL argument");
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    int k = 0, n = 0;
    for (const SubPlan& sp : p->subs)
        for (int g = 0; g < sp.grid; ++g, ++k) {
            if (k < cap) cta_start[k] = n;
            cta_pieces(p, sp, g, [&](int, int, int, int) { ++n; });
        }
    if (k < cap) cta_start[k] = n;
    return KV_OK;
}

int attn_decode_plan(kvp_pool* p, int nseq, const int* seq_ids, void* stream) {
    return attn_decode_plan_ex(p, nseq, seq_ids, nullptr, nullptr, stream);
}

static int decode_call(kvp_pool* p, int layer, const float* q, const float* k_new, const float* v_new,
                       float* out, float* m, float* l, void* stream, kvx_exch* x = nullptr,
                       float* x_out = nullptr, kvn_comm* nc = nullptr) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    if (int rc = require_device(p)) return rc;
    if (layer < 0 || layer >= p->layers) return fail(KV_ERR_INVAL, "layer %d out of range", layer);
    if (!q || !k_new || !v_new || !out) return fail(KV_ERR_INVAL, "NULL tensor");
    if (((uintptr_t)q | (uintptr_t)k_new | (uintptr_t)v_new) & 7)
        return fail(KV_ERR_INVAL, "q/k_new/v_new must be 8-byte aligned");
    XchgArgs xa;
    const int rows = (int)p->plan_seqs.size() * p->q_heads;
    if (x) {
        // the local states go to this rank's slot of the exchange area
        if (int rc = xchg_prepare(x, p->device, rows, p->pv.status, x_out, &xa, &m, &l, &out)) return rc;
    }
    if (nc) {
        // the local states go to the communicator's send buffer
        if (int rc = nccl_prepare(nc, p->device, rows, &m, &l, &out)) return rc;
    }
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    // With kvp_set_overlap, programmatic dependent launches: the decode grid
    // starts while the previous kernel in the stream finishes and copies its
    // first tiles then.  Only on a created stream (the legacy default stream
    // keeps ordinary launches), and not while timing: events between
    // launches would serialise them anyway.
    const bool pdl = p->overlap && !p->timing && st != nullptr && st != cudaStreamLegacy;
    for (const SubPlan& sp : p->subs) {
        int flags = 0;
        if (pdl && !p->dirty) flags |= kDecEarly;
        if (!p->plan_patched) flags |= kDecPatch;
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
        CombineArgs ca;
        ca.nsegs = (int)sp.comb.size();
        ca.row0 = sp.row0;
        ca.pad[0] = ca.pad[1] = 0;
        for (size_t i = 0; i < sp.comb.size(); ++i) ca.seg[i] = sp.comb[i];
        if (x && p->subs.size() == 1 && ca.nsegs > 0 && ca.nsegs <= kMaxXchgSplit) {
            // The exchange kernel merges the split segments itself (one
            // launch fewer per layer): hand it the pieces, skip the merge.
            xa.partials = p->pv.partials;
            xa.nsplit = ca.nsegs;
            xa.q_heads = p->q_heads;
            xa.group = p->q_heads / p->kv_heads;
            for (int i = 0; i < ca.nsegs; ++i) xa.seg[i] = ca.seg[i];
            ca.nsegs = 0;
        }
        if (sp.nslots <= kSlotsSmall && (int)sp.seg.size() <= kSegsPerSlot * kSlotsSmall) {
            DecodeArgs<kSlotsSmall> a;
            fill_args(p, sp, layer, flags, a);
            KV_CUDA(launch_decode(p->pv, a, ca, sp.max_pieces, q, k_new, v_new, out, m, l, pdl, st));
        } else {
            static thread_local DecodeArgs<kSlotsLarge> a;  // 7 KB: kept off the stack
            fill_args(p, sp, layer, flags, a);
            KV_CUDA(launch_decode(p->pv, a, ca, sp.max_pieces, q, k_new, v_new, out, m, l, pdl, st));
        }
        if (te) KV_CUDA(cudaEventRecord(te->second, st));
        for (const DecodeSlot& sl : sp.slots)
            if (sl.new_block >= 0) {
                Seq& sq = p->seqs[sl.seq];
                sq.app_serial = p->launch_serial;
                sq.app_pos = sl.kv_len - 1;
            }
        p->last_layer = layer;
        p->last_patched = (flags & kDecPatch) != 0;
        p->launch_serial++;
        p->dirty = false;
    }
    p->plan_patched = true;
    if (x) {
        KV_CUDA(launch_xchg(xa, st));
        xchg_commit(x);
    }
    if (nc) return nccl_gather_combine(nc, rows, x_out, st);
    return KV_OK;
}

int kvp_set_overlap(kvp_pool* p, int enable) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (int rc = require_device(p)) return rc;
    p->overlap = enable != 0;
    return KV_OK;
}

int kvp_set_merge_mode(kvp_pool* p, int mode) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    if (mode != KVP_MERGE_GRID && mode != KVP_MERGE_CLUSTER) return fail(KV_ERR_INVAL, "unknown merge mode %d", mode);
    std::lock_guard<std::mutex> lk(p->mu);
    p->merge_mode = mode;
    return KV_OK;
}

int kvp_plan_clusters(const kvp_pool* p, int* clustered_launches, int* launches) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    int c = 0;
    for (const SubPlan& sp : p->subs) c += sp.cluster > 1;
    if (clustered_launches) *clustered_launches = c;
    if (launches) *launches = (int)p->subs.size();
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

int attn_decode_append_nccl(kvp_pool* p, int layer, const float* q, const float* k_new, const float* v_new,
                            float* out, kvn_comm* c, void* stream) {
    if (!c || !out) return fail(KV_ERR_INVAL, "NULL argument");
    float* dummy = out;  // replaced by the communicator's send buffer inside decode_call
    return decode_call(p, layer, q, k_new, v_new, dummy, dummy, dummy, stream, nullptr, out, c);
}

int attn_decode_commit(kvp_pool* p) {
    if (!p) return fail(KV_ERR_INVAL, "pool is NULL");
    std::lock_guard<std::mutex> lk(p->mu);
    if (!p->plan_active) return fail(KV_ERR_STATE, "no active decode plan");
    // New blocks of a plan that no layer call entered in the table are
    // queued; the next call that touches the device applies them.
    queue_plan_patches(p);
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
