// kvattn_kvcache.hpp -- C++ adapter for the Qwen2 worker (C++14, header only).
//
// PagedKVCache keeps the method names of the reference's KVCache
// (worker/include/model/kv_cache.h:19-41: init, reset, cur_pos, set_cur_pos,
// capacity, kv_dim) over one sequence of the paged B200 pool (kvattn.h), and
// adds the calls that replace the per-layer RoPE + append + attention of
// Qwen2Model::forward (worker/src/model/qwen2_model.cpp:180-206).  The
// reference's k_ptr(layer)/v_ptr(layer) hand out contiguous host rows; the
// pool is paged device memory, so gather() copies a layer's rows out in that
// same [pos][kv_dim] layout instead.
//
// kvattn::op_attention has op_attention's signature and meaning
// (worker/include/ops/op_attention.h:19-26) on DEVICE pointers with fp16
// contiguous caches, through the allocation-free entry point.
#pragma once

#include <cstdint>
#include <cstdio>

#include "kvattn.h"

namespace kvattn {

struct KVCacheConfig {
    int device = 0;          // CUDA device, or KVP_HOST_ONLY (bookkeeping only)
    int num_q_heads = 12;    // Qwen2-1.5B: 12 query heads over kv_dim / 128 KV heads
    int dtype = KV_F16;      // the reference stores fp16
    float rope_theta = 1e6f;
    void* stream = nullptr;  // stream of every call (nullptr: legacy default stream)
};

class PagedKVCache {
public:
    explicit PagedKVCache(const KVCacheConfig& cfg = KVCacheConfig()) : cfg_(cfg) {}
    ~PagedKVCache() { release(); }
    PagedKVCache(const PagedKVCache&) = delete;
    PagedKVCache& operator=(const PagedKVCache&) = delete;

    // KVCache::init (kv_cache.cpp:4-10): room for `capacity` positions of one
    // sequence in every layer, zero-filled.  false (kv_last_error() says why)
    // on an unsupported shape or a CUDA failure.
    bool init(int num_layers, int capacity, int kv_dim) {
        release();
        if (kv_dim <= 0 || kv_dim % 128 != 0 || capacity <= 0) return false;
        const int blocks = (capacity + 15) / 16;
        if (kvp_create(cfg_.device, num_layers, cfg_.num_q_heads, kv_dim / 128, 128, 16, blocks,
                       cfg_.dtype, 1, capacity, cfg_.rope_theta, &pool_) != KV_OK)
            return false;
        capacity_ = capacity;
        kv_dim_ = kv_dim;
        return open_sequence();
    }

    // KVCache::reset (kv_cache.cpp:12-16): position 0, storage zeroed.
    void reset() {
        if (!pool_) return;
        if (kvp_reset(pool_, cfg_.stream) != KV_OK || !open_sequence())
            std::fprintf(stderr, "[kvattn] reset: %s\n", kv_last_error());
    }

    int cur_pos() const {
        int n = 0;
        if (pool_) kvp_seq_len(pool_, seq_, &n);
        return n;
    }
    void set_cur_pos(int pos) {
        if (pool_ && kvp_seq_set_len(pool_, seq_, pos) != KV_OK)
            std::fprintf(stderr, "[kvattn] set_cur_pos(%d): %s\n", pos, kv_last_error());
    }
    int capacity() const { return capacity_; }
    int kv_dim() const { return kv_dim_; }

    // What k_ptr(layer)/v_ptr(layer) would hold at [0, cur_pos()): rows
    // [cur_pos()][kv_dim] 16-bit, written to device buffers.
    bool gather(int layer, uint16_t* k_rows, uint16_t* v_rows) const {
        return kvp_gather(pool_, layer, seq_, k_rows, v_rows, cfg_.stream) == KV_OK;
    }

    // ---- decode (seq = 1), qwen2_model.cpp:140, 180-206, 268 ----
    // begin_step once before the layer loop; decode_layer(li, ...) replaces
    // op_rope + the append loop + op_attention of layer li (q, k, v fp32
    // after bias add, out fp32, all device pointers); end_step replaces
    // set_cur_pos(pos + 1) after the last layer.
    bool begin_step() { return attn_decode_plan(pool_, 1, &seq_, cfg_.stream) == KV_OK; }
    bool decode_layer(int layer, const float* q, const float* k, const float* v, float* out) {
        return attn_decode_append(pool_, layer, q, k, v, out, cfg_.stream) == KV_OK;
    }
    bool end_step() { return attn_decode_commit(pool_) == KV_OK; }

    // ---- prefill (seq = n > 1) ----
    // RoPE + append of n new rows k, v [n][kv_dim] fp32 (device) at
    // positions cur_pos().. of `layer`; after the last layer advance with
    // set_cur_pos(cur_pos() + n), as qwen2_model.cpp:268.
    bool append_prefill(int layer, int n, const float* k, const float* v) {
        return kv_append_chunk(pool_, layer, seq_, cur_pos(), n, k, v, cfg_.stream) == KV_OK;
    }

    kvp_pool* pool() const { return pool_; }
    int seq() const { return seq_; }

private:
    bool open_sequence() {
        return kvp_seq_alloc(pool_, &seq_) == KV_OK && kvp_seq_reserve(pool_, seq_, capacity_) == KV_OK;
    }
    void release() {
        if (pool_) kvp_destroy(pool_);
        pool_ = nullptr;
        seq_ = -1;
    }

    KVCacheConfig cfg_;
    kvp_pool* pool_ = nullptr;
    int seq_ = -1;
    int capacity_ = 0;
    int kv_dim_ = 0;
};

// op_attention (op_attention.h:19-26): causal GQA attention, q [seq][n_heads
// * head_dim] fp32 already rotated, caches [total_len][n_kv_heads *
// head_dim] fp16, out [seq][n_heads * head_dim] fp32, query s at absolute
// position pos_base + s -- on device pointers, on the legacy default stream.
// Like the reference it returns nothing; a rejected call is reported on
// stderr (kv_last_error() has the status message).
inline void op_attention(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                         float* out, int seq, int total_len, int n_heads, int n_kv_heads,
                         int head_dim, int pos_base) {
    const int rc = attn_contig_noalloc(q, k_cache, v_cache, out, seq, total_len, n_heads,
                                       n_kv_heads, head_dim, pos_base, KV_F16, nullptr);
    if (rc != KV_OK) std::fprintf(stderr, "[kvattn] op_attention: %s\n", kv_status_str(rc));
}

}  // namespace kvattn
