// ref_shim.cpp -- C entry points around the reference's OWN functions.
//
// TEST INFRASTRUCTURE ONLY (the checker and the CPU baseline).  Built by
// oracle/Makefile together with the unmodified reference sources
//   worker/src/ops/op_attention.cpp, op_softmax.cpp, op_rope.cpp,
//   worker/src/model/kv_cache.cpp, worker/include/core/half.h
// into oracle/_ref/libkvref.so.  Nothing here re-implements the reference:
// each function forwards to the reference symbol it names.  The only loop
// written here is the KV append of qwen2_model.cpp:188-200, which the
// reference has inline in Qwen2Model::forward rather than as a function.
#include <cstdint>
#include <thread>
#include <vector>

#include "core/half.h"
#include "model/kv_cache.h"
#include "ops/op_attention.h"
#include "ops/op_rope.h"
#include "ops/op_softmax.h"

extern "C" {

void ref_f32_to_f16(const float* src, uint16_t* dst, long n) {
    for (long i = 0; i < n; ++i) dst[i] = f32_to_f16(src[i]);  // half.h:24-32
}
void ref_f16_to_f32(const uint16_t* src, float* dst, long n) {
    for (long i = 0; i < n; ++i) dst[i] = f16_to_f32(src[i]);  // half.h:34-43
}
void ref_f32_to_bf16(const float* src, uint16_t* dst, long n) {
    for (long i = 0; i < n; ++i) dst[i] = f32_to_bf16(src[i]);  // half.h:17-20
}
void ref_bf16_to_f32(const uint16_t* src, float* dst, long n) {
    for (long i = 0; i < n; ++i) dst[i] = bf16_to_f32(src[i]);  // half.h:12-15
}

void ref_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_dim, int pos,
              float theta) {
    op_rope(q, k, n_heads, n_kv_heads, head_dim, pos, theta);  // op_rope.cpp:21-30
}

void ref_softmax(float* x, int rows, int cols) { op_softmax(x, rows, cols); }

void ref_attention(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                   float* out, int seq, int total_len, int n_heads, int n_kv_heads,
                   int head_dim, int pos_base) {
    op_attention(q, k_cache, v_cache, out, seq, total_len, n_heads, n_kv_heads, head_dim,
                 pos_base);  // op_attention.cpp:9-56
}

// ---- KVCache handle (kv_cache.h:19-41) ----
void* ref_kvc_create(int num_layers, int capacity, int kv_dim) {
    KVCache* c = new KVCache();
    c->init(num_layers, capacity, kv_dim);
    return c;
}
void ref_kvc_destroy(void* h) { delete static_cast<KVCache*>(h); }
void ref_kvc_reset(void* h) { static_cast<KVCache*>(h)->reset(); }
int ref_kvc_cur_pos(void* h) { return static_cast<KVCache*>(h)->cur_pos(); }
void ref_kvc_set_cur_pos(void* h, int p) { static_cast<KVCache*>(h)->set_cur_pos(p); }
int ref_kvc_capacity(void* h) { return static_cast<KVCache*>(h)->capacity(); }
uint16_t* ref_kvc_k_ptr(void* h, int layer) { return static_cast<KVCache*>(h)->k_ptr(layer); }
uint16_t* ref_kvc_v_ptr(void* h, int layer) { return static_cast<KVCache*>(h)->v_ptr(layer); }

// Steps 3-5 of Qwen2Model::forward for one layer (qwen2_model.cpp:180-206):
// RoPE every new token at pos+s, write the fp16 rows, attend over pos+seq.
// q [seq][n_heads*head_dim], k/v [seq][kv_dim] fp32 (bias already added);
// q and k are rotated in place as the reference does.
void ref_layer_step(float* q, float* k, const float* v, uint16_t* kc, uint16_t* vc,
                    float* out, int seq, int pos, int n_heads, int n_kv_heads, int head_dim,
                    float theta) {
    const int H = n_heads * head_dim;
    const int kv_dim = n_kv_heads * head_dim;
    for (int s = 0; s < seq; ++s)
        op_rope(q + s * H, k + s * kv_dim, n_heads, n_kv_heads, head_dim, pos + s, theta);
    for (int s = 0; s < seq; ++s) {
        const float* ksrc = k + s * kv_dim;
        const float* vsrc = v + s * kv_dim;
        uint16_t* kdst = kc + (pos + s) * kv_dim;
        uint16_t* vdst = vc + (pos + s) * kv_dim;
        for (int d = 0; d < kv_dim; ++d) {
            kdst[d] = f32_to_f16(ksrc[d]);
            vdst[d] = f32_to_f16(vsrc[d]);
        }
    }
    op_attention(q, kc, vc, out, seq, pos + seq, n_heads, n_kv_heads, head_dim, pos);
}

// The same layer step for `nseq` independent sequences, run by `threads` host
// threads that each take whole sequences (a harness-level loop around the
// unmodified functions; the reference itself is single-threaded).
// kc/vc[i] point at sequence i's contiguous cache; q/k/v/out are packed
// [nseq][...]; pos[i] is sequence i's position.
void ref_batch_step(float* q, float* k, const float* v, uint16_t** kc, uint16_t** vc,
                    float* out, const int* pos, int nseq, int n_heads, int n_kv_heads,
                    int head_dim, float theta, int threads) {
    const int H = n_heads * head_dim;
    const int kv_dim = n_kv_heads * head_dim;
    auto work = [&](int t) {
        for (int i = t; i < nseq; i += threads)
            ref_layer_step(q + (long)i * H, k + (long)i * kv_dim, v + (long)i * kv_dim, kc[i],
                           vc[i], out + (long)i * H, 1, pos[i], n_heads, n_kv_heads, head_dim,
                           theta);
    };
    if (threads <= 1) {
        threads = 1;
        work(0);
        return;
    }
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) pool.emplace_back(work, t);
    for (auto& th : pool) th.join();
}

}  // extern "C"
