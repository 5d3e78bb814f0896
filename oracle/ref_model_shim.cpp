// ref_model_shim.cpp -- C entry points around the reference's OWN Qwen2 model
// and engine (Qwen2Model, LLMEngine), compiled unmodified from its sources.
//
// TEST INFRASTRUCTURE ONLY (golden token streams and the CPU baseline of the
// full-model workload).  Built by oracle/Makefile (`make model`) together with
//   worker/src/model/qwen2_model.cpp, weight_loader.cpp, kv_cache.cpp,
//   worker/src/api/llm_engine.cpp and the ops it calls
// into oracle/_ref/libqwen2ref.so.
//
// The one piece that is not the reference's: the linear backend.  The
// reference's only backend is NpuLinear (worker/src/backend/npu_linear.cpp:
// 84-98), which needs librknnrt (not shipped).  make_linear() below returns a
// CPU stand-in with the ILinearOp contract of worker/include/ops/op_linear.h:
// A [M][K] fp16, weights [K][N] fp16, C [M][N] fp16, computed as
//     C[m][n] = f32_to_f16( sum_{k=0..K-1} f16_to_f32(A[m][k]) * f16_to_f32(B[k][n]) )
// with fp32 accumulation in k order and the reference's truncating
// f32_to_f16 (worker/include/core/half.h).  The NPU's own rounding cannot be
// observed here; the device model follows this same rule.  Columns are split
// across threads; every output keeps its sequential k order, so the thread
// count never changes a result.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "api/llm_engine.h"
#include "core/half.h"
#include "model/qwen2_model.h"
#include "ops/op_linear.h"
#include "ops/op_sampling.h"

namespace {

int g_threads = 0;    // 0: hardware concurrency
int g_sum_order = 0;  // 0: k = 0..K-1 (the contract); 1: k = K-1..0; 2: 32-lane tree (probes only)

int n_threads() {
    if (g_threads > 0) return g_threads;
    const unsigned h = std::thread::hardware_concurrency();
    return h ? (int)h : 1;
}

class CpuLinear : public ILinearOp {
public:
    bool init(int K, int N, const uint16_t* weight_kn) override {
        K_ = K;
        N_ = N;
        w_.resize((size_t)K * N);
        for (size_t i = 0; i < w_.size(); ++i) w_[i] = f16_to_f32(weight_kn[i]);
        return true;
    }

    bool forward(const uint16_t* input_f16, int M, uint16_t* output_f16) override {
        std::vector<float> a((size_t)K_);
        const int T = std::max(1, std::min(n_threads(), N_ / 64));
        for (int m = 0; m < M; ++m) {
            for (int k = 0; k < K_; ++k) a[k] = f16_to_f32(input_f16[(size_t)m * K_ + k]);
            uint16_t* out = output_f16 + (size_t)m * N_;
            auto work = [&](int t) {
                const int n0 = (int)((long long)N_ * t / T), n1 = (int)((long long)N_ * (t + 1) / T);
                std::vector<float> acc((size_t)(n1 - n0), 0.0f);
                if (g_sum_order == 2) {
                    // 32 lanes, lane l summing the 8-element chunks l, l + 32, ...
                    // in order, then a butterfly over the lanes (a parallel order)
                    std::vector<float> lanes((size_t)(n1 - n0) * 32, 0.0f);
                    for (int c = 0; c < K_ / 8; ++c)
                        for (int e = 0; e < 8; ++e) {
                            const int k = c * 8 + e;
                            const float ak = a[k];
                            const float* wr = w_.data() + (size_t)k * N_ + n0;
                            float* lr = lanes.data() + (c % 32);
                            for (int j = 0; j < n1 - n0; ++j) lr[(size_t)j * 32] += ak * wr[j];
                        }
                    for (int j = 0; j < n1 - n0; ++j) {
                        float* l = lanes.data() + (size_t)j * 32;
                        for (int o = 16; o > 0; o >>= 1)
                            for (int x = 0; x < o; ++x) l[x] = l[x] + l[x + o];
                        acc[j] = l[0];
                    }
                } else {
                    for (int i = 0; i < K_; ++i) {
                        const int k = g_sum_order ? K_ - 1 - i : i;
                        const float ak = a[k];
                        const float* wr = w_.data() + (size_t)k * N_ + n0;
                        for (int j = 0; j < n1 - n0; ++j) acc[j] += ak * wr[j];
                    }
                }
                for (int j = 0; j < n1 - n0; ++j) out[n0 + j] = f32_to_f16(acc[j]);
            };
            std::vector<std::thread> pool;
            for (int t = 1; t < T; ++t) pool.emplace_back(work, t);
            work(0);
            for (auto& th : pool) th.join();
        }
        return true;
    }

    void destroy() override {
        w_.clear();
        w_.shrink_to_fit();
    }

private:
    int K_ = 0, N_ = 0;
    std::vector<float> w_;  // [K][N] as fp32 (every fp16 value is exact in fp32)
};

}  // namespace

std::unique_ptr<ILinearOp> make_linear(LinearBackend) { return std::unique_ptr<ILinearOp>(new CpuLinear()); }

extern "C" {

void ref_set_threads(int n) { g_threads = n; }

// Order of the stand-in's fp32 sums: 0 the contract above; 1 reversed; 2 the
// order of a 32-lane parallel reduction.  1 and 2 change nothing but rounding.  Used only to measure how far rounding noise
// alone moves the model's logits (the noise floor any other summation order,
// e.g. a parallel one, meets).
void ref_set_sum_order(int order) { g_sum_order = order; }

// ---- Qwen2Model (worker/include/model/qwen2_model.h:23-56) ----
void* ref_qwen2_load(const char* model_dir) {
    Qwen2Model* m = new Qwen2Model();
    if (!m->load(model_dir)) {
        delete m;
        return nullptr;
    }
    return m;
}
void ref_qwen2_free(void* h) { delete static_cast<Qwen2Model*>(h); }
void ref_qwen2_reset(void* h) { static_cast<Qwen2Model*>(h)->reset_kv_cache(); }

// Qwen2Model::forward (qwen2_model.cpp:131-274): logits of the last token.
int ref_qwen2_forward(void* h, const int* tokens, int n, float* logits, int cap) {
    std::vector<int> ids(tokens, tokens + n);
    std::vector<float> out = static_cast<Qwen2Model*>(h)->forward(ids);
    const int v = (int)out.size();
    std::memcpy(logits, out.data(), sizeof(float) * (size_t)std::min(v, cap));
    return v;
}

// op_greedy_sample (op_sampling.cpp:4-11).
int ref_greedy_sample(const float* logits, int n) {
    return op_greedy_sample(std::vector<float>(logits, logits + n));
}

// ---- LLMEngine (worker/include/api/llm_engine.h) ----
void* ref_engine_load(const char* model_dir) {
    LLMEngine* e = new LLMEngine();
    if (!e->load(model_dir)) {
        delete e;
        return nullptr;
    }
    return e;
}
void ref_engine_free(void* h) { delete static_cast<LLMEngine*>(h); }
void ref_engine_reset(void* h) { static_cast<LLMEngine*>(h)->reset(); }

// LLMEngine::generate (llm_engine.cpp:53-103) with the given stop tokens and
// repetition window; returns the number of generated ids (<= cap copied).
int ref_engine_generate(void* h, const int* ids, int n, int max_new, const int* stops, int nstops,
                        int repetition_window, int* out_ids, int cap) {
    GenerationConfig cfg;
    cfg.max_new_tokens = max_new;
    cfg.stop_tokens.assign(stops, stops + nstops);
    cfg.repetition_window = repetition_window;
    GenerationResult r = static_cast<LLMEngine*>(h)->generate(std::vector<int>(ids, ids + n), cfg);
    const int k = (int)r.output_ids.size();
    for (int i = 0; i < k && i < cap; ++i) out_ids[i] = r.output_ids[i];
    return k;
}

}  // extern "C"
