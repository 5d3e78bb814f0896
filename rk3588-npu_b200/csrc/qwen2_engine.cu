// qwen2_engine.cu -- host runtime of the Qwen2 model and greedy engine on one
// GPU (the qw2_* C ABI of include/qwen2_engine.h).
//
// Replaces Qwen2Model (worker/src/model/qwen2_model.cpp) and LLMEngine
// (worker/src/api/llm_engine.cpp).  Weights are fp16 in HBM in the file's
// [out][in] layout (q, k, v rows of a layer stacked into one [H + 2 kv_dim][H]
// matrix with one bias vector); the KV cache is a kvattn pool (fp16, one
// sequence); one forward is a stream-ordered sequence of launches:
//   embed -> per layer { RMSNorm + QKV GEMV (+bias) -> attention (fused
//   RoPE + append + decode for one token, append chunk + tcgen05 prefill
//   attention for a prompt) -> O GEMV (+residual) -> RMSNorm + gate/up GEMV
//   (SiLU product) -> down GEMV (+residual) } -> RMSNorm + lm_head GEMV ->
//   argmax (each RMSNorm fused into the projection that consumes it),
// then one device-to-host read of the argmax (and the logits when asked),
// which is also the forward's only synchronisation.
#include <cuda_runtime.h>

#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "kvattn.h"
#include "kvattn_internal.h"
#include "qwen2_engine.h"

using namespace kvattn;

namespace {

int qfail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return set_error(status, buf);
}

#define QW_CUDA(call)                                                                             \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) return qfail(KV_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

#define QW_OK(call)                \
    do {                           \
        int s_ = (call);           \
        if (s_ != KV_OK) return s_; \
    } while (0)

// Per-layer tensors in the file (qwen2_model.cpp:83-100).
enum Field { F_LN1, F_WQ, F_BQ, F_WK, F_BK, F_WV, F_BV, F_WO, F_LN2, F_WG, F_WU, F_WD, F_COUNT };
const char* const kFieldName[F_COUNT] = {
    "input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.q_proj.bias", "self_attn.k_proj.weight",
    "self_attn.k_proj.bias",  "self_attn.v_proj.weight", "self_attn.v_proj.bias", "self_attn.o_proj.weight",
    "post_attention_layernorm.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"};

// fp16 -> fp32 as worker/include/core/half.h:34-43.
float host_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    uint32_t x;
    if (e == 0) x = sign | (mant << 13);
    else if (e == 31) x = sign | 0x7F800000u | (mant << 13);
    else x = sign | ((e + 112u) << 23) | (mant << 13);
    float f;
    memcpy(&f, &x, 4);
    return f;
}

constexpr size_t kStagingBytes = 64u << 20;

}  // namespace

namespace {

// One generation request moving through LLMEngine::generate's loop
// (llm_engine.cpp:66-98) one engine step at a time.
struct Job {
    int id = 0;
    int session = 0;
    std::vector<int> input;       // ids still to append (prefill)
    int n_input = 0;
    int max_new = 0;
    int rep_window = 0;
    std::vector<int> stops;
    qw2_token_cb cb = nullptr;
    void* user = nullptr;
    std::vector<int> out;
    int next = 0;                 // greedy choice of the last forward
    int step = 0;                 // decode step (loop counter of the reference)
    bool prefilled = false;
    bool decoding = false;        // `next` is pushed and waits for its forward
    bool done = false;
    std::atomic<bool> cancel{false};  // set by qw2_cancel from another thread
    qw2_result res{};
    std::chrono::steady_clock::time_point t0, t_prefill, t_step;
};

}  // namespace

struct qw2_model {
    int device = 0;
    qw2_config c{};
    int kvd = 0;
    cudaStream_t st = nullptr;
    bool own_stream = false;
    kvp_pool* pool = nullptr;
    int kv_dtype = KV_F16;
    int max_sessions = 1;
    int rows_cap = 0;              // rows of one forward (activation buffers)
    std::vector<int> session_seq;  // session -> pool sequence id, -1 = free
    std::vector<char> session_busy;  // an async request runs on it

    // async engine
    std::mutex mu;                 // one model operation at a time
    std::mutex qmu;                // the queue and the finished jobs
    std::condition_variable qcv;
    std::deque<std::shared_ptr<Job>> queue;
    std::map<int, std::shared_ptr<Job>> finished;
    std::map<int, std::shared_ptr<Job>> running;
    std::thread worker;
    bool stop_worker = false;
    int next_job = 1;

    struct Layer {
        float* ln1 = nullptr;
        uint16_t* wqkv = nullptr;  // [H + 2 kvd][H]
        float* bqkv = nullptr;     // [H + 2 kvd]
        uint16_t* wo = nullptr;    // [H][H]
        float* ln2 = nullptr;
        uint16_t* wg = nullptr;    // [IS][H]
        uint16_t* wu = nullptr;    // [IS][H]
        uint16_t* wd = nullptr;    // [H][IS]
        bool have[F_COUNT] = {};
    };
    std::vector<Layer> L;
    uint16_t* embed = nullptr;  // [V][H], also lm_head
    float* norm = nullptr;
    bool have_embed = false, have_norm = false;

    // activations, up to max_position rows
    float* hidden = nullptr;  // [R][H]
    float* q = nullptr;       // [R][H]
    float* k = nullptr;       // [R][kvd]
    float* v = nullptr;       // [R][kvd]
    float* attn = nullptr;    // [R][H]
    uint16_t* h16 = nullptr;  // [R][IS]
    float* logits = nullptr;  // [S][V]: one row per session of a forward
    float* last = nullptr;    // [S][H]: the last hidden row of each session
    int* ids = nullptr;       // [R + S]: token ids, then the last-row index of each session
    unsigned long long* best = nullptr;  // [S]
    void* staging = nullptr;

    // forward in the reference's operation order (qw2_set_exact): buffers
    // allocated on first use
    bool exact = false;
    uint16_t* ex_x16 = nullptr;    // [R][max(H, IS)] projection inputs
    uint16_t* ex_qkv16 = nullptr;  // [R][H + 2 kvd]
    uint16_t* ex_g16 = nullptr;    // [R][IS]
    uint16_t* ex_u16 = nullptr;    // [R][IS]
    uint16_t* ex_y16 = nullptr;    // [max(R H, V)] projection outputs
    uint16_t* ex_kc = nullptr;     // [max_position][kvd] one layer's cache rows
    uint16_t* ex_vc = nullptr;
    ExpTab ex_exp;                 // the host expf's deviations from the correctly rounded exp

    std::vector<void*> allocs;

    int alloc(void** p, size_t bytes) {
        cudaError_t e = cudaMalloc(p, bytes);
        if (e != cudaSuccess) return qfail(KV_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
        allocs.push_back(*p);
        return KV_OK;
    }
    template <class T>
    int alloc_n(T** p, size_t n) {
        return alloc(reinterpret_cast<void**>(p), n * sizeof(T));
    }
    void release() {
        for (void* p : allocs) cudaFree(p);
        allocs.clear();
    }
};

namespace {

int check_cfg(const qw2_config* c) {
    if (!c) return qfail(KV_ERR_INVAL, "NULL config");
    if (c->head_dim != kHeadDim) return qfail(KV_ERR_INVAL, "head_dim %d unsupported (128 only)", c->head_dim);
    if (c->layers <= 0 || c->q_heads <= 0 || c->kv_heads <= 0 || c->vocab <= 0 || c->max_position <= 0 ||
        c->intermediate <= 0)
        return qfail(KV_ERR_INVAL, "non-positive size in config");
    if (c->hidden != c->q_heads * c->head_dim) return qfail(KV_ERR_INVAL, "hidden != q_heads * head_dim");
    if (c->q_heads % c->kv_heads || c->q_heads / c->kv_heads > kMaxGroup)
        return qfail(KV_ERR_INVAL, "q_heads / kv_heads must be an integer <= %d", kMaxGroup);
    if (c->hidden % 32 || c->intermediate % 32)
        return qfail(KV_ERR_INVAL, "hidden and intermediate must be multiples of 32");
    return KV_OK;
}

// Where a named tensor goes: a matrix (fp16, row offset inside a stacked
// matrix) or a vector (fp32, element offset).
struct Target {
    bool matrix = false;
    uint16_t* m16 = nullptr;
    float* f32 = nullptr;
    int64_t rows = 0, cols = 0;  // expected shape ([n] for vectors: rows = n, cols = 0)
    bool* have = nullptr;
};

int resolve(qw2_model* m, const char* name, Target* t) {
    const qw2_config& c = m->c;
    const int H = c.hidden, kvd = m->kvd, IS = c.intermediate;
    std::string s(name);
    if (s == "model.embed_tokens.weight") {
        *t = Target{true, m->embed, nullptr, c.vocab, H, &m->have_embed};
        return KV_OK;
    }
    if (s == "model.norm.weight") {
        *t = Target{false, nullptr, m->norm, H, 0, &m->have_norm};
        return KV_OK;
    }
    const std::string pre = "model.layers.";
    if (s.compare(0, pre.size(), pre) == 0) {
        size_t p = pre.size(), q = p;
        while (q < s.size() && s[q] >= '0' && s[q] <= '9') ++q;
        if (q > p && q < s.size() && s[q] == '.' && q - p < 6) {
            const int li = atoi(s.substr(p, q - p).c_str());
            const std::string f = s.substr(q + 1);
            if (li >= 0 && li < c.layers) {
                qw2_model::Layer& Ly = m->L[li];
                for (int i = 0; i < F_COUNT; ++i) {
                    if (f != kFieldName[i]) continue;
                    bool* hv = &Ly.have[i];
                    switch (i) {
                        case F_LN1: *t = Target{false, nullptr, Ly.ln1, H, 0, hv}; break;
                        case F_WQ: *t = Target{true, Ly.wqkv, nullptr, H, H, hv}; break;
                        case F_BQ: *t = Target{false, nullptr, Ly.bqkv, H, 0, hv}; break;
                        case F_WK: *t = Target{true, Ly.wqkv + (size_t)H * H, nullptr, kvd, H, hv}; break;
                        case F_BK: *t = Target{false, nullptr, Ly.bqkv + H, kvd, 0, hv}; break;
                        case F_WV: *t = Target{true, Ly.wqkv + (size_t)(H + kvd) * H, nullptr, kvd, H, hv}; break;
                        case F_BV: *t = Target{false, nullptr, Ly.bqkv + H + kvd, kvd, 0, hv}; break;
                        case F_WO: *t = Target{true, Ly.wo, nullptr, H, H, hv}; break;
                        case F_LN2: *t = Target{false, nullptr, Ly.ln2, H, 0, hv}; break;
                        case F_WG: *t = Target{true, Ly.wg, nullptr, IS, H, hv}; break;
                        case F_WU: *t = Target{true, Ly.wu, nullptr, IS, H, hv}; break;
                        case F_WD: *t = Target{true, Ly.wd, nullptr, H, IS, hv}; break;
                    }
                    return KV_OK;
                }
            }
        }
    }
    return qfail(KV_ERR_INVAL, "unknown tensor name '%s'", name);
}


// ---- a minimal reader of the safetensors header (a JSON object) ----
struct JsonTensor {
    std::string dtype;
    std::vector<int64_t> shape;
    int64_t begin = -1, end = -1;
};

struct JsonReader {
    const char* p;
    const char* e;
    bool ok = true;
    bool fail() {
        ok = false;
        return false;
    }
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool lit(char ch) {
        ws();
        if (p < e && *p == ch) {
            ++p;
            return true;
        }
        return false;
    }
    bool str(std::string* out) {
        ws();
        if (p >= e || *p != '"') return fail();
        ++p;
        out->clear();
        while (p < e && *p != '"') {
            if (*p == '\\' && p + 1 < e) ++p;
            out->push_back(*p++);
        }
        if (p >= e) return fail();
        ++p;
        return true;
    }
    bool num(int64_t* out) {
        ws();
        bool neg = false;
        if (p < e && *p == '-') {
            neg = true;
            ++p;
        }
        if (p >= e || *p < '0' || *p > '9') return fail();
        int64_t v = 0;
        while (p < e && *p >= '0' && *p <= '9') v = v * 10 + (*p++ - '0');
        *out = neg ? -v : v;
        return true;
    }
    bool skip() {  // any value
        ws();
        if (p >= e) return fail();
        if (*p == '"') {
            std::string t;
            return str(&t);
        }
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            ++p;
            if (lit(close)) return true;
            do {
                if (obj) {
                    std::string k;
                    if (!str(&k) || !lit(':')) return fail();
                }
                if (!skip()) return false;
            } while (lit(','));
            return lit(close) || fail();
        }
        while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
        return true;
    }
};

int parse_header(const std::string& json, std::unordered_map<std::string, JsonTensor>* out) {
    JsonReader r{json.data(), json.data() + json.size()};
    if (!r.lit('{')) return qfail(KV_ERR_INVAL, "safetensors header is not a JSON object");
    if (r.lit('}')) return KV_OK;
    do {
        std::string key;
        if (!r.str(&key) || !r.lit(':')) break;
        if (key == "__metadata__") {
            if (!r.skip()) break;
            continue;
        }
        JsonTensor t;
        if (!r.lit('{')) break;
        if (!r.lit('}')) {
            do {
                std::string f;
                if (!r.str(&f) || !r.lit(':')) break;
                if (f == "dtype") {
                    r.str(&t.dtype);
                } else if (f == "shape") {
                    if (!r.lit('[')) break;
                    if (!r.lit(']')) {
                        do {
                            int64_t d;
                            if (!r.num(&d)) break;
                            t.shape.push_back(d);
                        } while (r.lit(','));
                        if (!r.lit(']')) r.ok = false;
                    }
                } else if (f == "data_offsets") {
                    if (!r.lit('[') || !r.num(&t.begin) || !r.lit(',') || !r.num(&t.end) || !r.lit(']')) r.ok = false;
                } else {
                    r.skip();
                }
            } while (r.ok && r.lit(','));
            if (r.ok && !r.lit('}')) r.ok = false;
        }
        if (!r.ok) break;
        (*out)[key] = t;
    } while (r.lit(','));
    if (!r.ok || !r.lit('}')) return qfail(KV_ERR_INVAL, "malformed safetensors header");
    return KV_OK;
}

// detect_repetition (llm_engine.cpp:22-36): the last `window` ids repeat with
// some period p in [1, window/2].  Where the reference's loop would index
// before the first id (it reads ids[i - p] before testing i - p < 0), it
// returns false for that p; so does this.
bool detect_repetition(const std::vector<int>& ids, int window) {
    const int n = (int)ids.size();
    if (window <= 0 || n < window) return false;
    for (int p = 1; p <= window / 2; ++p) {
        if (n - window - p < 0) continue;
        bool rep = true;
        for (int i = n - 1; i >= n - window; --i)
            if (ids[i] != ids[i - p]) {
                rep = false;
                break;
            }
        if (rep) return true;
    }
    return false;
}

}  // namespace

namespace {

int session_check(const qw2_model* m, int session) {
    if (session < 0 || session >= m->max_sessions || m->session_seq[session] < 0)
        return qfail(KV_ERR_BADSEQ, "no session %d", session);
    return KV_OK;
}

// n tokens of one session, at its current position.
struct Group {
    int session = 0;
    const int* tokens = nullptr;
    int n = 0;
    float* logits_host = nullptr;  // [vocab] or NULL
    int argmax = 0;
};

// The float inputs where this process's C library expf (the exp the
// reference's loops call) differs from the correctly rounded exponential --
// (float)exp((double)x) -- and its results there, found once per process by
// evaluating both over every float with a finite, nonzero result
// (|x| < 104, about 2.2e9 inputs, on all host threads).  Sorted by bits,
// with an index over the top 16 bits (see ExpTab).
struct HostExpTable {
    std::vector<uint32_t> keys, vals, bucket;
};

const HostExpTable& host_exp_table() {
    static HostExpTable t;
    static std::once_flag once;
    std::call_once(once, [] {
        // positive inputs [0, 104) then negative ones, as bit ranges
        const uint32_t kPosEnd = 0x42D00000u, kNegBeg = 0x80000000u, kNegEnd = 0xC2D00000u;
        const uint64_t total = (uint64_t)kPosEnd + (kNegEnd - kNegBeg);
        unsigned nt = std::max(1u, std::thread::hardware_concurrency());
        std::vector<std::vector<std::pair<uint32_t, uint32_t>>> part(nt);
        std::vector<std::thread> th;
        for (unsigned w = 0; w < nt; ++w)
            th.emplace_back([&, w] {
                const uint64_t a = total * w / nt, b = total * (w + 1) / nt;
                for (uint64_t i = a; i < b; ++i) {
                    const uint32_t bits = i < kPosEnd ? (uint32_t)i : (uint32_t)(kNegBeg + (i - kPosEnd));
                    float x;
                    memcpy(&x, &bits, 4);
                    const float lib = std::exp(x), cr = (float)std::exp((double)x);
                    if (lib != cr) {
                        uint32_t lb;
                        memcpy(&lb, &lib, 4);
                        part[w].emplace_back(bits, lb);
                    }
                }
            });
        for (auto& x : th) x.join();
        std::vector<std::pair<uint32_t, uint32_t>> all;
        for (auto& p : part) all.insert(all.end(), p.begin(), p.end());
        std::sort(all.begin(), all.end());
        t.keys.reserve(all.size());
        t.vals.reserve(all.size());
        for (auto& kv : all) {
            t.keys.push_back(kv.first);
            t.vals.push_back(kv.second);
        }
        t.bucket.assign(65537, 0);
        for (uint32_t k : t.keys) ++t.bucket[(k >> 16) + 1];
        for (int b = 0; b < 65536; ++b) t.bucket[b + 1] += t.bucket[b];
    });
    return t;
}

// Qwen2Model::forward in the reference's operation order (qw2_set_exact):
// the groups one after another, each with the exact_kernels.cu kernels --
// RMSNorm, projections, biases, q RoPE, the pool's bit-exact append, the
// layer's cache rows gathered into the reference layout, attention,
// residuals, SiLU, lm_head -- then the greedy argmax of its last row.
int forward_exact(qw2_model* m, std::vector<Group>& gs) {
    const qw2_config& c = m->c;
    const int G = (int)gs.size();
    if (G == 0) return qfail(KV_ERR_INVAL, "forward of no tokens");
    if (G > m->max_sessions) return qfail(KV_ERR_INVAL, "%d groups > %d sessions", G, m->max_sessions);
    QW_OK(qw2_ready(m));
    std::vector<char> seen(m->max_sessions, 0);
    std::vector<int> pos(G), seq(G);
    for (int g = 0; g < G; ++g) {
        const Group& gr = gs[g];
        QW_OK(session_check(m, gr.session));
        if (seen[gr.session]) return qfail(KV_ERR_INVAL, "session %d twice in one forward", gr.session);
        seen[gr.session] = 1;
        if (gr.n <= 0 || !gr.tokens) return qfail(KV_ERR_INVAL, "forward of %d tokens", gr.n);
        for (int i = 0; i < gr.n; ++i)
            if (gr.tokens[i] < 0 || gr.tokens[i] >= c.vocab)
                return qfail(KV_ERR_RANGE, "token id %d outside [0, %d)", gr.tokens[i], c.vocab);
        seq[g] = m->session_seq[gr.session];
        QW_OK(kvp_seq_len(m->pool, seq[g], &pos[g]));
        if (pos[g] + gr.n > c.max_position)
            return qfail(KV_ERR_RANGE, "positions %d..%d pass max_position %d", pos[g], pos[g] + gr.n - 1,
                         c.max_position);
        if (gr.n > m->rows_cap) return qfail(KV_ERR_RANGE, "%d rows in one forward > %d", gr.n, m->rows_cap);
    }
    DeviceGuard dg(m->device);
    cudaStream_t st = m->st;
    const int H = c.hidden, kvd = m->kvd, IS = c.intermediate, V = c.vocab;
    const float scale = 1.0f / std::sqrt((float)c.head_dim);  // op_attention.cpp:20
    const float2* rope = pool_rope_table(m->pool);
    for (int g = 0; g < G; ++g) {
        const Group& gr = gs[g];
        const int n = gr.n, p0 = pos[g], T = p0 + n;
        QW_OK(kvp_seq_reserve(m->pool, seq[g], T));
        QW_OK(kvp_seq_set_len(m->pool, seq[g], T));  // the gathers below read positions [0, T)
        QW_CUDA(cudaMemcpyAsync(m->ids, gr.tokens, sizeof(int) * n, cudaMemcpyHostToDevice, st));
        QW_CUDA(launch_embed(m->ids, n, m->embed, m->hidden, H, st));
        for (int li = 0; li < c.layers; ++li) {
            const qw2_model::Layer& Ly = m->L[li];
            QW_CUDA(launch_rmsnorm_exact(m->hidden, Ly.ln1, c.rms_eps, n, H, m->ex_x16, st));
            QW_CUDA(launch_gemv_exact(m->ex_x16, n, H, Ly.wqkv, H + 2 * kvd, m->ex_qkv16, st));
            QW_CUDA(launch_qkv_bias_exact(m->ex_qkv16, Ly.bqkv, n, H, kvd, m->q, m->k, m->v, st));
            QW_CUDA(launch_rope_q_exact(m->q, n, c.q_heads, p0, rope, st));
            QW_OK(kv_append_chunk(m->pool, li, seq[g], p0, n, m->k, m->v, st));
            QW_OK(kvp_gather(m->pool, li, seq[g], m->ex_kc, m->ex_vc, st));
            QW_CUDA(launch_attn_exact(m->q, m->ex_kc, m->ex_vc, m->attn, n, T, c.q_heads, c.kv_heads, p0, scale, m->ex_exp,
                                      st));
            QW_CUDA(launch_to_f16_exact(m->attn, (long)n * H, m->ex_x16, st));
            QW_CUDA(launch_gemv_exact(m->ex_x16, n, H, Ly.wo, H, m->ex_y16, st));
            QW_CUDA(launch_resid_exact(m->hidden, m->ex_y16, (long)n * H, st));
            QW_CUDA(launch_rmsnorm_exact(m->hidden, Ly.ln2, c.rms_eps, n, H, m->ex_x16, st));
            QW_CUDA(launch_gemv_exact(m->ex_x16, n, H, Ly.wg, IS, m->ex_g16, st));
            QW_CUDA(launch_gemv_exact(m->ex_x16, n, H, Ly.wu, IS, m->ex_u16, st));
            QW_CUDA(launch_silu_mul_exact(m->ex_g16, m->ex_u16, (long)n * IS, m->h16, m->ex_exp, st));
            QW_CUDA(launch_gemv_exact(m->h16, n, IS, Ly.wd, H, m->ex_y16, st));
            QW_CUDA(launch_resid_exact(m->hidden, m->ex_y16, (long)n * H, st));
        }
        // final RMSNorm of the last row, lm_head (the tied embedding), argmax
        QW_CUDA(launch_rmsnorm_exact(m->hidden + (size_t)(n - 1) * H, m->norm, c.rms_eps, 1, H, m->ex_x16, st));
        QW_CUDA(launch_gemv_exact(m->ex_x16, 1, H, m->embed, V, m->ex_y16, st));
        float* lg = m->logits + (size_t)g * V;
        QW_CUDA(launch_f16_to_f32_exact(m->ex_y16, V, lg, st));
        QW_CUDA(launch_argmax(lg, V, 1, m->best + g, st));
        if (gr.logits_host)
            QW_CUDA(cudaMemcpyAsync(gr.logits_host, lg, sizeof(float) * (size_t)V, cudaMemcpyDeviceToHost, st));
    }
    std::vector<unsigned long long> keys(G);
    QW_CUDA(cudaMemcpyAsync(keys.data(), m->best, sizeof(unsigned long long) * G, cudaMemcpyDeviceToHost, st));
    int status = 0;
    QW_OK(kvp_device_status(m->pool, st, &status));  // synchronises the stream
    if (status != 0) return status;
    for (int g = 0; g < G; ++g)
        gs[g].argmax = keys[g] ? (int)(0xFFFFFFFFu - (uint32_t)(keys[g] & 0xFFFFFFFFu)) : 0;
    return KV_OK;
}

// Qwen2Model::forward (qwen2_model.cpp:131-274) over several sessions at
// once.  Rows: the one-token groups first (in the given order: one planned
// decode-attention launch covers them), then every longer group (appended
// as a chunk and attended with the prefill kernel).  The projections run
// once over all rows; lm_head and the argmax over each group's last row.
int forward_groups(qw2_model* m, std::vector<Group>& gs) {
    if (m->exact) return forward_exact(m, gs);
    const qw2_config& c = m->c;
    const int G = (int)gs.size();
    if (G == 0) return qfail(KV_ERR_INVAL, "forward of no tokens");
    if (G > m->max_sessions) return qfail(KV_ERR_INVAL, "%d groups > %d sessions", G, m->max_sessions);
    QW_OK(qw2_ready(m));
    std::vector<int> order;  // decode groups first
    for (int pass = 0; pass < 2; ++pass)
        for (int g = 0; g < G; ++g)
            if ((gs[g].n == 1) == (pass == 0)) order.push_back(g);
    std::vector<int> pos(G), seq(G), off(G);
    std::vector<char> seen(m->max_sessions, 0);
    int rows = 0, nD = 0;
    for (int g : order) {
        Group& gr = gs[g];
        QW_OK(session_check(m, gr.session));
        if (seen[gr.session]) return qfail(KV_ERR_INVAL, "session %d twice in one forward", gr.session);
        seen[gr.session] = 1;
        if (gr.n <= 0 || !gr.tokens) return qfail(KV_ERR_INVAL, "forward of %d tokens", gr.n);
        for (int i = 0; i < gr.n; ++i)
            if (gr.tokens[i] < 0 || gr.tokens[i] >= c.vocab)
                return qfail(KV_ERR_RANGE, "token id %d outside [0, %d)", gr.tokens[i], c.vocab);
        seq[g] = m->session_seq[gr.session];
        QW_OK(kvp_seq_len(m->pool, seq[g], &pos[g]));
        if (pos[g] + gr.n > c.max_position)
            return qfail(KV_ERR_RANGE, "positions %d..%d pass max_position %d", pos[g], pos[g] + gr.n - 1,
                         c.max_position);
        off[g] = rows;
        rows += gr.n;
        nD += gr.n == 1;
    }
    if (rows > m->rows_cap) return qfail(KV_ERR_RANGE, "%d rows in one forward > %d", rows, m->rows_cap);
    DeviceGuard dg(m->device);
    cudaStream_t st = m->st;
    const int H = c.hidden, kvd = m->kvd, IS = c.intermediate;

    // token ids, then the index of each group's last row (in `order`)
    std::vector<int> host(rows + G);
    for (int g : order) memcpy(host.data() + off[g], gs[g].tokens, sizeof(int) * gs[g].n);
    for (int i = 0; i < G; ++i) host[rows + i] = off[order[i]] + gs[order[i]].n - 1;
    QW_CUDA(cudaMemcpyAsync(m->ids, host.data(), sizeof(int) * host.size(), cudaMemcpyHostToDevice, st));
    QW_CUDA(launch_embed(m->ids, rows, m->embed, m->hidden, H, st));
    if (nD) {
        std::vector<int> dseq;
        for (int i = 0; i < nD; ++i) dseq.push_back(seq[order[i]]);
        QW_OK(attn_decode_plan(m->pool, nD, dseq.data(), st));
    }
    for (int i = nD; i < G; ++i) QW_OK(kvp_seq_reserve(m->pool, seq[order[i]], pos[order[i]] + gs[order[i]].n));
    // the prompt chunks: consecutive rows from off[order[nD]], appended and
    // attended together (shared launches)
    std::vector<int> cseq, cpos, cn;
    for (int i = nD; i < G; ++i) {
        cseq.push_back(seq[order[i]]);
        cpos.push_back(pos[order[i]]);
        cn.push_back(gs[order[i]].n);
    }
    const size_t crow = nD < G ? (size_t)off[order[nD]] : 0;

    for (int li = 0; li < c.layers; ++li) {
        const qw2_model::Layer& Ly = m->L[li];
        // 1-2: input RMSNorm fused into the Q/K/V projections (+ biases)
        GemvArgs a;
        a.w = Ly.wqkv;
        a.N = H + 2 * kvd;
        a.K = H;
        a.M = rows;
        a.x = m->hidden;
        a.norm_w = Ly.ln1;
        a.eps = c.rms_eps;
        a.bias = Ly.bqkv;
        a.out0 = m->q;
        a.out1 = m->k;
        a.out2 = m->v;
        a.n0 = H;
        a.n1 = kvd;
        QW_CUDA(launch_gemv(0, 2, a, st));
        // 3-5: RoPE, KV append, attention
        if (nD) QW_OK(attn_decode_append(m->pool, li, m->q, m->k, m->v, m->attn, st));
        if (nD < G) {
            const int nc = G - nD;
            QW_OK(kv_append_chunk_batch(m->pool, li, nc, cseq.data(), cpos.data(), cn.data(), m->k + crow * kvd,
                                        m->v + crow * kvd, st));
            QW_OK(attn_prefill_batch(m->pool, li, nc, cseq.data(), cpos.data(), cn.data(), m->q + crow * H,
                                     m->attn + crow * H, st));
        }
        // 6-7: O projection + residual
        GemvArgs o;
        o.w = Ly.wo;
        o.N = H;
        o.K = H;
        o.M = rows;
        o.x = m->attn;
        o.resid = m->hidden;
        QW_CUDA(launch_gemv(1, 1, o, st));
        // 8-10: post-attention RMSNorm fused into gate/up (+ SiLU product), down + residual
        GemvArgs gu;
        gu.w = Ly.wg;
        gu.w2 = Ly.wu;
        gu.N = IS;
        gu.K = H;
        gu.M = rows;
        gu.x = m->hidden;
        gu.norm_w = Ly.ln2;
        gu.eps = c.rms_eps;
        gu.out16 = m->h16;
        QW_CUDA(launch_gemv(2, 2, gu, st));
        GemvArgs d;
        d.w = Ly.wd;
        d.N = H;
        d.K = IS;
        d.M = rows;
        d.x = m->h16;
        d.resid = m->hidden;
        QW_CUDA(launch_gemv(1, 0, d, st));
    }
    if (nD) QW_OK(attn_decode_commit(m->pool));
    for (int i = nD; i < G; ++i) QW_OK(kvp_seq_set_len(m->pool, seq[order[i]], pos[order[i]] + gs[order[i]].n));

    // final RMSNorm of each group's last token fused into lm_head (tied embedding), argmax
    const float* last = m->hidden;
    if (!(G == rows)) {  // one-token groups only: the last rows are rows 0..G-1 already
        QW_CUDA(launch_gather_rows(m->hidden, m->ids + rows, G, m->last, H, st));
        last = m->last;
    }
    GemvArgs lm;
    lm.w = m->embed;
    lm.N = c.vocab;
    lm.K = H;
    lm.M = G;
    lm.x = last;
    lm.norm_w = m->norm;
    lm.eps = c.rms_eps;
    lm.logits = m->logits;
    QW_CUDA(launch_gemv(3, 2, lm, st));
    QW_CUDA(launch_argmax(m->logits, c.vocab, G, m->best, st));
    std::vector<unsigned long long> keys(G);
    QW_CUDA(cudaMemcpyAsync(keys.data(), m->best, sizeof(unsigned long long) * G, cudaMemcpyDeviceToHost, st));
    for (int i = 0; i < G; ++i)
        if (gs[order[i]].logits_host)
            QW_CUDA(cudaMemcpyAsync(gs[order[i]].logits_host, m->logits + (size_t)i * c.vocab,
                                    sizeof(float) * (size_t)c.vocab, cudaMemcpyDeviceToHost, st));
    int status = 0;
    QW_OK(kvp_device_status(m->pool, st, &status));  // synchronises the stream
    if (status != 0) return status;
    for (int i = 0; i < G; ++i) {
        const unsigned long long key = keys[i];
        gs[order[i]].argmax = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu)) : 0;
    }
    return KV_OK;
}

using Clock = std::chrono::steady_clock;

float ms_since(Clock::time_point t) {
    return std::chrono::duration<float, std::milli>(Clock::now() - t).count();
}

void job_finish(Job& j, int status) {
    j.done = true;
    j.res.status = status;
    j.res.n_out = (int)j.out.size();
    j.res.decode_tokens = (int)j.out.size();
    if (j.prefilled) j.res.decode_ms = ms_since(j.t_prefill);
}

// The loop head of llm_engine.cpp:76-90 once `next` holds the greedy choice
// of the job's last forward: stop at max_new or a stop token (not emitted),
// emit `next`, stop on a repetition (emitted, never forwarded), else its
// forward is due.
void job_advance(Job& j) {
    if (j.step >= j.max_new) {
        job_finish(j, KV_OK);
        return;
    }
    for (int s : j.stops)
        if (s == j.next) {
            j.res.hit_stop = 1;
            job_finish(j, KV_OK);
            return;
        }
    j.out.push_back(j.next);
    if (j.rep_window > 0 && detect_repetition(j.out, j.rep_window)) {
        j.res.hit_repetition = 1;
        job_finish(j, KV_OK);
        return;
    }
    j.decoding = true;
    j.t_step = Clock::now();
}

constexpr int kPrefillChunk = 256;  // prompt tokens of one request appended per engine step

// One engine step over the live jobs: every decoding job forwards its pushed
// id, every prefilling job appends its next prompt chunk (as rows allow),
// all in one forward_groups.  Returns the forward's status (a failure ends
// every job of the step).
int engine_step(qw2_model* m, std::vector<Job*>& jobs) {
    std::vector<Group> gs;
    std::vector<Job*> gj;
    int rows = 0;
    for (Job* j : jobs) {
        if (j->done) continue;
        if (j->cancel) {  // cancel_generation: ends at this step boundary
            j->res.cancelled = 1;
            job_finish(*j, KV_OK);
            continue;
        }
        if (j->prefilled && j->decoding) {
            Group g;
            g.session = j->session;
            g.tokens = &j->out.back();
            g.n = 1;
            gs.push_back(g);
            gj.push_back(j);
            ++rows;
        }
    }
    for (Job* j : jobs) {
        if (j->done || j->prefilled) continue;
        int n = std::min((int)j->input.size(), std::min(kPrefillChunk, m->c.max_position));
        n = std::min(n, m->rows_cap - rows);
        if (n <= 0) continue;
        Group g;
        g.session = j->session;
        g.tokens = j->input.data();
        g.n = n;
        gs.push_back(g);
        gj.push_back(j);
        rows += n;
    }
    if (gs.empty()) return KV_OK;
    const int rc = forward_groups(m, gs);
    if (rc != KV_OK) {
        for (Job* j : gj) job_finish(*j, rc);
        return rc;
    }
    for (size_t i = 0; i < gs.size(); ++i) {
        Job& j = *gj[i];
        j.next = gs[i].argmax;
        if (!j.prefilled) {
            j.input.erase(j.input.begin(), j.input.begin() + gs[i].n);
            if (!j.input.empty()) continue;
            j.prefilled = true;
            j.t_prefill = Clock::now();
            j.res.prefill_ms = ms_since(j.t0);
            j.res.prefill_tokens = j.n_input;
        } else {
            j.decoding = false;
            if (j.cb) j.cb(j.user, j.session, j.step, j.out.back(), ms_since(j.t_step));
            ++j.step;
        }
        job_advance(j);
    }
    return KV_OK;
}

std::shared_ptr<Job> make_job(const qw2_request& r) {
    auto j = std::make_shared<Job>();
    j->session = r.session;
    j->input.assign(r.input_ids, r.input_ids + r.n_input);
    j->n_input = r.n_input;
    j->max_new = r.cfg.max_new_tokens;
    j->rep_window = r.cfg.repetition_window;
    if (r.cfg.n_stop > 0) j->stops.assign(r.cfg.stop_tokens, r.cfg.stop_tokens + r.cfg.n_stop);
    j->cb = r.on_token;
    j->user = r.user;
    j->t0 = Clock::now();
    return j;
}

int check_request(const qw2_model* m, const qw2_request& r) {
    QW_OK(session_check(m, r.session));
    if (r.n_input < 0 || (r.n_input > 0 && !r.input_ids) || (r.cfg.n_stop > 0 && !r.cfg.stop_tokens) ||
        r.cfg.n_stop < 0 || (r.out_cap > 0 && !r.out_ids))
        return qfail(KV_ERR_INVAL, "malformed request for session %d", r.session);
    return KV_OK;
}

// Run jobs to completion on the calling thread (the model lock held).
int run_jobs(qw2_model* m, std::vector<Job*>& jobs) {
    for (Job* j : jobs)
        if (j->n_input == 0) job_finish(*j, KV_OK);  // llm_engine.cpp:59: nothing to do
    for (;;) {
        bool live = false;
        for (Job* j : jobs) live = live || !j->done;
        if (!live) return KV_OK;
        const int rc = engine_step(m, jobs);
        if (rc != KV_OK) {
            for (Job* j : jobs)
                if (!j->done) job_finish(*j, rc);
            return rc;
        }
    }
}

void worker_loop(qw2_model* m) {
    std::vector<std::shared_ptr<Job>> active;
    for (;;) {
        {
            std::unique_lock<std::mutex> lk(m->qmu);
            m->qcv.wait(lk, [&] { return m->stop_worker || !m->queue.empty() || !active.empty(); });
            if (m->stop_worker) {
                for (auto& j : active) {
                    job_finish(*j, KV_ERR_STATE);
                    m->finished[j->id] = j;
                }
                for (auto& j : m->queue) {
                    job_finish(*j, KV_ERR_STATE);
                    m->finished[j->id] = j;
                }
                m->queue.clear();
                m->qcv.notify_all();
                return;
            }
            while (!m->queue.empty()) {
                active.push_back(m->queue.front());
                m->queue.pop_front();
            }
        }
        std::vector<Job*> raw;
        for (auto& j : active) {
            if (j->n_input == 0 && !j->done) job_finish(*j, KV_OK);
            raw.push_back(j.get());
        }
        {
            std::lock_guard<std::mutex> mk(m->mu);
            const int rc = engine_step(m, raw);
            if (rc != KV_OK)
                for (Job* j : raw)
                    if (!j->done) job_finish(*j, rc);
        }
        std::lock_guard<std::mutex> lk(m->qmu);
        std::vector<std::shared_ptr<Job>> still;
        for (auto& j : active) {
            if (j->done) {
                m->running.erase(j->id);
                m->session_busy[j->session] = 0;
                m->finished[j->id] = j;
            } else {
                still.push_back(j);
            }
        }
        active.swap(still);
        m->qcv.notify_all();
    }
}

}  // namespace

extern "C" {

int qw2_config_default(qw2_config* c) {
    if (!c) return qfail(KV_ERR_INVAL, "NULL config");
    // Qwen2Config defaults (model_config.h:8-23)
    c->hidden = 1536;
    c->layers = 28;
    c->q_heads = 12;
    c->kv_heads = 2;
    c->head_dim = 128;
    c->intermediate = 8960;
    c->vocab = 151936;
    c->rms_eps = 1e-6f;
    c->rope_theta = 1000000.0f;
    c->max_position = 512;
    return KV_OK;
}

int qw2_destroy(qw2_model* m) {
    if (!m) return KV_OK;
    {
        std::lock_guard<std::mutex> lk(m->qmu);
        m->stop_worker = true;
    }
    m->qcv.notify_all();
    if (m->worker.joinable()) m->worker.join();
    DeviceGuard g(m->device);
    if (m->st) cudaStreamSynchronize(m->st);
    if (m->pool) kvp_destroy(m->pool);
    m->release();
    if (m->own_stream && m->st) cudaStreamDestroy(m->st);
    delete m;
    return KV_OK;
}

int qw2_create_kv(int device, const qw2_config* cfg, int max_sessions, int kv_dtype, qw2_model** out) {
    if (!out) return qfail(KV_ERR_INVAL, "NULL out");
    *out = nullptr;
    QW_OK(check_cfg(cfg));
    if (kv_dtype != KV_F16 && kv_dtype != KV_BF16 && kv_dtype != KV_I8)
        return qfail(KV_ERR_INVAL, "KV cache type %d is not KV_F16, KV_BF16 or KV_I8", kv_dtype);
    if (max_sessions < 1 || max_sessions > 1024) return qfail(KV_ERR_INVAL, "max_sessions %d outside [1, 1024]", max_sessions);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return qfail(KV_ERR_INVAL, "no CUDA device %d", device);
    DeviceGuard g(device);
    if (!g.ok) return qfail(KV_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    qw2_model* m = new qw2_model();
    m->device = device;
    m->c = *cfg;
    m->kvd = cfg->kv_heads * cfg->head_dim;
    m->kv_dtype = kv_dtype;
    m->max_sessions = max_sessions;
    m->rows_cap = cfg->max_position + max_sessions;
    m->session_seq.assign(max_sessions, -1);
    m->session_busy.assign(max_sessions, 0);
    const size_t H = cfg->hidden, kvd = m->kvd, IS = cfg->intermediate, V = cfg->vocab, R = m->rows_cap,
                 S = max_sessions;
    int rc = KV_OK;
    auto step = [&](int s) {
        if (rc == KV_OK) rc = s;
    };
    m->L.resize(cfg->layers);
    step(m->alloc_n(&m->embed, V * H));
    step(m->alloc_n(&m->norm, H));
    for (auto& Ly : m->L) {
        step(m->alloc_n(&Ly.ln1, H));
        step(m->alloc_n(&Ly.wqkv, (H + 2 * kvd) * H));
        step(m->alloc_n(&Ly.bqkv, H + 2 * kvd));
        step(m->alloc_n(&Ly.wo, H * H));
        step(m->alloc_n(&Ly.ln2, H));
        step(m->alloc_n(&Ly.wg, IS * H));
        step(m->alloc_n(&Ly.wu, IS * H));
        step(m->alloc_n(&Ly.wd, H * IS));
    }
    step(m->alloc_n(&m->hidden, R * H));
    step(m->alloc_n(&m->q, R * H));
    step(m->alloc_n(&m->k, R * kvd));
    step(m->alloc_n(&m->v, R * kvd));
    step(m->alloc_n(&m->attn, R * H));
    step(m->alloc_n(&m->h16, R * IS));
    step(m->alloc_n(&m->logits, S * V));
    step(m->alloc_n(&m->last, S * H));
    step(m->alloc_n(&m->ids, R + S));
    step(m->alloc_n(&m->best, S));
    step(m->alloc(&m->staging, kStagingBytes));
    if (rc == KV_OK) {
        if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess)
            rc = qfail(KV_ERR_CUDA, "cudaStreamCreate failed");
        else
            m->own_stream = true;
    }
    if (rc == KV_OK) {
        const int blocks = max_sessions * ((cfg->max_position + kBlockTokens - 1) / kBlockTokens);
        step(kvp_create(device, cfg->layers, cfg->q_heads, cfg->kv_heads, cfg->head_dim, kBlockTokens, blocks,
                        kv_dtype, max_sessions, cfg->max_position, cfg->rope_theta, &m->pool));
    }
    // every forward ends with a host synchronisation, so no decode launch
    // overlaps a kernel that writes the cache (kvp_set_overlap's contract)
    if (rc == KV_OK) step(kvp_set_overlap(m->pool, 1));
    if (rc == KV_OK) step(kvp_seq_alloc(m->pool, &m->session_seq[0]));  // session 0
    if (rc != KV_OK) {
        const std::string msg = kv_last_error();
        qw2_destroy(m);
        return qfail(rc, "%s", msg.c_str());
    }
    *out = m;
    return KV_OK;
}

int qw2_create_sessions(int device, const qw2_config* cfg, int max_sessions, qw2_model** out) {
    return qw2_create_kv(device, cfg, max_sessions, KV_F16, out);
}

int qw2_create(int device, const qw2_config* cfg, qw2_model** out) {
    return qw2_create_sessions(device, cfg, 1, out);
}

int qw2_set_exact(qw2_model* m, int on) {
    if (!m) return qfail(KV_ERR_INVAL, "NULL model");
    std::lock_guard<std::mutex> lk(m->mu);
    if (on && m->kv_dtype != KV_F16)
        return qfail(KV_ERR_INVAL, "the reference-order forward needs the fp16 KV cache (the reference's)");
    if (on && !m->ex_x16) {
        DeviceGuard g(m->device);
        const size_t H = m->c.hidden, kvd = m->kvd, IS = m->c.intermediate, V = m->c.vocab, R = m->rows_cap;
        QW_OK(m->alloc_n(&m->ex_x16, R * std::max(H, IS)));
        QW_OK(m->alloc_n(&m->ex_qkv16, R * (H + 2 * kvd)));
        QW_OK(m->alloc_n(&m->ex_g16, R * IS));
        QW_OK(m->alloc_n(&m->ex_u16, R * IS));
        QW_OK(m->alloc_n(&m->ex_y16, std::max(R * H, V)));
        QW_OK(m->alloc_n(&m->ex_kc, (size_t)m->c.max_position * kvd));
        QW_OK(m->alloc_n(&m->ex_vc, (size_t)m->c.max_position * kvd));
        const HostExpTable& t = host_exp_table();
        uint32_t *keys = nullptr, *vals = nullptr, *bucket = nullptr;
        const size_t ne = std::max<size_t>(1, t.keys.size());
        QW_OK(m->alloc_n(&keys, ne));
        QW_OK(m->alloc_n(&vals, ne));
        QW_OK(m->alloc_n(&bucket, t.bucket.size()));
        if (!t.keys.empty()) {
            QW_CUDA(cudaMemcpy(keys, t.keys.data(), t.keys.size() * 4, cudaMemcpyHostToDevice));
            QW_CUDA(cudaMemcpy(vals, t.vals.data(), t.vals.size() * 4, cudaMemcpyHostToDevice));
        }
        QW_CUDA(cudaMemcpy(bucket, t.bucket.data(), t.bucket.size() * 4, cudaMemcpyHostToDevice));
        m->ex_exp.keys = keys;
        m->ex_exp.vals = vals;
        m->ex_exp.bucket = bucket;
    }
    m->exact = on != 0;
    return KV_OK;
}

int qw2_set_stream(qw2_model* m, void* stream) {
    if (!m) return qfail(KV_ERR_INVAL, "NULL model");
    DeviceGuard g(m->device);
    QW_CUDA(cudaStreamSynchronize(m->st));
    if (m->own_stream) cudaStreamDestroy(m->st);
    m->st = (cudaStream_t)stream;
    m->own_stream = false;
    return KV_OK;
}

int qw2_set_tensor(qw2_model* m, const char* name, int dtype, const int64_t* shape, int ndim, const void* host) {
    if (!m || !name || !shape || !host) return qfail(KV_ERR_INVAL, "NULL argument");
    if (dtype != QW2_F16 && dtype != QW2_BF16 && dtype != QW2_F32)
        return qfail(KV_ERR_INVAL, "tensor '%s': unsupported dtype %d", name, dtype);
    std::lock_guard<std::mutex> lk(m->mu);
    Target t;
    QW_OK(resolve(m, name, &t));
    const bool shape_ok = t.matrix ? (ndim == 2 && shape[0] == t.rows && shape[1] == t.cols)
                                   : (ndim == 1 && shape[0] == t.rows);
    if (!shape_ok)
        return qfail(KV_ERR_INVAL, "tensor '%s': shape [%lld%s%lld] expected [%lld%s%lld]", name,
                     (long long)shape[0], ndim > 1 ? "," : "", ndim > 1 ? (long long)shape[1] : 0LL,
                     (long long)t.rows, t.matrix ? "," : "", t.matrix ? (long long)t.cols : 0LL);
    DeviceGuard g(m->device);
    const size_t esz = dtype == QW2_F32 ? 4 : 2;
    if (t.matrix) {
        const size_t n = (size_t)t.rows * (size_t)t.cols, per = kStagingBytes / esz;
        for (size_t i = 0; i < n; i += per) {
            const size_t cnt = n - i < per ? n - i : per;
            QW_CUDA(cudaMemcpyAsync(m->staging, static_cast<const uint8_t*>(host) + i * esz, cnt * esz,
                                    cudaMemcpyHostToDevice, m->st));
            QW_CUDA(launch_weight_to_f16(m->staging, dtype, t.m16 + i, cnt, m->st));
        }
    } else {
        // load_tensor_f32 (weight_loader.cpp:207-235)
        std::vector<float> f((size_t)t.rows);
        for (size_t i = 0; i < f.size(); ++i) {
            if (dtype == QW2_F32) {
                f[i] = static_cast<const float*>(host)[i];
            } else {
                const uint16_t h = static_cast<const uint16_t*>(host)[i];
                if (dtype == QW2_BF16) {
                    const uint32_t u = (uint32_t)h << 16;
                    memcpy(&f[i], &u, 4);
                } else {
                    f[i] = host_f16_to_f32(h);
                }
            }
        }
        QW_CUDA(cudaMemcpyAsync(t.f32, f.data(), f.size() * 4, cudaMemcpyHostToDevice, m->st));
    }
    QW_CUDA(cudaStreamSynchronize(m->st));
    *t.have = true;
    return KV_OK;
}

int qw2_load_safetensors(qw2_model* m, const char* path) {
    if (!m || !path) return qfail(KV_ERR_INVAL, "NULL argument");
    FILE* fp = fopen(path, "rb");
    if (!fp) return qfail(KV_ERR_INVAL, "cannot open %s", path);
    uint64_t hlen = 0;
    int rc = KV_OK;
    std::unordered_map<std::string, JsonTensor> meta;
    if (fread(&hlen, 1, 8, fp) != 8 || hlen > (1u << 30)) {
        rc = qfail(KV_ERR_INVAL, "%s: bad safetensors header", path);
    } else {
        std::string json(hlen, '\0');
        if (fread(&json[0], 1, hlen, fp) != hlen) rc = qfail(KV_ERR_INVAL, "%s: short header", path);
        else rc = parse_header(json, &meta);
    }
    const int64_t base = 8 + (int64_t)hlen;
    std::vector<std::string> names = {"model.embed_tokens.weight", "model.norm.weight"};
    for (int i = 0; i < m->c.layers; ++i)
        for (int f = 0; f < F_COUNT; ++f) names.push_back("model.layers." + std::to_string(i) + "." + kFieldName[f]);
    std::vector<uint8_t> buf;
    for (const std::string& nm : names) {
        if (rc != KV_OK) break;
        auto it = meta.find(nm);
        if (it == meta.end()) {
            rc = qfail(KV_ERR_INVAL, "%s: tensor '%s' missing", path, nm.c_str());
            break;
        }
        const JsonTensor& t = it->second;
        const int dt = t.dtype == "F16" ? QW2_F16 : t.dtype == "BF16" ? QW2_BF16 : t.dtype == "F32" ? QW2_F32 : -1;
        if (dt < 0) {
            rc = qfail(KV_ERR_INVAL, "%s: tensor '%s' has unsupported dtype %s", path, nm.c_str(), t.dtype.c_str());
            break;
        }
        int64_t n = 1;
        for (int64_t d : t.shape) n *= d;
        const int64_t bytes = n * (dt == QW2_F32 ? 4 : 2);
        if (t.begin < 0 || t.end - t.begin != bytes || t.shape.empty() || t.shape.size() > 2) {
            rc = qfail(KV_ERR_INVAL, "%s: tensor '%s' has inconsistent offsets or shape", path, nm.c_str());
            break;
        }
        buf.resize((size_t)bytes);
        if (fseeko(fp, (off_t)(base + t.begin), SEEK_SET) != 0 || fread(buf.data(), 1, (size_t)bytes, fp) != (size_t)bytes) {
            rc = qfail(KV_ERR_INVAL, "%s: tensor '%s' read failed", path, nm.c_str());
            break;
        }
        rc = qw2_set_tensor(m, nm.c_str(), dt, t.shape.data(), (int)t.shape.size(), buf.data());
    }
    fclose(fp);
    return rc;
}

int qw2_ready(qw2_model* m) {
    if (!m) return qfail(KV_ERR_INVAL, "NULL model");
    if (!m->have_embed) return qfail(KV_ERR_STATE, "tensor model.embed_tokens.weight not set");
    if (!m->have_norm) return qfail(KV_ERR_STATE, "tensor model.norm.weight not set");
    for (int i = 0; i < m->c.layers; ++i)
        for (int f = 0; f < F_COUNT; ++f)
            if (!m->L[i].have[f]) return qfail(KV_ERR_STATE, "tensor model.layers.%d.%s not set", i, kFieldName[f]);
    return KV_OK;
}

int qw2_reset(qw2_model* m) {
    if (!m) return qfail(KV_ERR_INVAL, "NULL model");
    std::lock_guard<std::mutex> lk(m->mu);
    if (m->session_busy[0]) return qfail(KV_ERR_STATE, "session 0 has a running request");
    DeviceGuard g(m->device);
    bool others = false;
    for (int s = 1; s < m->max_sessions; ++s) others = others || m->session_seq[s] >= 0;
    if (!others) {
        // Qwen2Model::reset_kv_cache: the whole cache zeroed (kv_cache.cpp:12-16)
        QW_OK(kvp_reset(m->pool, m->st));
    } else {
        QW_OK(kvp_seq_free(m->pool, m->session_seq[0]));  // other sessions keep their blocks
    }
    QW_OK(kvp_seq_alloc(m->pool, &m->session_seq[0]));
    QW_CUDA(cudaStreamSynchronize(m->st));
    return KV_OK;
}

int qw2_cur_pos(const qw2_model* m, int* pos) { return qw2_session_len(m, 0, pos); }

int qw2_session_create(qw2_model* m, int* session) {
    if (!m || !session) return qfail(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(m->mu);
    for (int s = 0; s < m->max_sessions; ++s)
        if (m->session_seq[s] < 0) {
            QW_OK(kvp_seq_alloc(m->pool, &m->session_seq[s]));
            *session = s;
            return KV_OK;
        }
    return qfail(KV_ERR_OOM, "all %d sessions in use", m->max_sessions);
}

int qw2_session_destroy(qw2_model* m, int session) {
    if (!m) return qfail(KV_ERR_INVAL, "NULL model");
    std::lock_guard<std::mutex> lk(m->mu);
    QW_OK(session_check(m, session));
    {
        std::lock_guard<std::mutex> qk(m->qmu);
        if (m->session_busy[session]) return qfail(KV_ERR_STATE, "session %d has a running request", session);
    }
    QW_OK(kvp_seq_free(m->pool, m->session_seq[session]));
    m->session_seq[session] = -1;
    return KV_OK;
}

int qw2_session_exists(const qw2_model* m, int session, int* exists) {
    if (!m || !exists) return qfail(KV_ERR_INVAL, "NULL argument");
    *exists = session >= 0 && session < m->max_sessions && m->session_seq[session] >= 0;
    return KV_OK;
}

int qw2_session_len(const qw2_model* m, int session, int* len) {
    if (!m || !len) return qfail(KV_ERR_INVAL, "NULL argument");
    QW_OK(session_check(m, session));
    return kvp_seq_len(m->pool, m->session_seq[session], len);
}

int qw2_session_seq(const qw2_model* m, int session, int* seq_id) {
    if (!m || !seq_id) return qfail(KV_ERR_INVAL, "NULL argument");
    QW_OK(session_check(m, session));
    *seq_id = m->session_seq[session];
    return KV_OK;
}

int qw2_forward_session(qw2_model* m, int session, const int* tokens, int n, float* logits_host, int* argmax) {
    if (!m || !tokens) return qfail(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(m->mu);
    QW_OK(session_check(m, session));
    {
        std::lock_guard<std::mutex> qk(m->qmu);
        if (m->session_busy[session]) return qfail(KV_ERR_STATE, "session %d has a running request", session);
    }
    std::vector<Group> gs(1);
    gs[0].session = session;
    gs[0].tokens = tokens;
    gs[0].n = n;
    gs[0].logits_host = logits_host;
    QW_OK(forward_groups(m, gs));
    if (argmax) *argmax = gs[0].argmax;
    return KV_OK;
}

int qw2_forward(qw2_model* m, const int* tokens, int n, float* logits_host, int* argmax) {
    return qw2_forward_session(m, 0, tokens, n, logits_host, argmax);
}

int qw2_generate_batch(qw2_model* m, int n_requests, const qw2_request* requests, qw2_result* results) {
    if (!m || n_requests < 0 || (n_requests > 0 && (!requests || !results)))
        return qfail(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(m->mu);
    std::vector<char> seen(m->max_sessions, 0);
    for (int i = 0; i < n_requests; ++i) {
        QW_OK(check_request(m, requests[i]));
        if (seen[requests[i].session]) return qfail(KV_ERR_INVAL, "session %d twice in one batch", requests[i].session);
        seen[requests[i].session] = 1;
        std::lock_guard<std::mutex> qk(m->qmu);
        if (m->session_busy[requests[i].session])
            return qfail(KV_ERR_STATE, "session %d has a running request", requests[i].session);
    }
    std::vector<std::shared_ptr<Job>> jobs;
    std::vector<Job*> raw;
    for (int i = 0; i < n_requests; ++i) {
        jobs.push_back(make_job(requests[i]));
        raw.push_back(jobs.back().get());
    }
    const int rc = run_jobs(m, raw);
    for (int i = 0; i < n_requests; ++i) {
        const Job& j = *jobs[i];
        results[i] = j.res;
        for (int k = 0; k < (int)j.out.size() && k < requests[i].out_cap; ++k) requests[i].out_ids[k] = j.out[k];
    }
    return rc;
}

int qw2_generate_session(qw2_model* m, int session, const int* input_ids, int n_input, const qw2_gen_config* cfg,
                         int* out_ids, int out_cap, qw2_result* result) {
    if (!m || !cfg || !result) return qfail(KV_ERR_INVAL, "NULL argument");
    qw2_request r{};
    r.session = session;
    r.input_ids = input_ids;
    r.n_input = n_input;
    r.cfg = *cfg;
    r.out_ids = out_ids;
    r.out_cap = out_cap;
    return qw2_generate_batch(m, 1, &r, result);
}

int qw2_generate(qw2_model* m, const int* prompt, int n_prompt, int max_new, const int* stop_tokens, int n_stop,
                 int repetition_window, int* out_ids, int cap, int* n_out) {
    if (!m || !n_out) return qfail(KV_ERR_INVAL, "NULL argument");
    *n_out = 0;
    if (n_prompt <= 0 || !prompt) return KV_OK;  // llm_engine.cpp:59
    qw2_gen_config cfg{max_new, repetition_window, stop_tokens, n_stop};
    qw2_result res{};
    QW_OK(qw2_generate_session(m, 0, prompt, n_prompt, &cfg, out_ids, cap, &res));
    *n_out = res.n_out;
    return res.status;
}

int qw2_submit(qw2_model* m, const qw2_request* request, int* job) {
    if (!m || !request || !job) return qfail(KV_ERR_INVAL, "NULL argument");
    QW_OK(check_request(m, *request));
    auto j = make_job(*request);
    {
        std::lock_guard<std::mutex> lk(m->qmu);
        if (m->stop_worker) return qfail(KV_ERR_STATE, "model is being destroyed");
        if (m->session_busy[request->session])
            return qfail(KV_ERR_STATE, "session %d has a running request", request->session);
        m->session_busy[request->session] = 1;
        j->id = m->next_job++;
        m->running[j->id] = j;
        m->queue.push_back(j);
        if (!m->worker.joinable()) m->worker = std::thread(worker_loop, m);
    }
    m->qcv.notify_all();
    *job = j->id;
    return KV_OK;
}

int qw2_wait(qw2_model* m, int job, int timeout_ms, int* out_ids, int out_cap, qw2_result* result) {
    if (!m || !result || (out_cap > 0 && !out_ids)) return qfail(KV_ERR_INVAL, "NULL argument");
    std::unique_lock<std::mutex> lk(m->qmu);
    auto ready = [&] { return m->finished.count(job) > 0; };
    if (!ready() && !m->running.count(job)) return qfail(KV_ERR_INVAL, "no job %d", job);
    if (timeout_ms < 0) m->qcv.wait(lk, ready);
    else if (!m->qcv.wait_for(lk, std::chrono::milliseconds(timeout_ms), ready))
        return qfail(KV_ERR_TIMEOUT, "job %d still running", job);
    std::shared_ptr<Job> j = m->finished[job];
    m->finished.erase(job);
    *result = j->res;
    for (int k = 0; k < (int)j->out.size() && k < out_cap; ++k) out_ids[k] = j->out[k];
    return KV_OK;
}

int qw2_cancel(qw2_model* m, int session) {
    if (!m) return qfail(KV_ERR_INVAL, "NULL model");
    std::lock_guard<std::mutex> lk(m->qmu);
    bool any = false;
    for (auto& kv : m->running)
        if (kv.second->session == session) {
            kv.second->cancel = true;
            any = true;
        }
    if (!any) return qfail(KV_ERR_BADSEQ, "no request running on session %d", session);
    m->qcv.notify_all();
    return KV_OK;
}

int qw2_kv_pool(qw2_model* m, kvp_pool** pool) {
    if (!m || !pool) return qfail(KV_ERR_INVAL, "NULL argument");
    *pool = m->pool;
    return KV_OK;
}

int qw2_weight_bytes(const qw2_model* m, long long* bytes) {
    if (!m || !bytes) return qfail(KV_ERR_INVAL, "NULL argument");
    const long long H = m->c.hidden, kvd = m->kvd, IS = m->c.intermediate, V = m->c.vocab;
    const long long per_layer = (H + 2 * kvd) * H + H * H + 3 * IS * H;
    *bytes = 2 * (per_layer * m->c.layers + V * H);
    return KV_OK;
}

}  // extern "C"
