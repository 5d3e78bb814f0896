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

#include <string>
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

struct qw2_model {
    int device = 0;
    qw2_config c{};
    int kvd = 0;
    cudaStream_t st = nullptr;
    bool own_stream = false;
    kvp_pool* pool = nullptr;
    int seq = -1;

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
    float* logits = nullptr;  // [V]
    int* ids = nullptr;       // [R]
    unsigned long long* best = nullptr;
    void* staging = nullptr;

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
    if (c->hidden % 8 || c->intermediate % 8) return qfail(KV_ERR_INVAL, "hidden and intermediate must be multiples of 8");
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

int new_sequence(qw2_model* m) {
    QW_OK(kvp_seq_alloc(m->pool, &m->seq));
    return KV_OK;
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
    DeviceGuard g(m->device);
    if (m->st) cudaStreamSynchronize(m->st);
    if (m->pool) kvp_destroy(m->pool);
    m->release();
    if (m->own_stream && m->st) cudaStreamDestroy(m->st);
    delete m;
    return KV_OK;
}

int qw2_create(int device, const qw2_config* cfg, qw2_model** out) {
    if (!out) return qfail(KV_ERR_INVAL, "NULL out");
    *out = nullptr;
    QW_OK(check_cfg(cfg));
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return qfail(KV_ERR_INVAL, "no CUDA device %d", device);
    DeviceGuard g(device);
    if (!g.ok) return qfail(KV_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    qw2_model* m = new qw2_model();
    m->device = device;
    m->c = *cfg;
    m->kvd = cfg->kv_heads * cfg->head_dim;
    const size_t H = cfg->hidden, kvd = m->kvd, IS = cfg->intermediate, V = cfg->vocab, R = cfg->max_position;
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
    step(m->alloc_n(&m->logits, V));
    step(m->alloc_n(&m->ids, R));
    step(m->alloc_n(&m->best, 1));
    step(m->alloc(&m->staging, kStagingBytes));
    if (rc == KV_OK) {
        if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess)
            rc = qfail(KV_ERR_CUDA, "cudaStreamCreate failed");
        else
            m->own_stream = true;
    }
    if (rc == KV_OK) {
        const int blocks = (cfg->max_position + kBlockTokens - 1) / kBlockTokens;
        step(kvp_create(device, cfg->layers, cfg->q_heads, cfg->kv_heads, cfg->head_dim, kBlockTokens, blocks,
                        KV_F16, 1, cfg->max_position, cfg->rope_theta, &m->pool));
    }
    // every forward ends with a host synchronisation, so no decode launch
    // overlaps a kernel that writes the cache (kvp_set_overlap's contract)
    if (rc == KV_OK) step(kvp_set_overlap(m->pool, 1));
    if (rc == KV_OK) step(new_sequence(m));
    if (rc != KV_OK) {
        const std::string msg = kv_last_error();
        qw2_destroy(m);
        return qfail(rc, "%s", msg.c_str());
    }
    *out = m;
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
    DeviceGuard g(m->device);
    QW_OK(kvp_reset(m->pool, m->st));
    QW_OK(new_sequence(m));
    QW_CUDA(cudaStreamSynchronize(m->st));
    return KV_OK;
}

int qw2_cur_pos(const qw2_model* m, int* pos) {
    if (!m || !pos) return qfail(KV_ERR_INVAL, "NULL argument");
    return kvp_seq_len(m->pool, m->seq, pos);
}

int qw2_forward(qw2_model* m, const int* tokens, int n, float* logits_host, int* argmax) {
    if (!m || !tokens) return qfail(KV_ERR_INVAL, "NULL argument");
    if (n <= 0) return qfail(KV_ERR_INVAL, "forward of %d tokens", n);
    QW_OK(qw2_ready(m));
    const qw2_config& c = m->c;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= c.vocab) return qfail(KV_ERR_RANGE, "token id %d outside [0, %d)", tokens[i], c.vocab);
    int pos = 0;
    QW_OK(kvp_seq_len(m->pool, m->seq, &pos));
    if (pos + n > c.max_position)
        return qfail(KV_ERR_RANGE, "positions %d..%d pass max_position %d", pos, pos + n - 1, c.max_position);
    DeviceGuard g(m->device);
    cudaStream_t st = m->st;
    const int H = c.hidden, kvd = m->kvd, IS = c.intermediate;

    QW_CUDA(cudaMemcpyAsync(m->ids, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, st));
    QW_CUDA(launch_embed(m->ids, n, m->embed, m->hidden, H, st));
    if (n == 1) QW_OK(attn_decode_plan(m->pool, 1, &m->seq, st));
    else QW_OK(kvp_seq_reserve(m->pool, m->seq, pos + n));

    for (int li = 0; li < c.layers; ++li) {
        const qw2_model::Layer& Ly = m->L[li];
        // 1-2: input RMSNorm fused into the Q/K/V projections (+ biases)
        GemvArgs a;
        a.w = Ly.wqkv;
        a.N = H + 2 * kvd;
        a.K = H;
        a.M = n;
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
        if (n == 1) {
            QW_OK(attn_decode_append(m->pool, li, m->q, m->k, m->v, m->attn, st));
        } else {
            QW_OK(kv_append_chunk(m->pool, li, m->seq, pos, n, m->k, m->v, st));
            QW_OK(attn_prefill(m->pool, li, m->seq, pos, n, m->q, m->attn, st));
        }
        // 6-7: O projection + residual
        GemvArgs o;
        o.w = Ly.wo;
        o.N = H;
        o.K = H;
        o.M = n;
        o.x = m->attn;
        o.resid = m->hidden;
        QW_CUDA(launch_gemv(1, 1, o, st));
        // 8-10: post-attention RMSNorm fused into gate/up (+ SiLU product), down + residual
        GemvArgs gu;
        gu.w = Ly.wg;
        gu.w2 = Ly.wu;
        gu.N = IS;
        gu.K = H;
        gu.M = n;
        gu.x = m->hidden;
        gu.norm_w = Ly.ln2;
        gu.eps = c.rms_eps;
        gu.out16 = m->h16;
        QW_CUDA(launch_gemv(2, 2, gu, st));
        GemvArgs d;
        d.w = Ly.wd;
        d.N = H;
        d.K = IS;
        d.M = n;
        d.x = m->h16;
        d.resid = m->hidden;
        QW_CUDA(launch_gemv(1, 0, d, st));
    }
    if (n == 1) QW_OK(attn_decode_commit(m->pool));
    else QW_OK(kvp_seq_set_len(m->pool, m->seq, pos + n));

    // final RMSNorm of the last token fused into lm_head (tied embedding), argmax
    GemvArgs lm;
    lm.w = m->embed;
    lm.N = c.vocab;
    lm.K = H;
    lm.M = 1;
    lm.x = m->hidden + (size_t)(n - 1) * H;
    lm.norm_w = m->norm;
    lm.eps = c.rms_eps;
    lm.logits = m->logits;
    QW_CUDA(launch_gemv(3, 2, lm, st));
    QW_CUDA(launch_argmax(m->logits, c.vocab, m->best, st));
    unsigned long long key = 0;
    QW_CUDA(cudaMemcpyAsync(&key, m->best, sizeof key, cudaMemcpyDeviceToHost, st));
    if (logits_host)
        QW_CUDA(cudaMemcpyAsync(logits_host, m->logits, sizeof(float) * (size_t)c.vocab, cudaMemcpyDeviceToHost, st));
    int status = 0;
    QW_OK(kvp_device_status(m->pool, st, &status));  // synchronises the stream
    if (status != 0) return status;
    if (argmax) *argmax = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu)) : 0;
    return KV_OK;
}

int qw2_generate(qw2_model* m, const int* prompt, int n_prompt, int max_new, const int* stop_tokens, int n_stop,
                 int repetition_window, int* out_ids, int cap, int* n_out) {
    if (!m || !n_out || (n_stop > 0 && !stop_tokens) || (cap > 0 && !out_ids))
        return qfail(KV_ERR_INVAL, "NULL argument");
    *n_out = 0;
    if (n_prompt <= 0 || !prompt) return KV_OK;  // llm_engine.cpp:59
    auto is_stop = [&](int id) {
        for (int i = 0; i < n_stop; ++i)
            if (stop_tokens[i] == id) return true;
        return false;
    };
    int next = 0;
    QW_OK(qw2_forward(m, prompt, n_prompt, nullptr, &next));
    std::vector<int> out;
    for (int step = 0; step < max_new; ++step) {
        if (is_stop(next)) break;
        out.push_back(next);
        if (repetition_window > 0 && detect_repetition(out, repetition_window)) break;
        const int id = next;
        QW_OK(qw2_forward(m, &id, 1, nullptr, &next));
    }
    for (size_t i = 0; i < out.size() && (int)i < cap; ++i) out_ids[i] = out[i];
    *n_out = (int)out.size();
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
