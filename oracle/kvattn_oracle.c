/*
 * kvattn_oracle.c -- CPU restatement of the reference's decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it.  The product library never links or calls it.
 *
 * What it restates (paths are relative to the Bobchasm/rk3588-npu project):
 *   - fp16/bf16 <-> fp32 conversions        worker/include/core/half.h:10-48
 *   - RoPE (NeoX half-split pairing)       worker/src/ops/op_rope.cpp:8-30
 *   - row softmax                          worker/src/ops/op_softmax.cpp:6-16
 *   - causal GQA attention                 worker/src/ops/op_attention.cpp:9-56
 *   - KV append loop at the call site      worker/src/model/qwen2_model.cpp:180-206
 *   - INT8 KV (planned by the reference, docs/work_division.md:72): the
 *     scheme the device implements, restated (orc_quantize_i8 ...)
 *
 * The loops keep the reference's accumulation order exactly, so with
 * `-O2 -ffp-contract=off` on x86-64 this file reproduces the reference
 * bit-for-bit (pinned in tests/test_oracle.py against the reference compiled
 * from its own sources and against the committed golden vectors).
 *
 * The bf16 KV variants are a restatement beyond the reference (which stores
 * fp16 only): identical loops with half.h's bf16 encoder/decoder
 * (truncating f32->bf16 at half.h:17-20, shift decode at half.h:12-15).
 */
#include <math.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_F16 0
#define ORC_BF16 1

/* ---- half.h:12-15 ---- */
float orc_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* ---- half.h:17-20: truncation, no rounding ---- */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    return (uint16_t)(u >> 16);
}

/* ---- half.h:24-32: mantissa truncation, exp<=0 -> signed zero,
 *      exp>=31 -> signed inf (NaN becomes inf) ---- */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    int32_t e = (int32_t)((x >> 23) & 0xFFu) - 127 + 15;
    uint32_t mant = x & 0x7FFFFFu;
    if (e <= 0) return sign;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | (uint16_t)((e << 10) | (mant >> 13)));
}

/* ---- half.h:34-43: exp==0 is decoded as sign|(mant<<13), which is not the
 *      IEEE value of an fp16 subnormal; kept as the reference has it ---- */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t x;
    if (e == 0) x = sign | (mant << 13);
    else if (e == 31) x = sign | 0x7F800000u | (mant << 13);
    else x = sign | ((e + 112u) << 23) | (mant << 13);
    float r;
    memcpy(&r, &x, sizeof r);
    return r;
}

static inline float dec(uint16_t v, int dtype) {
    return dtype == ORC_BF16 ? orc_bf16_to_f32(v) : orc_f16_to_f32(v);
}

static inline uint16_t enc(float v, int dtype) {
    return dtype == ORC_BF16 ? orc_f32_to_bf16(v) : orc_f32_to_f16(v);
}

void orc_encode(const float* src, uint16_t* dst, long n, int dtype) {
    for (long i = 0; i < n; ++i) dst[i] = enc(src[i], dtype);
}

void orc_decode(const uint16_t* src, float* dst, long n, int dtype) {
    for (long i = 0; i < n; ++i) dst[i] = dec(src[i], dtype);
}

/* ---- op_rope.cpp:8-19: one head, pairs (v[i], v[i+half]) ---- */
static void rope_one_head(float* v, int head_dim, int pos, float theta) {
    const int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
        float angle = (float)pos * freq;
        float c = cosf(angle);
        float s = sinf(angle);
        float v0 = v[i];
        float v1 = v[i + half];
        v[i] = v0 * c - v1 * s;
        v[i + half] = v0 * s + v1 * c;
    }
}

/* ---- op_rope.cpp:21-30 ---- */
void orc_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_dim,
              int pos, float theta) {
    for (int h = 0; h < n_heads; ++h) rope_one_head(q + h * head_dim, head_dim, pos, theta);
    for (int h = 0; h < n_kv_heads; ++h) rope_one_head(k + h * head_dim, head_dim, pos, theta);
}

/* The cos/sin values rope_one_head uses for (pos, i): the same three libm
 * calls in float, laid out [npos][half] cos then [npos][half] sin.  Used by
 * the tests to check the product's host-built table value for value. */
void orc_rope_table(float theta, int head_dim, int pos0, int npos, float* cos_out,
                    float* sin_out) {
    const int half = head_dim / 2;
    for (int p = 0; p < npos; ++p)
        for (int i = 0; i < half; ++i) {
            float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
            float angle = (float)(pos0 + p) * freq;
            cos_out[(long)p * half + i] = cosf(angle);
            sin_out[(long)p * half + i] = sinf(angle);
        }
}

/* ---- op_softmax.cpp:6-16 (std::max(a,b) == (a<b)?b:a) ---- */
void orc_softmax(float* x, int rows, int cols) {
    for (int r = 0; r < rows; ++r) {
        float* row = x + (long)r * cols;
        float mx = -FLT_MAX;
        for (int i = 0; i < cols; ++i) mx = (mx < row[i]) ? row[i] : mx;
        float sum = 0.0f;
        for (int i = 0; i < cols; ++i) {
            row[i] = expf(row[i] - mx);
            sum += row[i];
        }
        float inv = 1.0f / sum;
        for (int i = 0; i < cols; ++i) row[i] *= inv;
    }
}

/* ---- op_attention.cpp:9-56; dtype selects the cache decoder ----
 * q [seq][n_heads*head_dim] fp32, caches [total_len][n_kv_heads*head_dim],
 * out [seq][n_heads*head_dim] fp32.  Returns 0, or -1 if scratch allocation
 * fails. */
int orc_attention(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                  float* out, int seq, int total_len, int n_heads, int n_kv_heads,
                  int head_dim, int pos_base, int dtype) {
    const int hidden = n_heads * head_dim;
    const int kv_dim = n_kv_heads * head_dim;
    const float scale = 1.0f / sqrtf((float)head_dim);
    memset(out, 0, sizeof(float) * (size_t)seq * hidden);
    float* scores = (float*)malloc(sizeof(float) * ((size_t)seq * total_len + 1));
    if (!scores) return -1;
    for (int h = 0; h < n_heads; ++h) {
        int kv_h = h / (n_heads / n_kv_heads);
        for (int sq = 0; sq < seq; ++sq) {
            int abs_sq = pos_base + sq;
            for (int sk = 0; sk < total_len; ++sk) {
                if (sk > abs_sq) {
                    scores[(long)sq * total_len + sk] = -1e9f;
                    continue;
                }
                float dot = 0.0f;
                const float* qh = q + (long)sq * hidden + h * head_dim;
                const uint16_t* kh = k_cache + (long)sk * kv_dim + kv_h * head_dim;
                for (int d = 0; d < head_dim; ++d) dot += qh[d] * dec(kh[d], dtype);
                scores[(long)sq * total_len + sk] = dot * scale;
            }
        }
        orc_softmax(scores, seq, total_len);
        for (int sq = 0; sq < seq; ++sq) {
            float* out_row = out + (long)sq * hidden + h * head_dim;
            for (int sk = 0; sk < total_len; ++sk) {
                const uint16_t* vh = v_cache + (long)sk * kv_dim + kv_h * head_dim;
                float w = scores[(long)sq * total_len + sk];
                for (int d = 0; d < head_dim; ++d) out_row[d] += w * dec(vh[d], dtype);
            }
        }
    }
    free(scores);
    return 0;
}

/* ---- qwen2_model.cpp:180-200: RoPE each new token at pos+s, then write the
 * encoded K/V rows at (pos+s)*kv_dim.  q and k are rotated IN PLACE, as the
 * reference's op_rope does. ---- */
void orc_rope_append(float* q, float* k, const float* v, uint16_t* k_cache,
                     uint16_t* v_cache, int seq, int pos, int n_heads, int n_kv_heads,
                     int head_dim, float theta, int dtype) {
    const int hidden = n_heads * head_dim;
    const int kv_dim = n_kv_heads * head_dim;
    for (int s = 0; s < seq; ++s)
        orc_rope(q + (long)s * hidden, k + (long)s * kv_dim, n_heads, n_kv_heads, head_dim,
                 pos + s, theta);
    for (int s = 0; s < seq; ++s) {
        const float* ksrc = k + (long)s * kv_dim;
        const float* vsrc = v + (long)s * kv_dim;
        uint16_t* kdst = k_cache + (long)(pos + s) * kv_dim;
        uint16_t* vdst = v_cache + (long)(pos + s) * kv_dim;
        for (int d = 0; d < kv_dim; ++d) {
            kdst[d] = enc(ksrc[d], dtype);
            vdst[d] = enc(vsrc[d], dtype);
        }
    }
}

/* ---- qwen2_model.cpp:180-206 as one call: steps 3 (RoPE), 4 (append) and
 * 5 (attention) of one layer for `seq` new tokens starting at `pos`.
 * The caches are contiguous [capacity][kv_dim] rows, the reference layout. */
int orc_layer_step(float* q, float* k, const float* v, uint16_t* k_cache,
                   uint16_t* v_cache, float* out, int seq, int pos, int n_heads,
                   int n_kv_heads, int head_dim, float theta, int dtype) {
    orc_rope_append(q, k, v, k_cache, v_cache, seq, pos, n_heads, n_kv_heads, head_dim,
                    theta, dtype);
    return orc_attention(q, k_cache, v_cache, out, seq, pos + seq, n_heads, n_kv_heads,
                         head_dim, pos, dtype);
}

/* Merge G partial states (m, l, o) per row, the log-sum-exp combine the
 * split-KV paths use: o are normalised outputs, m the row max of the scaled
 * scores, l = sum exp(s - m).  Double precision: this is a checker. */
void orc_lse_combine(const float* m, const float* l, const float* o, int G, int rows,
                     int dim, float* out) {
    for (int r = 0; r < rows; ++r) {
        double M = -INFINITY;
        for (int g = 0; g < G; ++g)
            if (l[(long)g * rows + r] > 0 && m[(long)g * rows + r] > M) M = m[(long)g * rows + r];
        double L = 0;
        for (int g = 0; g < G; ++g)
            if (l[(long)g * rows + r] > 0) L += l[(long)g * rows + r] * exp(m[(long)g * rows + r] - M);
        for (int d = 0; d < dim; ++d) {
            double acc = 0;
            for (int g = 0; g < G; ++g) {
                double lg = l[(long)g * rows + r];
                if (lg > 0)
                    acc += lg * exp(m[(long)g * rows + r] - M) * o[((long)g * rows + r) * dim + d];
            }
            out[(long)r * dim + d] = (float)(L > 0 ? acc / L : 0.0);
        }
    }
}

/* ---- INT8 KV cache ----
 * The reference plans an FP16 -> INT8 KV compression to cut memory traffic
 * (docs/work_division.md:72, docs/worker_arch.md:330: a QuantizedKVCache
 * behind the same interface) but ships no implementation, so this restates
 * the scheme the device implements:
 *   one fp32 scale per (token, KV head) row of head_dim values,
 *   scale = max|x| / 127, code = round-half-away(x / scale) clamped to
 *   [-127, 127] (0 for an all-zero row or a NaN element),
 *   dequantised value = code * scale.
 * K is quantised after RoPE, like the 16-bit append.  Every operation is
 * exactly rounded (fabsf, fmaxf, division, roundf), so the device's codes and
 * scales are reproducible bit for bit. */
void orc_quantize_i8(const float* x, int n, int8_t* q, float* scale) {
    float amax = 0.0f;
    for (int i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const float s = amax / 127.0f;
    *scale = s;
    for (int i = 0; i < n; ++i) {
        float r = (s > 0.0f) ? roundf(x[i] / s) : 0.0f;
        if (r != r) r = 0.0f;
        if (r > 127.0f) r = 127.0f;
        if (r < -127.0f) r = -127.0f;
        q[i] = (int8_t)r;
    }
}

/* op_attention (op_attention.cpp:9-56) over INT8 caches: the same loops with
 * every cached value dequantised as code * scale.  kq/vq [T][kv_dim] codes,
 * ks/vs [T][n_kv_heads] scales. */
int orc_attention_i8(const float* q, const int8_t* kq, const float* ks, const int8_t* vq,
                     const float* vs, float* out, int seq, int total_len, int n_heads,
                     int n_kv_heads, int head_dim, int pos_base) {
    const int hidden = n_heads * head_dim;
    const int kv_dim = n_kv_heads * head_dim;
    const float scale = 1.0f / sqrtf((float)head_dim);
    memset(out, 0, sizeof(float) * (size_t)seq * hidden);
    float* scores = (float*)malloc(sizeof(float) * ((size_t)seq * total_len + 1));
    if (!scores) return -1;
    for (int h = 0; h < n_heads; ++h) {
        int kv_h = h / (n_heads / n_kv_heads);
        for (int sq = 0; sq < seq; ++sq) {
            int abs_sq = pos_base + sq;
            for (int sk = 0; sk < total_len; ++sk) {
                if (sk > abs_sq) {
                    scores[(long)sq * total_len + sk] = -1e9f;
                    continue;
                }
                float dot = 0.0f;
                const float* qh = q + (long)sq * hidden + h * head_dim;
                const int8_t* kh = kq + (long)sk * kv_dim + kv_h * head_dim;
                const float kscale = ks[(long)sk * n_kv_heads + kv_h];
                for (int d = 0; d < head_dim; ++d) dot += qh[d] * ((float)kh[d] * kscale);
                scores[(long)sq * total_len + sk] = dot * scale;
            }
        }
        orc_softmax(scores, seq, total_len);
        for (int sq = 0; sq < seq; ++sq) {
            float* out_row = out + (long)sq * hidden + h * head_dim;
            for (int sk = 0; sk < total_len; ++sk) {
                const int8_t* vh = vq + (long)sk * kv_dim + kv_h * head_dim;
                const float vscale = vs[(long)sk * n_kv_heads + kv_h];
                float w = scores[(long)sq * total_len + sk];
                for (int d = 0; d < head_dim; ++d) out_row[d] += w * ((float)vh[d] * vscale);
            }
        }
    }
    free(scores);
    return 0;
}

/* One layer step over INT8 caches: RoPE at pos+s, quantise and append every
 * (token, KV head) row, attend over pos+seq. */
int orc_layer_step_i8(float* q, float* k, const float* v, int8_t* kq, float* ks, int8_t* vq,
                      float* vs, float* out, int seq, int pos, int n_heads, int n_kv_heads,
                      int head_dim, float theta) {
    const int hidden = n_heads * head_dim;
    const int kv_dim = n_kv_heads * head_dim;
    for (int s = 0; s < seq; ++s)
        orc_rope(q + (long)s * hidden, k + (long)s * kv_dim, n_heads, n_kv_heads, head_dim,
                 pos + s, theta);
    for (int s = 0; s < seq; ++s)
        for (int hh = 0; hh < n_kv_heads; ++hh) {
            const long row = (long)(pos + s);
            orc_quantize_i8(k + (long)s * kv_dim + hh * head_dim, head_dim,
                            kq + row * kv_dim + hh * head_dim, ks + row * n_kv_heads + hh);
            orc_quantize_i8(v + (long)s * kv_dim + hh * head_dim, head_dim,
                            vq + row * kv_dim + hh * head_dim, vs + row * n_kv_heads + hh);
        }
    return orc_attention_i8(q, kq, ks, vq, vs, out, seq, pos + seq, n_heads, n_kv_heads,
                            head_dim, pos);
}
