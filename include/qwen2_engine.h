/* qwen2_engine.h -- the Qwen2 model and its greedy engine on one B200 (C ABI).
 *
 * Replaces the reference's model and engine for one sequence at a time:
 *   Qwen2Model   worker/include/model/qwen2_model.h:23-56   (load, reset_kv_cache, forward)
 *   LLMEngine    worker/include/api/llm_engine.h            (generate)
 *   Qwen2Config  worker/include/core/model_config.h:8-23
 *   ILinearOp    worker/include/ops/op_linear.h             (every projection, on the device)
 * Weights, KV cache (a kvattn paged pool, fp16) and activations live in HBM;
 * one forward is a sequence of stream-ordered kernel launches (RMSNorm,
 * GEMVs with fused bias / residual / SiLU epilogues, the fused RoPE + append +
 * attention of kvattn.h, lm_head, greedy argmax).
 *
 * Numerics follow the reference's forward (qwen2_model.cpp:131-274) with its
 * linear contract: each projection takes fp16 inputs (the reference's
 * truncating f32_to_f16, half.h), multiplies fp16 weights with fp32
 * accumulation and rounds the result to fp16 with the same truncation;
 * biases, residuals, RMSNorm and SiLU stay fp32.  Only the order of the fp32
 * sums differs from a sequential loop.
 *
 * Status codes and kv_last_error() are those of kvattn.h.
 */
#ifndef QWEN2_ENGINE_H
#define QWEN2_ENGINE_H

#include <stdint.h>

#include "kvattn.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct qw2_model qw2_model;

/* Qwen2Config (model_config.h:8-23).  Constraints here: head_dim 128,
 * hidden == q_heads * head_dim, hidden and intermediate multiples of 8,
 * q_heads / kv_heads <= 8. */
typedef struct qw2_config {
    int hidden;        /* 1536 */
    int layers;        /* 28 */
    int q_heads;       /* 12 */
    int kv_heads;      /* 2 */
    int head_dim;      /* 128 */
    int intermediate;  /* 8960 */
    int vocab;         /* 151936 */
    float rms_eps;     /* 1e-6 */
    float rope_theta;  /* 1e6 */
    int max_position;  /* 512: KV capacity in tokens (kv_cache_.init, qwen2_model.cpp:115) */
} qw2_config;

/* Tensor dtypes accepted by qw2_set_tensor (the safetensors dtypes the
 * reference loader accepts, weight_loader.cpp:184-194). */
enum { QW2_F16 = 0, QW2_BF16 = 1, QW2_F32 = 2 };

/* The reference's defaults (Qwen2-1.5B). */
int qw2_config_default(qw2_config* cfg);

/* Allocate the model on `device`: weights (uninitialised until set), the
 * fp16 KV pool with one sequence, activations.  Qwen2Model() + the
 * allocation half of Qwen2Model::load. */
int qw2_create(int device, const qw2_config* cfg, qw2_model** out);
int qw2_destroy(qw2_model* m);

/* Run on this stream from now on (default: a stream the model created). */
int qw2_set_stream(qw2_model* m, void* stream);

/* One tensor from host memory, named as in the safetensors file
 * (qwen2_model.cpp:72-111: model.embed_tokens.weight, model.layers.<i>.
 * input_layernorm.weight, ...self_attn.{q,k,v}_proj.{weight,bias},
 * ...self_attn.o_proj.weight, ...post_attention_layernorm.weight,
 * ...mlp.{gate,up,down}_proj.weight, model.norm.weight).  Shape as in the
 * file ([out][in] for matrices).  Matrices are stored as fp16 with the
 * loader's conversions (load_tensor_f16: BF16 -> bf16_to_f16, F32 ->
 * f32_to_f16, F16 as is except that subnormal fp16 values become signed
 * zero); vectors as fp32 (load_tensor_f32).  lm_head is the embedding
 * (tied, qwen2_model.cpp:109-112). */
int qw2_set_tensor(qw2_model* m, const char* name, int dtype, const int64_t* shape, int ndim,
                   const void* host_data);

/* Qwen2Model::load: every tensor of <path> (a model.safetensors file) that
 * the model uses.  KV_ERR_INVAL if one is missing or malformed. */
int qw2_load_safetensors(qw2_model* m, const char* path);

/* KV_OK when every tensor has been set, else KV_ERR_STATE naming a missing one. */
int qw2_ready(qw2_model* m);

/* Qwen2Model::reset_kv_cache (qwen2_model.cpp:44-46): position 0, cache zeroed. */
int qw2_reset(qw2_model* m);
int qw2_cur_pos(const qw2_model* m, int* pos);

/* Qwen2Model::forward (qwen2_model.cpp:131-274): run n tokens at positions
 * cur_pos.. and advance cur_pos by n.  n == 1 uses the fused decode
 * attention, n > 1 the chunked-prefill append + attention.  Writes the last
 * token's fp32 logits to `logits_host` (vocab floats, may be NULL) and their
 * greedy argmax (op_greedy_sample, op_sampling.cpp:4-11) to `argmax` (may
 * be NULL).  KV_ERR_RANGE if a token id is outside [0, vocab) or the
 * positions would pass max_position. */
int qw2_forward(qw2_model* m, const int* tokens, int n, float* logits_host, int* argmax);

/* LLMEngine::generate (llm_engine.cpp:53-103): prefill `prompt`, then up to
 * max_new greedy tokens, stopping at a stop token (not emitted) or when the
 * last `repetition_window` ids repeat with a period <= window/2 (0
 * disables).  Generated ids go to out_ids (cap entries), their count to
 * n_out.  Does not reset the cache first (the reference does not either). */
int qw2_generate(qw2_model* m, const int* prompt, int n_prompt, int max_new, const int* stop_tokens,
                 int n_stop, int repetition_window, int* out_ids, int cap, int* n_out);

/* The model's KV pool (sequence 0), for inspection with kvp_gather etc. */
int qw2_kv_pool(qw2_model* m, kvp_pool** pool);

/* Bytes of weights one decode step reads (all projections + lm_head). */
int qw2_weight_bytes(const qw2_model* m, long long* bytes);

#ifdef __cplusplus
}
#endif

#endif /* QWEN2_ENGINE_H */
