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
 * hidden == q_heads * head_dim, hidden and intermediate multiples of 32,
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

/* on != 0: every forward from now on repeats the reference's float
 * operations in the reference's order (Qwen2Model::forward,
 * qwen2_model.cpp:131-274: RMSNorm, projections and attention with their
 * sums taken sequentially, separately rounded products, softmax and SiLU
 * with the exp of this process's C library), so the logits equal those of
 * the reference's own loops on this host bit for bit -- a parity mode, far
 * slower than the default forward.  Groups of one engine step run one after
 * another.  Needs the fp16 KV cache.  The first call with on != 0 allocates
 * the mode's buffers and, once per process, finds the float inputs where the
 * C library's expf is not correctly rounded (a scan of every float with a
 * finite, nonzero exp on all host threads: seconds). */
int qw2_set_exact(qw2_model* m, int on);

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

/* The model's KV pool, for inspection with kvp_gather etc.; qw2_session_seq
 * gives a session's sequence id in it. */
int qw2_kv_pool(qw2_model* m, kvp_pool** pool);

/* ------------------------------------------------------------ sessions
 * The reference plans multi-session, batch and async interfaces on top of
 * LLMEngine (docs/api_requirements.md:90-151: create_session /
 * destroy_session / session_exists, generate_session, generate_batch,
 * generate_async + cancel_generation).  Here a session is one sequence of
 * the model's paged KV pool; qw2_create's model has one session (id 0, the
 * one qw2_forward / qw2_generate / qw2_reset use), qw2_create_sessions's has
 * up to max_sessions, all sharing the weights. */
int qw2_create_sessions(int device, const qw2_config* cfg, int max_sessions, qw2_model** out);
/* The same with the KV cache in another element type: KV_F16 (the
 * reference's KVCache, what qw2_create_sessions uses), KV_BF16, or KV_I8 --
 * the INT8 compression the reference plans (docs/work_division.md:72; the
 * scheme of kvattn.h), a quarter of the fp16 cache's bytes per token plus
 * one fp32 scale per (token, KV head) row.  The prompt and decode paths are
 * the same calls; only the cache changes, so the logits move by the
 * quantisation error. */
int qw2_create_kv(int device, const qw2_config* cfg, int max_sessions, int kv_dtype, qw2_model** out);
int qw2_session_create(qw2_model* m, int* session);
int qw2_session_destroy(qw2_model* m, int session);
int qw2_session_exists(const qw2_model* m, int session, int* exists);
int qw2_session_len(const qw2_model* m, int session, int* len);
int qw2_session_seq(const qw2_model* m, int session, int* seq_id);
/* Qwen2Model::forward on one session (its cache continues). */
int qw2_forward_session(qw2_model* m, int session, const int* tokens, int n, float* logits_host, int* argmax);

/* GenerationConfig (worker/include/api/generation_config.h:9-25) and
 * GenerationResult (generation_config.h:28-36). */
typedef struct qw2_gen_config {
    int max_new_tokens;
    int repetition_window;  /* 0 disables */
    const int* stop_tokens;
    int n_stop;
} qw2_gen_config;

typedef struct qw2_result {
    int n_out;           /* generated ids (the first out_cap are stored) */
    int prefill_tokens;
    int decode_tokens;
    float prefill_ms;    /* host clock; in a batch the forwards are shared */
    float decode_ms;
    int hit_stop;
    int hit_repetition;
    int cancelled;
    int status;          /* KV_OK, or the status that ended the request */
} qw2_result;

/* TokenCallback (llm_engine.h): called after the forward of each generated
 * id, with its decode step and the step's host time. */
typedef void (*qw2_token_cb)(void* user, int session, int step, int id, float elapsed_ms);

typedef struct qw2_request {
    int session;
    const int* input_ids;
    int n_input;
    qw2_gen_config cfg;
    int* out_ids;        /* generate_batch: where the generated ids go */
    int out_cap;
    qw2_token_cb on_token;
    void* user;
} qw2_request;

/* generate_session: LLMEngine::generate's loop on a session whose cache holds
 * the earlier turns (the input is appended at the session's position). */
int qw2_generate_session(qw2_model* m, int session, const int* input_ids, int n_input, const qw2_gen_config* cfg,
                         int* out_ids, int out_cap, qw2_result* result);
/* generate_batch: every request at once (distinct sessions).  Each engine
 * step runs one forward over all of them: one-token rows of the decoding
 * requests share every projection and one planned decode-attention launch;
 * prompts are appended in chunks of up to 256 tokens beside them. */
int qw2_generate_batch(qw2_model* m, int n_requests, const qw2_request* requests, qw2_result* results);
/* generate_async: queue a request (input and stop ids are copied) and return
 * at once; a worker thread runs every queued request, batched as above.
 * qw2_wait blocks up to timeout_ms (< 0: no limit) for job `job`: KV_OK with
 * its ids and result when it finished (the job is then retired),
 * KV_ERR_TIMEOUT if still running.  qw2_cancel ends the session's queued or
 * running request at the next step (result.cancelled = 1). */
int qw2_submit(qw2_model* m, const qw2_request* request, int* job);
int qw2_wait(qw2_model* m, int job, int timeout_ms, int* out_ids, int out_cap, qw2_result* result);
int qw2_cancel(qw2_model* m, int session);

/* Bytes of weights one decode step reads (all projections + lm_head). */
int qw2_weight_bytes(const qw2_model* m, long long* bytes);

#ifdef __cplusplus
}
#endif

#endif /* QWEN2_ENGINE_H */
