/*
 * kvattn.h -- C ABI of the B200 decode hot path: a paged KV-cache block pool
 * with on-device RoPE'd append, and grouped-query split-KV decode attention.
 *
 * It replaces, behind plain C entry points, the Qwen2 worker's
 *   KVCache                 worker/include/model/kv_cache.h:19-41
 *                           worker/src/model/kv_cache.cpp:4-16
 *   op_rope                 worker/include/ops/op_rope.h:17-19
 *   the KV append loop      worker/src/model/qwen2_model.cpp:188-200
 *   op_attention            worker/include/ops/op_attention.h:19-26
 *                           (with op_softmax, worker/src/ops/op_softmax.cpp:6-16)
 * and the call-site contract around them (qwen2_model.cpp:140-141,203-206,268:
 * the position is read before the layers and advanced once after the last).
 *
 * Conventions
 *  - Every function returns an int status (KV_OK == 0).  kv_last_error()
 *    gives the message of the calling thread's last failure.
 *  - Tensors are DEVICE pointers on the pool's device; host pointers are used
 *    only for control arguments (sequence ids, block ids, counts).
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    Device work is stream-ordered; a decode step's plan, layer calls and any
 *    gather of its results must be issued on one stream.
 *  - One pool per GPU.  Host calls on one pool are serialised internally.
 *  - Numerics (the reference's, kept bit-exact where they are integer work):
 *    appended K is RoPE'd in fp32 with non-fused multiply/add, using cos/sin
 *    values computed on the host with the same float libm calls as
 *    op_rope.cpp:11-14, then stored with half.h's TRUNCATING encoders
 *    (f32_to_f16 half.h:24-32, or f32_to_bf16 half.h:17-20); V is stored the
 *    same way without rotation.  Attention reads fp32 q, decodes the cache to
 *    fp32 and accumulates in fp32; outputs are fp32.
 */
#ifndef KVATTN_H
#define KVATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kvp_pool kvp_pool; /* opaque: one paged KV pool on one GPU */

enum kv_status {
    KV_OK = 0,
    KV_ERR_INVAL = 1,   /* bad argument or unsupported shape */
    KV_ERR_OOM = 2,     /* the pool has too few free blocks (nothing was changed) */
    KV_ERR_BADSEQ = 3,  /* sequence id unknown or not live */
    KV_ERR_CUDA = 4,    /* a CUDA runtime call failed */
    KV_ERR_RANGE = 5,   /* position beyond max_seq_len or beyond reserved blocks */
    KV_ERR_STATE = 6,   /* call order violated (e.g. layer call without a plan) */
    KV_ERR_TIMEOUT = 7  /* a device-side bounded wait gave up (see kvp_device_status) */
};

/* KV cache element types.  KV_I8: the INT8 compression the reference plans
 * (docs/work_division.md:72): per (token, KV head) row of 128 values one fp32
 * scale = max|x| / 127 and codes round-half-away(x / scale) in [-127, 127];
 * attention reads code * scale.  INT8 pools serve the decode path
 * (attn_decode_*), the prompt path (kv_append_chunk(_batch), and
 * attn_prefill(_batch) / attn_prefill_mma on the mma.sync prefill kernel)
 * and kvp_import_i8 / kvp_gather_i8; the 16-bit import / gather reject them. */
enum kv_dtype { KV_F16 = 0, KV_BF16 = 1, KV_I8 = 2 };

/* Pass as `device` to kvp_create for a bookkeeping-only pool: allocator,
 * block tables and decode planning run on the host with no device memory
 * (plans are sized for a nominal 148-SM part).  Data-movement and attention
 * calls on it return KV_ERR_STATE.  Used to test host logic without a GPU. */
#define KVP_HOST_ONLY (-1)

/* Message for the calling thread's last non-OK status ("" if none). */
const char* kv_last_error(void);
/* Process-wide number of CUDA kernels this library has launched (every
 * entry point that launches counts its kernels). */
int kv_kernel_count(long long* n);
/* Static name of a status code. */
const char* kv_status_str(int status);
/* Library version, "major.minor.patch". */
const char* kv_version(void);

/* ------------------------------------------------------------------ pool */

/* Create a pool on `device`.  Replaces KVCache::init (kv_cache.h:21,
 * kv_cache.cpp:4-10): the contiguous per-layer [capacity][kv_dim] arrays
 * become `num_blocks` blocks of `block_tokens` token rows shared by all
 * sequences, zero-filled like init's assign(..., 0).
 * Supported shapes: head_dim 128, block_tokens 16, num_q_heads a multiple of
 * num_kv_heads with num_q_heads/num_kv_heads <= 8.  max_seq_len bounds any
 * position (it sizes the RoPE table and the per-sequence block table). */
int kvp_create(int device, int num_layers, int num_q_heads, int num_kv_heads, int head_dim,
               int block_tokens, int num_blocks, int dtype, int max_seqs, int max_seq_len,
               float rope_theta, kvp_pool** out);
int kvp_destroy(kvp_pool* pool);

/* Free every sequence and zero the pool's K/V memory (KVCache::reset,
 * kv_cache.cpp:12-16).  Stream-ordered. */
int kvp_reset(kvp_pool* pool, void* stream);

/* Pool facts: number of free blocks / total blocks. */
int kvp_free_blocks(const kvp_pool* pool, int* n_free);
int kvp_num_blocks(const kvp_pool* pool, int* n_blocks);

/* Device pointers of the raw storage, for callers that manage layout
 * themselves (tests, zero-copy consumers).  Layout of one layer:
 * [num_blocks][num_kv_heads][4096-byte tile]; a tile holds 16 token rows of
 * 128 dims in the swizzled order documented in the design notes. */
int kvp_storage(const kvp_pool* pool, void** k_base, void** v_base, size_t* layer_bytes);

/* ------------------------------------------------------------- sequences */

/* A new empty sequence (length 0).  KVCache has exactly one implicit
 * sequence; the pool holds up to max_seqs. */
int kvp_seq_alloc(kvp_pool* pool, int* seq_id);
/* Return the sequence's blocks to the free list and retire the id. */
int kvp_seq_free(kvp_pool* pool, int seq_id);
/* Grow the sequence's block table to hold n_tokens positions, taking blocks
 * from the free list (all or nothing: KV_ERR_OOM leaves it unchanged). */
int kvp_seq_reserve(kvp_pool* pool, int seq_id, int n_tokens);
/* Append explicit block ids (each must be free) to the sequence's table,
 * e.g. a random permutation of the pool.  All or nothing. */
int kvp_seq_set_blocks(kvp_pool* pool, int seq_id, const int* block_ids, int n);
/* Current length: KVCache::cur_pos / set_cur_pos (kv_cache.h:24-25).  A new
 * length may not exceed the reserved capacity. */
int kvp_seq_len(const kvp_pool* pool, int seq_id, int* len);
int kvp_seq_set_len(kvp_pool* pool, int seq_id, int len);
/* Copy the host block table of a sequence (n_out receives its length). */
int kvp_seq_blocks(const kvp_pool* pool, int seq_id, int* block_ids, int cap, int* n_out);

/* --------------------------------------------------------- data movement */

/* Write n already-encoded rows [n][num_kv_heads*128] (the reference layout
 * of k_ptr(layer)/v_ptr(layer), kv_cache.h:30-33) at positions pos0.. of a
 * sequence.  Blocks must be reserved.  Does not change the length. */
int kvp_import(kvp_pool* pool, int layer, int seq_id, int pos0, int n, const void* k_rows,
               const void* v_rows, void* stream);
/* Read positions [0, len) of a sequence back into the reference layout
 * [len][num_kv_heads*128] (what k_ptr(layer)/v_ptr(layer) would hold). */
int kvp_gather(kvp_pool* pool, int layer, int seq_id, void* k_rows, void* v_rows,
               void* stream);

/* INT8 pools: the same, with codes [n][num_kv_heads*128] int8 (16-byte
 * aligned) and scales [n][num_kv_heads] fp32 for K and for V. */
int kvp_import_i8(kvp_pool* pool, int layer, int seq_id, int pos0, int n, const void* k_codes,
                  const void* v_codes, const float* k_scales, const float* v_scales, void* stream);
int kvp_gather_i8(kvp_pool* pool, int layer, int seq_id, void* k_codes, void* v_codes, float* k_scales,
                  float* v_scales, void* stream);

/* Prefill append: RoPE (positions pos0..pos0+n-1) and encode n new tokens'
 * k/v [n][num_kv_heads*128] fp32 into the sequence's blocks, as
 * qwen2_model.cpp:180-200 does for seq=n.  Blocks must be reserved; the
 * length is not changed (set it after the last layer, as qwen2_model.cpp:268). */
int kv_append_chunk(kvp_pool* pool, int layer, int seq_id, int pos0, int n, const float* k,
                    const float* v, void* stream);

/* Causal attention of a prompt chunk over the pool: op_attention with
 * seq = n > 1 (op_attention.cpp:9-56).  Query s sits at position pos0 + s of
 * the sequence and attends to positions [0, pos0 + s]; the chunk's own K/V
 * must already be in the pool for `layer` (kv_append_chunk).  q [n][num_q_heads
 * * 128] fp32 straight from the projections (16-byte aligned): it is rotated
 * here at pos0 + s with the append's RoPE arithmetic.  out [n][num_q_heads *
 * 128] fp32 (both 16-byte aligned).  The length is not changed.  Runs on the
 * 5th-generation tensor cores (tcgen05 MMA with accumulators in tensor memory). */
int attn_prefill(kvp_pool* pool, int layer, int seq_id, int pos0, int n, const float* q,
                 float* out, void* stream);
/* Several prompt chunks at once (chunked prefill of a continuous-batching
 * step): chunk i appends / attends n[i] tokens at positions pos0[i].. of
 * sequence seq_ids[i] (distinct sequences); its rows are rows
 * [n[0] + ... + n[i-1], ... + n[i]) of k / v / q / out, laid out as in the
 * single-chunk calls.  Same results as one call per chunk; the chunks share
 * launches (up to 32 chunks per launch), with the key splits of the
 * attention planned over all of them.  Replaces the per-request loop around
 * the append (qwen2_model.cpp:180-200) and op_attention (op_attention.cpp:
 * 9-56) when several requests prefill in one step. */
int kv_append_chunk_batch(kvp_pool* pool, int layer, int nreq, const int* seq_ids, const int* pos0,
                          const int* n, const float* k, const float* v, void* stream);
int attn_prefill_batch(kvp_pool* pool, int layer, int nreq, const int* seq_ids, const int* pos0,
                       const int* n, const float* q, float* out, void* stream);
/* The same computation on the legacy mma.sync tensor path (the baseline
 * attn_prefill's tcgen05 kernel is measured against). */
int attn_prefill_mma(kvp_pool* pool, int layer, int seq_id, int pos0, int n, const float* q,
                     float* out, void* stream);

/* ---------------------------------------------------------------- decode */

/* Plan one decode step for nseq sequences (host ids).  For each sequence:
 * position p = its length; one block is reserved for p+1 if needed (all or
 * nothing); the split-KV work partition is built on the host and passed to
 * every layer's launch as kernel parameters (nothing is uploaded; block-table
 * entries queued by reserve / set_blocks are applied on `stream`).  The plan
 * stays valid for every layer until the next plan or commit.  A plan of more
 * than 256 sequences runs as one launch per 256 sequences per layer. */
int attn_decode_plan(kvp_pool* pool, int nseq, const int* seq_ids, void* stream);

/* The same with per-sequence control, for a sequence whose positions are
 * split across GPUs: rope_pos[i] is the GLOBAL position of the new token
 * (used for q and k rotation); append[i] = 1 writes the new token at local
 * slot `length` and attends [0, length]; append[i] = 0 attends [0, length)
 * only and writes nothing.  NULL arrays mean rope_pos = length, append = 1. */
int attn_decode_plan_ex(kvp_pool* pool, int nseq, const int* seq_ids, const int* rope_pos,
                        const int* append, void* stream);

/* One layer of the planned step, fused in one launch: RoPE q and the new k,
 * append the encoded k/v row, grouped-query attention over the sequence's
 * blocks with an online softmax, split-KV partials merged on device.
 *   q     [nseq][num_q_heads*128]  fp32 (pre-RoPE, bias added)
 *   k_new [nseq][num_kv_heads*128] fp32 (pre-RoPE, bias added)
 *   v_new [nseq][num_kv_heads*128] fp32
 *   out   [nseq][num_q_heads*128]  fp32
 * Row i belongs to seq_ids[i] of the plan.  Replaces op_rope + the append
 * loop + op_attention for seq=1 (qwen2_model.cpp:180-206). */
int attn_decode_append(kvp_pool* pool, int layer, const float* q, const float* k_new,
                       const float* v_new, float* out, void* stream);

/* The same, also writing each row's softmax state for a cross-GPU merge:
 * m [nseq][num_q_heads] = max of the scaled scores, l = sum of exp(s - m);
 * out holds the normalised partial output.  Rows with nothing to attend get
 * m = -inf, l = 0, out = 0. */
int attn_decode_append_partial(kvp_pool* pool, int layer, const float* q, const float* k_new,
                               const float* v_new, float* out, float* m, float* l,
                               void* stream);

/* Advance the planned sequences by one position (set_cur_pos(total_len),
 * qwen2_model.cpp:268) and retire the plan. */
int attn_decode_commit(kvp_pool* pool);

/* Log-sum-exp merge of G partial states per row (split-KV across GPUs):
 *   m, l [G][rows], o [G][rows][dim] (normalised partial outputs) ->
 *   out [rows][dim] = sum_g l_g e^(m_g-M) o_g / sum_g l_g e^(m_g-M).
 * No reference counterpart (the reference has no split-KV). */
int attn_combine_lse(int G, int rows, int dim, const float* m, const float* l, const float* o,
                     float* out, void* stream);
/* ---- Split-KV across GPUs over peer memory ---------------------------------
 * No counterpart in the reference.  One exchange object per rank (one process
 * per GPU, all on one node): kvx_create allocates this rank's area on
 * `device` for up to max_rows (sequence x query head) rows; kvx_handle gives
 * its CUDA IPC handle (KVX_HANDLE_BYTES bytes) for the caller to pass to the
 * other ranks (e.g. through torch.distributed); kvx_open maps a peer's area.
 * attn_decode_append_xgpu then runs one layer of a sequence-split step: the
 * local decode over this rank's slice (as attn_decode_append_partial), and,
 * launched right behind it, an exchange kernel that pushes every row's
 * (m, l, o) to every peer over NVLink, waits (bounded, ~1 s, then
 * KV_ERR_TIMEOUT in kvp_device_status) for every peer's states of the same
 * call and writes the merged out [rows][128].  Every rank must make the same
 * sequence of calls.  Destroy after a barrier, when no rank calls any more. */
typedef struct kvx_exch kvx_exch;
#define KVX_HANDLE_BYTES 64
int kvx_create(int device, int rank, int world, int max_rows, kvx_exch** out);
int kvx_handle(const kvx_exch* x, void* handle);
int kvx_open(kvx_exch* x, int peer, const void* handle);
int kvx_destroy(kvx_exch* x);
int attn_decode_append_xgpu(kvp_pool* pool, int layer, const float* q, const float* k_new,
                            const float* v_new, float* out, kvx_exch* x, void* stream);

/* ---- Split-KV across GPUs over NCCL -----------------------------------------
 * No counterpart in the reference.  One communicator per rank (one process
 * per GPU): rank 0 makes a unique id with kvn_unique_id and passes its
 * KVN_UNIQUE_ID_BYTES bytes to the other ranks by any means (its own RPC, a
 * file, a framework's broadcast); then every rank calls kvn_create with its
 * rank (a collective: it returns once all ranks joined), for up to max_rows
 * (sequence x query head) rows.  attn_decode_append_nccl then runs one layer
 * of a sequence-split step on `stream`: the local decode over this rank's
 * slice of the planned sequences (as attn_decode_append_partial), an NCCL
 * all-gather of every rank's packed (m, l, o) states, and their log-sum-exp
 * merge into out [rows][128] -- one host call per layer.  Every rank must
 * make the same sequence of calls.  NCCL is loaded at run time (the copy
 * already in the process if there is one, else libnccl.so.2): KV_ERR_STATE
 * if none is found.  Destroy after the last call of every rank. */
typedef struct kvn_comm kvn_comm;
#define KVN_UNIQUE_ID_BYTES 128
int kvn_unique_id(void* id);
int kvn_create(int device, int rank, int world, const void* id, int max_rows, kvn_comm** out);
int kvn_destroy(kvn_comm* c);
int attn_decode_append_nccl(kvp_pool* pool, int layer, const float* q, const float* k_new,
                            const float* v_new, float* out, kvn_comm* c, void* stream);

/* The same merge over the packed buffer an all-gather of per-rank states
 * yields: packed [G][rows*(2+dim)], rank g's part laid out as
 * [m rows][l rows][o rows x dim].  No reference counterpart. */
int attn_combine_lse_packed(int G, int rows, int dim, const float* packed, float* out,
                            void* stream);

/* Attention for callers that cannot allocate device memory (a host that
 * owns all GPU memory in its own arena and forbids plugin allocations, or a
 * decode loop that may not call into the allocator).  It creates no pool and
 * calls no cudaMalloc/cudaFree: split-KV partial states go to a fixed
 * file-scope device array of 4 MiB that every GPU loading this library holds
 * until the process exits.  No counterpart in the reference.  The math: for
 * query row s (absolute position pos_base + s) and query head h of KV group
 * g = h / (n_heads / n_kv_heads), out[s][h] = softmax(q[s][h] . K_g^T /
 * sqrt(128)) V_g over keys 0 .. min(pos_base + s, total_len - 1), with
 * q [seq][n_heads*128] fp32 already rotated, contiguous caches
 * [total_len][n_kv_heads*128] of `dtype` (KV_F16 or KV_BF16) and out
 * [seq][n_heads*128] fp32, all device pointers; q and the caches 16-byte
 * aligned.  Limit: seq * n_kv_heads <= 1008 (else KV_ERR_RANGE).  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress)
 * with that device current, so make that first call before any stream
 * capture; the address is kept for the process, so the entry point is not
 * for use across cudaDeviceReset.  All calls share the array: calls that
 * overlap on the GPU (concurrent streams) race and must be serialised by the
 * caller; nothing in it needs clearing, every value read is written first
 * in the same call. */
int attn_contig_noalloc(const float* q, const void* k_cache, const void* v_cache, float* out,
                        int seq, int total_len, int n_heads, int n_kv_heads, int head_dim,
                        int pos_base, int dtype, void* stream);

/* Device status word of the pool: 0, or KV_ERR_TIMEOUT if a kernel's
 * bounded wait gave up.  Synchronises `stream`; clears the word. */
int kvp_device_status(kvp_pool* pool, void* stream, int* status);

/* The active plan's work list (host copy): number of pieces, CTAs the
 * layer calls launch, new block-table entries, and up to `cap` pieces'
 * (slot, kv head, first block, end block).  Any output pointer may be NULL. */
int kvp_plan_info(const kvp_pool* pool, int* nitems, int* grid, int* npatch, int* item_slot,
                  int* item_head, int* item_b0, int* item_b1, int cap);
/* cta_start[0..grid] of the active plan: CTA g runs pieces
 * [cta_start[g], cta_start[g+1]). */
int kvp_plan_cta_start(const kvp_pool* pool, int* cta_start, int cap);

/* Launch timing: when enabled, CUDA events are recorded on the launching
 * stream immediately before and after every decode launch of this pool.
 * kvp_timing_read synchronises on the last event and returns the summed
 * launch durations (ms) and the launch count since enabling, then resets. */
int kvp_timing_enable(kvp_pool* pool, int enable);

/* With overlap enabled, every decode launch on a created stream (not the
 * legacy default stream) is a programmatic dependent launch: its CTAs start
 * while the previous kernel in the stream finishes and copy their first K/V
 * tiles then, while everything that reads other state that kernel may write
 * (q / k_new / v_new) or writes anything waits for it inside the kernel.
 * Valid when that kernel writes
 * none of this pool's blocks or block-table entries -- or is itself a decode
 * launch (or merge) of this pool: the rows and table entries the previous
 * decode launch of the pool appended are read only after it.  The library
 * turns the early copies off by itself for the first decode launch after any
 * other of its calls that writes the pool (import, prompt append, reset,
 * reserve / set_blocks).  Default off. */
int kvp_set_overlap(kvp_pool* pool, int enable);
int kvp_timing_read(kvp_pool* pool, double* total_ms, int* launches);

/* Number of SMs and of resident decode CTAs per SM used for grid sizing. */
int kvp_launch_info(const kvp_pool* pool, int* num_sms, int* ctas_per_sm);

/* How a decode launch merges a sequence's K/V heads split over several CTAs
 * (long contexts are cut so every SM gets an equal share).  GRID (default):
 * a merge launch right behind the decode launch (a programmatic dependent
 * launch, so the next decode launch's first copies overlap it).  CLUSTER:
 * the planner keeps every split inside a thread-block cluster of 8 CTAs and
 * merges it there over distributed shared memory -- one launch per layer --
 * when the cluster packing balances about as well as the grid-wide cut
 * (else the plan stays GRID).  Measured on B200 for 32 sequences of
 * U[256,4096] tokens, CLUSTER is slower (19.1-19.9 against 18.6 us per
 * step): only 33 clusters of 8 fit at once (264 CTAs against 292), and each
 * next launch can start only in whole free clusters.  Applies to plans made
 * after the call. */
#define KVP_MERGE_GRID 0
#define KVP_MERGE_CLUSTER 1
int kvp_set_merge_mode(kvp_pool* pool, int mode);
/* Merge clusters of the active plan's launches (0: every split merged by
 * the merge launch). */
int kvp_plan_clusters(const kvp_pool* pool, int* clustered_launches, int* launches);

/* ---- Placement of requests onto GPUs --------------------------------------
 * No counterpart in the reference: its engine runs one sequence on one
 * device (worker/src/engine/llm_engine.cpp:68-98).  A request is placed
 * whole on the GPU holding the fewest resident KV blocks among those with
 * room for it (ties: lowest index); its blocks are counted as
 * ceil(tokens / block_tokens).  The state is plain host data: every process
 * that makes the same calls in the same order reaches the same placement,
 * so a scheduler replicated on every rank needs no communication.  Calls on
 * one scheduler are serialised internally.  Request ids are the caller's.
 * An OOM (no GPU has room) changes nothing. */
typedef struct kvs_sched kvs_sched;

int kvs_create(int n_gpus, int block_tokens, const long long* blocks_per_gpu, kvs_sched** out);
int kvs_destroy(kvs_sched* s);
/* Place a new request that needs `tokens` tokens of cache; *gpu = its GPU. */
int kvs_place(kvs_sched* s, long long request, int tokens, int* gpu);
/* The request now needs `tokens` tokens (growth by decode, or a prefill
 * chunk); KV_ERR_OOM if its GPU has no room for the extra blocks. */
int kvs_resize(kvs_sched* s, long long request, int tokens);
/* The request completed: its blocks leave its GPU's load. */
int kvs_release(kvs_sched* s, long long request);
int kvs_gpu_of(const kvs_sched* s, long long request, int* gpu);
/* Resident blocks and requests of one GPU (either pointer may be NULL). */
int kvs_load(const kvs_sched* s, int gpu, long long* resident_blocks, int* resident_requests);

#ifdef __cplusplus
}
#endif
#endif /* KVATTN_H */
