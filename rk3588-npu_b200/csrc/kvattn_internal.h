// kvattn_internal.h -- structures shared by the host runtime and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

struct kvx_exch;  // split-KV exchange object of the C ABI (xgpu_exchange.cu)
struct kvn_comm;  // split-KV NCCL communicator of the C ABI (nccl_split.cu)
struct kvp_pool;  // paged pool of the C ABI (kvattn_host.cu)

namespace kvattn {

constexpr int kHeadDim = 128;          // dims per head (the only supported value)
constexpr int kBlockTokens = 16;       // token rows per block
constexpr int kTileBytes = kBlockTokens * kHeadDim * 2;  // one (block, kv head) tile: 4 KiB
// INT8 pools: a (block, kv head) tile is 16 rows x 128 int8 codes (row t at
// byte 128 t, its 16-byte chunks swizzled: i8_offset) followed by the 16
// rows' fp32 scales.
constexpr int kTileBytesI8 = kBlockTokens * kHeadDim + kBlockTokens * 4;  // 2112 bytes
constexpr int kMaxGroup = 8;           // query heads per KV head handled by one MMA tile
constexpr int kPartialFloats = kMaxGroup * (kHeadDim + 2);  // m[8], l[8], o[8][128]
constexpr int kMaxCtaItems = 64;       // pieces per decode CTA (the planner never assigns more)

// Byte offset of element (token t, dim d) inside a 4 KiB tile.
// Two 2 KiB halves (dims 0-63, 64-127); each half has 16 rows of 128 bytes;
// the 16-byte chunk index inside a row is XORed with (t & 7).  This is the
// 128-byte-swizzle K-major layout, so ldmatrix rows of 8 consecutive tokens at
// one logical chunk land in 8 different bank groups.
__host__ __device__ inline uint32_t tile_offset(int t, int d) {
    return (uint32_t)(((d >> 6) * 16 + t) * 128 + ((((d >> 3) & 7) ^ (t & 7)) << 4) + (d & 7) * 2);
}

// Byte offset of code (token t, dim d) inside an INT8 tile: 16 rows of 128
// codes, the 16-byte chunk index inside a row XORed with (t & 7) so that one
// logical chunk of eight consecutive tokens lies in eight different bank
// groups (ldmatrix reads the codes in place); the 16 fp32 row scales follow
// the codes (kBlockTokens * kHeadDim bytes in).
__host__ __device__ inline uint32_t i8_offset(int t, int d) {
    return (uint32_t)(t * kHeadDim + ((((d >> 4) ^ t) & 7) << 4) + (d & 15));
}

// A block-table entry to write before use: table[seq][idx] = block.
struct TablePatch {
    int seq;
    int idx;
    int block;
    int pad;
};

// ---- decode plans (kernel parameters) ---------------------------------
// A decode step is passed to its launches by value: the host owns the block
// tables and lengths, so it builds the work partition in O(sequences + CTAs)
// and no plan is uploaded.  Work is a flat sequence of 16-token blocks made
// of segments, one per (slot i, KV head h) with blocks: segment k is flat
// blocks [seg_f0[k], seg_f0[k + 1]), all ceil(kv_len_i / 16) blocks of
// (seg[k] & 0xffff, seg[k] >> 16).  CTA g owns flat blocks [cta_f0[g],
// cta_f0[g + 1]); its pieces are the maximal runs of one segment inside that
// range.  Only a CTA's first and last piece can be part of a segment that
// other CTAs share (a split segment).  Two ways to merge split segments:
//  * grid-wide (cluster == 1): the pieces' partial states go to partials[2g]
//    (first piece) and partials[2g + 1] (last piece), merged by the combine
//    kernel launched right behind the decode grid;
//  * in a thread-block cluster (cluster == C > 1): the launch runs in
//    clusters of C consecutive CTAs and the plan keeps every segment inside
//    one cluster; a split piece's state stays in its CTA's shared memory and
//    the CTA holding the segment's first block merges the others' states
//    over distributed shared memory once the cluster has finished (no
//    combine launch).
constexpr int kMaxGrid = 320;       // decode CTAs per launch (B200: 148 SMs x 2 resident)
constexpr int kSlotsSmall = 64;     // slot capacities of the two kernel-parameter layouts
constexpr int kSlotsLarge = 256;    // (a step with more sequences runs as several launches)
constexpr int kSegsPerSlot = 2;     // segment capacity per slot (KV heads beyond 2: fewer slots per launch)
constexpr int kClusterCtas = 8;     // CTAs of a merge cluster (portable cluster size)

struct DecodeSlot {
    int seq;        // row of the block table
    int kv_len;     // tokens attended (including the new one when it appends)
    int rope_pos;   // position used to rotate q and the new k
    int new_block;  // block holding slot kv_len-1 when the launch appends; -1: attend only
};

// Flags of a decode launch.
constexpr int kDecEarly = 1;  // copy the first ring round before the previous kernel finishes
constexpr int kDecPatch = 2;  // write table[seq][(kv_len-1)/16] = new_block for appending slots

template <int S>
struct DecodeArgs {
    int nslots;
    int grid;
    int layer;
    int flags;
    int total;                  // flat blocks of the launch
    int row0;                   // row of slot 0 in q / k_new / v_new / out / m / l
    int nsegs;                  // segments (slots with kv_len > 0, times KV heads)
    int cluster;                // 1: grid-wide merge; kClusterCtas: merge inside clusters
    int seg_f0[kSegsPerSlot * S + 1];  // flat offset of segment k; seg_f0[nsegs] = total
    int seg[kSegsPerSlot * S];  // slot | KV head << 16
    DecodeSlot slot[S];
    int defer_blk[S];           // block of slot i the previous decode launch may still write (-1: none)
    int cta_f0[kMaxGrid + 1];   // flat range of every CTA
};

// A split segment, for the combine kernel: x = slot | head << 16, y =
// first_part | npieces << 16.  Its pieces' partial states are at
// first_part, then 2 * (first_part / 2 + u) for u = 1 .. npieces - 1.
struct CombineArgs {
    int nsegs;
    int row0;
    int pad[2];
    int2 seg[kMaxGrid];
};

// Device view of the pool handed to kernels by value.
struct PoolView {
    uint8_t* k;              // [layers][num_blocks][kv_heads][kTileBytes]
    uint8_t* v;
    const float2* rope;      // [max_seq_len][kHeadDim/2] (cos, sin)
    int* table;              // [max_seqs][max_blocks_per_seq]
    float* partials;         // [2 * kMaxGrid][kPartialFloats]: split-piece states of a decode launch
    int* status;             // device status: [0] code, [1] item index, [2] detail
    int num_blocks;
    int kv_heads;
    int q_heads;
    int group;               // q_heads / kv_heads
    int max_blocks_per_seq;
    int max_seq_len;
    int max_seqs;
    int dtype;               // 0 f16, 1 bf16, 2 int8 codes + per-row fp32 scales
    int tile_bytes;          // kTileBytes, or kTileBytesI8 for int8
    size_t layer_bytes;      // num_blocks * kv_heads * tile_bytes
};

// ---- launchers (kernels.cu) ----
// One decode launch (and, when the plan splits segments, its combine launch
// right behind it).  pdl: launch as a programmatic dependent of the previous
// kernel in the stream (every read of state that kernel may write waits for
// it inside the kernel).
template <int S>
cudaError_t launch_decode(const PoolView& pv, const DecodeArgs<S>& a, const CombineArgs& c, int max_pieces,
                          const float* q, const float* k_new, const float* v_new, float* out, float* m_out,
                          float* l_out, bool pdl, cudaStream_t st);
// ctas_per_sm: resident decode CTAs per SM; clusters: resident merge
// clusters (kClusterCtas CTAs each) on the device, 0 if none fit.
cudaError_t decode_occupancy(int dtype, int* ctas_per_sm, int* clusters);
cudaError_t launch_import(const PoolView& pv, int layer, int seq, int pos0, int n,
                          const uint16_t* k_rows, const uint16_t* v_rows, cudaStream_t st);
cudaError_t launch_gather(const PoolView& pv, int layer, int seq, int len, uint16_t* k_rows,
                          uint16_t* v_rows, cudaStream_t st);
// Prompt chunks of several sequences in one launch: chunk i is rows
// [row0[i], row0[i+1]) of the concatenated k / v (or q / out) rows, at
// positions pos0[i].. of sequence seq[i].  Passed by value (kernel parameter).
constexpr int kMaxChunkBatch = 32;
struct ChunkBatch {
    int nreq;
    int seq[kMaxChunkBatch];
    int pos0[kMaxChunkBatch];
    int row0[kMaxChunkBatch + 1];
};
cudaError_t launch_append_batch(const PoolView& pv, int layer, const ChunkBatch& cb, const float* k,
                                const float* v, cudaStream_t st);
cudaError_t launch_import_i8(const PoolView& pv, int layer, int seq, int pos0, int n, const int8_t* k_codes,
                             const int8_t* v_codes, const float* k_scales, const float* v_scales, cudaStream_t st);
cudaError_t launch_gather_i8(const PoolView& pv, int layer, int seq, int len, int8_t* k_codes, int8_t* v_codes,
                             float* k_scales, float* v_scales, cudaStream_t st);
cudaError_t launch_patch(const PoolView& pv, const TablePatch* patches, int npatch,
                         cudaStream_t st);
cudaError_t launch_prefill(const PoolView& pv, int layer, int seq, int pos0, int n, const float* q,
                           float* out, float* part, int nsplit, int tiles_per_split, cudaStream_t st);
// One chunk of a tcgen05 prefill launch: its CTAs are [cta0, cta0 + nq *
// kv_heads * nsplit) (token group fastest, then KV head, then key split);
// with nsplit > 1 its partials start at part0 floats and its merge rows at
// mrow0 (both running totals over the chunks before it).
struct TcReq {
    int seq, pos0, n, row0;
    int nq, nsplit, tps, cta0;
    int mrow0, pad;
    long long part0;
};
struct TcBatch {
    int nreq, pad;
    TcReq r[kMaxChunkBatch];  // in launch order (cta0 ascending)
};
cudaError_t launch_prefill_tc(const PoolView& pv, int layer, const TcBatch& b, int total_ctas, int merge_rows,
                              const float* q, float* out, float* part, cudaStream_t st);
int prefill_tc_tokens_per_cta(int group);
int prefill_tc_stage_tiles();  // key tiles per stage of the tcgen05 prefill (a split is a whole number of them)
size_t prefill_tc_part_floats(int q_heads, int n, int nsplit);
cudaError_t launch_combine(int G, int rows, int dim, const float* m, const float* l,
                           const float* o, size_t gstride_ml, size_t gstride_o, float* out,
                           cudaStream_t st);

// ---- split-KV exchange over peer memory (xgpu_exchange.cu) ----
// Every rank owns one area in its own device memory, mapped by every peer:
//   local   [m max_rows][l max_rows][o max_rows x 128] floats: this rank's
//           states, written by its decode (never read by peers);
//   inbox   [2 buffers][world sources][max_rows][2 + 128] words of 8 bytes,
//           each {value bits, epoch}: a source writes a word with one 8-byte
//           store, so a reader that sees the epoch of the current call sees
//           its value (m, l, then the 128 dims of o).
// Layer call e uses inbox buffer e & 1.
constexpr int kMaxRanks = 8;

constexpr int kMaxXchgSplit = 64;  // split segments whose merge the exchange kernel takes over
struct XchgArgs {
    float* base[kMaxRanks];  // every rank's area (this rank's is local)
    int world, me, rows, max_rows;
    unsigned epoch;          // >= 1, one more per layer call
    float* out;              // [rows][128]
    int* status;             // the pool's status words
    // nsplit > 0: the decode launch's split segments (CombineArgs::seg
    // layout, slot = plan row of the only launch) are merged here from
    // `partials`, in place of a merge launch; their rows of the local slot
    // are not written.
    const float* partials;
    int nsplit, q_heads, group, pad;
    int2 seg[kMaxXchgSplit];
};

__host__ __device__ inline size_t xchg_local_floats(int max_rows) { return (size_t)max_rows * (2 + kHeadDim); }
__host__ __device__ inline uint2* xchg_inbox(float* base, int world, int max_rows, int buf, int src) {
    return reinterpret_cast<uint2*>(base + xchg_local_floats(max_rows)) +
           ((size_t)buf * world + src) * (size_t)max_rows * (2 + kHeadDim);
}
inline size_t xchg_bytes(int world, int max_rows) {
    return xchg_local_floats(max_rows) * 4 + 2 * (size_t)world * max_rows * (2 + kHeadDim) * 8;
}

cudaError_t launch_xchg(const XchgArgs& a, cudaStream_t st);
// Fill the arguments of the next layer call on `x` and point m/l/o at this
// rank's own slot (where the local decode writes its states); the epoch
// advances only on xchg_commit, after the launches succeeded.
int xchg_prepare(::kvx_exch* x, int device, int rows, int* status, float* out, XchgArgs* a,
                 float** m, float** l, float** o);
void xchg_commit(::kvx_exch* x);

// ---- split-KV merge over an NCCL all-gather (nccl_split.cu) ----
// Point m / l / o at this rank's packed state buffer of the communicator.
int nccl_prepare(::kvn_comm* c, int device, int rows, float** m, float** l, float** o);
// All-gather every rank's packed states on `st` and merge them into out.
int nccl_gather_combine(::kvn_comm* c, int rows, float* out, cudaStream_t st);

// ---- Qwen2 forward kernels (model_kernels.cu) ----
// One projection y = epilogue(x W^T): W fp16 [N][K], x [M][K]: in = 0 fp16
// bits, 1 fp32 rounded through fp16, 2 fp32 rows RMSNorm'd with norm_w / eps
// and rounded through fp16.  Modes: 0 QKV (fp16-rounded + bias,
// rows n < n0 to out0 [M][n0], then n1 rows to out1 [M][n1], the rest to out2),
// 1 residual (resid [M][N] += rounded), 2 gate/up (w = gate, w2 = up; out16
// [M][N] = fp16(silu(g) * u)), 3 logits (logits [M][N] = rounded).
struct GemvArgs {
    const uint16_t* w = nullptr;
    const uint16_t* w2 = nullptr;
    int N = 0, K = 0, M = 0, ks = 1;
    const void* x = nullptr;
    const float* bias = nullptr;
    float* out0 = nullptr;
    float* out1 = nullptr;
    float* out2 = nullptr;
    int n0 = 0, n1 = 0;
    float* resid = nullptr;
    uint16_t* out16 = nullptr;
    float* logits = nullptr;
    const float* norm_w = nullptr;
    float eps = 0.f;
};
cudaError_t launch_gemv(int mode, int in, GemvArgs a, cudaStream_t st);
int gemv_split(int K);
cudaError_t launch_rmsnorm_f16(const float* x, const float* w, uint16_t* y, int rows, int H, float eps,
                               cudaStream_t st);
cudaError_t launch_embed(const int* ids, int n, const uint16_t* table, float* hidden, int H, cudaStream_t st);
cudaError_t launch_argmax(const float* v, int n, int rows, unsigned long long* best, cudaStream_t st);
cudaError_t launch_gather_rows(const float* src, const int* idx, int rows, float* dst, int H, cudaStream_t st);
cudaError_t launch_weight_to_f16(const void* src, int dtype, uint16_t* dst, size_t n, cudaStream_t st);

// ---- the Qwen2 forward in the reference's operation order (exact_kernels.cu) ----
// The float inputs where the host C library's expf is not the correctly
// rounded exponential, with its result: keys (float bits, ascending) and
// vals of n entries; bucket[b] .. bucket[b + 1] are the entries whose top
// 16 key bits are b (65537 offsets).  All NULL: the correctly rounded value
// everywhere.
struct ExpTab {
    const uint32_t* keys = nullptr;
    const uint32_t* vals = nullptr;
    const uint32_t* bucket = nullptr;
};
cudaError_t launch_rmsnorm_exact(const float* x, const float* w, float eps, int rows, int H, uint16_t* y16,
                                 cudaStream_t st);
cudaError_t launch_gemv_exact(const uint16_t* x16, int M, int K, const uint16_t* W, int N, uint16_t* y16,
                              cudaStream_t st);
cudaError_t launch_qkv_bias_exact(const uint16_t* qkv16, const float* bias, int rows, int H, int kvd, float* q, float* k,
                                  float* v, cudaStream_t st);
cudaError_t launch_rope_q_exact(float* q, int rows, int heads, int pos0, const float2* rope, cudaStream_t st);
cudaError_t launch_attn_exact(const float* q, const uint16_t* kc, const uint16_t* vc, float* out, int seq, int total_len,
                              int n_heads, int n_kv_heads, int pos_base, float scale, ExpTab et, cudaStream_t st);
cudaError_t launch_to_f16_exact(const float* x, long n, uint16_t* y, cudaStream_t st);
cudaError_t launch_resid_exact(float* hidden, const uint16_t* y16, long n, cudaStream_t st);
cudaError_t launch_silu_mul_exact(const uint16_t* g16, const uint16_t* u16, long n, uint16_t* h16, ExpTab et,
                                  cudaStream_t st);
cudaError_t launch_f16_to_f32_exact(const uint16_t* y16, long n, float* y, cudaStream_t st);
// The pool's device RoPE table [max_seq_len][64] (cos, sin), host-built with
// the reference's float libm calls.
const float2* pool_rope_table(const ::kvp_pool* p);

// Sets a device for the scope of a call and restores the caller's.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (dev < 0) return;  // host-only object: no device calls
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Sets the calling thread's kv_last_error() message; returns `status`.
int set_error(int status, const char* msg);

// Process-wide count of kernels this library launched (kv_kernel_count):
// a launcher passes its launch's status through counted().
void count_launch();
inline cudaError_t counted(cudaError_t e) {
    if (e == cudaSuccess) count_launch();
    return e;
}

}  // namespace kvattn
