// internal.h -- launchers shared between the kernel files and the C ABI.
#pragma once

#include "common.cuh"

namespace odi_cuda {

cudaError_t launch_act_quant(const float* x, int64_t M, int64_t K, uint8_t* tiles, uint8_t* blocks,
                             bool pdl, cudaStream_t stream);
cudaError_t launch_act_q8_records(const float* x, int64_t ldx, int64_t M, int64_t K, uint8_t* recs, bool pdl,
                                  cudaStream_t stream);
struct GemvFuse;
cudaError_t launch_act_records_fused(const float* x, int64_t ldx, int64_t M, int64_t K, const GemvFuse& fu,
                                    uint8_t* recs, bool pdl, cudaStream_t stream);
cudaError_t launch_act_pack_f32(const float* x, int64_t M, int64_t K, float* tiles, bool pdl,
                                cudaStream_t stream);
cudaError_t launch_repack(int dt, const void* gguf, void* tiled, int64_t N, int64_t K, cudaStream_t s);
cudaError_t launch_unpack(int dt, const void* tiled, void* gguf, int64_t N, int64_t K, cudaStream_t s);
cudaError_t launch_dequant(int dt, const void* tiled, float* out, int64_t N, int64_t K, cudaStream_t s);
// Copy `bytes` (a multiple of 4) from page-locked host memory, given by its
// device address, into device memory with a small kernel whose host loads
// start before the programmatic dependency wait (pdl) and whose stores follow
// it (hostio.cu).
cudaError_t launch_pull_host(const void* src_dev_view, void* dst, size_t bytes, bool pdl, cudaStream_t stream);

// Outputs parked in a device ring, to be copied to page-locked host buffers
// by one launch (hostio.cu): entry e is bytes[e] bytes (a multiple of 4) at
// ring + 16 off16[e], for the host buffer whose device address is dst[e].
// Passed by value (kernel parameters: under 4 KB).
constexpr int GATHER_MAX = 200;
struct GatherTable {
  unsigned long long dst[GATHER_MAX];
  unsigned off16[GATHER_MAX];
  unsigned bytes[GATHER_MAX];
  int n;
};
static_assert(sizeof(GatherTable) <= 4000, "kernel parameter space");
cudaError_t launch_gather_to_host(const void* ring, const GatherTable& t, bool pdl, cudaStream_t stream);

cudaError_t launch_quant_weights(int dt, const float* w, void* out, int64_t N, int64_t K, cudaStream_t s);

// Work split of the streaming GEMV.  The weight is G row tiles of KB units.
// Each row tile is handled by one thread-block cluster of C CTAs; CTA rank j
// takes the contiguous chunk of spans [j*chunk, min(KB, (j+1)*chunk)) and the
// C partial tiles are added in rank order through distributed shared memory.
struct GemvPlan {
  int G, KB;
  int C;             // cluster size (CTAs per row tile), 1..8
  int chunk;         // spans per CTA
  int stages;        // weight ring depth
  int stage_bytes;   // one unit, 128-aligned
  int xq_bytes;      // staged activations: chunk * mt records, 128-aligned
  int smem_bytes;    // dynamic shared memory per CTA
  int mt;            // tokens per pass (template instantiation)
  int pre;           // activations arrive as Q8 records (Q8_REC_BYTES), quantized beforehand
  int rs;            // the cluster reduce-scatters (every rank writes 64/C rows; needs C a power of two)
  int ctas_per_sm;   // CTAs of smem_bytes that fit one SM (up to the launch bound)
};

// Output scatter of a row shard into every rank's gathered buffer (the
// all-gather of a row-sharded product, fused into the GEMV epilogue).  With
// n == 0 the product is written to GemvArgs::y as usual.
constexpr int MAX_PEERS = 8;
struct GemvScatter {
  float* out[MAX_PEERS];                 // rank p's gathered output [M][ld] (own rank included)
  unsigned long long* cnt[MAX_PEERS];    // rank p's arrival counters; this rank adds to [src]
  int n;                                 // ranks; 0 = no scatter
  int src;                               // this rank
  int64_t row0, ld;                      // first row of this shard in the full output, full rows
  unsigned* done;                        // local completion count of the launch (workspace, zero)
  int writers;                           // CTAs of the launch that write outputs (one per row tile)
};
constexpr int WS_DONE_OFFSET = 64;       // byte offset of GemvScatter::done in the workspace

// Transforms fused into the GEMV (decode step): the activation row is first
// RMS-normalised (norm_w) or is silu(gate) * up of a [gate K | up K] row
// (swiglu); the result is added to y (accumulate) instead of stored.
struct GemvFuse {
  const float* norm_w;  // non-null: x <- x / sqrt(mean(x^2) + eps) * norm_w, per token over K
  float eps;
  int swiglu;           // x rows are [gate | up], 2K values
  int accumulate;       // y += product
  const float* ssq_in;  // norm: sums of squares of x in ssq_n slots per token (else summed from x)
  int ssq_n;
  float* ssq_out;       // sums of squares of the stored y, one slot per 64-row tile: [M][G]
  // Pre-quantized input (plan.pre) that holds u = x * norm weights: scale its
  // records by each token's 1 / sqrt(mean(x^2) + eps), from ssq_in / ssq_n.
  int rec_scale;
  // Records of the stored y for the next product, [ceil(N/256)][rec_out_ld]
  // (this pass's first token at rec_out): of y * rec_norm_w (the next
  // RMSNorm's weights; y itself when null), or -- rec_swiglu, the rows of
  // each 64-row tile being 32 gate rows then the 32 matching up rows -- of
  // silu(gate) * up, N / 2 values.
  uint8_t* rec_out;
  int64_t rec_out_ld;
  const float* rec_norm_w;
  int rec_swiglu;
};

struct GemvArgs {
  const uint8_t* w;   // tiled weight
  const float* x;     // activations of this pass [M][ldx] fp32
  float* y;           // outputs of this pass [M][N] fp32, row stride N
  int* err;           // device error word
  int64_t N, K;
  int64_t ldx;        // row stride of x (K, or 2K for swiglu)
  int M;              // tokens in this pass (<= mt)
  GemvScatter sc;     // row offset of this pass's tokens is folded into sc.out
  GemvFuse fu;
  // Pre-quantized activations (plan.pre): Q8 records of this pass's first
  // token, record (kb, m) at recs + (kb * rec_ld + m) * Q8_REC_BYTES
  const uint8_t* recs;
  int64_t rec_ld;
};

// Plan for dtype / tokens / fp32-activation mode on a device with num_sms SMs.
// pre: the activations are quantized beforehand into Q8 records (ACT_Q8
// only), so a record takes Q8_REC_BYTES of shared memory, not the fp32 staging.
GemvPlan make_gemv_plan(int dt, int64_t N, int64_t K, int M, bool f32act, int num_sms, bool pre = false,
                        bool rs_ok = false);
cudaError_t launch_gemv(int dt, bool f32act, const GemvPlan& plan, const GemvArgs& a, bool pdl,
                        cudaStream_t s);

// Peer signalling (peer.cu): wait until every source rank's counter has
// advanced by inc[src] past what this rank consumed, then consume.
constexpr int ERR_PEER_WAIT = 32;
struct PeerWait {
  unsigned long long inc[MAX_PEERS];
  unsigned long long timeout_ns;  // give up after this long (device global timer)
  int n;
};
constexpr unsigned long long PEER_WAIT_DEFAULT_NS = 1000000000ull;  // one second
cudaError_t launch_wait_peers(const unsigned long long* cnt, unsigned long long* consumed, const PeerWait& w,
                              int* err, cudaStream_t s);

// The C ABI's error record (capi.cu): sets the thread's message, returns code.
int set_error(int code, const char* msg);

// NCCL, opened at run time (shard.cu).  Each returns 0, or -1 with *why set.
bool nccl_available();
int nccl_unique_id(void* out, const char** why);
int nccl_comm_init(const void* id, int nranks, int rank, void** comm, const char** why);
int nccl_comm_destroy(void* comm, const char** why);
int nccl_all_gather_f32(const float* send, float* recv, size_t count, void* comm, cudaStream_t s, const char** why);
// y [M][N] from a rank-major gather buffer [g][M][S]
cudaError_t launch_unshard(const float* src, float* y, int64_t M, int64_t N, int64_t S, int g, cudaStream_t s);

// Decode-step kernels (decode_ops.cu).  The token and position live on the
// device; argmax advances them, so one captured graph serves every step.
struct DecodeState {
  int token;  // input token of the next step
  int pos;    // its position (KV slot)
  int step;   // tokens generated so far (index into the token record)
  int reserved;
};
constexpr int ATT_CHUNK = 64;  // positions per CTA in the attention's first pass (8 per warp)
int attention_chunks(int ctx);
// attention scratch: the error word (int at 0), per-kv-head arrival counters
// from byte 16 (zero between launches), then the per-split partials
// [heads][splits][hd + 2] fp32 from the next 256-byte boundary
constexpr int ATT_CNT_OFFSET = 16;
inline size_t att_part_offset(int heads) { return (ATT_CNT_OFFSET + (size_t)heads * sizeof(int) + 255) / 256 * 256; }
size_t attention_scratch(int heads, int hd, int ctx);
int attention_splits(int kv_heads, int ctx, int num_sms);
cudaError_t launch_embed(const float* table, int64_t vocab, int64_t E, const DecodeState* st, float* x, float* ssq,
                         const float* norm_w, uint8_t* recs, cudaStream_t s);
cudaError_t launch_rms_norm(const float* x, const float* w, float* y, int64_t rows, int64_t n, float eps,
                            cudaStream_t s);
cudaError_t launch_rope_kv(float* q, float* k, const float* v, __half* kc, __half* vc, const DecodeState* st,
                           int heads, int kv_heads, int hd, int ctx, float theta, cudaStream_t s);
// rope_kv fused into the attention: this step's raw k and v (k == nullptr:
// q is already rotated and the caches already hold pos)
struct AttRope {
  const float* k = nullptr;
  const float* v = nullptr;
  float theta = 0.f;
  uint8_t* out_recs = nullptr;  // also write the outputs as one token's Q8 records
};
cudaError_t launch_attention(const float* q, const __half* kc, const __half* vc, float* o, void* scratch,
                             const DecodeState* st, int heads, int kv_heads, int hd, int ctx, float scale,
                             const AttRope& rp, cudaStream_t s);
cudaError_t launch_silu_mul(const float* gu, float* a, int64_t F, cudaStream_t s);
cudaError_t launch_add(float* x, const float* d, int64_t n, cudaStream_t s);
cudaError_t launch_argmax(const float* logits, int64_t V, DecodeState* st, int* record, int record_len,
                          cudaStream_t s);

// Prefill-shaped GEMM on the tensor cores (qgemm_tc.cu).  Weights decoded to
// fp16 in shared memory, activations packed to fp16 operand tiles in the
// workspace by launch_act_pack_f16, fp32 accumulation in tensor memory.
struct TcArgs {
  const uint8_t* w;    // tiled weight
  const uint8_t* x16;  // packed fp16 activation tiles (tc_x16_bytes)
  float* y;            // [M][N] fp32
  int* err;            // device error word
  int64_t N;
  int M, M_pad, KB;    // tokens, tokens rounded up to 256 (packed rows), 256-column spans
};
constexpr int TC_X16_OFFSET = 1024;  // packed activations start here in the workspace
bool tc_supported(int dt);
struct TcPlan {
  int BN;     // tokens per CTA (UMMA N): 32, 64, 128 or 256
  int C;      // K split: CTAs per cluster, each with `chunk` spans
  int chunk;
};
TcPlan make_tc_plan(int64_t M, int64_t N, int64_t K, int num_sms);
int64_t tc_x16_bytes(int64_t M, int64_t K);
cudaError_t launch_act_pack_f16(const float* x, int M, int64_t K, int M_pad, uint8_t* x16, cudaStream_t s);
cudaError_t launch_qgemm_tc(int dt, const TcPlan& p, const TcArgs& a, cudaStream_t s);

}  // namespace odi_cuda
