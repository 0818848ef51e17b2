/*
 * odi_cuda.h -- C ABI of the B200 (sm_100a) quantized matrix-product backend
 * for ODIEngine.
 *
 * Every entry point is plain C: pointers, sizes, int status codes, and an
 * opaque cudaStream_t passed as void* (NULL = the legacy default stream).
 * Nothing here throws.  Status codes are odi_error_t values from the
 * reference's include/odi/odi_error.h:11-48 so the C++ backend can hand them
 * to the C API unchanged; a thread-local message explains the last failure.
 *
 * Weight matrices follow the reference's GGUF convention: a weight of
 * GGUF shape [K, N] (ne0 = K inputs, ne1 = N outputs) is stored as N output
 * rows of ceil(K / block) packed blocks (src/compute/cpu/cpu_backend.cpp:804,
 * 839).  On the device it lives in a "tiled" layout: rows grouped in tiles of
 * 64, columns in spans of 256, each (tile, span) unit contiguous, so one
 * bulk copy moves one unit.  The transform is a byte permutation and is
 * invertible (odi_cuda_unpack).
 *
 * dtype ids are odi_dtype_t values (include/odi/odi_types.h:32-49):
 *   ODI_DTYPE_Q8_0 = 6, ODI_DTYPE_Q4_0 = 7, ODI_DTYPE_Q4_1 = 8,
 *   ODI_DTYPE_Q5_0 = 9, ODI_DTYPE_Q5_1 = 10, ODI_DTYPE_Q4_K = 11,
 *   ODI_DTYPE_Q5_K = 12, ODI_DTYPE_Q6_K = 13.
 * Q4_1 / Q5_0 / Q5_1 give the product their block format defines
 * (cpu_backend.cpp:704-767 decode); the reference CPU backend's
 * dequantize + matmul_f32 fallback for them reads the weight transposed
 * (cpu_backend.cpp:211-216) and is not reproduced.
 */
#ifndef ODI_CUDA_H
#define ODI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: the odi_error_t values (odi_error.h:11-48). */
enum {
  ODI_CUDA_OK = 0,
  ODI_CUDA_ERR_INVALID_ARGUMENT = 2,
  ODI_CUDA_ERR_OUT_OF_MEMORY = 3,
  ODI_CUDA_ERR_NOT_IMPLEMENTED = 4,
  ODI_CUDA_ERR_INVALID_STATE = 5,
  ODI_CUDA_ERR_OPERATION_FAILED = 6,
  ODI_CUDA_ERR_UNSUPPORTED_DTYPE = 202,
  ODI_CUDA_ERR_BACKEND_UNAVAILABLE = 300,
  ODI_CUDA_ERR_BACKEND_INIT_FAILED = 301,
  ODI_CUDA_ERR_GPU_OUT_OF_MEMORY = 303
};

/* Activation modes for odi_cuda_matmul.
 *   ODI_CUDA_ACT_Q8  -- activations are quantised to Q8_0 first (bit-exact
 *                       with the GGUF Q8_0 quantiser) and dotted against the
 *                       weight codes in integer arithmetic; fp32 block scales.
 *                       Streaming GEMV, 8 tokens per launch (decode).
 *   ODI_CUDA_ACT_F32 -- fp32 activations times the fp32-decoded weights, the
 *                       arithmetic of the reference's matmul_q4_0 /
 *                       matmul_q8_0 (cpu_backend.cpp:786-854) up to
 *                       summation order.  Streaming GEMV.
 *   ODI_CUDA_ACT_F16 -- tensor cores (tcgen05): weights decoded to fp16
 *                       (fp16(d*sc) * q - fp16(dmin*m)), activations rounded
 *                       to fp16, exact products, fp32 sums (prefill).  For
 *                       the dtypes odi_cuda_tc_supported accepts.
 *   ODI_CUDA_ACT_AUTO -- ODI_CUDA_ACT_F16 when M >= ODI_CUDA_TC_MIN_TOKENS
 *                       and the dtype has a tensor-core path, else
 *                       ODI_CUDA_ACT_Q8. */
enum { ODI_CUDA_ACT_Q8 = 0, ODI_CUDA_ACT_F32 = 1, ODI_CUDA_ACT_F16 = 2, ODI_CUDA_ACT_AUTO = 3 };
/* From 9 tokens the streaming GEMV needs a second pass over the weight,
 * and the tensor-core path is faster on every measured decode shape. */
#define ODI_CUDA_TC_MIN_TOKENS 9

/* Flags for odi_cuda_matmul. */
enum {
  /* Launch with programmatic dependent launch: the kernel may start, and
   * prefetch weights, while earlier kernels on the stream are still running.
   * Only valid when no kernel still in flight on the stream writes the
   * weight buffer. */
  ODI_CUDA_FLAG_PDL = 1
};

/* --- device / backend ---------------------------------------------------- */

/* Select and initialise a CUDA device.  Replaces the CPU fallback that
 * create_backend(ODI_BACKEND_CUDA) returns today (cpu_backend.cpp:1010-1013):
 * fails with ODI_CUDA_ERR_BACKEND_UNAVAILABLE when there is no usable device
 * or it is not sm_100. */
int odi_cuda_init(int device);

/* Number of CUDA devices (0 if none).  Backs is_backend_available
 * (backend.hpp:150). */
int odi_cuda_device_count(void);

/* Backend::device_info (backend.hpp:23): "NVIDIA B200 (sm_100, 148 SMs, ...)". */
int odi_cuda_device_info(char* buf, size_t len);

/* Backend::available_memory / used_memory (backend.hpp:26-27). */
int odi_cuda_memory_info(size_t* free_bytes, size_t* total_bytes);

/* Backend::supports_dtype (backend.hpp:30): 1 for Q8_0, Q4_0, Q4_1, Q5_0,
 * Q5_1, Q4_K, Q5_K, Q6_K, else 0. */
int odi_cuda_supports_dtype(int dtype);

/* Message for the last non-zero status returned on this thread
 * (odi_get_last_error_message, odi_error.h:55). */
const char* odi_cuda_last_error(void);

/* Block until all work on `stream` is done (Backend::sync, backend.hpp:130). */
int odi_cuda_sync(void* stream);

/* --- layout ----------------------------------------------------------------- */

/* Bytes of the GGUF packing of an N x K weight: N * ceil(K/block) * block
 * bytes (Tensor::nbytes, tensor.cpp:281-288).  -1 for unsupported dtypes. */
int64_t odi_cuda_gguf_bytes(int dtype, int64_t N, int64_t K);

/* Bytes of the tiled device layout (rows padded to 64, columns to 256). */
int64_t odi_cuda_tiled_bytes(int dtype, int64_t N, int64_t K);

/* GGUF blocks -> tiled layout and back, both buffers in device memory.
 * K-quant rows must be whole 256-value super-blocks (K % 256 == 0). */
int odi_cuda_repack(int dtype, const void* d_gguf, void* d_tiled, int64_t N, int64_t K,
                    void* stream);
int odi_cuda_unpack(int dtype, const void* d_tiled, void* d_gguf, int64_t N, int64_t K,
                    void* stream);

/* --- weights: upload packed blocks to HBM once (gguf_parser.cpp:614-628) ----- */

typedef struct odi_cuda_weight odi_cuda_weight;

/* Copy host GGUF blocks to the device and repack them into the tiled layout.
 * The returned handle owns the device copy until odi_cuda_weight_free. */
int odi_cuda_weight_upload(const void* host_blocks, int dtype, int64_t N, int64_t K,
                           odi_cuda_weight** out);
int odi_cuda_weight_free(odi_cuda_weight* w);
/* Device pointer of the tiled bytes, and the weight's shape. */
const void* odi_cuda_weight_data(const odi_cuda_weight* w);
int odi_cuda_weight_shape(const odi_cuda_weight* w, int* dtype, int64_t* N, int64_t* K);

/* fp32 weights [N, K] (device) -> GGUF blocks [N][ceil(K/block)] (device).
 * Q4_0 / Q8_0 / Q4_1 / Q5_0 / Q5_1 are byte-identical to the GGUF quantisers
 * (gguf 0.19.0); Q4_K / Q5_K / Q6_K
 * use this library's own quantisers of the GGML formats.  The reference has
 * no quantiser (Tensor::to throws for quantized dtypes, tensor.cpp:654-656);
 * this brings fp32 checkpoints and synthetic models up on the device. */
int odi_cuda_quantize_weight(int dtype, const float* d_w, void* d_blocks, int64_t N, int64_t K,
                             void* stream);

/* --- activation quantisation -------------------------------------------------- */

/* x fp32 [M, K] (device) -> GGUF Q8_0 blocks [M][ceil(K/32)] x 34 bytes
 * (device), bit-exact with the GGUF Q8_0 quantiser: d = amax/127,
 * q = round-half-away(x / d), d stored as fp16.  A partial last block is
 * quantised as if zero-padded. */
int odi_cuda_quantize_q8_0(const float* d_x, void* d_blocks, int64_t M, int64_t K, void* stream);

/* --- the quantized matrix product ------------------------------------------ */

/* Device scratch needed by odi_cuda_matmul: 256 bytes holding the device
 * error word for the streaming GEMV with one token (its activations are
 * staged on chip); with 2 or more tokens in ACT_Q8 mode the tokens are
 * quantized once into Q8 records after those 256 bytes
 * (ceil(K/256) * M * 384 bytes), so each pass of up to 8 tokens streams the
 * weight once; the tensor-core path adds its fp16 activation tiles
 * (1024 + ceil(M/256)*256 * ceil(K/256)*256 * 2 bytes). */
size_t odi_cuda_matmul_workspace_bytes(int dtype, int64_t M, int64_t N, int64_t K, int act_mode);

/* How the streaming GEMV splits one product of M tokens (ODI_CUDA_ACT_Q8 /
 * ODI_CUDA_ACT_F32, or ACT_AUTO below ODI_CUDA_TC_MIN_TOKENS), for sizing and
 * diagnosis: the same plan odi_cuda_matmul launches for a product whose
 * epilogue only stores y.  Host arithmetic only (no device is touched; without
 * one the SM count is taken as 148).  A diagnostic of this backend, with no
 * counterpart in the reference. */
typedef struct odi_cuda_gemv_plan {
  int tokens_per_pass;  /* tokens per launch: 1, 2, 4 or 8 */
  int passes;           /* launches for the M tokens */
  int cluster;          /* CTAs per 64-row tile (thread-block cluster size) */
  int spans_per_cta;    /* 256-column spans each CTA streams */
  int stages;           /* weight ring depth (units in flight per CTA) */
  int reduce_scatter;   /* 1: the cluster reduce-scatters its partials */
  int ctas_per_sm;      /* CTAs of this shared-memory size resident per SM (4 is the design point) */
  int64_t ctas;         /* CTAs per launch */
  size_t shared_bytes;  /* dynamic shared memory per CTA */
} odi_cuda_gemv_plan;
int odi_cuda_gemv_plan_info(int dtype, int64_t M, int64_t N, int64_t K, int act_mode, odi_cuda_gemv_plan* out);

/* 1 if `dtype` has the tensor-core (ODI_CUDA_ACT_F16) path, else 0. */
int odi_cuda_tc_supported(int dtype);

/* y[M, N] = x[M, K] . dequant(W)^T in fp32 -- Backend::matmul /
 * quantized_matmul (backend.hpp:38, 114) with a = x, b = W.
 *   d_w_tiled : tiled weight (odi_cuda_repack / odi_cuda_weight_data)
 *   d_x, d_y  : device fp32, row-major, contiguous
 *   d_workspace: at least odi_cuda_matmul_workspace_bytes, zero before its
 *     first use (a call leaves it zero unless a kernel wait gave up; see
 *     odi_cuda_workspace_status).
 * One kernel launch per 8 tokens (plus one quantizing the tokens when there
 * are 2 or more in ACT_Q8 mode).  Asynchronous on `stream`. */
int odi_cuda_matmul(int dtype, const void* d_w_tiled, const float* d_x, float* d_y, int64_t M,
                    int64_t N, int64_t K, int act_mode, void* d_workspace,
                    size_t workspace_bytes, int flags, void* stream);

/* Operations fused into the streaming GEMV of odi_cuda_matmul (decode
 * step): the activation row is RMS-normalised first (Backend::rms_norm,
 * cpu_backend.cpp:388-414: x / sqrt(mean(x^2) + eps) * norm_weight), or is
 * silu(gate) * up of a [gate K | up K] row (the SwiGLU of context.cpp:
 * 272-275; x rows then hold 2K values); the product is added to y
 * (the residual add of context.cpp:124, 130) instead of stored. */
typedef struct odi_cuda_matmul_opts {
  const float* norm_weight;  /* K weights, or NULL */
  float norm_eps;
  int swiglu;                /* exclusive with norm_weight */
  int accumulate;
  /* RMSNorm from partial sums instead of a pass over x: norm_ssq holds
   * norm_ssq_count sums of squares per token (e.g. out_ssq of the GEMV, or
   * the ssq of odi_cuda_embed, that wrote x).  NULL: sum x itself. */
  const float* norm_ssq;
  int norm_ssq_count;
  /* If non-NULL: the sum of squares of the stored y of every 64-row tile,
   * [M][ceil(N / 64)] -- what the next GEMV's RMSNorm needs. */
  float* out_ssq;
} odi_cuda_matmul_opts;

/* odi_cuda_matmul with the operations above (ACT_Q8 / ACT_F32, and AUTO
 * below ODI_CUDA_TC_MIN_TOKENS); opts == NULL is odi_cuda_matmul.  With an
 * RMSNorm or SwiGLU prologue the activations are staged on chip (256 bytes
 * of workspace suffice); otherwise the workspace rules of odi_cuda_matmul
 * apply (a smaller workspace is accepted and takes the on-chip path). */
int odi_cuda_matmul_fused(int dtype, const void* d_w_tiled, const float* d_x, float* d_y, int64_t M,
                          int64_t N, int64_t K, int act_mode, void* d_workspace, size_t workspace_bytes,
                          int flags, const odi_cuda_matmul_opts* opts, void* stream);

/* Pre-quantized activations.  A Q8 record holds one (256-column span,
 * token): 256 int8 codes (Q8_0 per 32 values, the gguf quantiser), then 8 x
 * {scale, scale * sum of codes, ... of the first 16, ... of the last 16}
 * fp32; records are span-major, (span kb, token m) at (kb * M + m) * 384.
 * odi_cuda_q8_records_bytes gives the size for M rows of K values. */
size_t odi_cuda_q8_records_bytes(int64_t M, int64_t K);

/* fp32 rows x [M][K] -> Q8 records, after the optional prologue of opts
 * (norm_weight / norm_ssq: RMSNorm; swiglu: x rows are [gate K | up K]).
 * The records equal, bit for bit, the ones odi_cuda_matmul_fused builds on
 * chip from the same inputs; odi_cuda_matmul_q8rec on them then equals
 * odi_cuda_matmul_fused up to the order of the fp32 cross-CTA reduction,
 * which the two paths may split differently on products of several waves.
 * opts may be NULL. */
int odi_cuda_quantize_records(const float* d_x, int64_t M, int64_t K, const odi_cuda_matmul_opts* opts, void* d_recs,
                              int flags, void* stream);

/* Options of odi_cuda_matmul_q8rec (all zero / NULL: the plain product). */
typedef struct odi_cuda_q8rec_opts {
  int accumulate;              /* y += product */
  float* out_ssq;              /* as odi_cuda_matmul_opts.out_ssq */
  /* The input records hold u = x * w of an RMSNorm (x its input, w its
   * weights): each token's records are scaled by 1 / sqrt(sum(x^2) / K + eps)
   * first, the sum from norm_ssq_count slots per token (out_ssq of x's
   * writer).  The quantisation of u differs from that of the normalised row
   * only by the fp16 rounding of each block scale. */
  const float* norm_ssq;
  int norm_ssq_count;
  float norm_eps;
  /* Records of the stored y for the next product ([N/256][M], 16-byte
   * aligned; N a multiple of 256): of y * out_norm_weight (the next
   * RMSNorm's weights) or of y itself; or, with out_swiglu, the weight's
   * rows being 32 gate rows then the 32 matching up rows in every 64-row
   * tile (N a multiple of 512), of silu(gate) * up ([N/512][M] records). */
  void* out_records;
  const float* out_norm_weight;
  int out_swiglu;
} odi_cuda_q8rec_opts;

/* The streaming GEMV (ACT_Q8) on pre-quantized Q8 records, with the options
 * above (opts may be NULL).  Workspace: 256 bytes. */
int odi_cuda_matmul_q8rec(int dtype, const void* d_w_tiled, const void* d_recs, float* d_y, int64_t M, int64_t N,
                          int64_t K, void* d_workspace, size_t workspace_bytes, int flags,
                          const odi_cuda_q8rec_opts* opts, void* stream);

/* Reads and clears the device-side error word of a workspace (kernel waits
 * that gave up set it).  Synchronises `stream`.  *status = 0 when clean. */
int odi_cuda_workspace_status(void* d_workspace, int* status, void* stream);

/* Tiled weight -> fp32 [N, K] on the device (Backend::dequantize,
 * backend.hpp:111; cpu_backend.cpp:625-648). */
int odi_cuda_dequantize(int dtype, const void* d_w_tiled, float* d_out, int64_t N, int64_t K,
                        void* stream);

/* Host-buffer form of Backend::matmul as the reference Context calls it
 * (context.cpp:152, 188-190): h_x [M, K] and h_y [M, N] are host memory;
 * the call brings x in, runs the product on the weight's device copy,
 * brings y out and waits.  Uses a library-owned per-device workspace.
 * A page-locked h_x (cudaHostAlloc / cudaHostRegister) is read by a small
 * kernel whose loads overlap the start of the product's weight stream
 * (programmatic dependent launch); pageable x goes in with cudaMemcpyAsync.
 * A page-locked h_y is written by the product itself, saving a copy's
 * latency (the tensor-core path and pageable buffers copy y out).
 * Returns ODI_CUDA_ERR_OPERATION_FAILED (h_y not to be used) when a kernel's
 * bounded wait gave up, as cpu_backend.cpp:177-227 throws on failure. */
int odi_cuda_matmul_host(const odi_cuda_weight* w, const float* h_x, float* h_y, int64_t M,
                         int act_mode, void* stream);

/* odi_cuda_matmul_host without the wait: the product is queued on `stream`
 * and the call returns.  This is the Backend::matmul / Backend::sync pair
 * (backend.hpp:38, 130) with sync made meaningful, as a CUDA backend is
 * allowed to: a caller with several independent products (the seven
 * per-layer products of a batch of sequences, a prefill split into chunks)
 * queues them and syncs once, and each product's x arrives while the one
 * before it runs.  h_x must stay unchanged, and h_y unread, until
 * odi_cuda_host_sync(stream) returns; products on one stream run in call
 * order and share the device workspace, so they need not be separated by
 * syncs.  With page-locked buffers nothing waits; pageable ones make the
 * copy in or out synchronous.  A page-locked h_y is filled by the library
 * in batches (its output parked on the device, then copied out by one
 * launch per batch of up to 200 products and at the sync), so the products
 * themselves touch no host memory. */
int odi_cuda_matmul_host_async(const odi_cuda_weight* w, const float* h_x, float* h_y, int64_t M,
                               int act_mode, void* stream);

/* Waits for the host-buffer products queued on `stream` (current device)
 * and reads, then clears, the error word they report into:
 * ODI_CUDA_ERR_OPERATION_FAILED when a kernel's bounded wait gave up in any
 * of them (their h_y are then not to be used). */
int odi_cuda_host_sync(void* stream);

/* Host-buffer form of Backend::dequantize (backend.hpp:111;
 * cpu_backend.cpp:625-648) for an uploaded weight: h_out receives N*K fp32
 * values in block order ([N][K]).  Synchronous; the values pass through the
 * library's per-device output buffer (grown once to N*K*4 bytes, kept). */
int odi_cuda_dequantize_host(const odi_cuda_weight* w, float* h_out, void* stream);

/* --- decode step: the non-matmul operations of Context::forward ------------- */

/* Device-resident decode state: the next input token, its position (KV
 * slot) and the number of tokens generated.  Every decode operation reads
 * it from device memory and odi_cuda_argmax advances it, so one step can be
 * captured in a CUDA graph and replayed token after token. */
typedef struct odi_cuda_decode_state {
  int32_t token;
  int32_t pos;
  int32_t step;
  int32_t reserved;
} odi_cuda_decode_state;

/* x[E] = table[token] (Backend::embedding, cpu_backend.cpp:610-619; table
 * fp32 [vocab][E], an out-of-range token reads row 0).  d_ssq (or NULL):
 * the sum of squares of every 64 values, ceil(E / 64) floats, for a fused
 * RMSNorm (odi_cuda_matmul_opts.norm_ssq).  d_records (or NULL; E a
 * multiple of 256): x * d_norm_w (x itself when d_norm_w is NULL) as one
 * token's Q8 records, for odi_cuda_matmul_q8rec with norm_ssq. */
int odi_cuda_embed(const float* d_table, int64_t vocab, int64_t E, const odi_cuda_decode_state* d_state, float* d_x,
                   float* d_ssq, const float* d_norm_w, void* d_records, void* stream);

/* y = x / sqrt(mean(x^2) + eps) * w per row of n (Backend::rms_norm,
 * cpu_backend.cpp:388-414).  y may alias x. */
int odi_cuda_rms_norm(const float* d_x, const float* d_w, float* d_y, int64_t rows, int64_t n, float eps,
                      void* stream);

/* Rotary embedding of q [heads][head_dim] and k [kv_heads][head_dim] at the
 * state's pos (pairs i, i + head_dim/2, freq = theta^(-2i/head_dim):
 * Backend::rope, cpu_backend.cpp:500-539), then k and v appended to the fp16
 * caches [kv_heads][ctx][head_dim] at pos (context.cpp:205-214).
 * head_dim 64 or 128; pos >= ctx writes nothing. */
int odi_cuda_rope_kv(float* d_q, float* d_k, const float* d_v, void* d_kcache, void* d_vcache,
                     const odi_cuda_decode_state* d_state, int heads, int kv_heads, int head_dim, int ctx,
                     float theta, void* stream);

/* Attention of one query token over cache positions 0..pos (fp16 K, V;
 * fp32 scores and softmax), out [heads][head_dim] (Backend::attention,
 * cpu_backend.cpp:541-608, with the causal limit taken at the query's
 * absolute position).  Grouped-query heads share kv head h / (heads /
 * kv_heads); 1, 2, 4 or 8 query heads per kv head.  One launch: K and V
 * are streamed by bulk copies, split over about two CTAs per SM, and the
 * last CTA of each kv head folds the splits.  The caches must be 16-byte
 * aligned.  Needs odi_cuda_attention_scratch_bytes of 16-byte aligned
 * device scratch, zero-filled before its first use; each call leaves its
 * arrival counters zero again, so one scratch serves every layer and step
 * (calls on one stream only).  The scratch's first int is an error word
 * (odi_cuda_workspace_status reads it): non-zero if a bounded wait of the
 * kernel gave up. */
size_t odi_cuda_attention_scratch_bytes(int heads, int head_dim, int ctx);
int odi_cuda_attention_decode(const float* d_q, const void* d_kcache, const void* d_vcache, float* d_out,
                              const odi_cuda_decode_state* d_state, int heads, int kv_heads, int head_dim, int ctx,
                              float scale, void* d_scratch, size_t scratch_bytes, void* stream);

/* odi_cuda_rope_kv followed by odi_cuda_attention_decode, in one launch:
 * q [heads][head_dim], k and v [kv_heads][head_dim] are this step's raw
 * projections (q is rotated in registers and left unchanged in memory);
 * the rotated k and v are written as fp16 into the caches at the state's
 * pos (nothing is written when pos >= ctx).  Same results as the two calls;
 * same scratch and alignment rules as odi_cuda_attention_decode.  If
 * d_out_records is non-NULL (16-byte aligned,
 * odi_cuda_q8_records_bytes(1, heads * head_dim) bytes), the output row is
 * also written as the Q8 records odi_cuda_quantize_records would make of
 * it, ready for odi_cuda_matmul_q8rec. */
int odi_cuda_rope_attention(const float* d_q, const float* d_k, const float* d_v, void* d_kcache, void* d_vcache,
                            float* d_out, void* d_out_records, const odi_cuda_decode_state* d_state, int heads,
                            int kv_heads, int head_dim, int ctx, float theta, float scale, void* d_scratch,
                            size_t scratch_bytes, void* stream);

/* out[F] = silu(gate) * up with gate_up = [gate F | up F] (context.cpp:272-275). */
int odi_cuda_silu_mul(const float* d_gate_up, float* d_out, int64_t F, void* stream);

/* x += d (the residual adds of context.cpp:124, 130). */
int odi_cuda_add(float* d_x, const float* d_d, int64_t n, void* stream);

/* Greedy next token (first index of the largest logit): sets state.token,
 * stores it at d_record[state.step] when step < record_len, then advances
 * step and pos. */
int odi_cuda_argmax(const float* d_logits, int64_t V, odi_cuda_decode_state* d_state, int32_t* d_record,
                    int record_len, void* stream);

/* --- the decode step as one call per token ----------------------------------
 * A device-resident decoder of a Llama-shaped model: one token's forward
 * pass (context.cpp:84-282 for a single token, with cpu_backend.cpp:388-619's
 * element-wise ops on the device) captured once as a CUDA graph and replayed
 * per token; the token and position stay on the device and the greedy
 * argmax advances them.  For a C++ engine that calls it once per token
 * instead of one Backend call per operation. */
typedef struct odi_cuda_decoder_config {
  int layers, hidden, heads, kv_heads, head_dim, ffn, vocab;
  int ctx;          /* KV cache positions */
  float eps;        /* RMSNorm epsilon */
  float theta;      /* RoPE base */
  int attn_dtype;   /* Q|K|V, O and gate|up weights */
  int down_dtype;   /* down and output weights */
} odi_cuda_decoder_config;

/* One layer's device weights, tiled (odi_cuda_weight_data / odi_cuda_repack):
 * wqkv has (heads + 2 kv_heads) * head_dim rows, Q, K and V stacked; wgu
 * has 2 * ffn rows, gate and up interleaved 32 rows each per 64-row tile
 * (row p is gate row 32t + p % 64 when p % 64 < 32, else up row
 * 32t + p % 64 - 32, t = p / 64).  Norm weights fp32 [hidden]. */
typedef struct odi_cuda_decoder_layer {
  const float* attn_norm;
  const void* wqkv;
  const void* wo;
  const float* ffn_norm;
  const void* wgu;
  const void* wdown;
} odi_cuda_decoder_layer;

typedef struct odi_cuda_decoder odi_cuda_decoder;

/* Builds the decoder on the current device: its buffers (fp16 KV cache of
 * layers * kv_heads * ctx * head_dim per K and V, activations, Q8 records),
 * one eager step, then the captured step.  The weights stay the caller's
 * and must outlive the decoder.  token_embd fp32 [vocab][hidden]; output
 * [vocab rows x hidden]; max_record: tokens the device record holds
 * between resets.  hidden, ffn and heads * head_dim multiples of 256. */
int odi_cuda_decoder_create(const odi_cuda_decoder_config* cfg, const float* d_token_embd,
                            const odi_cuda_decoder_layer* layers, const float* d_out_norm, const void* d_output,
                            int max_record, odi_cuda_decoder** decoder);
int odi_cuda_decoder_free(odi_cuda_decoder* decoder);
/* Next step reads `token` at position `pos`; the record restarts; with
 * clear_cache the KV cache is zeroed (a new sequence). */
int odi_cuda_decoder_reset(odi_cuda_decoder* decoder, int token, int pos, int clear_cache);
/* The prompt into the cache: one step per token at positions pos0.. */
int odi_cuda_decoder_prefill(odi_cuda_decoder* decoder, const int32_t* tokens, int n, int pos0);
/* n greedy steps from the current state; out_tokens receives them.  Fails
 * with ODI_CUDA_ERR_OPERATION_FAILED if a bounded device wait gave up. */
int odi_cuda_decoder_generate(odi_cuda_decoder* decoder, int n, int32_t* out_tokens);
/* n greedy steps timed on the device (CUDA events around the replays). */
int odi_cuda_decoder_time(odi_cuda_decoder* decoder, int n, float* ms);
/* Tokens [start, start + n) of the device record since the last reset. */
int odi_cuda_decoder_tokens(odi_cuda_decoder* decoder, int start, int n, int32_t* out_tokens);
/* The last step's logits, vocab fp32 values. */
int odi_cuda_decoder_logits(odi_cuda_decoder* decoder, float* out);
/* Kernel launches in one step. */
int odi_cuda_decoder_launches_per_step(const odi_cuda_decoder* decoder);

/* A plain device copy of host bytes (norm weights, embedding tables) and its
 * release. */
int odi_cuda_buffer_upload(const void* host, size_t bytes, void** d_ptr);
int odi_cuda_buffer_free(void* d_ptr);

/* --- row-sharded product with the all-gather fused into the GEMV ------------ */

/* A weight sharded by output rows over nranks GPUs (one process each): rank
 * r holds rows [row0, row0 + N) of the full ld-row weight.  Instead of a
 * GEMV followed by an all-gather of the slices (ncclAllGather), each rank's
 * GEMV stores its slice straight into every rank's gathered output buffer
 * (peer stores over NVLink); the last CTA of each launch then adds one
 * arrival to its slot [rank] of every rank's counter array (release, system
 * scope).  The workspace's first 256 bytes hold the launch's completion
 * count: zero at start, left zero by every launch that completes.
 *   out[p]      : rank p's gathered output, [M][ld] fp32 (own rank included)
 *   counters[p] : rank p's arrival counters, nranks uint64 (zero at start)
 * Peer addresses come from odi_cuda_sym_alloc / odi_cuda_ipc_open.  No TMA
 * and no multicast: plain stores and system-scope atomics. */
#define ODI_CUDA_MAX_PEERS 8
#define ODI_CUDA_IPC_HANDLE_BYTES 64
typedef struct odi_cuda_scatter {
  float* out[ODI_CUDA_MAX_PEERS];
  unsigned long long* counters[ODI_CUDA_MAX_PEERS];
  int nranks;
  int rank;
  int64_t row0;
  int64_t ld;
} odi_cuda_scatter;

/* Arrivals one odi_cuda_matmul_scatter call of this shard shape adds to
 * its slot on every rank (one per launch: ceil(M / tokens per pass)); -1 if
 * the shape / mode has no fused path (the tensor-core modes). */
int64_t odi_cuda_scatter_signals(int dtype, int64_t M, int64_t N, int64_t K, int act_mode);

/* The GEMV of odi_cuda_matmul on this rank's shard (N = shard rows), with
 * the output scattered as described above.  ACT_Q8 / ACT_F32 (and AUTO
 * below ODI_CUDA_TC_MIN_TOKENS).  Asynchronous on `stream`. */
int odi_cuda_matmul_scatter(int dtype, const void* d_w_tiled, const float* d_x, int64_t M, int64_t N,
                            int64_t K, int act_mode, void* d_workspace, size_t workspace_bytes, int flags,
                            const odi_cuda_scatter* sc, void* stream);

/* Before using the gathered output: waits (one small kernel on `stream`)
 * until every source rank p's counter reached d_consumed[p] +
 * increments[p] (increments = odi_cuda_scatter_signals of rank p's shard),
 * then advances d_consumed.  d_counters / d_consumed are this rank's own
 * arrays (nranks uint64, zero at start).  Bounded: a rank that has not
 * arrived after one second sets ODI_CUDA_WS_ERR_PEER_WAIT in the workspace
 * error word (see odi_cuda_workspace_status) and the kernel returns; the
 * gathered output is then invalid.  The counterpart of the all-gather that
 * follows a row-sharded Backend::matmul (backend.hpp:38); the reference has
 * no multi-GPU path. */
int odi_cuda_wait_peers(const unsigned long long* d_counters, unsigned long long* d_consumed,
                        const unsigned long long* increments, int nranks, void* d_workspace, void* stream);

/* odi_cuda_wait_peers with the give-up time chosen by the caller
 * (1 us .. 60 s), for failure detection that must answer faster than the
 * default second. */
int odi_cuda_wait_peers_timeout(const unsigned long long* d_counters, unsigned long long* d_consumed,
                                const unsigned long long* increments, int nranks, uint64_t timeout_us,
                                void* d_workspace, void* stream);

/* Bits of the workspace error word (odi_cuda_workspace_status): a bounded
 * device wait that gave up. */
#define ODI_CUDA_WS_ERR_FULL_WAIT 1
#define ODI_CUDA_WS_ERR_EMPTY_WAIT 2
#define ODI_CUDA_WS_ERR_DRAIN_WAIT 4
#define ODI_CUDA_WS_ERR_REDUCE_WAIT 8
#define ODI_CUDA_WS_ERR_PEER_WAIT 32

/* Zeroed device buffer for sharing with other processes: *d_ptr and the
 * ODI_CUDA_IPC_HANDLE_BYTES-byte handle to pass to the other ranks. */
int odi_cuda_sym_alloc(size_t bytes, void** d_ptr, void* ipc_handle);
int odi_cuda_sym_free(void* d_ptr);
/* Map another rank's buffer (handle from its odi_cuda_sym_alloc). */
int odi_cuda_ipc_open(const void* ipc_handle, void** d_ptr);
int odi_cuda_ipc_close(void* d_ptr);

/* --- row-sharded product over an NCCL communicator ---------------------------
 * A weight too large (or too slow) for one GPU is split by output rows across
 * the GPUs of one node, one process each; every rank computes its rows and the
 * slices are all-gathered with NCCL over NVLink.  This is the C-ABI form of
 * the row sharding a Backend::matmul (backend.hpp:38) needs once the model
 * spans GPUs; the reference has no multi-GPU path.  NCCL (libnccl.so.2) is
 * opened at run time: these calls fail with ODI_CUDA_ERR_BACKEND_UNAVAILABLE
 * where it is absent, and nothing else depends on it. */
#define ODI_CUDA_NCCL_ID_BYTES 128
typedef struct odi_cuda_comm odi_cuda_comm;

/* A new communicator id: one rank makes it and hands the bytes to the others
 * over any host channel. */
int odi_cuda_nccl_unique_id(void* id /* ODI_CUDA_NCCL_ID_BYTES */);
/* Joins the communicator as `rank` of `nranks` on the current device (every
 * rank calls it; it returns when all have joined). */
int odi_cuda_nccl_init(const void* id, int nranks, int rank, odi_cuda_comm** comm);
int odi_cuda_nccl_free(odi_cuda_comm* comm);
int odi_cuda_comm_ranks(const odi_cuda_comm* comm, int* nranks, int* rank);

/* Device workspace of odi_cuda_matmul_sharded: the product's workspace for
 * the shard, then the gather buffer of nranks * M * S fp32. */
size_t odi_cuda_sharded_workspace_bytes(const odi_cuda_comm* comm, int dtype, int64_t M, int64_t S, int64_t K,
                                        int act_mode);

/* d_y [M, N] = d_x [M, K] . W^T on every rank, W [N rows] split by rows:
 * rank r holds rows [r*S, min(N, (r+1)*S)) as its own tiled weight of S rows
 * (rows past N zero; S = ceil(N / nranks) is the usual split).  The rank
 * computes its S rows, the slices are all-gathered in place (ncclAllGather
 * on `stream`), and -- unless M = 1 and N = nranks * S, where the gathered
 * slices are y itself -- one small kernel lays them out as [M, N].  All
 * ranks call it with the same M, N, S, K and act_mode, in the same order
 * as their other collectives. */
int odi_cuda_matmul_sharded(odi_cuda_comm* comm, int dtype, const void* d_w_shard, const float* d_x, float* d_y,
                            int64_t M, int64_t N, int64_t S, int64_t K, int act_mode, void* d_workspace,
                            size_t workspace_bytes, int flags, void* stream);

/* Size of the static device array behind odi_cuda_matmul_host_noalloc. */
#define ODI_CUDA_NOALLOC_SCRATCH_BYTES (8u << 20)

/* The product of odi_cuda_matmul_host, for callers that must not allocate
 * device memory once they are running.  No counterpart in the reference.
 *
 * Who needs it: an engine that reserves HBM for its weights and KV cache up
 * front cannot have a later cudaMalloc fail or carve into that reservation;
 * a process whose device memory belongs to another allocator's pool must
 * not allocate behind that pool's back; a decode loop cannot afford the
 * device-wide synchronisation that cudaMalloc / cudaFree may cause.
 * odi_cuda_matmul_host grows a per-device buffer with cudaMalloc whenever it
 * meets a larger M; this call allocates nothing.  It stages x, y and the
 * kernels' error word in one static device array of
 * ODI_CUDA_NOALLOC_SCRATCH_BYTES per GPU, part of the library's device image:
 * every GPU that loads the library holds that array until the process exits.
 * (The weight itself is uploaded beforehand, at load time, by
 * odi_cuda_weight_upload.)
 *
 * Limit: round_up(W, 256) + round_up(M*K*4, 256) + M*N*4 <=
 * ODI_CUDA_NOALLOC_SCRATCH_BYTES, W = odi_cuda_matmul_workspace_bytes (256
 * for one token or fp32 activations, so M=1 fits any N up to about two
 * million; 256 + ceil(K/256)*M*384 for a multi-token Q8 product; the fp16
 * activation tiles on the tensor-core path); a larger call returns
 * ODI_CUDA_ERR_INVALID_ARGUMENT and runs nothing.
 *
 * The call itself allocates nothing, but the first call of each kernel
 * variant (dtype x activation mode x tokens per pass) may make the CUDA
 * driver load that kernel's code under lazy module loading, which can
 * reserve device memory: make one call of each variant in use (or run with
 * CUDA_MODULE_LOADING=EAGER) before the phase that must not allocate.
 *
 * The first call on a device, with that device current, looks up the
 * array's device address; make that first call before any stream capture on
 * the device.  All calls share the one array per device: each call clears
 * the error word (the only part that must start at zero) and overwrites the
 * x and y regions.  Calls whose GPU work overlaps -- e.g. two host threads
 * on two streams of the same device -- race on the array and corrupt each
 * other's results, so serialise them.  Synchronous: returns once h_y holds
 * the result; ODI_CUDA_ERR_OPERATION_FAILED if a kernel wait gave up. */
int odi_cuda_matmul_host_noalloc(const odi_cuda_weight* w, const float* h_x, float* h_y, int64_t M,
                                 int act_mode, void* stream);

#ifdef __cplusplus
}
#endif
#endif
