// decoder.cu -- the device-resident decode step behind the C ABI
// (odi_cuda_decoder_*): one token of a Llama-shaped model per step, the
// reference's Context::forward for a single token (src/core/context.cpp:84-282)
// with the CPU backend's element-wise ops (cpu_backend.cpp:388-619) done on
// the device, for a C++ engine to call once per token.
//
// The step (5 launches per layer, every product on the Q8 records its
// producer wrote; the token and position live on the device and argmax
// advances them):
//   embed (x, its sums of squares, records of x * attn_norm[0])
//   per layer:
//     QKV GEMV on the records, scaled by 1/rms from the sums of squares
//     attention with RoPE and the fp16 KV append fused in; writes the O
//       GEMV's records
//     O GEMV, x += ...; leaves x's sums of squares and records of x * ffn_norm
//     gate|up GEMV (rows interleaved 32 gate / 32 up per 64-row tile) on the
//       scaled records; writes the records of silu(gate) * up
//     down GEMV, x += ...; leaves the sums of squares and records of
//       x * the next norm's weights
//   output GEMV (records scaled by 1/rms), argmax
// The step is captured once as a CUDA graph on the decoder's stream and
// replayed per token: prefill replays it per prompt token (the state copied
// in first), generate replays it n times and reads the recorded tokens back.
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/odi_cuda.h"
#include "internal.h"

namespace {

// errors go to the C ABI's record (odi_cuda_last_error)
int dec_fail(int code, const std::string& msg) { return odi_cuda::set_error(code, msg.c_str()); }

size_t round256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

struct odi_cuda_decoder {
  odi_cuda_decoder_config cfg;
  std::vector<odi_cuda_decoder_layer> layers;
  const float* token_embd = nullptr;
  const float* out_norm = nullptr;
  const void* output = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  // one device allocation carved into the step's buffers
  void* arena = nullptr;
  float *x = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr, *logits = nullptr, *ssq = nullptr;
  uint8_t *rec_e = nullptr, *rec_a = nullptr, *rec_f = nullptr;
  __half *kc = nullptr, *vc = nullptr;
  void* att_scratch = nullptr;
  size_t att_scratch_bytes = 0;
  uint8_t* gemv_ws = nullptr;  // one WS_HEADER slot per product of the step (error words)
  int n_gemv = 0;
  odi_cuda_decode_state* state = nullptr;
  int32_t* record = nullptr;
  int max_record = 0;
  odi_cuda_decode_state* h_state = nullptr;  // page-locked staging for state copies
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int generated = 0;  // steps replayed since the last reset
};

namespace {

// Enqueue one decode step on d->stream.
int enqueue_step(odi_cuda_decoder* d) {
  const odi_cuda_decoder_config& c = d->cfg;
  const int E = c.hidden, H = c.heads, KV = c.kv_heads, hd = c.head_dim, F = c.ffn;
  const int qkv_rows = (H + 2 * KV) * hd;
  const int slots = (E + 63) / 64;
  void* s = d->stream;
  float* q = d->qkv;
  float* k = q + (size_t)H * hd;
  float* v = k + (size_t)KV * hd;
  const float scale = 1.0f / sqrtf((float)hd);
  int rc = odi_cuda_embed(d->token_embd, c.vocab, E, d->state, d->x, d->ssq, d->layers[0].attn_norm, d->rec_e, s);
  if (rc) return rc;
  int g = 0;
  auto q8rec = [&](int dtype, const void* w, const uint8_t* rec, float* y, int64_t N, int64_t K,
                   const odi_cuda_q8rec_opts& o) {
    uint8_t* ws = d->gemv_ws + (size_t)(g++) * odi_cuda::WS_HEADER;
    return odi_cuda_matmul_q8rec(dtype, w, rec, y, 1, N, K, ws, odi_cuda::WS_HEADER, ODI_CUDA_FLAG_PDL, &o, s);
  };
  for (int li = 0; li < c.layers; ++li) {
    const odi_cuda_decoder_layer& L = d->layers[li];
    const float* next_norm = li + 1 < c.layers ? d->layers[li + 1].attn_norm : d->out_norm;
    const size_t kvoff = (size_t)li * KV * c.ctx * hd;
    odi_cuda_q8rec_opts o{};
    o.norm_ssq = d->ssq;
    o.norm_ssq_count = slots;
    o.norm_eps = c.eps;
    if ((rc = q8rec(c.attn_dtype, L.wqkv, d->rec_e, d->qkv, qkv_rows, E, o))) return rc;
    if ((rc = odi_cuda_rope_attention(q, k, v, d->kc + kvoff, d->vc + kvoff, d->attn, d->rec_a, d->state, H, KV, hd,
                                      c.ctx, c.theta, scale, d->att_scratch, d->att_scratch_bytes, s)))
      return rc;
    o = odi_cuda_q8rec_opts{};
    o.accumulate = 1;
    o.out_ssq = d->ssq;
    o.out_records = d->rec_e;
    o.out_norm_weight = L.ffn_norm;
    if ((rc = q8rec(c.attn_dtype, L.wo, d->rec_a, d->x, E, (int64_t)H * hd, o))) return rc;
    o = odi_cuda_q8rec_opts{};
    o.norm_ssq = d->ssq;
    o.norm_ssq_count = slots;
    o.norm_eps = c.eps;
    o.out_records = d->rec_f;
    o.out_swiglu = 1;
    if ((rc = q8rec(c.attn_dtype, L.wgu, d->rec_e, d->gu, 2 * (int64_t)F, E, o))) return rc;
    o = odi_cuda_q8rec_opts{};
    o.accumulate = 1;
    o.out_ssq = d->ssq;
    o.out_records = d->rec_e;
    o.out_norm_weight = next_norm;
    if ((rc = q8rec(c.down_dtype, L.wdown, d->rec_f, d->x, E, F, o))) return rc;
  }
  odi_cuda_q8rec_opts o{};
  o.norm_ssq = d->ssq;
  o.norm_ssq_count = slots;
  o.norm_eps = c.eps;
  if ((rc = q8rec(c.down_dtype, d->output, d->rec_e, d->logits, c.vocab, E, o))) return rc;
  return odi_cuda_argmax(d->logits, c.vocab, d->state, d->record, d->max_record, s);
}

int dec_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ODI_CUDA_OK;
  return dec_fail(e == cudaErrorMemoryAllocation ? ODI_CUDA_ERR_GPU_OUT_OF_MEMORY : ODI_CUDA_ERR_OPERATION_FAILED,
                  std::string(what) + ": " + cudaGetErrorString(e));
}

// OR of every error word of the step (the products' workspaces and the
// attention scratch); synchronises the stream.
int dec_status(odi_cuda_decoder* d, int* word) {
  std::vector<int> w((size_t)d->n_gemv * (odi_cuda::WS_HEADER / sizeof(int)));
  int a = 0;
  cudaError_t e = cudaMemcpyAsync(w.data(), d->gemv_ws, w.size() * sizeof(int), cudaMemcpyDeviceToHost, d->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&a, d->att_scratch, sizeof(int), cudaMemcpyDeviceToHost, d->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
  if (e != cudaSuccess) return dec_cuda(e, "reading the error words");
  int v = a;
  for (int i = 0; i < d->n_gemv; ++i) v |= w[(size_t)i * (odi_cuda::WS_HEADER / sizeof(int))];
  *word = v;
  return ODI_CUDA_OK;
}

int dec_check(odi_cuda_decoder* d) {
  int v = 0;
  int rc = dec_status(d, &v);
  if (rc) return rc;
  if (v) {
    char buf[96];
    snprintf(buf, sizeof buf, "decode step: a bounded device wait gave up (error word 0x%x)", v);
    return dec_fail(ODI_CUDA_ERR_OPERATION_FAILED, buf);
  }
  return ODI_CUDA_OK;
}

void dec_free(odi_cuda_decoder* d) {
  if (!d) return;
  if (d->exec) cudaGraphExecDestroy(d->exec);
  if (d->graph) cudaGraphDestroy(d->graph);
  if (d->arena) cudaFree(d->arena);
  if (d->h_state) cudaFreeHost(d->h_state);
  if (d->stream) cudaStreamDestroy(d->stream);
  delete d;
}

}  // namespace

extern "C" {

int odi_cuda_decoder_create(const odi_cuda_decoder_config* cfg, const float* d_token_embd,
                            const odi_cuda_decoder_layer* layers, const float* d_out_norm, const void* d_output,
                            int max_record, odi_cuda_decoder** out) {
  if (!cfg || !d_token_embd || !layers || !d_out_norm || !d_output || !out)
    return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: null argument");
  *out = nullptr;
  const odi_cuda_decoder_config& c = *cfg;
  if (c.layers < 1 || c.hidden < 256 || c.hidden % 256 || c.heads < 1 || c.kv_heads < 1 || c.heads % c.kv_heads ||
      (c.head_dim != 64 && c.head_dim != 128) || c.ffn < 256 || c.ffn % 256 || c.vocab < 1 || c.ctx < 1 ||
      max_record < 0)
    return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT,
                    "decoder: shape needs hidden and ffn multiples of 256, head_dim 64 or 128, heads a multiple of "
                    "kv_heads");
  if ((c.heads * c.head_dim) % 256)
    return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: heads * head_dim must be a multiple of 256");
  if (odi_cuda_supports_dtype(c.attn_dtype) != 1 || odi_cuda_supports_dtype(c.down_dtype) != 1)
    return dec_fail(ODI_CUDA_ERR_UNSUPPORTED_DTYPE, "decoder: weight dtype not supported");
  for (int i = 0; i < c.layers; ++i)
    if (!layers[i].attn_norm || !layers[i].wqkv || !layers[i].wo || !layers[i].ffn_norm || !layers[i].wgu ||
        !layers[i].wdown)
      return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: null weight in layer " + std::to_string(i));
  odi_cuda_decoder* d = new (std::nothrow) odi_cuda_decoder;
  if (!d) return dec_fail(ODI_CUDA_ERR_OUT_OF_MEMORY, "decoder: host allocation failed");
  d->cfg = c;
  d->layers.assign(layers, layers + c.layers);
  d->token_embd = d_token_embd;
  d->out_norm = d_out_norm;
  d->output = d_output;
  d->max_record = max_record;
  int rc = dec_cuda(cudaGetDevice(&d->device), "cudaGetDevice");
  if (!rc) rc = dec_cuda(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  if (!rc) rc = dec_cuda(cudaHostAlloc(reinterpret_cast<void**>(&d->h_state), 64 * sizeof(odi_cuda_decode_state), 0),
                         "cudaHostAlloc (state)");
  if (rc) {
    dec_free(d);
    return rc;
  }
  // layout of the arena
  const size_t E = c.hidden, F = c.ffn, H = c.heads, KV = c.kv_heads, hd = c.head_dim;
  const size_t qkv_rows = (H + 2 * KV) * hd;
  d->n_gemv = 4 * c.layers + 1;
  d->att_scratch_bytes = round256(odi_cuda_attention_scratch_bytes((int)H, (int)hd, c.ctx));
  const size_t kv_bytes = (size_t)c.layers * KV * c.ctx * hd * sizeof(__half);
  size_t off = 0;
  auto take = [&](size_t b) { const size_t o = off; off += round256(b); return o; };
  const size_t o_x = take(E * 4), o_qkv = take(qkv_rows * 4), o_attn = take(H * hd * 4), o_gu = take(2 * F * 4),
               o_logits = take((size_t)c.vocab * 4), o_ssq = take((E + 63) / 64 * 4),
               o_rec_e = take(odi_cuda_q8_records_bytes(1, E)), o_rec_a = take(odi_cuda_q8_records_bytes(1, H * hd)),
               o_rec_f = take(odi_cuda_q8_records_bytes(1, F)), o_att = take(d->att_scratch_bytes),
               o_ws = take((size_t)d->n_gemv * odi_cuda::WS_HEADER), o_state = take(sizeof(odi_cuda_decode_state)),
               o_rec = take((size_t)(max_record > 0 ? max_record : 1) * 4), o_kc = take(kv_bytes), o_vc = take(kv_bytes);
  rc = dec_cuda(cudaMalloc(&d->arena, off), "cudaMalloc (decoder buffers)");
  if (!rc) rc = dec_cuda(cudaMemsetAsync(d->arena, 0, off, d->stream), "cudaMemset (decoder buffers)");
  if (rc) {
    dec_free(d);
    return rc;
  }
  uint8_t* base = static_cast<uint8_t*>(d->arena);
  d->x = reinterpret_cast<float*>(base + o_x);
  d->qkv = reinterpret_cast<float*>(base + o_qkv);
  d->attn = reinterpret_cast<float*>(base + o_attn);
  d->gu = reinterpret_cast<float*>(base + o_gu);
  d->logits = reinterpret_cast<float*>(base + o_logits);
  d->ssq = reinterpret_cast<float*>(base + o_ssq);
  d->rec_e = base + o_rec_e;
  d->rec_a = base + o_rec_a;
  d->rec_f = base + o_rec_f;
  d->att_scratch = base + o_att;
  d->gemv_ws = base + o_ws;
  d->state = reinterpret_cast<odi_cuda_decode_state*>(base + o_state);
  d->record = reinterpret_cast<int32_t*>(base + o_rec);
  d->kc = reinterpret_cast<__half*>(base + o_kc);
  d->vc = reinterpret_cast<__half*>(base + o_vc);
  // One eager step (kernel attributes, lazy module loading), then the graph.
  rc = enqueue_step(d);
  if (!rc) rc = dec_cuda(cudaStreamSynchronize(d->stream), "first step");
  if (!rc) rc = dec_check(d);
  if (!rc) rc = dec_cuda(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
  if (!rc) {
    const int src = enqueue_step(d);
    const cudaError_t e = cudaStreamEndCapture(d->stream, &d->graph);
    rc = src ? src : dec_cuda(e, "end capture");
  }
  if (!rc) rc = dec_cuda(cudaGraphInstantiate(&d->exec, d->graph, 0), "graph instantiate");
  // the eager step wrote KV position 0 and the record: start clean
  if (!rc) rc = dec_cuda(cudaMemsetAsync(d->arena, 0, off, d->stream), "cudaMemset (decoder buffers)");
  if (!rc) rc = dec_cuda(cudaStreamSynchronize(d->stream), "sync");
  if (rc) {
    dec_free(d);
    return rc;
  }
  *out = d;
  return ODI_CUDA_OK;
}

int odi_cuda_decoder_free(odi_cuda_decoder* d) {
  if (!d) return ODI_CUDA_OK;
  cudaStreamSynchronize(d->stream);
  dec_free(d);
  return ODI_CUDA_OK;
}

int odi_cuda_decoder_reset(odi_cuda_decoder* d, int token, int pos, int clear_cache) {
  if (!d) return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: null");
  if (token < 0 || token >= d->cfg.vocab || pos < 0 || pos >= d->cfg.ctx)
    return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: token or position out of range");
  int rc = dec_cuda(cudaStreamSynchronize(d->stream), "sync");
  if (rc) return rc;
  d->h_state[0] = odi_cuda_decode_state{token, pos, 0, 0};
  rc = dec_cuda(cudaMemcpyAsync(d->state, d->h_state, sizeof(odi_cuda_decode_state), cudaMemcpyHostToDevice,
                                d->stream), "state copy");
  if (!rc && d->max_record > 0)
    rc = dec_cuda(cudaMemsetAsync(d->record, 0xff, (size_t)d->max_record * 4, d->stream), "record reset");
  if (!rc && clear_cache) {
    const size_t kv_bytes = (size_t)d->cfg.layers * d->cfg.kv_heads * d->cfg.ctx * d->cfg.head_dim * sizeof(__half);
    rc = dec_cuda(cudaMemsetAsync(d->kc, 0, kv_bytes, d->stream), "cache clear");
    if (!rc) rc = dec_cuda(cudaMemsetAsync(d->vc, 0, kv_bytes, d->stream), "cache clear");
  }
  if (!rc) rc = dec_cuda(cudaStreamSynchronize(d->stream), "sync");
  d->generated = 0;
  return rc;
}

int odi_cuda_decoder_prefill(odi_cuda_decoder* d, const int32_t* tokens, int n, int pos0) {
  if (!d || (n > 0 && !tokens)) return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: null argument");
  if (n < 0 || pos0 < 0 || (int64_t)pos0 + n > d->cfg.ctx)
    return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: prompt runs past the context");
  int rc = dec_cuda(cudaStreamSynchronize(d->stream), "sync");
  // One step per prompt token: its state (token, position) goes in first,
  // through page-locked staging slots reused once the stream has passed them.
  for (int i = 0; i < n && !rc; ++i) {
    const int slot = i & 63;
    if (slot == 0 && i) rc = dec_cuda(cudaStreamSynchronize(d->stream), "sync");
    if (tokens[i] < 0 || tokens[i] >= d->cfg.vocab) {
      rc = dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: prompt token out of range");
      break;
    }
    d->h_state[slot] = odi_cuda_decode_state{tokens[i], pos0 + i, 0, 0};
    if (!rc)
      rc = dec_cuda(cudaMemcpyAsync(d->state, d->h_state + slot, sizeof(odi_cuda_decode_state),
                                    cudaMemcpyHostToDevice, d->stream), "state copy");
    if (!rc) rc = dec_cuda(cudaGraphLaunch(d->exec, d->stream), "graph launch");
  }
  if (rc) return rc;
  d->generated = 0;
  return dec_check(d);
}

int odi_cuda_decoder_generate(odi_cuda_decoder* d, int n, int32_t* out_tokens) {
  if (!d || (n > 0 && !out_tokens)) return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: null argument");
  if (n < 0 || d->generated + n > d->max_record)
    return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: more tokens than the record holds");
  int rc = ODI_CUDA_OK;
  for (int i = 0; i < n && !rc; ++i) rc = dec_cuda(cudaGraphLaunch(d->exec, d->stream), "graph launch");
  if (!rc)
    rc = dec_cuda(cudaMemcpyAsync(out_tokens, d->record + d->generated, (size_t)n * 4, cudaMemcpyDeviceToHost,
                                  d->stream), "token copy");
  if (!rc) rc = dec_check(d);  // synchronises
  if (!rc) d->generated += n;
  return rc;
}

int odi_cuda_decoder_time(odi_cuda_decoder* d, int n, float* ms) {
  if (!d || !ms || n < 1) return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: bad argument");
  if (d->generated + n > d->max_record)
    return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: more tokens than the record holds");
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  int rc = dec_cuda(cudaEventCreate(&e0), "event");
  if (!rc) rc = dec_cuda(cudaEventCreate(&e1), "event");
  if (!rc) rc = dec_cuda(cudaEventRecord(e0, d->stream), "event record");
  for (int i = 0; i < n && !rc; ++i) rc = dec_cuda(cudaGraphLaunch(d->exec, d->stream), "graph launch");
  if (!rc) rc = dec_cuda(cudaEventRecord(e1, d->stream), "event record");
  if (!rc) rc = dec_cuda(cudaEventSynchronize(e1), "event sync");
  if (!rc) rc = dec_cuda(cudaEventElapsedTime(ms, e0, e1), "elapsed time");
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (!rc) rc = dec_check(d);
  if (!rc) d->generated += n;
  return rc;
}

int odi_cuda_decoder_tokens(odi_cuda_decoder* d, int start, int n, int32_t* out_tokens) {
  if (!d || !out_tokens || start < 0 || n < 0 || start + n > d->max_record)
    return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: bad token range");
  int rc = dec_cuda(cudaMemcpyAsync(out_tokens, d->record + start, (size_t)n * 4, cudaMemcpyDeviceToHost, d->stream),
                    "token copy");
  if (!rc) rc = dec_cuda(cudaStreamSynchronize(d->stream), "sync");
  return rc;
}

int odi_cuda_decoder_logits(odi_cuda_decoder* d, float* out) {
  if (!d || !out) return dec_fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "decoder: null argument");
  int rc = dec_cuda(cudaMemcpyAsync(out, d->logits, (size_t)d->cfg.vocab * 4, cudaMemcpyDeviceToHost, d->stream),
                    "logits copy");
  if (!rc) rc = dec_cuda(cudaStreamSynchronize(d->stream), "sync");
  return rc;
}

int odi_cuda_decoder_launches_per_step(const odi_cuda_decoder* d) {
  return d ? 1 + 5 * d->cfg.layers + 2 : 0;
}

}  // extern "C"
