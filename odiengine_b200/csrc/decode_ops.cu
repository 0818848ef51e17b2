// decode_ops.cu -- the non-matmul kernels of one decode step of a
// Llama-shaped model, device resident: the reference Context runs them on
// the host CPU backend (src/core/context.cpp:84-282, cpu_backend.cpp:354-619).
//
// The token and the position live in device memory (DecodeState), read by
// every kernel and advanced by the argmax kernel, so the whole step can be
// captured once in a CUDA graph and replayed token after token.
//
//   embed        x = token_embd[token]                 (cpu_backend.cpp:610-619)
//   rms_norm     y = x / sqrt(mean(x^2) + eps) * w     (cpu_backend.cpp:388-414)
//   rope_kv      NeoX rotation of q and k at pos (pairs i, i + hd/2,
//                freq = theta^(-2i/hd), cpu_backend.cpp:500-539); k and v
//                written to the fp16 KV cache [kv_head][ctx][hd] at pos
//                (the cache layout of context.cpp:205-214)
//   attention    softmax(q.K^T * scale) V over positions 0..pos, split over
//                chunks of positions (flash decoding) and combined
//   silu_mul     a = silu(gate) * up                    (context.cpp:272-275)
//   add          x += d                                 (context.cpp:124,130)
//   argmax       greedy next token; advances token and pos
#include <math.h>

#include "internal.h"

namespace odi_cuda {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One CTA of 64 threads per 64 values; with ssq, each CTA also leaves the
// sum of squares of its values (the slot a fused RMSNorm reads).
__global__ void embed_kernel(const float* __restrict__ table, const DecodeState* st, float* __restrict__ x,
                             float* __restrict__ ssq, int64_t E, int64_t vocab) {
  __shared__ float red[2];
  pdl_launch_dependents();
  pdl_wait();
  int tok = st->token;
  if (tok < 0 || tok >= vocab) tok = 0;  // out-of-range ids are rejected on the host; never read outside
  const int64_t i = blockIdx.x * 64ll + threadIdx.x;
  const float v = i < E ? table[(int64_t)tok * E + i] : 0.f;
  if (i < E) x[i] = v;
  if (ssq) {
    const float s = warp_sum(v * v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) ssq[blockIdx.x] = red[0] + red[1];
  }
}

// One CTA per row.
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                                int64_t n, float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  const float* xr = x + blockIdx.x * n;
  float* yr = y + blockIdx.x * n;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rms = 1.0f / sqrtf(red[0] / (float)n + eps);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) yr[i] = xr[i] * rms * w[i];
}

// grid: heads (q) + kv_heads (k and v); block hd/2 threads.
__global__ void rope_kv_kernel(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v,
                               __half* __restrict__ kc, __half* __restrict__ vc, const DecodeState* st, int heads,
                               int kv_heads, int hd, int ctx, float theta) {
  pdl_launch_dependents();
  pdl_wait();
  const int pos = st->pos;
  if (pos < 0 || pos >= ctx) return;  // the host keeps pos < ctx; never write outside the cache
  const int i = threadIdx.x, half = hd >> 1;
  if (i >= half) return;
  const float freq = 1.0f / powf(theta, 2.0f * (float)i / (float)hd);
  float sn, cs;
  sincosf((float)pos * freq, &sn, &cs);
  const int h = blockIdx.x;
  if (h < heads) {
    float* qh = q + (int64_t)h * hd;
    const float q0 = qh[i], q1 = qh[i + half];
    qh[i] = q0 * cs - q1 * sn;
    qh[i + half] = q0 * sn + q1 * cs;
  } else {
    const int kh = h - heads;
    float* kk = k + (int64_t)kh * hd;
    const float k0 = kk[i], k1 = kk[i + half];
    const float r0 = k0 * cs - k1 * sn, r1 = k0 * sn + k1 * cs;
    kk[i] = r0;
    kk[i + half] = r1;
    __half* kd = kc + ((int64_t)kh * ctx + pos) * hd;
    __half* vd = vc + ((int64_t)kh * ctx + pos) * hd;
    const float* vv = v + (int64_t)kh * hd;
    kd[i] = __float2half_rn(r0);
    kd[i + half] = __float2half_rn(r1);
    vd[i] = __float2half_rn(vv[i]);
    vd[i + half] = __float2half_rn(vv[i + half]);
  }
}

// Flash decoding in one launch.  CTA (h, c) covers positions
// [c*ATT_CHUNK, +ATT_CHUNK) of kv_len = pos + 1; its 8 warps take
// PW = ATT_CHUNK/8 positions each.  Lane l holds dims [l*HD/32, +HD/32) of q
// and of its running output.  A warp first loads all PW positions' k and v
// (coalesced: each position is HD contiguous halves), so the loads are in
// flight together, then reduces the PW dots across lanes and folds them into
// an online softmax (running max m, sum l, output acc).  The CTA folds its
// warps and writes (m, l, acc[HD]) for the chunk.  The last CTA of head h
// to finish (arrival counter cnt[h]) folds the chunks in chunk order and
// writes the head's output, then zeroes cnt[h] for the next launch.
template <int HD>
__global__ void __launch_bounds__(256) attn_kernel(const float* __restrict__ q, const __half* __restrict__ kc,
                                                   const __half* __restrict__ vc, float* __restrict__ o,
                                                   float* __restrict__ part, int* __restrict__ cnt,
                                                   const DecodeState* st, int heads, int kv_heads, int ctx,
                                                   int nch, float scale) {
  constexpr int DPL = HD / 32;         // dims per lane
  constexpr int PW = ATT_CHUNK / 8;    // positions per warp
  __shared__ float sm[8], sl[8], sacc[8][HD];
  __shared__ int is_last;
  pdl_launch_dependents();
  pdl_wait();  // q and the cache are written by the kernels before
  const int h = blockIdx.x, c = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv_len = min(st->pos + 1, ctx);
  const int kvh = h / (heads / kv_heads);
  const __half* kb = kc + (int64_t)kvh * ctx * HD;
  const __half* vb = vc + (int64_t)kvh * ctx * HD;
  float qr[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) qr[e] = q[(int64_t)h * HD + lane * DPL + e] * scale;
  float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) acc[e] = 0.f;
  const int j0 = c * ATT_CHUNK + warp * PW;
  const int nj = max(0, min(kv_len - j0, PW));
  __half2 kr[PW][DPL / 2], vr[PW][DPL / 2];
#pragma unroll
  for (int t = 0; t < PW; ++t) {
    if (t < nj) {
      const __half2* kp = reinterpret_cast<const __half2*>(kb + (int64_t)(j0 + t) * HD + lane * DPL);
      const __half2* vp = reinterpret_cast<const __half2*>(vb + (int64_t)(j0 + t) * HD + lane * DPL);
#pragma unroll
      for (int e = 0; e < DPL / 2; ++e) {
        kr[t][e] = kp[e];
        vr[t][e] = vp[e];
      }
    }
  }
  float sc[PW];
#pragma unroll
  for (int t = 0; t < PW; ++t) {
    float d = 0.f;
#pragma unroll
    for (int e = 0; e < DPL / 2; ++e) {
      const float2 kk = __half22float2(kr[t][e]);
      d = fmaf(qr[2 * e], kk.x, d);
      d = fmaf(qr[2 * e + 1], kk.y, d);
    }
    sc[t] = d;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
#pragma unroll
    for (int t = 0; t < PW; ++t) sc[t] += __shfl_xor_sync(0xffffffffu, sc[t], o);
  }
#pragma unroll
  for (int t = 0; t < PW; ++t) {
    if (t < nj) {
      const float s = sc[t];
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn), p = expf(s - mn);
      l = l * corr + p;
#pragma unroll
      for (int e = 0; e < DPL / 2; ++e) {
        const float2 vv = __half22float2(vr[t][e]);
        acc[2 * e] = fmaf(p, vv.x, acc[2 * e] * corr);
        acc[2 * e + 1] = fmaf(p, vv.y, acc[2 * e + 1] * corr);
      }
      m = mn;
    }
  }
  if (lane == 0) {
    sm[warp] = m;
    sl[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < DPL; ++e) sacc[warp][lane * DPL + e] = acc[e];
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < 8; ++w) M = fmaxf(M, sm[w]);
  float* out = part + ((int64_t)h * nch + c) * (HD + 2);
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float a = 0.f;
    for (int w = 0; w < 8; ++w)
      if (sm[w] != -INFINITY) a += sacc[w][d] * expf(sm[w] - M);
    out[2 + d] = a;
  }
  if (threadIdx.x == 0) {
    float L = 0.f;
    for (int w = 0; w < 8; ++w)
      if (sm[w] != -INFINITY) L += sl[w] * expf(sm[w] - M);
    out[0] = M;
    out[1] = L;
  }
  // every writer's partial is visible device-wide before the arrival
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(&cnt[h], 1) == nch - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const int nc = (kv_len + ATT_CHUNK - 1) / ATT_CHUNK;
  const float* p = part + (int64_t)h * nch * (HD + 2);
  float Mx = -INFINITY;
  for (int cc = 0; cc < nc; ++cc) Mx = fmaxf(Mx, __ldcg(p + cc * (HD + 2)));
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float L = 0.f, a = 0.f;
    for (int cc = 0; cc < nc; ++cc) {
      const float mc = __ldcg(p + cc * (HD + 2));
      if (mc == -INFINITY) continue;
      const float f = expf(mc - Mx);
      L += __ldcg(p + cc * (HD + 2) + 1) * f;
      a += __ldcg(p + cc * (HD + 2) + 2 + d) * f;
    }
    o[(int64_t)h * HD + d] = a / L;
  }
  if (threadIdx.x == 0) cnt[h] = 0;
}

__global__ void silu_mul_kernel(const float* __restrict__ gu, float* __restrict__ a, int64_t F) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < F; i += (int64_t)gridDim.x * blockDim.x) {
    const float g = gu[i];
    a[i] = g / (1.0f + expf(-g)) * gu[F + i];
  }
}

__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ d, int64_t n) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] += d[i];
}

// Greedy sampling: the first index of the largest logit; writes the token
// into the state and the token record, advances pos and the step count.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int64_t V, DecodeState* st,
                                                      int* __restrict__ record, int record_len) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_launch_dependents();
  pdl_wait();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = logits[i];
    if (v > bv) {  // ascending scan: the first maximum of this thread's stride wins
      bv = v;
      bi = (int)i;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    bv = threadIdx.x < (blockDim.x >> 5) ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < (blockDim.x >> 5) ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) {
      if (bi == 0x7fffffff) bi = 0;  // all logits NaN: token 0
      st->token = bi;
      if (record && st->step >= 0 && st->step < record_len) record[st->step] = bi;
      st->step += 1;
      st->pos += 1;
    }
  }
}

}  // namespace

}  // namespace odi_cuda

namespace odi_cuda {

// Every kernel here triggers its dependents on entry and waits for the
// kernels before it (griddepcontrol) before touching global memory, so all
// are launched with programmatic stream serialisation: the next kernel (a
// GEMV streaming its weights) may start while this one runs.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

static int grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 8) b = 148 * 8;
  return (int)(b < 1 ? 1 : b);
}

cudaError_t launch_embed(const float* table, int64_t vocab, int64_t E, const DecodeState* st, float* x, float* ssq,
                         cudaStream_t s) {
  return launch_pdl(embed_kernel, dim3((unsigned)((E + 63) / 64)), dim3(64), s, table, st, x, ssq, E, vocab);
}

cudaError_t launch_rms_norm(const float* x, const float* w, float* y, int64_t rows, int64_t n, float eps,
                            cudaStream_t s) {
  return launch_pdl(rms_norm_kernel, dim3((unsigned)rows), dim3(512), s, x, w, y, n, eps);
}

cudaError_t launch_rope_kv(float* q, float* k, const float* v, __half* kc, __half* vc, const DecodeState* st,
                           int heads, int kv_heads, int hd, int ctx, float theta, cudaStream_t s) {
  return launch_pdl(rope_kv_kernel, dim3(heads + kv_heads), dim3(hd / 2), s, q, k, v, kc, vc, st, heads, kv_heads,
                    hd, ctx, theta);
}

int attention_chunks(int ctx) { return (ctx + ATT_CHUNK - 1) / ATT_CHUNK; }

size_t attention_scratch(int heads, int hd, int ctx) {
  return att_part_offset(heads) + (size_t)heads * attention_chunks(ctx) * (hd + 2) * sizeof(float);
}

cudaError_t launch_attention(const float* q, const __half* kc, const __half* vc, float* o, void* scratch,
                             const DecodeState* st, int heads, int kv_heads, int hd, int ctx, float scale,
                             cudaStream_t s) {
  const int nch = attention_chunks(ctx);
  int* cnt = static_cast<int*>(scratch);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + att_part_offset(heads));
  const dim3 grid(heads, nch);
  if (hd == 128)
    return launch_pdl(attn_kernel<128>, grid, dim3(256), s, q, kc, vc, o, part, cnt, st, heads, kv_heads, ctx, nch,
                      scale);
  if (hd == 64)
    return launch_pdl(attn_kernel<64>, grid, dim3(256), s, q, kc, vc, o, part, cnt, st, heads, kv_heads, ctx, nch,
                      scale);
  return cudaErrorInvalidValue;
}

cudaError_t launch_silu_mul(const float* gu, float* a, int64_t F, cudaStream_t s) {
  return launch_pdl(silu_mul_kernel, dim3(grid_for(F, 256)), dim3(256), s, gu, a, F);
}

cudaError_t launch_add(float* x, const float* d, int64_t n, cudaStream_t s) {
  return launch_pdl(add_kernel, dim3(grid_for(n, 256)), dim3(256), s, x, d, n);
}

cudaError_t launch_argmax(const float* logits, int64_t V, DecodeState* st, int* record, int record_len,
                          cudaStream_t s) {
  return launch_pdl(argmax_kernel, dim3(1), dim3(1024), s, logits, V, st, record, record_len);
}

}  // namespace odi_cuda
