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
// sum of squares of its values (the slot a fused RMSNorm reads); with recs,
// the row times norm_w (or the row) as Q8 records for the first product.
__global__ void embed_kernel(const float* __restrict__ table, const DecodeState* st, float* __restrict__ x,
                             float* __restrict__ ssq, int64_t E, int64_t vocab, const float* __restrict__ norm_w,
                             uint8_t* __restrict__ recs) {
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
  if (recs) {  // E is a multiple of 256: whole warps, whole records
    const float u = (norm_w && i < E) ? v * norm_w[i] : v;
    q8_block_to_record(u, threadIdx.x & 31, recs + (i >> 8) * Q8_REC_BYTES, (int)((i & 255) >> 5));
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

// Flash decoding in one launch, streamed by the bulk-copy engine.
// (With orec, the outputs are also written as Q8 records for the next GEMV.)
// CTA (kvh, split) serves the G = heads / kv_heads query heads of kv head
// kvh over the 64-position chunks c = split, split + nsplit, ... of
// kv_len = pos + 1.  Thread 0 streams each chunk's K and V tiles (64 x HD
// fp16 each, contiguous in the [kv_head][ctx][HD] cache) into a two-stage
// shared-memory ring with cp.async.bulk (no multicast), completing on an
// mbarrier; its warps take ATT_PW positions each.  Scores: lane l holds
// dims [l*HD/32, +HD/32) of q; the partial dots are summed across lanes by
// a halving butterfly, after which lanes 32/ATT_PW * t .. hold position t's
// score.  Online softmax per warp and head (running max m,
// sum l, output acc), then the CTA folds its warps and writes (m, l,
// acc[HD]) per head for its split.  The last CTA of kv head kvh to finish
// (arrival counter) folds the splits in split order, writes the heads'
// outputs and zeroes its counter for the next launch.
// With rope (the rope_kv step fused in): q, k and v are this step's raw
// projections; every CTA rotates q in registers (the arithmetic of
// rope_kv_kernel), and the CTA whose chunk holds pos writes the rotated k and
// v as fp16 into its shared K / V tiles (after the chunk landed) and into the
// caches, for the steps after.
// Every mbarrier wait is bounded: a wait that gives up sets the error word,
// the CTA stops consuming (the decision is made uniform by a CTA-wide vote),
// drains its copies in flight and still arrives, so counters stay balanced.
constexpr int ATT_STAGES = 2;
constexpr int ATT_PW = 8;                       // positions per warp per chunk
constexpr int ATT_WARPS = ATT_CHUNK / ATT_PW;   // warps per CTA
constexpr int ATT_THREADS = 32 * ATT_WARPS;

template <int HD, int G>
constexpr int att_smem_bytes() {
  return ATT_STAGES * 2 * ATT_CHUNK * HD * 2 + ATT_WARPS * G * (HD + 2) * 4 + ATT_STAGES * 8;
}

template <int HD, int G>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(const float* __restrict__ q,
                                                           const __half* __restrict__ kc,
                                                           const __half* __restrict__ vc, float* __restrict__ o,
                                                           float* __restrict__ part, int* __restrict__ cnt,
                                                           int* __restrict__ err, const DecodeState* st, int ctx,
                                                           int nsplit, float scale, const float* __restrict__ kraw,
                                                           const float* __restrict__ vraw, float theta, int rope,
                                                           __half* __restrict__ kcw, __half* __restrict__ vcw,
                                                           uint8_t* __restrict__ orec) {
  constexpr int DPL = HD / 32;           // dims per lane
  constexpr int TILE = ATT_CHUNK * HD;   // halves per K (or V) tile
  constexpr int PW = ATT_PW;             // positions per warp per chunk
  constexpr int LPP = 32 / PW;           // lanes per position after the butterfly
  constexpr int NW = ATT_WARPS;
  extern __shared__ __align__(128) uint8_t att_smem[];
  __half* tiles = reinterpret_cast<__half*>(att_smem);  // [stage][K | V][TILE]
  float* fold = reinterpret_cast<float*>(att_smem + ATT_STAGES * 2 * TILE * 2);  // [NW][G][HD + 2]
  uint64_t* full = reinterpret_cast<uint64_t*>(fold + NW * G * (HD + 2));
  __shared__ int is_last;
  pdl_launch_dependents();
  pdl_wait();  // q and the cache are written by the kernels before
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv_len = min(st->pos + 1, ctx);
  const int nc = kv_len > 0 ? (kv_len + ATT_CHUNK - 1) / ATT_CHUNK : 0;
  const int nmine = split < nc ? (nc - 1 - split) / nsplit + 1 : 0;
  const __half* kb = kc + (int64_t)kvh * ctx * HD;
  const __half* vb = vc + (int64_t)kvh * ctx * HD;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ATT_STAGES; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;
  auto issue = [&](int i) {  // thread 0: chunk i of this CTA into stage i % ATT_STAGES
    const int p0 = (split + i * nsplit) * ATT_CHUNK;
    const int n = min(ATT_CHUNK, kv_len - p0);
    const uint32_t bytes = (uint32_t)n * HD * 2;
    const int s = i % ATT_STAGES;
    mbar_arrive_expect_tx(&full[s], 2 * bytes);
    bulk_g2s(tiles + (2 * s) * TILE, kb + (int64_t)p0 * HD, bytes, &full[s]);
    bulk_g2s(tiles + (2 * s + 1) * TILE, vb + (int64_t)p0 * HD, bytes, &full[s]);
  };
  if (threadIdx.x == 0)
    for (; issued < nmine && issued < ATT_STAGES; ++issued) issue(issued);

  constexpr int HALF = HD / 2;
  const int pos = st->pos;
  const bool rot = rope && pos >= 0 && pos < ctx;
  // rotary angles of this lane's dims (pair index d mod HD/2), as rope_kv_kernel
  float rsn[DPL], rcs[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) {
    rsn[e] = 0.f;
    rcs[e] = 1.f;
    if (rot) {
      const int pi = (lane * DPL + e) % HALF;
      const float freq = 1.0f / powf(theta, 2.0f * (float)pi / (float)HD);
      sincosf((float)pos * freq, &rsn[e], &rcs[e]);
    }
  }
  const bool lower = lane * DPL < HALF;  // partner dims d + HD/2 live on lane ^ 16
  float qr[G][DPL], acc[G][DPL], m[G], l[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      float v = q[(int64_t)(kvh * G + g) * HD + lane * DPL + e];
      if (rot) {
        const float pv = __shfl_xor_sync(0xffffffffu, v, 16);
        v = lower ? v * rcs[e] - pv * rsn[e] : pv * rsn[e] + v * rcs[e];
      }
      qr[g][e] = v * scale;
      acc[g][e] = 0.f;
    }
    m[g] = -INFINITY;
    l[g] = 0.f;
  }
  // the CTA whose chunks include pos appends this step's k and v: its local
  // chunk index, and each of the first HD/2 threads' rotated pair
  const int cpos = rot ? pos / ATT_CHUNK : -1;
  const int ipos = (rot && cpos % nsplit == split) ? cpos / nsplit : -1;
  __half k0h = __float2half_rn(0.f), k1h = k0h, v0h = k0h, v1h = k0h;
  if (ipos >= 0 && threadIdx.x < HALF) {
    const int t = threadIdx.x;
    const float freq = 1.0f / powf(theta, 2.0f * (float)t / (float)HD);
    float sn, cs;
    sincosf((float)pos * freq, &sn, &cs);
    const float k0 = kraw[(int64_t)kvh * HD + t], k1 = kraw[(int64_t)kvh * HD + t + HALF];
    k0h = __float2half_rn(k0 * cs - k1 * sn);
    k1h = __float2half_rn(k0 * sn + k1 * cs);
    v0h = __float2half_rn(vraw[(int64_t)kvh * HD + t]);
    v1h = __float2half_rn(vraw[(int64_t)kvh * HD + t + HALF]);
  }
  const int pidx = (lane / LPP) & (PW - 1);  // the position whose score this lane ends with
  int i = 0;
  for (; i < nmine; ++i) {
    const int s = i % ATT_STAGES;
    const bool ok = mbar_wait(&full[s], (uint32_t)(i / ATT_STAGES) & 1u, err, ERR_FULL_WAIT);
    if (__syncthreads_or(!ok)) break;  // uniform: every thread stops at the same chunk
    const int p0 = (split + i * nsplit) * ATT_CHUNK;
    if (i == ipos) {  // this step's k and v: into the landed tiles and the caches
      if (threadIdx.x < HALF) {
        const int t = threadIdx.x, row = pos - p0;
        __half* kt = tiles + (2 * s) * TILE + row * HD;
        __half* vt = kt + TILE;
        kt[t] = k0h;
        kt[t + HALF] = k1h;
        vt[t] = v0h;
        vt[t + HALF] = v1h;
        __half* kg = kcw + ((int64_t)kvh * ctx + pos) * HD;
        __half* vg = vcw + ((int64_t)kvh * ctx + pos) * HD;
        kg[t] = k0h;
        kg[t + HALF] = k1h;
        vg[t] = v0h;
        vg[t + HALF] = v1h;
      }
      __syncthreads();
    }
    const __half* Ks = tiles + (2 * s) * TILE + warp * PW * HD + lane * DPL;
    const __half* Vs = Ks + TILE;
    const int nvalid = min(PW, kv_len - p0 - warp * PW);  // this warp's positions in the chunk
    if (nvalid > 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float sc[PW];
#pragma unroll
        for (int t = 0; t < PW; ++t) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < DPL / 2; ++e) {
            const float2 kk = __half22float2(reinterpret_cast<const __half2*>(Ks + t * HD)[e]);
            d = fmaf(qr[g][2 * e], kk.x, d);
            d = fmaf(qr[g][2 * e + 1], kk.y, d);
          }
          sc[t] = d;
        }
        // halving butterfly: PW positions x 32 lanes -> position pidx on lanes LPP*pidx .. +LPP-1
#pragma unroll
        for (int w = 16, n = PW / 2; n >= 1; w >>= 1, n >>= 1) {
          const bool up = lane & w;
#pragma unroll
          for (int t = 0; t < n; ++t) {
            const float send = up ? sc[t] : sc[t + n];
            const float keep = up ? sc[t + n] : sc[t];
            sc[t] = keep + __shfl_xor_sync(0xffffffffu, send, w);
          }
        }
        float sfull = sc[0];
#pragma unroll
        for (int w = LPP / 2; w; w >>= 1) sfull += __shfl_xor_sync(0xffffffffu, sfull, w);
        const bool valid = pidx < nvalid;
        const float sv = valid ? sfull : -INFINITY;
        float mx = sv;
#pragma unroll
        for (int w = 16; w; w >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, w));
        const float mn = fmaxf(m[g], mx);  // finite: nvalid > 0
        const float corr = expf(m[g] - mn);
        const float pv = valid ? expf(sv - mn) : 0.f;
        float ps = (lane & (LPP - 1)) ? 0.f : pv;
#pragma unroll
        for (int w = 16; w; w >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, w);
        l[g] = l[g] * corr + ps;
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[g][e] *= corr;
        for (int t = 0; t < nvalid; ++t) {  // rows past the chunk's end hold stale data: not read
          const float pt = __shfl_sync(0xffffffffu, pv, LPP * t);
#pragma unroll
          for (int e = 0; e < DPL / 2; ++e) {
            const float2 vv = __half22float2(reinterpret_cast<const __half2*>(Vs + t * HD)[e]);
            acc[g][2 * e] = fmaf(pt, vv.x, acc[g][2 * e]);
            acc[g][2 * e + 1] = fmaf(pt, vv.y, acc[g][2 * e + 1]);
          }
        }
        m[g] = mn;
      }
    }
    fence_proxy_async_smem();  // this thread's reads of stage s before its refill
    __syncthreads();           // every warp is done with stage s
    if (threadIdx.x == 0 && issued < nmine) issue(issued++);
  }
  if (threadIdx.x == 0) {
    // copies still in flight (only after a wait gave up) land before the CTA may exit
    for (int j = i; j < issued; ++j)
      mbar_wait(&full[j % ATT_STAGES], (uint32_t)(j / ATT_STAGES) & 1u, err, ERR_DRAIN_WAIT);
  }
  // fold the warps, per head
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* f = fold + (warp * G + g) * (HD + 2);
    if (lane == 0) {
      f[0] = m[g];
      f[1] = l[g];
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e) f[2 + lane * DPL + e] = acc[g][e];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += ATT_THREADS) {
    const int g = idx / HD, d = idx - g * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, fold[(w * G + g) * (HD + 2)]);
    float a = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float* f = fold + (w * G + g) * (HD + 2);
      if (f[0] != -INFINITY) {
        const float sc = expf(f[0] - M);
        a += f[2 + d] * sc;
        L += f[1] * sc;
      }
    }
    float* out = part + ((int64_t)(kvh * G + g) * nsplit + split) * (HD + 2);
    out[2 + d] = a;
    if (d == 0) {
      out[0] = M;
      out[1] = L;
    }
  }
  // every writer's partial is visible device-wide before the arrival
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(&cnt[kvh], 1) == nsplit - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Online merge of the splits in split order; the partials of up to 16
  // splits are loaded together, so the merge costs one L2 round trip per 16.
  constexpr int SB = 16;
  for (int idx = threadIdx.x; idx < G * HD; idx += ATT_THREADS) {
    const int g = idx / HD, d = idx - g * HD;
    const int h = kvh * G + g;
    const float* p = part + (int64_t)h * nsplit * (HD + 2);
    float M = -INFINITY, L = 0.f, a = 0.f;
    for (int s0 = 0; s0 < nsplit; s0 += SB) {
      float mc[SB], lc[SB], ac[SB];
#pragma unroll
      for (int u = 0; u < SB; ++u) {
        const bool in = s0 + u < nsplit;
        const float* ps = p + (s0 + u) * (HD + 2);
        mc[u] = in ? __ldcg(ps) : -INFINITY;
        lc[u] = in ? __ldcg(ps + 1) : 0.f;
        ac[u] = in ? __ldcg(ps + 2 + d) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < SB; ++u) {
        if (mc[u] == -INFINITY) continue;
        const float mn = fmaxf(M, mc[u]);
        const float fo = expf(M - mn), fn = expf(mc[u] - mn);
        L = L * fo + lc[u] * fn;
        a = a * fo + ac[u] * fn;
        M = mn;
      }
    }
    const float val = L > 0.f ? a / L : 0.f;
    o[(int64_t)h * HD + d] = val;
    if (orec) {
      // The output row as the next GEMV's Q8 record (one token): each warp
      // holds 32 consecutive values = one Q8 block; the quantisation of
      // act_q8_records_kernel, bit for bit.
      const int64_t col = (int64_t)h * HD + d;
      q8_block_to_record(val, threadIdx.x & 31, orec + (col >> 8) * Q8_REC_BYTES, (int)((col & 255) >> 5));
    }
  }
  if (threadIdx.x == 0) cnt[kvh] = 0;
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
static cudaError_t launch_pdl_smem(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  return launch_pdl_smem(kern, grid, block, 0, s, args...);
}

static int grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 8) b = 148 * 8;
  return (int)(b < 1 ? 1 : b);
}

cudaError_t launch_embed(const float* table, int64_t vocab, int64_t E, const DecodeState* st, float* x, float* ssq,
                         const float* norm_w, uint8_t* recs, cudaStream_t s) {
  return launch_pdl(embed_kernel, dim3((unsigned)((E + 63) / 64)), dim3(64), s, table, st, x, ssq, E, vocab, norm_w,
                    recs);
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

// Splits per kv head: about two CTAs per SM in all (the ring takes 64 KB of
// shared memory, so a streaming GEMV CTA still fits beside two of them),
// never more than the context's chunks.
int attention_splits(int kv_heads, int ctx, int num_sms) {
  const int want = (2 * num_sms + kv_heads / 2) / kv_heads;
  const int nch = attention_chunks(ctx);
  return want < 1 ? 1 : want > nch ? nch : want;
}

template <int HD, int G>
static cudaError_t launch_att_t(const float* q, const __half* kc, const __half* vc, float* o, void* scratch,
                                const DecodeState* st, int heads, int kv_heads, int ctx, float scale,
                                const AttRope& rp, cudaStream_t s) {
  auto kern = attn_kernel<HD, G>;
  constexpr int smem = att_smem_bytes<HD, G>();
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int nsplit = attention_splits(kv_heads, ctx, sms);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  int* err = reinterpret_cast<int*>(base);
  int* cnt = reinterpret_cast<int*>(base + ATT_CNT_OFFSET);
  float* part = reinterpret_cast<float*>(base + att_part_offset(heads));
  return launch_pdl_smem(kern, dim3(kv_heads, nsplit), dim3(ATT_THREADS), smem, s, q, kc, vc, o, part, cnt, err, st,
                         ctx, nsplit, scale, rp.k, rp.v, rp.theta, rp.k ? 1 : 0, const_cast<__half*>(kc),
                         const_cast<__half*>(vc), rp.out_recs);
}

template <int HD>
static cudaError_t launch_att_hd(const float* q, const __half* kc, const __half* vc, float* o, void* scratch,
                                 const DecodeState* st, int heads, int kv_heads, int ctx, float scale,
                                 const AttRope& rp, cudaStream_t s) {
  switch (heads / kv_heads) {
    case 1: return launch_att_t<HD, 1>(q, kc, vc, o, scratch, st, heads, kv_heads, ctx, scale, rp, s);
    case 2: return launch_att_t<HD, 2>(q, kc, vc, o, scratch, st, heads, kv_heads, ctx, scale, rp, s);
    case 4: return launch_att_t<HD, 4>(q, kc, vc, o, scratch, st, heads, kv_heads, ctx, scale, rp, s);
    case 8: return launch_att_t<HD, 8>(q, kc, vc, o, scratch, st, heads, kv_heads, ctx, scale, rp, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_attention(const float* q, const __half* kc, const __half* vc, float* o, void* scratch,
                             const DecodeState* st, int heads, int kv_heads, int hd, int ctx, float scale,
                             const AttRope& rp, cudaStream_t s) {
  if (hd == 128) return launch_att_hd<128>(q, kc, vc, o, scratch, st, heads, kv_heads, ctx, scale, rp, s);
  if (hd == 64) return launch_att_hd<64>(q, kc, vc, o, scratch, st, heads, kv_heads, ctx, scale, rp, s);
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
