// act.cu -- activation staging kernels.
//
// act_quant_q8: fp32 x [M, K] -> Q8_0, one warp per 32-value block.  The
// arithmetic is the GGUF Q8_0 quantiser's, in IEEE fp32 with no contraction:
//   amax = max |x|;  d = amax / 127;  id = d ? 1 / d : 0;
//   q = round-half-away(x * id);  d stored as fp16 (round to nearest even).
// It writes the span-major activation tiles the GEMV kernels stream (codes,
// fp32-widened scale, half-block code sums) and/or GGUF Q8_0 blocks.
//
// act_pack_f32: fp32 x [M, K] -> span-major fp32 tiles, zero past K.
#include "internal.h"

namespace odi_cuda {

__global__ void act_quant_q8_kernel(const float* __restrict__ x, int64_t M, int64_t K, int64_t Kp,
                                    uint8_t* __restrict__ tiles, uint8_t* __restrict__ blocks) {
  pdl_wait();  // x may be written by the previous kernel on the stream
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t nbp = Kp / 32;
  const int64_t nbk = (K + 31) / 32;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < M * nbp; w += nwarps) {
    const int64_t m = w / nbp, b = w - m * nbp;
    const int64_t k = b * 32 + lane;
    const float v = k < K ? x[m * K + k] : 0.0f;
    float a = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float d = q8_scale(a);
    const float id = q8_inv(d);
    const int q = q8_round(__fmul_rn(v, id));
    const __half dh = __float2half_rn(d);
    int s = q;
#pragma unroll
    for (int o = 8; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);  // within 16-lane halves
    const int s_lo = __shfl_sync(0xffffffffu, s, 0);
    const int s_hi = __shfl_sync(0xffffffffu, s, 16);
    if (tiles) {
      const int64_t kb = b >> 3;
      const int j = (int)(b & 7);
      uint8_t* rec = tiles + (kb * M + m) * ACT_Q8_BYTES;
      rec[j * 32 + lane] = (uint8_t)(int8_t)q;
      if (lane == 0) {
        ActRec r;
        r.d = __half2float(dh);
        r.s_lo = (short)s_lo;
        r.s_hi = (short)s_hi;
        *reinterpret_cast<ActRec*>(rec + 256 + 8 * j) = r;
      }
    }
    if (blocks && b < nbk) {
      uint8_t* blk = blocks + (m * nbk + b) * 34;
      blk[2 + lane] = (uint8_t)(int8_t)q;
      if (lane == 0) {
        const uint16_t hb = __half_as_ushort(dh);
        blk[0] = (uint8_t)(hb & 0xFF);
        blk[1] = (uint8_t)(hb >> 8);
      }
    }
  }
}

// act_q8_records: fp32 x [M][ldx] -> the streaming GEMV's Q8 activation
// records, span-major: record (kb, m) at (kb * M + m) * Q8_REC_BYTES holds the
// 256 codes of span kb then 8 x {dx, sdx, sdx_lo, sdx_hi} (fp32: the fp16
// scale widened, and the block / half-block code sums times dx), zero past
// K.  One warp per 32-value block, lane = value; the arithmetic is the GEMV's
// own staging quantiser's, so the records are bit-identical to the ones it
// builds in shared memory.
__global__ void act_q8_records_kernel(const float* __restrict__ x, int64_t ldx, int64_t M, int64_t K, int64_t KB,
                                      uint8_t* __restrict__ recs) {
  pdl_wait();  // x may be written by the previous kernel on the stream
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = KB * M * 8;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total; w += nwarps) {
    const int64_t kb = w / (M * 8);
    const int64_t rem = w - kb * M * 8;
    const int64_t m = rem >> 3;
    const int j = (int)(rem & 7);
    const int64_t k = kb * 256 + 32 * j + lane;
    const float v = k < K ? x[m * ldx + k] : 0.0f;
    q8_block_to_record(v, lane, recs + (kb * M + m) * Q8_REC_BYTES, j);
  }
}

// act_q8_records with the decode step's activation prologues (GemvFuse):
// RMSNorm (x * rms * norm_w, rms from the token's sums-of-squares slots or
// from the row) or SwiGLU (silu(gate) * up of a [gate K | up K] row), then
// the same quantisation.  The arithmetic and its order are the streaming
// GEMV's own fused prologue (row_rms and stage_acts), so the records equal
// the ones that GEMV builds in shared memory.
__device__ __forceinline__ float act_silu(float g) { return g / (1.0f + expf(-g)); }

// 1 / sqrt(sum(x^2) / K + eps) for token m, summed as the GEMV's row_rms
// does with its 128 consumer threads: thread t (of 128) adds slots (or
// squares) t, t + 128, ...; each 32-thread group reduces by xor shuffles;
// the four group sums combine as (g0 + g1) + (g2 + g3).  One warp plays the
// 128 threads as four virtual groups.  With up to 128 slots (hidden sizes up
// to 8192) every slot is loaded at once, so the sum costs one round trip.
__device__ float act_rms(const GemvFuse& fu, const float* __restrict__ x, int64_t m, int64_t ldx, int64_t K,
                         int lane) {
  float g[4];
  if (fu.ssq_in && fu.ssq_n <= 128) {
    const float* sq = fu.ssq_in + m * fu.ssq_n;
    float v4[4];
#pragma unroll
    for (int v = 0; v < 4; ++v) v4[v] = 32 * v + lane < fu.ssq_n ? sq[32 * v + lane] : 0.f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      float s = 0.f + v4[v];
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      g[v] = s;
    }
  } else {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      float s = 0.f;
      const int t = 32 * v + lane;
      if (fu.ssq_in) {
        const float* sq = fu.ssq_in + m * fu.ssq_n;
        for (int i = t; i < fu.ssq_n; i += 128) s += sq[i];
      } else {
        const float* xm = x + m * ldx;
        for (int64_t k = t; k < K; k += 128) s = fmaf(xm[k], xm[k], s);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      g[v] = s;
    }
  }
  const float tot = (g[0] + g[1]) + (g[2] + g[3]);
  return 1.0f / sqrtf(tot / (float)K + fu.eps);
}

__global__ void act_records_fused_kernel(const float* __restrict__ x, int64_t ldx, int64_t M, int64_t K,
                                         int64_t KB, const GemvFuse fu, uint8_t* __restrict__ recs) {
  pdl_wait();  // x (and the sums of squares) are written by the kernels before
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = KB * M * 8;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total; w += nwarps) {
    const int64_t kb = w / (M * 8);
    const int64_t rem = w - kb * M * 8;
    const int64_t m = rem >> 3;
    const int j = (int)(rem & 7);
    const int64_t k = kb * 256 + 32 * j + lane;
    // every input of this value is requested before any is used
    float v = k < K ? x[m * ldx + k] : 0.0f;
    const float e = k >= K ? 0.0f : fu.swiglu ? x[m * ldx + K + k] : fu.norm_w ? fu.norm_w[k] : 0.0f;
    if (fu.swiglu) {
      v = k < K ? act_silu(v) * e : 0.0f;
    } else if (fu.norm_w) {
      const float r = act_rms(fu, x, m, ldx, K, lane);
      if (k < K) v = v * r * e;
    }
    q8_block_to_record(v, lane, recs + (kb * M + m) * Q8_REC_BYTES, j);
  }
}

__global__ void act_pack_f32_kernel(const float* __restrict__ x, int64_t M, int64_t K, int64_t Kp,
                                    float* __restrict__ tiles) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = M * Kp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    // i enumerates the tile layout: (kb, m, j)
    const int64_t kb = i / (M * 256);
    const int64_t rem = i - kb * M * 256;
    const int64_t m = rem / 256, j = rem & 255;
    const int64_t k = kb * 256 + j;
    tiles[i] = k < K ? x[m * K + k] : 0.0f;
  }
}

static int grid_for(int64_t threads_needed, int block) {
  int64_t g = (threads_needed + block - 1) / block;
  if (g < 1) g = 1;
  if (g > 148 * 32) g = 148 * 32;
  return (int)g;
}

static cudaLaunchConfig_t small_cfg(int grid, bool pdl, cudaStream_t stream, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

cudaError_t launch_act_quant(const float* x, int64_t M, int64_t K, uint8_t* tiles, uint8_t* blocks,
                             bool pdl, cudaStream_t stream) {
  const int64_t Kp = (K + 255) / 256 * 256;
  const int64_t warps = M * (Kp / 32);
  if (warps == 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(grid_for(warps * 32, 256), pdl, stream, attr);
  return cudaLaunchKernelEx(&cfg, act_quant_q8_kernel, x, M, K, Kp, tiles, blocks);
}

cudaError_t launch_act_q8_records(const float* x, int64_t ldx, int64_t M, int64_t K, uint8_t* recs, bool pdl,
                                  cudaStream_t stream) {
  const int64_t KB = (K + 255) / 256;
  const int64_t warps = KB * M * 8;
  if (warps == 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(grid_for(warps * 32, 256), pdl, stream, attr);
  return cudaLaunchKernelEx(&cfg, act_q8_records_kernel, x, ldx, M, K, KB, recs);
}

cudaError_t launch_act_records_fused(const float* x, int64_t ldx, int64_t M, int64_t K, const GemvFuse& fu,
                                    uint8_t* recs, bool pdl, cudaStream_t stream) {
  const int64_t KB = (K + 255) / 256;
  const int64_t warps = KB * M * 8;
  if (warps == 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(grid_for(warps * 32, 256), pdl, stream, attr);
  return cudaLaunchKernelEx(&cfg, act_records_fused_kernel, x, ldx, M, K, KB, fu, recs);
}

cudaError_t launch_act_pack_f32(const float* x, int64_t M, int64_t K, float* tiles, bool pdl,
                                cudaStream_t stream) {
  const int64_t Kp = (K + 255) / 256 * 256;
  if (M * Kp == 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(grid_for(M * Kp, 256), pdl, stream, attr);
  return cudaLaunchKernelEx(&cfg, act_pack_f32_kernel, x, M, K, Kp, tiles);
}

}  // namespace odi_cuda

