// quant_weights.cu -- fp32 weights -> GGUF blocks on the device.
//
// The reference cannot produce quantized weights (Tensor::to throws for
// quantized dtypes, src/tensor/tensor.cpp:654-656); models arrive
// pre-quantized in GGUF files.  This kernel quantizes fp32 weights on the
// GPU so synthetic models (and fp32 checkpoints) can be brought up without a
// host round trip.  One thread per block, IEEE fp32 with no contraction, so
// the bytes are identical to the CPU quantisers:
//   Q4_0, Q8_0, Q4_1, Q5_0, Q5_1 -- the GGUF quantisers (gguf 0.19.0):
//     Q4_0: m = signed value of largest |x| (first), d = m / -8,
//           q = min(15, trunc(x / d + 8.5)); Q8_0: d = amax / 127, q = round(x / d)
//     Q4_1 / Q5_1: d = (max - min) / 15 (31), q = min(15 (31), trunc((x - min) / d + 0.5)),
//           d and min stored as fp16
//     Q5_0: as Q4_0 with d = m / -16, q = min(31, trunc(x / d + 16.5))
//     (the fifth bits of Q5_0 / Q5_1 packed little-endian into qh, element
//     j at bit j)
//   Q4_K, Q5_K, Q6_K -- this project's own quantisers of the GGML formats:
//     Q4_K/Q5_K: per 32 values scale = (max - min<=0) / levels, min = -min;
//       6-bit codes of scale / d and min / dmin with d = max scale / 63,
//       dmin = max min / 63 (fp16); q = round((x + min') / scale')
//     Q6_K: per 16 values scale = (signed max) / -32; int8 codes of
//       scale / d with d = max |scale| / 127 (fp16); q = round(x / scale') + 32
#include "internal.h"

namespace odi_cuda {

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
__device__ __forceinline__ uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
// fp16 fields sit at even offsets of blocks whose sizes are even: one
// 16-bit store.
__device__ __forceinline__ void st16(uint8_t* p, uint16_t v) { *reinterpret_cast<uint16_t*>(p) = v; }

__device__ void q4_0_block(const float* x, uint8_t* blk) {
  float amax = -1.0f, mx = 0.0f;
  for (int j = 0; j < 32; ++j) {
    const float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      mx = x[j];
    }
  }
  const float d = __fdiv_rn(mx, -8.0f);
  const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
  st16(blk, f2h_bits(d));
  uint8_t q[32];
  for (int j = 0; j < 32; ++j) q[j] = (uint8_t)clampi((int)truncf(__fadd_rn(__fmul_rn(x[j], id), 8.5f)), 0, 15);
  for (int j = 0; j < 16; ++j) blk[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
}

__device__ void q8_0_block(const float* x, uint8_t* blk) {
  float amax = 0.0f;
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
  st16(blk, f2h_bits(d));
  for (int j = 0; j < 32; ++j) blk[2 + j] = (uint8_t)(int8_t)(int)roundf(__fmul_rn(x[j], id));
}

// Q4_1 (levels 15) and Q5_1 (levels 31): block [d][m][qh (Q5_1)][qs].
__device__ void qmin_block(const float* x, uint8_t* blk, int levels) {
  float mx = x[0], mn = x[0];
  for (int j = 1; j < 32; ++j) {
    mx = fmaxf(mx, x[j]);
    mn = fminf(mn, x[j]);
  }
  const float d = __fdiv_rn(__fsub_rn(mx, mn), (float)levels);
  const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
  st16(blk, f2h_bits(d));
  st16(blk + 2, f2h_bits(mn));
  uint8_t q[32];
  for (int j = 0; j < 32; ++j)
    q[j] = (uint8_t)clampi((int)truncf(__fadd_rn(__fmul_rn(__fsub_rn(x[j], mn), id), 0.5f)), 0, levels);
  uint8_t* qs = blk + (levels == 31 ? 8 : 4);
  for (int j = 0; j < 16; ++j) qs[j] = (uint8_t)((q[j] & 0x0F) | ((q[j + 16] & 0x0F) << 4));
  if (levels == 31) {
    uint32_t qh = 0;
    for (int j = 0; j < 32; ++j) qh |= (uint32_t)(q[j] >> 4) << j;
    for (int b = 0; b < 4; ++b) blk[4 + b] = (uint8_t)(qh >> (8 * b));
  }
}

// Q5_0: block [d][qh][qs].
__device__ void q5_0_block(const float* x, uint8_t* blk) {
  float amax = -1.0f, mx = 0.0f;
  for (int j = 0; j < 32; ++j) {
    const float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      mx = x[j];
    }
  }
  const float d = __fdiv_rn(mx, -16.0f);
  const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
  st16(blk, f2h_bits(d));
  uint8_t q[32];
  for (int j = 0; j < 32; ++j) q[j] = (uint8_t)clampi((int)truncf(__fadd_rn(__fmul_rn(x[j], id), 16.5f)), 0, 31);
  uint32_t qh = 0;
  for (int j = 0; j < 32; ++j) qh |= (uint32_t)(q[j] >> 4) << j;
  for (int b = 0; b < 4; ++b) blk[2 + b] = (uint8_t)(qh >> (8 * b));
  for (int j = 0; j < 16; ++j) blk[6 + j] = (uint8_t)((q[j] & 0x0F) | ((q[j + 16] & 0x0F) << 4));
}

__device__ void kq45_block(const float* x, uint8_t* blk, int levels, bool five) {
  float scale[8], mins[8], maxs = 0.0f, maxm = 0.0f;
  for (int j = 0; j < 8; ++j) {
    float mn = x[32 * j], mx = x[32 * j];
    for (int l = 1; l < 32; ++l) {
      const float v = x[32 * j + l];
      if (v < mn) mn = v;
      if (v > mx) mx = v;
    }
    if (mn > 0.0f) mn = 0.0f;
    scale[j] = __fdiv_rn(__fsub_rn(mx, mn), (float)levels);
    mins[j] = -mn;
    if (scale[j] > maxs) maxs = scale[j];
    if (mins[j] > maxm) maxm = mins[j];
  }
  const uint16_t dh = f2h_bits(__fdiv_rn(maxs, 63.0f)), mh = f2h_bits(__fdiv_rn(maxm, 63.0f));
  const float dd = h2f(dh), dm = h2f(mh);
  int ls[8], lm[8];
  for (int j = 0; j < 8; ++j) {
    ls[j] = dd > 0.0f ? clampi((int)roundf(__fdiv_rn(scale[j], dd)), 0, 63) : 0;
    lm[j] = dm > 0.0f ? clampi((int)roundf(__fdiv_rn(mins[j], dm)), 0, 63) : 0;
  }
  const int nb = five ? 176 : 144;
  for (int i = 0; i < nb; ++i) blk[i] = 0;
  st16(blk, dh);
  st16(blk + 2, mh);
  uint8_t* s = blk + 4;
  for (int j = 0; j < 4; ++j) {
    s[j] = (uint8_t)(ls[j] | ((ls[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)(lm[j] | ((lm[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((ls[j + 4] & 0x0F) | ((lm[j + 4] & 0x0F) << 4));
  }
  uint8_t* qh = blk + 16;
  uint8_t* qs = blk + (five ? 48 : 16);
  for (int j = 0; j < 8; ++j) {
    const float es = __fmul_rn(dd, (float)ls[j]), em = __fmul_rn(dm, (float)lm[j]);
    for (int l = 0; l < 32; ++l) {
      int q = 0;
      if (es > 0.0f) q = clampi((int)roundf(__fdiv_rn(__fadd_rn(x[32 * j + l], em), es)), 0, levels);
      qs[32 * (j >> 1) + l] |= (uint8_t)((q & 0x0F) << ((j & 1) ? 4 : 0));
      if (five) qh[l] |= (uint8_t)(((q >> 4) & 1) << j);
    }
  }
}

__device__ void q6_k_block(const float* x, uint8_t* blk) {
  float scale[16], amax = 0.0f;
  for (int j = 0; j < 16; ++j) {
    float best = -1.0f, v = 0.0f;
    for (int l = 0; l < 16; ++l) {
      const float a = fabsf(x[16 * j + l]);
      if (a > best) {
        best = a;
        v = x[16 * j + l];
      }
    }
    scale[j] = __fdiv_rn(v, -32.0f);
    if (fabsf(scale[j]) > amax) amax = fabsf(scale[j]);
  }
  const uint16_t dh = f2h_bits(__fdiv_rn(amax, 127.0f));
  const float d = h2f(dh);
  for (int i = 0; i < 210; ++i) blk[i] = 0;
  int8_t* sc = reinterpret_cast<int8_t*>(blk + 192);
  uint8_t q[256];
  for (int j = 0; j < 16; ++j) {
    const int s = d > 0.0f ? clampi((int)roundf(__fdiv_rn(scale[j], d)), -128, 127) : 0;
    sc[j] = (int8_t)s;
    const float es = __fmul_rn(d, (float)s);
    for (int l = 0; l < 16; ++l) {
      int v = 32;
      if (es != 0.0f) v = clampi((int)roundf(__fdiv_rn(x[16 * j + l], es)), -32, 31) + 32;
      q[16 * j + l] = (uint8_t)v;
    }
  }
  uint8_t* ql = blk;
  uint8_t* qh = blk + 128;
  for (int h = 0; h < 2; ++h) {
    for (int l = 0; l < 32; ++l) {
      const int q1 = q[128 * h + l], q2 = q[128 * h + l + 32], q3 = q[128 * h + l + 64], q4 = q[128 * h + l + 96];
      ql[64 * h + l] = (uint8_t)((q1 & 0x0F) | ((q3 & 0x0F) << 4));
      ql[64 * h + l + 32] = (uint8_t)((q2 & 0x0F) | ((q4 & 0x0F) << 4));
      qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  st16(blk + 208, dh);
}

template <int DT>
__global__ void quant_weights_kernel(const float* __restrict__ w, uint8_t* __restrict__ out, int64_t N,
                                     int64_t K) {
  constexpr int BE = block_elems(DT), BB = block_bytes(DT);
  const int64_t nb = (K + BE - 1) / BE;
  const int64_t total = N * nb;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / nb, b = i - n * nb;
    float x[BE];
    for (int j = 0; j < BE; ++j) {
      const int64_t k = b * BE + j;
      x[j] = k < K ? w[n * K + k] : 0.0f;
    }
    uint8_t* blk = out + i * BB;  // each thread owns one whole block of the output
    if (DT == Q4_0) q4_0_block(x, blk);
    else if (DT == Q8_0) q8_0_block(x, blk);
    else if (DT == Q4_1) qmin_block(x, blk, 15);
    else if (DT == Q5_1) qmin_block(x, blk, 31);
    else if (DT == Q5_0) q5_0_block(x, blk);
    else if (DT == Q4_K) kq45_block(x, blk, 15, false);
    else if (DT == Q5_K) kq45_block(x, blk, 31, true);
    else q6_k_block(x, blk);
  }
}

cudaError_t launch_quant_weights(int dt, const float* w, void* out, int64_t N, int64_t K, cudaStream_t s) {
  const int be = block_elems(dt);
  const int64_t total = N * ((K + be - 1) / be);
  if (total == 0) return cudaSuccess;
  const int block = 128;
  int64_t grid = (total + block - 1) / block;
  if (grid > 148 * 16) grid = 148 * 16;
  uint8_t* o = (uint8_t*)out;
  switch (dt) {
    case Q4_0: quant_weights_kernel<Q4_0><<<(int)grid, block, 0, s>>>(w, o, N, K); break;
    case Q8_0: quant_weights_kernel<Q8_0><<<(int)grid, block, 0, s>>>(w, o, N, K); break;
    case Q4_1: quant_weights_kernel<Q4_1><<<(int)grid, block, 0, s>>>(w, o, N, K); break;
    case Q5_0: quant_weights_kernel<Q5_0><<<(int)grid, block, 0, s>>>(w, o, N, K); break;
    case Q5_1: quant_weights_kernel<Q5_1><<<(int)grid, block, 0, s>>>(w, o, N, K); break;
    case Q4_K: quant_weights_kernel<Q4_K><<<(int)grid, block, 0, s>>>(w, o, N, K); break;
    case Q5_K: quant_weights_kernel<Q5_K><<<(int)grid, block, 0, s>>>(w, o, N, K); break;
    case Q6_K: quant_weights_kernel<Q6_K><<<(int)grid, block, 0, s>>>(w, o, N, K); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace odi_cuda
