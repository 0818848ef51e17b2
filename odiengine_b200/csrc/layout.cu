// layout.cu -- GGUF blocks <-> tiled device layout, and tiled -> fp32 decode.
//
// These run once per weight at load time (repack) or in tests and
// Backend::dequantize; they are plain byte gathers, one thread per output
// byte / element, grid-stride.
#include "internal.h"

namespace odi_cuda {

// Source byte in the GGUF buffer for tiled byte `idx`, or -1 for padding.
__device__ __forceinline__ int64_t tiled_src(int dt, int64_t idx, int64_t N, int64_t K, int64_t KB) {
  const int ub = unit_bytes(dt), sb = slice_bytes(dt), bb = block_bytes(dt);
  const int64_t unit = idx / ub;
  const int off = (int)(idx - unit * ub);
  const int64_t g = unit / KB, kb = unit - g * KB;
  if (dt == Q6_K && off >= UNIT_ROWS * sb) {
    const int t = off - UNIT_ROWS * sb, r = t >> 1;
    const int64_t n = g * UNIT_ROWS + r;
    if (n >= N) return -1;
    return (n * KB + kb) * bb + 208 + (t & 1);
  }
  const int r = off / sb, o = off - r * sb;
  const int64_t n = g * UNIT_ROWS + r;
  if (n >= N) return -1;
  if (dt == Q4_K || dt == Q5_K) return (n * KB + kb) * bb + o;
  if (dt == Q6_K) {
    const int64_t blk = (n * KB + kb) * bb;
    if (o < 16) return blk + 192 + o;
    if (o < 144) return blk + (o - 16);
    return blk + 128 + (o - 144);
  }
  // 32-value block types: 8 blocks per span, fields field-major in the slice
  const int64_t nb_row = (K + 31) / 32;
  int j, t;
  if (o < 16) {  // d
    j = o >> 1;
    t = o & 1;
  } else if (has_min(dt) && o < sl_qh(dt)) {  // m
    j = (o - 16) >> 1;
    t = 2 + ((o - 16) & 1);
  } else if (has_qh(dt) && o < sl_qs(dt)) {  // qh
    j = (o - sl_qh(dt)) >> 2;
    t = blk_qh(dt) + ((o - sl_qh(dt)) & 3);
  } else {  // qs, then the pad
    const int q = o - sl_qs(dt), qb = qs_bytes(dt);
    j = q / qb;
    if (j >= 8) return -1;
    t = blk_qs(dt) + (q - j * qb);
  }
  const int64_t b = kb * 8 + j;
  if (b >= nb_row) return -1;
  return (n * nb_row + b) * bb + t;
}

// Tiled byte for GGUF byte `idx` (always exists).
__device__ __forceinline__ int64_t gguf_dst(int dt, int64_t idx, int64_t K, int64_t KB) {
  const int ub = unit_bytes(dt), sb = slice_bytes(dt), bb = block_bytes(dt);
  const int64_t nb_row = (K + block_elems(dt) - 1) / block_elems(dt);
  const int64_t row_bytes = nb_row * bb;
  const int64_t n = idx / row_bytes;
  const int64_t rb = idx - n * row_bytes;
  const int64_t b = rb / bb;
  const int t = (int)(rb - b * bb);
  const int64_t g = n / UNIT_ROWS;
  const int r = (int)(n - g * UNIT_ROWS);
  if (is_block32(dt)) {
    const int64_t kb = b >> 3;
    const int j = (int)(b & 7);
    const int64_t base = (g * KB + kb) * ub + (int64_t)r * sb;
    if (t < 2) return base + 2 * j + t;
    if (has_min(dt) && t < 4) return base + sl_m(dt) + 2 * j + (t - 2);
    if (has_qh(dt) && t < blk_qs(dt)) return base + sl_qh(dt) + 4 * j + (t - blk_qh(dt));
    return base + sl_qs(dt) + (int64_t)qs_bytes(dt) * j + (t - blk_qs(dt));
  }
  const int64_t ubase = (g * KB + b) * ub;
  const int64_t base = ubase + (int64_t)r * sb;
  if (dt == Q4_K || dt == Q5_K) return base + t;
  // Q6_K
  if (t < 128) return base + 16 + t;
  if (t < 192) return base + 144 + (t - 128);
  if (t < 208) return base + (t - 192);
  return ubase + (int64_t)UNIT_ROWS * sb + 2 * r + (t - 208);
}

__global__ void repack_kernel(int dt, const uint8_t* __restrict__ gguf, uint8_t* __restrict__ tiled,
                              int64_t N, int64_t K, int64_t KB, int64_t total) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = tiled_src(dt, i, N, K, KB);
    tiled[i] = s >= 0 ? gguf[s] : 0;
  }
}

__global__ void unpack_kernel(int dt, const uint8_t* __restrict__ tiled, uint8_t* __restrict__ gguf,
                              int64_t K, int64_t KB, int64_t total) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    gguf[i] = tiled[gguf_dst(dt, i, K, KB)];
  }
}

__device__ __forceinline__ uint16_t ld16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// Decode element (n, k) from the tiled layout in the reference / gguf
// arithmetic: Q4_0 (q-8)*d, Q8_0 q*d, Q4_1 / Q5_1 q*d + m, Q5_0 (q-16)*d
// (cpu_backend.cpp:704-767; each operation rounded, as gguf's float32
// numpy and the reference built without contraction), Q4_K/Q5_K
// (d*sc)*q - dmin*m, Q6_K (d*sc)*(q-32).
__device__ float decode_tiled(int dt, const uint8_t* __restrict__ w, int64_t n, int64_t k, int64_t KB) {
  const int ub = unit_bytes(dt), sb = slice_bytes(dt);
  const int64_t g = n / UNIT_ROWS, kb = k / UNIT_COLS;
  const int r = (int)(n - g * UNIT_ROWS), e = (int)(k - kb * UNIT_COLS);
  const uint8_t* unit = w + (g * KB + kb) * ub;
  const uint8_t* sl = unit + (int64_t)r * sb;
  if (dt == Q4_0) {
    const int j = e >> 5, l = e & 31;
    const float d = h2f(ld16(sl + 2 * j));
    const uint8_t byte = sl[16 + 16 * j + (l & 15)];
    const int q = (l < 16 ? (byte & 15) : (byte >> 4)) - 8;
    return (float)q * d;
  }
  if (dt == Q8_0) {
    const int j = e >> 5, l = e & 31;
    return (float)(int8_t)sl[16 + 32 * j + l] * h2f(ld16(sl + 2 * j));
  }
  if (dt == Q4_1 || dt == Q5_0 || dt == Q5_1) {
    const int j = e >> 5, l = e & 31;
    const float d = h2f(ld16(sl + 2 * j));
    const uint8_t byte = sl[sl_qs(dt) + 16 * j + (l & 15)];
    int q = l < 16 ? (byte & 15) : (byte >> 4);
    if (has_qh(dt)) {
      const uint8_t* h = sl + sl_qh(dt) + 4 * j;
      const uint32_t qh = (uint32_t)h[0] | ((uint32_t)h[1] << 8) | ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
      q |= (int)((qh >> l) & 1u) << 4;
    }
    if (dt == Q5_0) return __fmul_rn((float)(q - 16), d);
    return __fadd_rn(__fmul_rn((float)q, d), h2f(ld16(sl + sl_m(dt) + 2 * j)));
  }
  if (dt == Q4_K || dt == Q5_K) {
    const float d = h2f(ld16(sl)), dmin = h2f(ld16(sl + 2));
    const uint8_t* s = sl + 4;
    const int j = e >> 5, l = e & 31;
    int sc, m;
    if (j < 4) {
      sc = s[j] & 63;
      m = s[j + 4] & 63;
    } else {
      sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
      m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const uint8_t* qs = sl + (dt == Q5_K ? 48 : 16);
    int q = (qs[32 * (j >> 1) + l] >> ((j & 1) ? 4 : 0)) & 15;
    if (dt == Q5_K) q |= ((sl[16 + l] >> j) & 1) << 4;
    return (d * (float)sc) * (float)q - dmin * (float)m;
  }
  // Q6_K
  const int h = e >> 7, rr = e & 127, c = rr >> 5, l = rr & 31;
  const int lo = (sl[16 + 64 * h + l + 32 * (c & 1)] >> (4 * (c >> 1))) & 15;
  const int hi = (sl[144 + 32 * h + l] >> (2 * c)) & 3;
  const float d = h2f(ld16(unit + (int64_t)UNIT_ROWS * sb + 2 * r));
  const int8_t sc = (int8_t)sl[e >> 4];
  return (d * (float)sc) * (float)((lo | (hi << 4)) - 32);
}

__global__ void dequant_kernel(int dt, const uint8_t* __restrict__ w, float* __restrict__ out,
                               int64_t N, int64_t K, int64_t KB) {
  const int64_t total = N * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / K, k = i - n * K;
    out[i] = decode_tiled(dt, w, n, k, KB);
  }
}

static int grid_for(int64_t n) {
  int64_t g = (n + 255) / 256;
  if (g < 1) g = 1;
  if (g > 148 * 64) g = 148 * 64;
  return (int)g;
}

cudaError_t launch_repack(int dt, const void* gguf, void* tiled, int64_t N, int64_t K, cudaStream_t s) {
  const int64_t KB = (K + UNIT_COLS - 1) / UNIT_COLS, G = (N + UNIT_ROWS - 1) / UNIT_ROWS;
  const int64_t total = G * KB * unit_bytes(dt);
  if (total == 0) return cudaSuccess;
  repack_kernel<<<grid_for(total), 256, 0, s>>>(dt, (const uint8_t*)gguf, (uint8_t*)tiled, N, K, KB, total);
  return cudaGetLastError();
}

cudaError_t launch_unpack(int dt, const void* tiled, void* gguf, int64_t N, int64_t K, cudaStream_t s) {
  const int64_t KB = (K + UNIT_COLS - 1) / UNIT_COLS;
  const int64_t nb_row = (K + block_elems(dt) - 1) / block_elems(dt);
  const int64_t total = N * nb_row * block_bytes(dt);
  if (total == 0) return cudaSuccess;
  unpack_kernel<<<grid_for(total), 256, 0, s>>>(dt, (const uint8_t*)tiled, (uint8_t*)gguf, K, KB, total);
  return cudaGetLastError();
}

cudaError_t launch_dequant(int dt, const void* tiled, float* out, int64_t N, int64_t K, cudaStream_t s) {
  const int64_t KB = (K + UNIT_COLS - 1) / UNIT_COLS;
  if (N * K == 0) return cudaSuccess;
  dequant_kernel<<<grid_for(N * K), 256, 0, s>>>(dt, (const uint8_t*)tiled, out, N, K, KB);
  return cudaGetLastError();
}

}  // namespace odi_cuda
