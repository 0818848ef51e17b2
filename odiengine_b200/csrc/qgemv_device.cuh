// qgemv_device.cuh -- the streaming quantized GEMV kernel (device side).
//
// y[M, N] = x[M, K] . dequant(W)^T for M <= 8 tokens per pass, W in the
// tiled layout (common.cuh).  Structure:
//   * The G*KB units of the weight (64 rows x 256 columns, contiguous) are cut
//     into P contiguous ranges, one per CTA (stream-K), so every SM streams
//     the same number of bytes.
//   * Warp 8 is the producer: one lane issues a bulk copy (cp.async.bulk, no
//     multicast) of each unit and of the matching activation slice into a
//     ring of shared-memory stages, completing on an mbarrier.
//   * Warps 0-7 consume.  Lane = output row: warp w owns rows 32*(w&1) ..+31
//     of the unit and the 64-column quarter kq = w>>1 of its 256 columns.
//     A lane reads its row's codes for that quarter with 128-bit shared
//     loads (the slice strides 144/176/208/272 B keep a quarter-warp on
//     distinct banks), decodes the header once per 64 weights, and
//     reads the activations as broadcast loads.
//       ACT_Q8 : codes x int8 activations with dp4a, exact int32 per
//                32-value block (16 for Q6_K), fp32 scale per block;
//       ACT_F32: codes widened to fp32 exactly (2^23 magic), fp32 FMA with
//                fp32 activations.
//   * At the end of a row tile the four quarter sums of each row meet in
//     shared memory (added in fixed order).  A tile wholly inside one CTA's
//     range is written to y; a tile cut between CTAs goes through the fixup:
//     partial sums into per-CTA slots, an atomic counter, and the last CTA to
//     arrive adds the slots in CTA order (deterministic) and writes y,
//     resetting the counter for the next call.
//   * Every mbarrier wait is bounded; a wait that gives up sets the error
//     word, and the producer drains its copies before the CTA exits.
#pragma once

#include "internal.h"

namespace odi_cuda {

constexpr int NCW = 8;                    // consumer warps: 2 row halves x 4 column quarters
constexpr int NTHREADS = (NCW + 1) * 32;  // + producer warp
constexpr int BAR_BYTES = 1024;           // mbarriers + flag
constexpr int MAX_STAGES = 16;
constexpr int MAX_MT = 8;
constexpr int RED_BYTES = 4 * UNIT_ROWS * MAX_MT * 4;  // quarter sums at tile end
constexpr int RING_OFFSET = BAR_BYTES + RED_BYTES;
constexpr int RING_BUDGET = 96 * 1024;    // two CTAs per SM

// Exact int -> float for |v| < 2^22 with two full-rate ops.
__device__ __forceinline__ float i2f(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }

// Byte B of w as the float 2^23 + byte (exact).
template <int B>
__device__ __forceinline__ float byte_magic(uint32_t w) {
  return __int_as_float(__byte_perm(w, 0x4Bu, 0x4550u | B));
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}

__device__ __forceinline__ int owner_of(int u, int P, int U) {
  return (int)(((int64_t)(u + 1) * P - 1) / U);
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t ldsu16(const uint8_t* p) {
  return *reinterpret_cast<const unsigned short*>(p);
}
__device__ __forceinline__ float h2f_lo(uint32_t w) { return h2f((uint16_t)(w & 0xFFFFu)); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return h2f((uint16_t)(w >> 16)); }

// ---------------------------------------------------------------------------
// One lane's share of a unit: 4 groups of 16 codes (4 bytes per word) of one
// row and one column quarter, with per-group scale A and min B
// (value = A * code - B; Q8_0 codes are signed, B = 0).
// Group g covers 16 consecutive columns starting at xoff(g) in the span and
// uses half (g & 1) of activation record rec(g).
// ---------------------------------------------------------------------------
struct LaneCodes {
  uint32_t cw[4][4];
  float A[4];
  float B[4];
};

// Bits s of each byte of h moved to bit 4 (s in 0..7).
__device__ __forceinline__ uint32_t bit_to4(uint32_t h, int s) {
  return (s <= 4 ? (h << (4 - s)) : (h >> (s - 4))) & 0x10101010u;
}
// Bits s, s+1 of each byte moved to bits 4, 5 (s even, 0..6).
__device__ __forceinline__ uint32_t bits2_to4(uint32_t h, int s) {
  return (s <= 4 ? (h << (4 - s)) : (h >> (s - 4))) & 0x30303030u;
}

template <int DT>
struct QuarterMap {
  // xoff: byte offset of group g's 16 activation codes in the 256-span
  __device__ __forceinline__ static int xoff(int kq, int g) {
    if (DT == Q6_K) {
      const int h = kq >> 1, cl = kq & 1;
      return 128 * h + 32 * cl + 16 * (g & 1) + 64 * (g >> 1);
    }
    return 64 * kq + 16 * g;
  }
  // record (32-value activation block) of group g
  __device__ __forceinline__ static int rec(int kq, int g) {
    if (DT == Q6_K) {
      const int h = kq >> 1, cl = kq & 1;
      return 4 * h + cl + 2 * (g >> 1);
    }
    return 2 * kq + (g >> 1);
  }
};

template <int DT>
__device__ __forceinline__ void lane_codes(const uint8_t* __restrict__ st, int row, int kq, LaneCodes& lc) {
  const uint8_t* sl = st + row * slice_bytes(DT);
  if (DT == Q4_K || DT == Q5_K) {
    const uint4 hd = lds128(sl);
    const float d = h2f_lo(hd.x), dmin = h2f_hi(hd.x);
    // 6-bit scales/mins of sub-blocks 0..3 (low) and 4..7 (high), one per byte
    const uint32_t scv = kq < 2 ? (hd.y & 0x3F3F3F3Fu) : ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u));
    const uint32_t mnv = kq < 2 ? (hd.z & 0x3F3F3F3Fu) : (((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u));
    const int sh = 16 * (kq & 1);
    lc.A[0] = lc.A[1] = d * i2f((scv >> sh) & 0xFF);
    lc.A[2] = lc.A[3] = d * i2f((scv >> (sh + 8)) & 0xFF);
    lc.B[0] = lc.B[1] = dmin * i2f((mnv >> sh) & 0xFF);
    lc.B[2] = lc.B[3] = dmin * i2f((mnv >> (sh + 8)) & 0xFF);
    const uint8_t* qs = sl + (DT == Q5_K ? 48 : 16) + 32 * kq;
    const uint4 qa = lds128(qs), qb = lds128(qs + 16);
    const uint32_t va[4] = {qa.x, qa.y, qa.z, qa.w}, vb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lc.cw[0][i] = va[i] & 0x0F0F0F0Fu;
      lc.cw[1][i] = vb[i] & 0x0F0F0F0Fu;
      lc.cw[2][i] = (va[i] >> 4) & 0x0F0F0F0Fu;
      lc.cw[3][i] = (vb[i] >> 4) & 0x0F0F0F0Fu;
    }
    if (DT == Q5_K) {
      const uint4 ha = lds128(sl + 16), hb = lds128(sl + 32);
      const uint32_t wa[4] = {ha.x, ha.y, ha.z, ha.w}, wb[4] = {hb.x, hb.y, hb.z, hb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        lc.cw[0][i] |= bit_to4(wa[i], 2 * kq);
        lc.cw[1][i] |= bit_to4(wb[i], 2 * kq);
        lc.cw[2][i] |= bit_to4(wa[i], 2 * kq + 1);
        lc.cw[3][i] |= bit_to4(wb[i], 2 * kq + 1);
      }
    }
  } else if (DT == Q6_K) {
    const int h = kq >> 1, cl = kq & 1;
    const uint4 a = lds128(sl + 16 + 64 * h + 32 * cl), b = lds128(sl + 16 + 64 * h + 32 * cl + 16);
    const uint4 ha = lds128(sl + 144 + 32 * h), hb = lds128(sl + 144 + 32 * h + 16);
    const uint32_t va[4] = {a.x, a.y, a.z, a.w}, vb[4] = {b.x, b.y, b.z, b.w};
    const uint32_t wa[4] = {ha.x, ha.y, ha.z, ha.w}, wb[4] = {hb.x, hb.y, hb.z, hb.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lc.cw[0][i] = (va[i] & 0x0F0F0F0Fu) | bits2_to4(wa[i], 2 * cl);
      lc.cw[1][i] = (vb[i] & 0x0F0F0F0Fu) | bits2_to4(wb[i], 2 * cl);
      lc.cw[2][i] = ((va[i] >> 4) & 0x0F0F0F0Fu) | bits2_to4(wa[i], 2 * cl + 4);
      lc.cw[3][i] = ((vb[i] >> 4) & 0x0F0F0F0Fu) | bits2_to4(wb[i], 2 * cl + 4);
    }
    const float d = h2f((uint16_t)ldsu16(st + UNIT_ROWS * 208 + 2 * row));
    const uint32_t s4 = ldsu16(sl + 8 * h + 2 * cl);      // int8 scales of sub-blocks sb, sb+1
    const uint32_t s6 = ldsu16(sl + 8 * h + 2 * cl + 4);  // sb+4, sb+5
    lc.A[0] = d * i2f((int)(signed char)(s4 & 0xFF));
    lc.A[1] = d * i2f((int)(signed char)((s4 >> 8) & 0xFF));
    lc.A[2] = d * i2f((int)(signed char)(s6 & 0xFF));
    lc.A[3] = d * i2f((int)(signed char)((s6 >> 8) & 0xFF));
#pragma unroll
    for (int g = 0; g < 4; ++g) lc.B[g] = 32.0f * lc.A[g];
  } else if (DT == Q8_0) {
    const uint32_t dd = lds32(sl + 4 * kq);
    lc.A[0] = lc.A[1] = h2f_lo(dd);
    lc.A[2] = lc.A[3] = h2f_hi(dd);
    lc.B[0] = lc.B[1] = lc.B[2] = lc.B[3] = 0.0f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint4 q = lds128(sl + 16 + 64 * kq + 16 * g);
      lc.cw[g][0] = q.x; lc.cw[g][1] = q.y; lc.cw[g][2] = q.z; lc.cw[g][3] = q.w;
    }
  } else {  // Q4_0
    const uint32_t dd = lds32(sl + 4 * kq);
    lc.A[0] = lc.A[1] = h2f_lo(dd);
    lc.A[2] = lc.A[3] = h2f_hi(dd);
#pragma unroll
    for (int g = 0; g < 4; ++g) lc.B[g] = 8.0f * lc.A[g];
    const uint4 q0 = lds128(sl + 16 + 32 * kq), q1 = lds128(sl + 32 + 32 * kq);
    const uint32_t v0[4] = {q0.x, q0.y, q0.z, q0.w}, v1[4] = {q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lc.cw[0][i] = v0[i] & 0x0F0F0F0Fu;
      lc.cw[1][i] = (v0[i] >> 4) & 0x0F0F0F0Fu;
      lc.cw[2][i] = v1[i] & 0x0F0F0F0Fu;
      lc.cw[3][i] = (v1[i] >> 4) & 0x0F0F0F0Fu;
    }
  }
}

__device__ __forceinline__ int dot16(const uint32_t (&cw)[4], uint4 x, int acc) {
  acc = __dp4a((int)cw[0], (int)x.x, acc);
  acc = __dp4a((int)cw[1], (int)x.y, acc);
  acc = __dp4a((int)cw[2], (int)x.z, acc);
  acc = __dp4a((int)cw[3], (int)x.w, acc);
  return acc;
}

// ---------------------------------------------------------------------------
// ACT_Q8 unit.  Groups (0,1) and (2,3) share scale and activation block for
// every type but Q6_K, so their integer dots are added before scaling.
// ---------------------------------------------------------------------------
template <int DT, int MT>
__device__ __forceinline__ void unit_q8(const uint8_t* __restrict__ st, const uint8_t* __restrict__ xs, int M,
                                        int row, int kq, float (&acc)[MT]) {
  LaneCodes lc;
  lane_codes<DT>(st, row, kq, lc);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m < M) {
      const uint8_t* xr = xs + m * ACT_Q8_BYTES;
      float v = acc[m];
      if (DT == Q6_K) {
        const uint4 x0 = lds128(xr + QuarterMap<DT>::xoff(kq, 0)), x1 = lds128(xr + QuarterMap<DT>::xoff(kq, 1));
        const uint4 x2 = lds128(xr + QuarterMap<DT>::xoff(kq, 2)), x3 = lds128(xr + QuarterMap<DT>::xoff(kq, 3));
        const uint2 ra = *reinterpret_cast<const uint2*>(xr + 256 + 8 * QuarterMap<DT>::rec(kq, 0));
        const uint2 rb = *reinterpret_cast<const uint2*>(xr + 256 + 8 * QuarterMap<DT>::rec(kq, 2));
        const float dxa = __uint_as_float(ra.x), dxb = __uint_as_float(rb.x);
        const int sa0 = (int)(short)(ra.y & 0xFFFFu), sa1 = (int)ra.y >> 16;
        const int sb0 = (int)(short)(rb.y & 0xFFFFu), sb1 = (int)rb.y >> 16;
        // (q - 32) . x = q . x - 32 * sum(x), exact in int32
        const int d0 = dot16(lc.cw[0], x0, -32 * sa0), d1 = dot16(lc.cw[1], x1, -32 * sa1);
        const int d2 = dot16(lc.cw[2], x2, -32 * sb0), d3 = dot16(lc.cw[3], x3, -32 * sb1);
        v = fmaf(i2f(d0), lc.A[0] * dxa, v);
        v = fmaf(i2f(d1), lc.A[1] * dxa, v);
        v = fmaf(i2f(d2), lc.A[2] * dxb, v);
        v = fmaf(i2f(d3), lc.A[3] * dxb, v);
      } else {
        const uint4 x0 = lds128(xr + 64 * kq), x1 = lds128(xr + 64 * kq + 16);
        const uint4 x2 = lds128(xr + 64 * kq + 32), x3 = lds128(xr + 64 * kq + 48);
        const uint4 rr = lds128(xr + 256 + 16 * kq);  // records 2kq, 2kq+1
        const float dxa = __uint_as_float(rr.x), dxb = __uint_as_float(rr.z);
        const int sa = (int)(short)(rr.y & 0xFFFFu) + ((int)rr.y >> 16);
        const int sb = (int)(short)(rr.w & 0xFFFFu) + ((int)rr.w >> 16);
        int da = DT == Q4_0 ? -8 * sa : 0, db = DT == Q4_0 ? -8 * sb : 0;
        da = dot16(lc.cw[1], x1, dot16(lc.cw[0], x0, da));
        db = dot16(lc.cw[3], x3, dot16(lc.cw[2], x2, db));
        v = fmaf(i2f(da), lc.A[0] * dxa, v);
        v = fmaf(i2f(db), lc.A[2] * dxb, v);
        if (DT == Q4_K || DT == Q5_K) {
          v = fmaf(-lc.B[0], i2f(sa) * dxa, v);
          v = fmaf(-lc.B[2], i2f(sb) * dxb, v);
        }
      }
      acc[m] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// ACT_F32 unit.
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ float dot16_f32(const uint32_t (&cw)[4], const float* __restrict__ x) {
  // Q8_0 codes are signed: flip to q + 128 and remove that bias too.
  constexpr float bias = DT == Q8_0 ? 8388608.0f + 128.0f : 8388608.0f;
  float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = DT == Q8_0 ? (cw[i] ^ 0x80808080u) : cw[i];
    const float4 xv = *reinterpret_cast<const float4*>(x + 4 * i);
    s0 = fmaf(xv.x, byte_magic<0>(w) - bias, s0);
    s1 = fmaf(xv.y, byte_magic<1>(w) - bias, s1);
    s0 = fmaf(xv.z, byte_magic<2>(w) - bias, s0);
    s1 = fmaf(xv.w, byte_magic<3>(w) - bias, s1);
  }
  return s0 + s1;
}

__device__ __forceinline__ float sum16(const float* __restrict__ x) {
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = *reinterpret_cast<const float4*>(x + 4 * i);
    s += (v.x + v.y) + (v.z + v.w);
  }
  return s;
}

template <int DT, int MT>
__device__ __forceinline__ void unit_f32(const uint8_t* __restrict__ st, const uint8_t* __restrict__ xs, int M,
                                         int row, int kq, float (&acc)[MT]) {
  LaneCodes lc;
  lane_codes<DT>(st, row, kq, lc);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m < M) {
      const float* xr = reinterpret_cast<const float*>(xs + m * ACT_F32_BYTES);
      float v = acc[m];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const float* xg = xr + QuarterMap<DT>::xoff(kq, g);
        v = fmaf(lc.A[g], dot16_f32<DT>(lc.cw[g], xg), v);
        if (DT != Q8_0) v = fmaf(-lc.B[g], sum16(xg), v);
      }
      acc[m] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Row-tile flush: quarter sums -> tile sums -> y or fixup.
// ---------------------------------------------------------------------------
template <int MT>
__device__ __forceinline__ void flush_tile(const GemvArgs& a, const GemvPlan& pl, int g, bool whole, int c,
                                           const float (&acc)[MT], int row, int kq, float* red,
                                           volatile int* flag) {
#pragma unroll
  for (int m = 0; m < MT; ++m)
    if (m < a.M) red[(kq * UNIT_ROWS + row) * MT + m] = acc[m];
  consumer_sync();
  const int tid = threadIdx.x;
  const int c_lo = whole ? c : owner_of(g * pl.KB, pl.P, pl.U);
  const int c_hi = whole ? c : owner_of((g + 1) * pl.KB - 1, pl.P, pl.U);
  float* slot = a.partial + ((int64_t)g * pl.maxc + (c - c_lo)) * (UNIT_ROWS * MT);
  for (int t = tid; t < UNIT_ROWS * a.M; t += NCW * 32) {
    const int m = t >> 6, r = t & 63;
    const float v = ((red[(0 * UNIT_ROWS + r) * MT + m] + red[(1 * UNIT_ROWS + r) * MT + m]) +
                     red[(2 * UNIT_ROWS + r) * MT + m]) + red[(3 * UNIT_ROWS + r) * MT + m];
    if (whole) {
      const int64_t n = (int64_t)g * UNIT_ROWS + r;
      if (n < a.N) a.y[(int64_t)m * a.N + n] = v;
    } else {
      slot[m * UNIT_ROWS + r] = v;
    }
  }
  if (!whole) {
    __threadfence();
    consumer_sync();
    if (tid == 0) {
      __threadfence();
      const int old = atomicAdd(&a.counters[g], 1);
      const int last = old == (c_hi - c_lo);
      if (last) atomicExch(&a.counters[g], 0);
      *flag = last;
    }
    consumer_sync();
    if (*flag) {
      __threadfence();
      const int nc = c_hi - c_lo + 1;
      const float* base = a.partial + (int64_t)g * pl.maxc * (UNIT_ROWS * MT);
      for (int t = tid; t < UNIT_ROWS * a.M; t += NCW * 32) {
        const int m = t >> 6, r = t & 63;
        const int64_t n = (int64_t)g * UNIT_ROWS + r;
        float s = 0.0f;
        for (int j = 0; j < nc; ++j) s += __ldcg(base + (int64_t)j * (UNIT_ROWS * MT) + m * UNIT_ROWS + r);
        if (n < a.N) a.y[(int64_t)m * a.N + n] = s;
      }
    }
  }
  consumer_sync();  // red and flag are reused by the next flush
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int DT, int MT, bool F32>
__global__ void __launch_bounds__(NTHREADS, 2) qgemv_kernel(const GemvArgs a, const GemvPlan pl) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAX_STAGES;
  volatile int* flag = reinterpret_cast<volatile int*>(smem + 512);
  float* red = reinterpret_cast<float*>(smem + BAR_BYTES);
  uint8_t* ring = smem + RING_OFFSET;
  constexpr int UB = unit_bytes(DT);
  constexpr int XB = F32 ? ACT_F32_BYTES : ACT_Q8_BYTES;
  const int S = pl.stages, SB = pl.stage_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int u0 = (int)((int64_t)pl.U * c / pl.P);
  const int u1 = (int)((int64_t)pl.U * (c + 1) / pl.P);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NCW) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint32_t xbytes = (uint32_t)a.M * XB;
      // Fill the ring with weight units first: weights are not written by the
      // kernels this one may overlap under programmatic dependent launch.
      const int first = (u1 - u0) < S ? (u1 - u0) : S;
      for (int i = 0; i < first; ++i) {
        mbar_arrive_expect_tx(&full[i], UB + xbytes);
        bulk_g2s(ring + i * SB, a.w + (int64_t)(u0 + i) * UB, UB, &full[i]);
      }
      pdl_wait();  // activation tiles are written by the previous kernel
      for (int i = 0; i < first; ++i) {
        const int kb = (u0 + i) % pl.KB;
        bulk_g2s(ring + i * SB + UB, a.act + ((int64_t)kb * a.M_total + a.m0) * XB, xbytes, &full[i]);
      }
      int i = first;
      for (int u = u0 + first; u < u1; ++u, ++i) {
        const int s = i % S;
        if (!mbar_wait(&empty[s], ((i / S) - 1) & 1, a.err, ERR_EMPTY_WAIT)) break;
        uint8_t* st = ring + s * SB;
        const int kb = u % pl.KB;
        mbar_arrive_expect_tx(&full[s], UB + xbytes);
        bulk_g2s(st, a.w + (int64_t)u * UB, UB, &full[s]);
        bulk_g2s(st + UB, a.act + ((int64_t)kb * a.M_total + a.m0) * XB, xbytes, &full[s]);
      }
      pdl_launch_dependents();
      // Drain: every copy issued must land before the CTA may exit.
      const int issued = i;
      for (int s = 0; s < S && s < issued; ++s) {
        const int last = s + S * ((issued - 1 - s) / S);
        mbar_wait(&full[s], (last / S) & 1, a.err, ERR_DRAIN_WAIT);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int row = 32 * (warp & 1) + lane;
  const int kq = warp >> 1;
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.0f;

  int i = 0;
  for (int u = u0; u < u1; ++u, ++i) {
    const int s = i % S;
    if (!mbar_wait(&full[s], (i / S) & 1, a.err, ERR_FULL_WAIT)) break;
    const uint8_t* st = ring + s * SB;
    if (F32) unit_f32<DT, MT>(st, st + UB, a.M, row, kq, acc);
    else unit_q8<DT, MT>(st, st + UB, a.M, row, kq, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    const int g = u / pl.KB, kb = u - g * pl.KB;
    if (kb == pl.KB - 1 || u == u1 - 1) {
      const bool whole = (u - kb >= u0) && (kb == pl.KB - 1);
      flush_tile<MT>(a, pl, g, whole, c, acc, row, kq, red, flag);
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    }
  }
}

}  // namespace odi_cuda
