// qgemv_device.cuh -- the streaming quantized GEMV kernel (device side).
//
// y[M, N] = x[M, K] . dequant(W)^T for M <= 8 tokens per pass, W in the
// tiled layout (common.cuh: units of 64 rows x 256 columns, contiguous).
//   * Each 64-row tile is handled by a thread-block cluster of C CTAs; CTA
//     rank j streams the contiguous chunk j of the tile's units (spans).
//   * Warp 4 is the producer: one lane issues a bulk copy (cp.async.bulk, no
//     multicast) of each unit into a ring of shared-memory stages, completing
//     on an mbarrier.  Weights do not depend on earlier kernels, so the
//     producer starts at once, also under programmatic dependent launch.
//   * Warps 0-3 consume.  After griddepcontrol.wait they stage the
//     activations of the chunk in shared memory (cp.async, all spans in
//     flight at once) and, in ACT_Q8 mode, quantise them in place to Q8_0
//     (bit-identical to odi_cuda_quantize_q8_0).  Then warp w takes every
//     other unit (parity w>>1) and lane l owns row 32*(w&1)+l across the
//     whole 256-column span: it decodes the row's header once per unit,
//     reads the codes with 128-bit shared loads (the slice strides
//     144/176/208/272 B keep each quarter-warp on distinct banks) and dots:
//       ACT_Q8 : codes x int8 activations with dp4a (high nibbles kept in
//                place, x16, via the unsigned x signed form), exact int32 per
//                32-value block (16 for Q6_K), fp32 scale per block;
//       ACT_F32: codes widened to fp32 exactly (2^23 magic), fp32 FMA with
//                fp32 activations.
//   * End of tile: the two unit-parity sums of each row are added in
//     shared memory; with C > 1 rank 0 adds the C partial tiles in rank
//     order over distributed shared memory (deterministic) and writes y.
//   * Every mbarrier wait is bounded (and sleeps in hardware while waiting);
//     a wait that gives up sets the error word, the producer drains its
//     copies, and every thread still reaches the cluster barriers.
#pragma once

#include "internal.h"

namespace odi_cuda {

constexpr int NCW = 4;                    // consumer warps
constexpr int NTHREADS = (NCW + 1) * 32;  // + producer warp
constexpr int CTAS_PER_SM = 4;
constexpr int BAR_BYTES = 1024;           // mbarriers
constexpr int MAX_STAGES = 16;
constexpr int MAX_MT = 8;
constexpr int SMEM_PER_CTA = 54 * 1024;   // the ring is sized to this
constexpr int SMEM_MAX_CTA = 56 * 1024;   // four CTAs per SM (228 KB less 1 KB reserved per CTA)
// Weight stages the producer fills before the activations are on their way
// when the kernel quantises fp32 activations itself: the rest wait until
// every consumer warp has issued its activation loads, so those loads are not
// queued in HBM behind a whole ring of weight copies (headline Q4_K
// 4096x14336: 8.02 -> 7.63 us; one early stage: 8.33).  Pre-quantized records
// come from L2, written by the kernel before: there all stages go out at once
// (holding two back cost the decode step 1%).
constexpr int EARLY_STAGES = 2;
constexpr int XR_BUDGET = 24 * 1024;      // staged activations per CTA
// One staged (span, token): 256 fp32 values, then 16 fp32 sums of 16 values.
// ACT_Q8 rewrites it in place as 256 codes followed by 8 XRec (one per
// 32-value block).
constexpr int XR_VALS = 1024;
constexpr int XR_STRIDE = XR_VALS + 64;
// Shared-memory stride of a staged (span, token) record: XR_STRIDE, or
// Q8_REC_BYTES for pre-quantized records.  8-token passes add 16 bytes so the
// records of the 8 tokens start in different banks: the tensor-core units
// read a word of every token's codes in one instruction (10% on the 8-token
// GEMVs; fewer tokens read each record by broadcast and keep the dense stride).
__host__ __device__ constexpr int stage_stride(bool pre, int mt) {
  return (pre ? Q8_REC_BYTES : XR_STRIDE) + (mt == 8 ? 16 : 0);
}

// Q8 activation record of one 32-value block, pre-scaled for the kernels:
// dx = the fp16 scale widened to fp32; sdx = (sum of codes) * dx, and the
// same for the first / second 16 codes.
struct XRec {
  float dx, sdx, sdx_lo, sdx_hi;
};

// Self-checking build (-DODI_GEMV_CHECKS): a failed index check records its
// code and two values in err[1..3] (first failure wins), sets bit 30 of
// err[0], and the guarded access is skipped.  Off in normal builds.
#ifdef ODI_GEMV_CHECKS
__device__ __forceinline__ bool gemv_check(bool ok, int* err, int code, long long x, long long y) {
  if (!ok && err) {
    atomicOr(err, 1 << 30);
    if (atomicCAS(err + 1, 0, code) == 0) {
      err[2] = (int)x;
      err[3] = (int)y;
    }
  }
  return ok;
}
#define GCHK(cond, code, x, y) gemv_check((cond), a.err, (code), (long long)(x), (long long)(y))
#else
#define GCHK(cond, code, x, y) true
#endif

// int -> float; exact here (|v| < 2^22).  One conversion instruction, not
// on the quarter-rate XU pipe on sm_100a (pipe counters), so it costs fewer
// issue slots than the two-op magic-number form.
__device__ __forceinline__ float i2f(int v) { return __int2float_rn(v); }

// Packed fp32 (sm_100 FFMA2 / FMUL2): two independent IEEE operations with
// round-to-nearest in one instruction, each element the same float as
// fmaf / __fmul_rn of its pair.  Used where two elements share an
// operation: two tokens of a pass, two rows of a tile, two scales.
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }

// Byte B of w as the float 2^23 + byte (exact).
template <int B>
__device__ __forceinline__ float byte_magic(uint32_t w) {
  return __int_as_float(__byte_perm(w, 0x4Bu, 0x4550u | B));
}
// d * (byte B of w), exactly rounded, in two ops: fma(d, 2^23 + b, -d*2^23).
template <int B>
__device__ __forceinline__ float scale_byte(float d, float nd23, uint32_t w) {
  return fmaf(d, byte_magic<B>(w), nd23);
}
// scale_byte of bytes B and B + 1 of w with the pair's own (d, -2^23 d)
template <int B>
__device__ __forceinline__ float2 scale_byte2(float2 d, float2 nd23, uint32_t w) {
  return fma2(d, f2(byte_magic<B>(w), byte_magic<B + 1>(w)), nd23);
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ float4 lds128f(const uint8_t* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ uint32_t ldsu16(const uint8_t* p) {
  return *reinterpret_cast<const unsigned short*>(p);
}
__device__ __forceinline__ float h2f_lo(uint32_t w) { return h2f((uint16_t)(w & 0xFFFFu)); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return h2f((uint16_t)(w >> 16)); }

// Signed x signed and unsigned x signed 4-way byte dot products.
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
template <bool US>
__device__ __forceinline__ int dot16(uint4 w, uint4 x, int acc) {
  if (US) {
    acc = dp4a_us(w.x, x.x, acc);
    acc = dp4a_us(w.y, x.y, acc);
    acc = dp4a_us(w.z, x.z, acc);
    return dp4a_us(w.w, x.w, acc);
  }
  acc = dp4a_ss(w.x, x.x, acc);
  acc = dp4a_ss(w.y, x.y, acc);
  acc = dp4a_ss(w.z, x.z, acc);
  return dp4a_ss(w.w, x.w, acc);
}
// The low bytes of four ints (codes in [-128, 127]) packed, a in byte 0.
__device__ __forceinline__ uint32_t pack4_s8(int a, int b, int c, int d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}
__device__ __forceinline__ uint4 and4(uint4 v, uint32_t m) { return make_uint4(v.x & m, v.y & m, v.z & m, v.w & m); }
__device__ __forceinline__ uint4 shr4(uint4 v, int s) { return make_uint4(v.x >> s, v.y >> s, v.z >> s, v.w >> s); }
__device__ __forceinline__ uint4 or4(uint4 a, uint4 b) { return make_uint4(a.x | b.x, a.y | b.y, a.z | b.z, a.w | b.w); }
// bits s..s+nb-1 of every byte moved to bit 4 (mask m selects the result bits)
__device__ __forceinline__ uint32_t mv4(uint32_t h, int s, uint32_t m) {
  return (s <= 4 ? (h << (4 - s)) : (h >> (s - 4))) & m;
}
__device__ __forceinline__ uint4 mv4x4(uint4 h, int s, uint32_t m) {
  return make_uint4(mv4(h.x, s, m), mv4(h.y, s, m), mv4(h.z, s, m), mv4(h.w, s, m));
}

// ---------------------------------------------------------------------------
// Activation staging (all 128 consumer threads).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// 1. cp.async copies of the raw fp32 values of the chunk's spans for every
//    token (16-byte copies when rows are 16-byte aligned, else 4-byte
//    copies; columns past K are zero-filled).
// 2. ACT_Q8: each 32-value block is quantised in place with the GGUF Q8_0
//    quantiser's arithmetic (d = amax/127 in fp32, q = round-half-away(
//    x * (1/d)), d kept as fp16): codes at [32*b, 32*b+32), XRec b at
//    256 + 16*b.  ACT_F32: the sums of each 16 values go after the values.
// Fused prologues (GemvFuse), applied to the staged fp32 values before the
// quantisation: SwiGLU builds silu(gate) * up from the staged gate and up
// halves; RMSNorm reduces sum(x^2) of every token of the pass -- from the
// sums of squares x's writer left in slots, else over the whole row -- while
// the copies are in flight, then scales the staged chunk by rms * norm_w.
__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

template <int MT>
__device__ __forceinline__ void row_rms(const GemvArgs& a, float* rms_out /* smem [MT] */, float* red /* smem */) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int m = 0; m < a.M; ++m) {
    float s = 0.f;
    if (a.fu.ssq_in) {  // the producer of x left its sums of squares in slots
      const float* sq = a.fu.ssq_in + (int64_t)m * a.fu.ssq_n;
      for (int i = tid; i < a.fu.ssq_n; i += NCW * 32) s += sq[i];
    } else {
      const float* xm = a.x + (int64_t)m * a.ldx;
      for (int64_t k = tid; k < a.K; k += NCW * 32) s = fmaf(xm[k], xm[k], s);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp * MT + m] = s;
  }
  consumer_sync();
  if (tid < a.M) {
    const float s = (red[0 * MT + tid] + red[1 * MT + tid]) + (red[2 * MT + tid] + red[3 * MT + tid]);
    rms_out[tid] = 1.0f / sqrtf(s / (float)a.K + a.fu.eps);
  }
  consumer_sync();
}

// Four fp32 values (nvalid of them real, the rest zero-filled) by cp.async.
__device__ __forceinline__ void copy4(uint8_t* dst, const float* src, int nvalid, bool vec) {
  if (vec) {
    cp_async16(dst, src, 4 * nvalid);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) cp_async4(dst + 4 * e, src + (e < nvalid ? e : 0), e < nvalid ? 4 : 0);
  }
}

// The prologue's second input for the 8 values [k, k+8) a lane quantises:
// the up half of record r's token (SwiGLU) or the norm weights (RMSNorm),
// read from L2 (ld.global.cg), zero past K.
__device__ __forceinline__ void prologue8(const GemvArgs& a, int kb0, int r, int off, float4& e0, float4& e1) {
  const int j = r / a.M, m = r - j * a.M;
  const int64_t k = (int64_t)(kb0 + j) * UNIT_COLS + off;
  const float* p = a.fu.swiglu ? a.x + (int64_t)m * a.ldx + a.K : a.fu.norm_w;
  if (k + 8 <= a.K && (reinterpret_cast<uintptr_t>(p + k) & 15) == 0) {
    e0 = __ldcg(reinterpret_cast<const float4*>(p + k));
    e1 = __ldcg(reinterpret_cast<const float4*>(p + k + 4));
  } else {
    float t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = k + e < a.K ? __ldcg(p + k + e) : 0.f;
    e0 = make_float4(t[0], t[1], t[2], t[3]);
    e1 = make_float4(t[4], t[5], t[6], t[7]);
  }
}

// Quantise two staged (span, token) records held in registers, one lane =
// block b = lane / 4, values [32b + 8 part, +8) with part = lane % 4, into
// Q8 records: codes at rec + 32b + 8part, XRec b at rec + 256 + 16b (the
// gguf Q8_0 quantiser's arithmetic; see stage_acts).  The second record is
// written only if `two`.  The caller orders reads of the records' old
// contents before the call (the codes may land on them).
__device__ __forceinline__ void q8_quantize2(const float (&vv)[2][8], uint8_t* const (&rec)[2], bool two, int lane) {
  const int b = lane >> 2, part = lane & 3;
  float dq[2], dx[2];
  int sh[2], sf[2], shi[2];
  uint32_t packed[2][2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float am = fmaxf(fmaxf(fmaxf(fabsf(vv[i][0]), fabsf(vv[i][1])), fmaxf(fabsf(vv[i][2]), fabsf(vv[i][3]))),
                     fmaxf(fmaxf(fabsf(vv[i][4]), fabsf(vv[i][5])), fmaxf(fabsf(vv[i][6]), fabsf(vv[i][7]))));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    dq[i] = q8_scale(am);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float id = q8_inv(dq[i]);
    int qq[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) qq[e] = q8_round(__fmul_rn(vv[i][e], id));
    packed[i][0] = pack4_s8(qq[0], qq[1], qq[2], qq[3]);
    packed[i][1] = pack4_s8(qq[4], qq[5], qq[6], qq[7]);
    const int sacc = __dp4a((int)packed[i][1], 0x01010101, __dp4a((int)packed[i][0], 0x01010101, 0));
    sh[i] = sacc + __shfl_xor_sync(0xffffffffu, sacc, 1);  // 16 codes: parts 0-1 or 2-3
    sf[i] = sh[i] + __shfl_xor_sync(0xffffffffu, sh[i], 2);
    shi[i] = __shfl_sync(0xffffffffu, sh[i], (lane & ~3) | 2);
    dx[i] = __half2float(__float2half_rn(dq[i]));
  }
  __syncwarp();  // every lane has read its fp32 values before codes land on them
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    if (i == 1 && !two) break;
    *reinterpret_cast<uint2*>(rec[i] + 32 * b + 8 * part) = make_uint2(packed[i][0], packed[i][1]);
    if (part == 0) {
      XRec rq;
      rq.dx = dx[i];
      rq.sdx = __fmul_rn((float)sf[i], dx[i]);
      rq.sdx_lo = __fmul_rn((float)sh[i], dx[i]);
      rq.sdx_hi = __fmul_rn((float)shi[i], dx[i]);
      *reinterpret_cast<XRec*>(rec[i] + 256 + 16 * b) = rq;
    }
  }
}

// ACT_Q8 staging without a prologue, x rows 16-byte aligned (K % 4 == 0):
// each lane loads the 8 values it quantises straight from global memory
// (ld.global.cg, 2 x 16 bytes per record, both records' loads in flight
// together) -- no shared-memory copy of the fp32 values, no barrier between
// load and quantisation; the records' bytes equal stage_acts'.
template <int MT>
__device__ __forceinline__ void stage_q8_direct(const GemvArgs& a, int kb0, int nsp, uint8_t* __restrict__ xr,
                                                uint64_t* xbar) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int off = 32 * (lane >> 2) + 8 * (lane & 3);
  const int nrec = nsp * a.M;
  if (warp >= nrec && lane == 0) mbar_arrive(xbar);  // no records: nothing to issue
  for (int r0 = warp; r0 < nrec; r0 += 2 * NCW) {
    const bool two = r0 + NCW < nrec;
    uint8_t* rec[2];
    float vv[2][8];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int ri = (i == 1 && two) ? r0 + NCW : r0;
      const int j = ri / a.M, m = ri - j * a.M;
      rec[i] = xr + (j * MT + m) * stage_stride(false, MT);
      const int64_t k = (int64_t)(kb0 + j) * UNIT_COLS + off;
      const float* p = a.x + (int64_t)m * a.ldx + k;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 v0 = k + 4 <= a.K ? __ldcg(reinterpret_cast<const float4*>(p)) : z;
      const float4 v1 = k + 8 <= a.K ? __ldcg(reinterpret_cast<const float4*>(p + 4)) : z;
      vv[i][0] = v0.x; vv[i][1] = v0.y; vv[i][2] = v0.z; vv[i][3] = v0.w;
      vv[i][4] = v1.x; vv[i][5] = v1.y; vv[i][6] = v1.z; vv[i][7] = v1.w;
    }
    if (r0 == warp && lane == 0) mbar_arrive(xbar);  // the first loads are in flight
    q8_quantize2(vv, rec, two, lane);
  }
  consumer_sync();
}

// Staging: x (or the gate half of a SwiGLU input) of every span of the chunk
// by cp.async in one group, so it costs one memory round trip whatever the
// chunk length.  The RMSNorm sum of squares is reduced while the copies fly.
// Then each warp applies the prologue to two staged (span, token) records at
// a time -- their second inputs loaded together -- and quantises them.
template <bool F32, int MT>
__device__ __forceinline__ void stage_acts(const GemvArgs& a, int kb0, int nsp, uint8_t* __restrict__ xr,
                                           float* __restrict__ fuse_smem, uint64_t* xbar) {
  const int tid = threadIdx.x;  // 0..127
  const int warp = tid >> 5, lane = tid & 31;
  const bool vec = (a.K & 3) == 0 && (a.ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
  if (!F32 && vec && !a.fu.swiglu && !a.fu.norm_w) {
    stage_q8_direct<MT>(a, kb0, nsp, xr, xbar);
    return;
  }
  // 64 chunks of 4 values per (span, token): threads 0-63 take even tokens, 64-127 odd
  const int q = tid & 63;
  for (int j = 0; j < nsp; ++j) {
    const int64_t k = (int64_t)(kb0 + j) * UNIT_COLS + 4 * q;
    const int64_t left = a.K - k;
    const int nvalid = left <= 0 ? 0 : (left >= 4 ? 4 : (int)left);
    for (int m = tid >> 6; m < a.M; m += 2)
      copy4(xr + (j * MT + m) * stage_stride(false, MT) + 16 * q, a.x + (int64_t)m * a.ldx + (nvalid ? k : 0), nvalid, vec);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  if ((threadIdx.x & 31) == 0) mbar_arrive(xbar);  // this warp's copies are in flight
  if (a.fu.norm_w) row_rms<MT>(a, fuse_smem, fuse_smem + MT);  // overlaps the copies
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  consumer_sync();
  // lane = (block b = lane/4, 8 values).  A warp takes two records per
  // iteration (records r and r + NCW), so their dependent chains (reduce,
  // divide, round, shuffle) interleave.
  const int b = lane >> 2, part = lane & 3;
  const int off = 32 * b + 8 * part;
  const int nrec = nsp * a.M;
  const bool pro = a.fu.swiglu || a.fu.norm_w;
  for (int r0 = warp; r0 < nrec; r0 += 2 * NCW) {
    const bool two = r0 + NCW < nrec;
    uint8_t* rec[2];
    float vv[2][8];
    int mi[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int ri = (i == 1 && two) ? r0 + NCW : r0;
      const int j = ri / a.M;
      mi[i] = ri - j * a.M;
      rec[i] = xr + (j * MT + mi[i]) * stage_stride(false, MT);
      const float4 v0 = lds128f(rec[i] + 4 * off), v1 = lds128f(rec[i] + 4 * (off + 4));
      vv[i][0] = v0.x; vv[i][1] = v0.y; vv[i][2] = v0.z; vv[i][3] = v0.w;
      vv[i][4] = v1.x; vv[i][5] = v1.y; vv[i][6] = v1.z; vv[i][7] = v1.w;
    }
    if (pro) {
      float4 e0[2], e1[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) prologue8(a, kb0, (i == 1 && two) ? r0 + NCW : r0, off, e0[i], e1[i]);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float ee[8] = {e0[i].x, e0[i].y, e0[i].z, e0[i].w, e1[i].x, e1[i].y, e1[i].z, e1[i].w};
        if (a.fu.swiglu) {
#pragma unroll
          for (int e = 0; e < 8; ++e) vv[i][e] = silu_f(vv[i][e]) * ee[e];  // past K: silu(0) * 0
        } else {
          const float rr = fuse_smem[mi[i]];
#pragma unroll
          for (int e = 0; e < 8; ++e) vv[i][e] = vv[i][e] * rr * ee[e];
        }
      }
      if (F32) {  // the fp32 dot reads the staged values
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (i == 1 && !two) break;
          *reinterpret_cast<float4*>(rec[i] + 4 * off) = make_float4(vv[i][0], vv[i][1], vv[i][2], vv[i][3]);
          *reinterpret_cast<float4*>(rec[i] + 4 * (off + 4)) = make_float4(vv[i][4], vv[i][5], vv[i][6], vv[i][7]);
        }
      }
    }
    if (F32) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float s = ((vv[i][0] + vv[i][1]) + (vv[i][2] + vv[i][3])) + ((vv[i][4] + vv[i][5]) + (vv[i][6] + vv[i][7]));
        s += __shfl_xor_sync(0xffffffffu, s, 1);  // 16-value sums (parts 0-1, 2-3)
        if ((part & 1) == 0 && (i == 0 || two)) reinterpret_cast<float*>(rec[i] + XR_VALS)[2 * b + (part >> 1)] = s;
      }
      continue;
    }
    q8_quantize2(vv, rec, two, lane);
    __syncwarp();
  }
  consumer_sync();
}

// Pre-quantized staging: the chunk's Q8 records, made by
// act_q8_records_kernel, copied as they are (16-byte cp.async by all 128
// consumer threads, one memory round trip); record (j, m) of the chunk to
// xr + (j * MT + m) * Q8_REC_BYTES.
template <int MT>
__device__ __forceinline__ void stage_records(const GemvArgs& a, int kb0, int nsp, uint8_t* __restrict__ xr,
                                              float* __restrict__ fuse_smem, uint64_t* xbar) {
  constexpr int V = Q8_REC_BYTES / 16;  // 16-byte pieces per record
  const int per_span = a.M * V;
  for (int c = threadIdx.x; c < nsp * per_span; c += NCW * 32) {
    const int j = c / per_span, rem = c - j * per_span;
    const int m = rem / V, v = rem - m * V;
    cp_async16(xr + (j * MT + m) * stage_stride(true, MT) + 16 * v,
               a.recs + ((int64_t)(kb0 + j) * a.rec_ld + m) * Q8_REC_BYTES + 16 * v, 16);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  if ((threadIdx.x & 31) == 0) mbar_arrive(xbar);  // this warp's copies are in flight
  if (a.fu.rec_scale) row_rms<MT>(a, fuse_smem, fuse_smem + MT);  // overlaps the copies
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  consumer_sync();
  if (a.fu.rec_scale) {
    // records of u = x * w: the token's 1 / rms scales every block factor
    for (int i = threadIdx.x; i < nsp * a.M * 32; i += NCW * 32) {
      const int rj = i >> 5, f = i & 31;
      const int j = rj / a.M, m = rj - j * a.M;
      float* xf = reinterpret_cast<float*>(xr + (j * MT + m) * stage_stride(true, MT) + 256);
      xf[f] = xf[f] * fuse_smem[m];
    }
    consumer_sync();
  }
}

// ---------------------------------------------------------------------------
// ACT_Q8 units: one lane, one row, the whole 256-column span, MT tokens.
// ---------------------------------------------------------------------------
template <int MT, int RS>
__device__ __forceinline__ void unit_q8_q4k(const uint8_t* __restrict__ sl, const uint8_t* __restrict__ xs, int M,
                                            float (&acc)[MT], bool five) {
  const uint4 hd = lds128(sl);
  const float d = h2f_lo(hd.x), dmin = h2f_hi(hd.x);
  const uint32_t scL = hd.y & 0x3F3F3F3Fu, mnL = hd.z & 0x3F3F3F3Fu;
  const uint32_t scH = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
  const uint32_t mnH = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
  // Q4_K keeps the high nibbles in place (x16): their scales carry 1/16.
  const float dh = five ? d : 0.0625f * d;
  const float nd = -8388608.0f * d, ndh = -8388608.0f * dh, nm = -8388608.0f * dmin;
  // A[j], B[j]: sub-block j's scale and min, in pairs (j even: d, odd: dh)
  const float2 dp = f2(d, dh), ndp = f2(nd, ndh), mp = f2(dmin, dmin), nmp = f2(nm, nm);
  float2 A[4], B[4];
  A[0] = scale_byte2<0>(dp, ndp, scL);
  A[1] = scale_byte2<2>(dp, ndp, scL);
  A[2] = scale_byte2<0>(dp, ndp, scH);
  A[3] = scale_byte2<2>(dp, ndp, scH);
  B[0] = scale_byte2<0>(mp, nmp, mnL);
  B[1] = scale_byte2<2>(mp, nmp, mnL);
  B[2] = scale_byte2<0>(mp, nmp, mnH);
  B[3] = scale_byte2<2>(mp, nmp, mnH);
  uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0;
  if (five) {
    h0 = lds128(sl + 16);
    h1 = lds128(sl + 32);
  }
  const uint8_t* qs = sl + (five ? 48 : 16);
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint4 q0 = lds128(qs + 32 * p), q1 = lds128(qs + 32 * p + 16);
    uint4 l0 = and4(q0, 0x0F0F0F0Fu), l1 = and4(q1, 0x0F0F0F0Fu), u0, u1;
    if (five) {
      l0 = or4(l0, mv4x4(h0, 2 * p, 0x10101010u));
      l1 = or4(l1, mv4x4(h1, 2 * p, 0x10101010u));
      u0 = or4(and4(shr4(q0, 4), 0x0F0F0F0Fu), mv4x4(h0, 2 * p + 1, 0x10101010u));
      u1 = or4(and4(shr4(q1, 4), 0x0F0F0F0Fu), mv4x4(h1, 2 * p + 1, 0x10101010u));
    } else {
      u0 = and4(q0, 0xF0F0F0F0u);
      u1 = and4(q1, 0xF0F0F0F0u);
    }
    // one token: its two sub-block dots and records
    auto dots = [&](int m, int& dl, int& du, float4& ra, float4& rb) {
      const uint8_t* xr = xs + m * RS;
      const uint4 x0 = lds128(xr + 64 * p), x1 = lds128(xr + 64 * p + 16);
      const uint4 x2 = lds128(xr + 64 * p + 32), x3 = lds128(xr + 64 * p + 48);
      ra = lds128f(xr + 256 + 32 * p);
      rb = lds128f(xr + 256 + 32 * p + 16);
      dl = dot16<false>(l1, x1, dot16<false>(l0, x0, 0));
      du = five ? dot16<false>(u1, x3, dot16<false>(u0, x2, 0)) : dot16<true>(u1, x3, dot16<true>(u0, x2, 0));
    };
    const float Al = A[p].x, Au = A[p].y, Bl = B[p].x, Bu = B[p].y;
    if (MT == 1) {
      int dl, du;
      float4 ra, rb;
      dots(0, dl, du, ra, rb);
      const float2 ar = mul2(A[p], f2(ra.x, rb.x));  // (Al * ra.x, Au * rb.x)
      float v = acc[0];
      v = fmaf(i2f(dl), ar.x, v);
      v = fmaf(-Bl, ra.y, v);
      v = fmaf(i2f(du), ar.y, v);
      v = fmaf(-Bu, rb.y, v);
      acc[0] = v;
    } else {
      // tokens in pairs: the same operations per token, two at a time (a
      // pass's unused second token reads stale records; its sum is dropped)
#pragma unroll
      for (int m = 0; m < MT; m += 2) {
        if (m < M) {
          int dl0, du0, dl1, du1;
          float4 ra0, rb0, ra1, rb1;
          dots(m, dl0, du0, ra0, rb0);
          dots(m + 1, dl1, du1, ra1, rb1);
          float2 v = f2(acc[m], acc[m + 1]);
          v = fma2(f2(i2f(dl0), i2f(dl1)), mul2(f2(Al, Al), f2(ra0.x, ra1.x)), v);
          v = fma2(f2(-Bl, -Bl), f2(ra0.y, ra1.y), v);
          v = fma2(f2(i2f(du0), i2f(du1)), mul2(f2(Au, Au), f2(rb0.x, rb1.x)), v);
          v = fma2(f2(-Bu, -Bu), f2(rb0.y, rb1.y), v);
          acc[m] = v.x;
          acc[m + 1] = v.y;
        }
      }
    }
  }
}

template <int MT, int RS>
__device__ __forceinline__ void unit_q8_q6k(const uint8_t* __restrict__ sl, float d, const uint8_t* __restrict__ xs,
                                            int M, float (&acc)[MT]) {
  const uint4 scv = lds128(sl);  // 16 int8 scales
  const uint32_t sw[4] = {scv.x ^ 0x80808080u, scv.y ^ 0x80808080u, scv.z ^ 0x80808080u, scv.w ^ 0x80808080u};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 qh0 = lds128(sl + 144 + 32 * h), qh1 = lds128(sl + 144 + 32 * h + 16);
#pragma unroll
    for (int cl = 0; cl < 2; ++cl) {
      const uint4 w0 = lds128(sl + 16 + 64 * h + 32 * cl), w1 = lds128(sl + 16 + 64 * h + 32 * cl + 16);
      // codes 0..63: low nibbles -> column group c = cl, high nibbles -> c = cl + 2
      const uint4 c0 = or4(and4(w0, 0x0F0F0F0Fu), mv4x4(qh0, 2 * cl, 0x30303030u));
      const uint4 c1 = or4(and4(w1, 0x0F0F0F0Fu), mv4x4(qh1, 2 * cl, 0x30303030u));
      const uint4 c2 = or4(and4(shr4(w0, 4), 0x0F0F0F0Fu), mv4x4(qh0, 2 * cl + 4, 0x30303030u));
      const uint4 c3 = or4(and4(shr4(w1, 4), 0x0F0F0F0Fu), mv4x4(qh1, 2 * cl + 4, 0x30303030u));
      const int sb = 8 * h + 2 * cl;  // sub-blocks sb, sb+1 (c0, c1) and sb+4, sb+5 (c2, c3)
      // scale d * sc with sc signed: the byte sc ^ 0x80 is sc + 128, so
      // magic - (2^23 + 128) is sc exactly
      // A01 = (A[0], A[1]) of sub-blocks sb, sb + 1, A23 of sb + 4, sb + 5
      float2 A01, A23;
      {
        const uint32_t w = sw[sb >> 2];
        const uint32_t w4 = sw[(sb + 4) >> 2];
        const int o = sb & 3;  // 0 or 2
        const float2 off = f2(-8388736.0f, -8388736.0f), dd = f2(d, d);
        const float2 a01 = __fadd2_rn(o == 0 ? f2(byte_magic<0>(w), byte_magic<1>(w))
                                             : f2(byte_magic<2>(w), byte_magic<3>(w)), off);
        const float2 a23 = __fadd2_rn(o == 0 ? f2(byte_magic<0>(w4), byte_magic<1>(w4))
                                             : f2(byte_magic<2>(w4), byte_magic<3>(w4)), off);
        A01 = mul2(dd, a01);
        A23 = mul2(dd, a23);
      }
      const float2 m32 = f2(-32.0f, -32.0f);
      const float2 N01 = mul2(m32, A01), N23 = mul2(m32, A23);  // -32 * A: the offset's factor
      // one token: its four integer dots and records
      auto dots = [&](int m, int (&dq)[4], float4& ra, float4& rb) {
        const uint8_t* xr = xs + m * RS;
        const int xo = 128 * h + 32 * cl;
        const uint4 x0 = lds128(xr + xo), x1 = lds128(xr + xo + 16);
        const uint4 x2 = lds128(xr + xo + 64), x3 = lds128(xr + xo + 80);
        ra = lds128f(xr + 256 + 16 * (4 * h + cl));
        rb = lds128f(xr + 256 + 16 * (4 * h + cl + 2));
        dq[0] = dot16<false>(c0, x0, 0);
        dq[1] = dot16<false>(c1, x1, 0);
        dq[2] = dot16<false>(c2, x2, 0);
        dq[3] = dot16<false>(c3, x3, 0);
      };
      if (MT == 1) {
        int dq[4];
        float4 ra, rb;
        dots(0, dq, ra, rb);
        const float2 Aa = mul2(A01, f2(ra.x, ra.x)), Ab = mul2(A23, f2(rb.x, rb.x));
        float v = acc[0];
        // (q - 32) . x: integer dot, then -32 * A * sum(x) in fp32
        v = fmaf(i2f(dq[0]), Aa.x, v);
        v = fmaf(N01.x, ra.z, v);
        v = fmaf(i2f(dq[1]), Aa.y, v);
        v = fmaf(N01.y, ra.w, v);
        v = fmaf(i2f(dq[2]), Ab.x, v);
        v = fmaf(N23.x, rb.z, v);
        v = fmaf(i2f(dq[3]), Ab.y, v);
        v = fmaf(N23.y, rb.w, v);
        acc[0] = v;
      } else {
#pragma unroll
        for (int m = 0; m < MT; m += 2) {
          if (m < M) {  // tokens in pairs (an unused second token's sum is dropped)
            int q0[4], q1[4];
            float4 ra0, rb0, ra1, rb1;
            dots(m, q0, ra0, rb0);
            dots(m + 1, q1, ra1, rb1);
            const float2 xa = f2(ra0.x, ra1.x), xb = f2(rb0.x, rb1.x);
            float2 v = f2(acc[m], acc[m + 1]);
            v = fma2(f2(i2f(q0[0]), i2f(q1[0])), mul2(f2(A01.x, A01.x), xa), v);
            v = fma2(f2(N01.x, N01.x), f2(ra0.z, ra1.z), v);
            v = fma2(f2(i2f(q0[1]), i2f(q1[1])), mul2(f2(A01.y, A01.y), xa), v);
            v = fma2(f2(N01.y, N01.y), f2(ra0.w, ra1.w), v);
            v = fma2(f2(i2f(q0[2]), i2f(q1[2])), mul2(f2(A23.x, A23.x), xb), v);
            v = fma2(f2(N23.x, N23.x), f2(rb0.z, rb1.z), v);
            v = fma2(f2(i2f(q0[3]), i2f(q1[3])), mul2(f2(A23.y, A23.y), xb), v);
            v = fma2(f2(N23.y, N23.y), f2(rb0.w, rb1.w), v);
            acc[m] = v.x;
            acc[m + 1] = v.y;
          }
        }
      }
    }
  }
}

template <int MT, int RS>
__device__ __forceinline__ void unit_q8_q8_0(const uint8_t* __restrict__ sl, const uint8_t* __restrict__ xs, int M,
                                             float (&acc)[MT]) {
  const uint4 dv = lds128(sl);
  const float dw[8] = {h2f_lo(dv.x), h2f_hi(dv.x), h2f_lo(dv.y), h2f_hi(dv.y),
                       h2f_lo(dv.z), h2f_hi(dv.z), h2f_lo(dv.w), h2f_hi(dv.w)};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 q0 = lds128(sl + 16 + 32 * j), q1 = lds128(sl + 32 + 32 * j);
    auto dot = [&](int m, float& dx) {
      const uint8_t* xr = xs + m * RS;
      const uint4 x0 = lds128(xr + 32 * j), x1 = lds128(xr + 32 * j + 16);
      dx = *reinterpret_cast<const float*>(xr + 256 + 16 * j);
      return dot16<false>(q1, x1, dot16<false>(q0, x0, 0));
    };
    if (MT == 1) {
      if (M > 0) {
        const uint8_t* xr = xs;
        const uint4 x0 = lds128(xr + 32 * j), x1 = lds128(xr + 32 * j + 16);
        const float dx = *reinterpret_cast<const float*>(xr + 256 + 16 * j);
        const int dd = dot16<false>(q1, x1, dot16<false>(q0, x0, 0));
        acc[0] = fmaf(i2f(dd), dw[j] * dx, acc[0]);
      }
    } else {
#pragma unroll
      for (int m = 0; m < MT; m += 2) {
        if (m < M) {  // tokens in pairs (an unused second token's sum is dropped)
          float dx0, dx1;
          const int d0 = dot(m, dx0), d1 = dot(m + 1, dx1);
          const float2 v = fma2(f2(i2f(d0), i2f(d1)), mul2(f2(dw[j], dw[j]), f2(dx0, dx1)), f2(acc[m], acc[m + 1]));
          acc[m] = v.x;
          acc[m + 1] = v.y;
        }
      }
    }
  }
}

template <int MT, int RS>
__device__ __forceinline__ void unit_q8_q4_0(const uint8_t* __restrict__ sl, const uint8_t* __restrict__ xs, int M,
                                             float (&acc)[MT]) {
  const uint4 dv = lds128(sl);
  const float dw[8] = {h2f_lo(dv.x), h2f_hi(dv.x), h2f_lo(dv.y), h2f_hi(dv.y),
                       h2f_lo(dv.z), h2f_hi(dv.z), h2f_lo(dv.w), h2f_hi(dv.w)};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 q = lds128(sl + 16 + 16 * j);
    const uint4 lo = and4(q, 0x0F0F0F0Fu), hi = and4(q, 0xF0F0F0F0u);  // hi kept x16
    // (q - 8) . x = lo . x0 + (hi . x1) / 16 - 8 * sum(x); the division is exact
    auto dot = [&](int m, float2& r) {
      const uint8_t* xr = xs + m * RS;
      const uint4 x0 = lds128(xr + 32 * j), x1 = lds128(xr + 32 * j + 16);
      r = *reinterpret_cast<const float2*>(xr + 256 + 16 * j);  // dx, sdx
      return dot16<false>(lo, x0, 0) + (dot16<true>(hi, x1, 0) >> 4);
    };
    if (MT == 1) {
      if (M > 0) {
        const uint8_t* xr = xs;
        const uint4 x0 = lds128(xr + 32 * j), x1 = lds128(xr + 32 * j + 16);
        const float2 r = *reinterpret_cast<const float2*>(xr + 256 + 16 * j);  // dx, sdx
        const int dd = dot16<false>(lo, x0, 0) + (dot16<true>(hi, x1, 0) >> 4);
        float v = fmaf(i2f(dd), dw[j] * r.x, acc[0]);
        acc[0] = fmaf(-8.0f * dw[j], r.y, v);
      }
    } else {
      const float n8 = -8.0f * dw[j];
#pragma unroll
      for (int m = 0; m < MT; m += 2) {
        if (m < M) {  // tokens in pairs (an unused second token's sum is dropped)
          float2 r0, r1;
          const int d0 = dot(m, r0), d1 = dot(m + 1, r1);
          float2 v = fma2(f2(i2f(d0), i2f(d1)), mul2(f2(dw[j], dw[j]), f2(r0.x, r1.x)), f2(acc[m], acc[m + 1]));
          v = fma2(f2(n8, n8), f2(r0.y, r1.y), v);
          acc[m] = v.x;
          acc[m + 1] = v.y;
        }
      }
    }
  }
}

// Bits 0..3 of h to bit 4 of bytes 0..3: the fifth bits of four 5-bit codes
// (the multiply places copies of h at bits 0, 7, 14, 21; no carries).
__device__ __forceinline__ uint32_t bit4_spread(uint32_t h) { return (((h & 0xFu) * 0x00204081u) << 4) & 0x10101010u; }
// The fifth bits of 16 codes: bits base..base+15 of a block's qh word.
__device__ __forceinline__ uint4 fifth_bits16(uint32_t qh, int base) {
  return make_uint4(bit4_spread(qh >> base), bit4_spread(qh >> (base + 4)), bit4_spread(qh >> (base + 8)),
                    bit4_spread(qh >> (base + 12)));
}

// Q4_1, Q5_0, Q5_1 (32-value blocks, cpu_backend.cpp:704-767): per block
// value = d * q + m (Q4_1, Q5_1) or d * (q - 16) (Q5_0), q the 4- or 5-bit
// code.  The integer dot of the codes with the int8 activations is exact;
// the min (or the -16 offset) folds into the block's sum of activation
// codes: sum((d q + m) x) = d dx sum(q xq) + m sdx.
template <int DT, int MT, int RS>
__device__ __forceinline__ void unit_q8_legacy(const uint8_t* __restrict__ sl, const uint8_t* __restrict__ xs,
                                               int M, float (&acc)[MT]) {
  constexpr bool FIVE = has_qh(DT), MIN = has_min(DT);
  const uint4 dv = lds128(sl);
  const float dw[8] = {h2f_lo(dv.x), h2f_hi(dv.x), h2f_lo(dv.y), h2f_hi(dv.y),
                       h2f_lo(dv.z), h2f_hi(dv.z), h2f_lo(dv.w), h2f_hi(dv.w)};
  float bw[8];  // the additive term per block: m, or -16 d
  if (MIN) {
    const uint4 mv = lds128(sl + sl_m(DT));
    const float t[8] = {h2f_lo(mv.x), h2f_hi(mv.x), h2f_lo(mv.y), h2f_hi(mv.y),
                        h2f_lo(mv.z), h2f_hi(mv.z), h2f_lo(mv.w), h2f_hi(mv.w)};
#pragma unroll
    for (int j = 0; j < 8; ++j) bw[j] = t[j];
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) bw[j] = -16.0f * dw[j];
  }
  uint32_t qhw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (FIVE) {
    const uint4 h0 = lds128(sl + sl_qh(DT)), h1 = lds128(sl + sl_qh(DT) + 16);
    qhw[0] = h0.x; qhw[1] = h0.y; qhw[2] = h0.z; qhw[3] = h0.w;
    qhw[4] = h1.x; qhw[5] = h1.y; qhw[6] = h1.z; qhw[7] = h1.w;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 q = lds128(sl + sl_qs(DT) + 16 * j);
    uint4 lo, hi;
    if (FIVE) {
      lo = or4(and4(q, 0x0F0F0F0Fu), fifth_bits16(qhw[j], 0));
      hi = or4(and4(shr4(q, 4), 0x0F0F0F0Fu), fifth_bits16(qhw[j], 16));
    } else {
      lo = and4(q, 0x0F0F0F0Fu);
      hi = and4(q, 0xF0F0F0F0u);  // kept x16
    }
    auto dot = [&](int m, float2& r) {
      const uint8_t* xr = xs + m * RS;
      const uint4 x0 = lds128(xr + 32 * j), x1 = lds128(xr + 32 * j + 16);
      r = *reinterpret_cast<const float2*>(xr + 256 + 16 * j);  // dx, sdx
      return FIVE ? dot16<false>(lo, x0, dot16<false>(hi, x1, 0))
                  : dot16<false>(lo, x0, 0) + (dot16<true>(hi, x1, 0) >> 4);  // exact division
    };
    if (MT == 1) {
      if (M > 0) {
        const uint8_t* xr = xs;
        const uint4 x0 = lds128(xr + 32 * j), x1 = lds128(xr + 32 * j + 16);
        const float2 r = *reinterpret_cast<const float2*>(xr + 256 + 16 * j);  // dx, sdx
        const int dd = FIVE ? dot16<false>(lo, x0, dot16<false>(hi, x1, 0))
                            : dot16<false>(lo, x0, 0) + (dot16<true>(hi, x1, 0) >> 4);  // exact division
        float v = fmaf(i2f(dd), dw[j] * r.x, acc[0]);
        acc[0] = fmaf(bw[j], r.y, v);
      }
    } else {
#pragma unroll
      for (int m = 0; m < MT; m += 2) {
        if (m < M) {  // tokens in pairs (an unused second token's sum is dropped)
          float2 r0, r1;
          const int d0 = dot(m, r0), d1 = dot(m + 1, r1);
          float2 v = fma2(f2(i2f(d0), i2f(d1)), mul2(f2(dw[j], dw[j]), f2(r0.x, r1.x)), f2(acc[m], acc[m + 1]));
          v = fma2(f2(bw[j], bw[j]), f2(r0.y, r1.y), v);
          acc[m] = v.x;
          acc[m + 1] = v.y;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// ACT_F32 units: 16 groups of 16 columns; value = A * code - B with integer
// codes widened to fp32 exactly, then fp32 FMA against fp32 activations.
// ---------------------------------------------------------------------------
struct Group16 {
  uint4 cw;  // 16 byte codes
  float A, B;
};

template <int DT>
__device__ __forceinline__ Group16 group16(const uint8_t* __restrict__ sl, float tail_d, int g) {
  Group16 G;
  if (DT == Q4_K || DT == Q5_K) {
    const int j = g >> 1, half = g & 1;  // sub-block j, 16-value half
    const uint4 hd = lds128(sl);
    const float d = h2f_lo(hd.x), dmin = h2f_hi(hd.x);
    const uint8_t* s = sl + 4;
    int sc, mn;
    if (j < 4) {
      sc = s[j] & 63;
      mn = s[j + 4] & 63;
    } else {
      sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
      mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    G.A = d * (float)sc;
    G.B = dmin * (float)mn;
    const uint8_t* qs = sl + (DT == Q5_K ? 48 : 16) + 32 * (j >> 1) + 16 * half;
    const uint4 q = lds128(qs);
    G.cw = (j & 1) ? and4(shr4(q, 4), 0x0F0F0F0Fu) : and4(q, 0x0F0F0F0Fu);
    if (DT == Q5_K) G.cw = or4(G.cw, mv4x4(lds128(sl + 16 + 16 * half), j, 0x10101010u));
  } else if (DT == Q6_K) {
    // group g = 16 columns [16g, 16g+16): h = g/8, c = (g/2)&3, l0 = 16*(g&1)
    const int h = g >> 3, c = (g >> 1) & 3, l0 = 16 * (g & 1);
    const uint4 w = lds128(sl + 16 + 64 * h + 32 * (c & 1) + l0);
    const uint4 qh = lds128(sl + 144 + 32 * h + l0);
    G.cw = or4(and4(shr4(w, 4 * (c >> 1)), 0x0F0F0F0Fu), mv4x4(qh, 2 * c, 0x30303030u));
    G.A = tail_d * (float)(int)(signed char)sl[g];
    G.B = 32.0f * G.A;
  } else if (DT == Q8_0) {
    const int j = g >> 1;
    G.cw = lds128(sl + 16 + 16 * g);
    G.A = h2f((uint16_t)ldsu16(sl + 2 * j));
    G.B = 0.0f;
  } else if (DT == Q4_1 || DT == Q5_0 || DT == Q5_1) {
    // block j = g/2: low nibbles = values 0..15, high = 16..31; value = A q - B
    const int j = g >> 1;
    const uint4 q = lds128(sl + sl_qs(DT) + 16 * j);
    G.cw = (g & 1) ? and4(shr4(q, 4), 0x0F0F0F0Fu) : and4(q, 0x0F0F0F0Fu);
    if (has_qh(DT))
      G.cw = or4(G.cw, fifth_bits16(*reinterpret_cast<const uint32_t*>(sl + sl_qh(DT) + 4 * j), 16 * (g & 1)));
    G.A = h2f((uint16_t)ldsu16(sl + 2 * j));
    G.B = DT == Q5_0 ? 16.0f * G.A : -h2f((uint16_t)ldsu16(sl + sl_m(DT) + 2 * j));
  } else {  // Q4_0: block j = g/2; low nibbles = values 0..15, high = 16..31
    const int j = g >> 1;
    const uint4 q = lds128(sl + 16 + 16 * j);
    G.cw = (g & 1) ? and4(shr4(q, 4), 0x0F0F0F0Fu) : and4(q, 0x0F0F0F0Fu);
    G.A = h2f((uint16_t)ldsu16(sl + 2 * j));
    G.B = 8.0f * G.A;
  }
  return G;
}

template <int DT>
__device__ __forceinline__ float dot16_f32(uint4 cw, const uint8_t* __restrict__ x) {
  // Q8_0 codes are signed: flip to q + 128 and remove that bias too.
  constexpr float bias = DT == Q8_0 ? 8388608.0f + 128.0f : 8388608.0f;
  const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
  float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t c = DT == Q8_0 ? (w[i] ^ 0x80808080u) : w[i];
    const float4 xv = lds128f(x + 16 * i);
    s0 = fmaf(xv.x, byte_magic<0>(c) - bias, s0);
    s1 = fmaf(xv.y, byte_magic<1>(c) - bias, s1);
    s0 = fmaf(xv.z, byte_magic<2>(c) - bias, s0);
    s1 = fmaf(xv.w, byte_magic<3>(c) - bias, s1);
  }
  return s0 + s1;
}

template <int DT, int MT>
__device__ __forceinline__ void unit_f32(const uint8_t* __restrict__ sl, float tail_d, const uint8_t* __restrict__ xs,
                                         int M, float (&acc)[MT]) {
#pragma unroll 2
  for (int g = 0; g < 16; ++g) {
    const Group16 G = group16<DT>(sl, tail_d, g);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < M) {
        const uint8_t* xr = xs + m * stage_stride(false, MT);
        float v = fmaf(G.A, dot16_f32<DT>(G.cw, xr + 64 * g), acc[m]);
        if (DT != Q8_0) v = fmaf(-G.B, reinterpret_cast<const float*>(xr + XR_VALS)[g], v);
        acc[m] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core units for a pass of 8 tokens (MT = 8, ACT_Q8).  At 8 tokens the
// dp4a units issue about 8x the M = 1 work per weight byte and the GEMV is
// instruction-bound; here the integer dot products of a warp's 32 rows run as
// mma.sync (m16n8k32 s8, m16n8k16 for Q6_K's 16-value scales), the tokens
// being the n = 8 columns, and the CUDA cores only unpack the codes and apply
// the per-(row, block, token) scales, which the format makes unavoidable (so
// tcgen05's larger tiles would not shorten this path).  Thread (g = lane / 4,
// t = lane % 4) holds rows g and g + 8 of each 16-row tile and tokens 2t and
// 2t + 1: acc[4 * mt + 2 * h + e] is unit row 32 * half + 16 * mt + 8 * h + g,
// token 2t + e.  The integer sums are exact and each block's scaling and
// accumulation follow the dp4a units' operations in the same order, so the
// results equal the dp4a path's.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%7, %7, %7, %7};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lo_nib(uint32_t w) { return w & 0x0F0F0F0Fu; }
__device__ __forceinline__ uint32_t hi_nib(uint32_t w) { return (w >> 4) & 0x0F0F0F0Fu; }
// d * (byte b of w), b known after unrolling: scale_byte with a run-time index
__device__ __forceinline__ float scale_byte_rt(float d, float nd23, uint32_t w, int b) {
  return fmaf(d, __int_as_float(__byte_perm(w, 0x4Bu, 0x4550u | b)), nd23);
}
// acc += D * (A_row * dx_token) [- C_row * sdx_token], the four elements of a
// tile, in the dp4a units' order of operations; the two tokens of a row as
// one packed pair
template <bool MIN>
__device__ __forceinline__ void tc_apply(float* acc, const int (&d)[4], float A0, float A1, float C0, float C1,
                                         float dx0, float dx1, float s0, float s1) {
  const float2 dx = f2(dx0, dx1), sx = f2(s0, s1);
  float2 v0 = fma2(f2(i2f(d[0]), i2f(d[1])), mul2(f2(A0, A0), dx), f2(acc[0], acc[1]));
  float2 v1 = fma2(f2(i2f(d[2]), i2f(d[3])), mul2(f2(A1, A1), dx), f2(acc[2], acc[3]));
  if (MIN) {
    v0 = fma2(f2(-C0, -C0), sx, v0);
    v1 = fma2(f2(-C1, -C1), sx, v1);
  }
  acc[0] = v0.x;
  acc[1] = v0.y;
  acc[2] = v1.x;
  acc[3] = v1.y;
}

// Q4_K / Q5_K header of one row (the unpacking of unit_q8_q4k): d, dmin and
// the 6-bit scales and mins as bytes.
struct KHead {
  float d, dmin, nd, nm;  // nd, nm: -2^23 d, -2^23 dmin for scale_byte
  uint32_t scL, mnL, scH, mnH;
};
__device__ __forceinline__ KHead khead(const uint8_t* sl) {
  const uint4 hd = lds128(sl);
  KHead h;
  h.d = h2f_lo(hd.x);
  h.dmin = h2f_hi(hd.x);
  h.nd = -8388608.0f * h.d;
  h.nm = -8388608.0f * h.dmin;
  h.scL = hd.y & 0x3F3F3F3Fu;
  h.mnL = hd.z & 0x3F3F3F3Fu;
  h.scH = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
  h.mnH = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
  return h;
}

template <int DT, int RS>
__device__ __forceinline__ void unit_tc(const uint8_t* __restrict__ st, int half, const uint8_t* __restrict__ xs,
                                        float (&acc)[8]) {
  constexpr int SB = slice_bytes(DT);
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint8_t* xg = xs + g * RS;                                // token g's codes (B fragments)
  const uint8_t* xr0 = xs + (2 * t) * RS + 256, *xr1 = xr0 + RS;  // tokens 2t, 2t+1: XRec per block
  const uint8_t* sl[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    sl[mt][0] = st + (32 * half + 16 * mt + g) * SB;
    sl[mt][1] = sl[mt][0] + 8 * SB;
  }
  if constexpr (DT == Q4_K || DT == Q5_K) {
    constexpr bool FIVE = DT == Q5_K;
    constexpr int QS = FIVE ? 48 : 16;
    KHead hd[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) hd[mt][h] = khead(sl[mt][h]);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      // codes of blocks 2p (low nibbles) and 2p + 1 (high): bytes 4t.. and 16 + 4t..
      uint32_t w[2][2][2], q5[2][2][2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            w[mt][h][u] = lds32(sl[mt][h] + QS + 32 * p + 16 * u + 4 * t);
            if (FIVE) q5[mt][h][u] = lds32(sl[mt][h] + 16 + 16 * u + 4 * t);
          }
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int j = 2 * p + hi;
        const uint32_t b0 = lds32(xg + 32 * j + 4 * t), b1 = lds32(xg + 32 * j + 16 + 4 * t);
        const float4 r0 = lds128f(xr0 + 16 * j), r1 = lds128f(xr1 + 16 * j);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t a[2][2];
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              a[h][u] = hi ? hi_nib(w[mt][h][u]) : lo_nib(w[mt][h][u]);
              if (FIVE) a[h][u] |= ((q5[mt][h][u] >> j) & 0x01010101u) << 4;
            }
          int d[4];
          mma_k32(d, a[0][0], a[1][0], a[0][1], a[1][1], b0, b1);
          // the scale and min of block j for rows g and g + 8, as pairs
          const KHead& k0 = hd[mt][0];
          const KHead& k1 = hd[mt][1];
          auto mag = [&](uint32_t w) { return __int_as_float(__byte_perm(w, 0x4Bu, 0x4550u | (j & 3))); };
          const float2 A = fma2(f2(k0.d, k1.d), f2(mag(j < 4 ? k0.scL : k0.scH), mag(j < 4 ? k1.scL : k1.scH)),
                                f2(k0.nd, k1.nd));
          const float2 C = fma2(f2(k0.dmin, k1.dmin), f2(mag(j < 4 ? k0.mnL : k0.mnH), mag(j < 4 ? k1.mnL : k1.mnH)),
                                f2(k0.nm, k1.nm));
          tc_apply<true>(acc + 4 * mt, d, A.x, A.y, C.x, C.y, r0.x, r1.x, r0.y, r1.y);
        }
      }
    }
  } else if constexpr (DT == Q8_0 || DT == Q4_0) {
    // value = d_j * q (Q8_0) or d_j * (q - 8) (Q4_0: the -8 folds into sdx)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t b0 = lds32(xg + 32 * j + 4 * t), b1 = lds32(xg + 32 * j + 16 + 4 * t);
      const float4 r0 = lds128f(xr0 + 16 * j), r1 = lds128f(xr1 + 16 * j);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t a[2][2];
        float A[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          A[h] = h2f((uint16_t)ldsu16(sl[mt][h] + 2 * j));
          if (DT == Q8_0) {
            a[h][0] = lds32(sl[mt][h] + 16 + 32 * j + 4 * t);
            a[h][1] = lds32(sl[mt][h] + 16 + 32 * j + 16 + 4 * t);
          } else {  // byte l: value l (low nibble), value l + 16 (high)
            const uint32_t q = lds32(sl[mt][h] + 16 + 16 * j + 4 * t);
            a[h][0] = lo_nib(q);
            a[h][1] = hi_nib(q);
          }
        }
        int d[4];
        mma_k32(d, a[0][0], a[1][0], a[0][1], a[1][1], b0, b1);
        tc_apply<DT == Q4_0>(acc + 4 * mt, d, A[0], A[1], 8.0f * A[0], 8.0f * A[1], r0.x, r1.x, r0.y, r1.y);
      }
    }
  } else {  // Q6_K: value = (d * sc) * (q - 32), q 6-bit, one int8 scale per 16 values
    float dd[2][2];
    uint4 scw[2][2];  // the row's 16 int8 scales, each byte + 128 (x ^ 0x80)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        dd[mt][h] = h2f((uint16_t)ldsu16(st + UNIT_ROWS * 208 + 2 * (32 * half + 16 * mt + 8 * h + g)));
        const uint4 v = lds128(sl[mt][h]);
        scw[mt][h] = make_uint4(v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u);
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c = (cc >> 1) | ((cc & 1) << 1);  // 0, 2, 1, 3: the dp4a unit's order
        // column group c of half hh: 32 values, block j = 4 hh + c of the span;
        // low nibbles of ql[64 hh + 32 (c & 1) + l] for c < 2, high for c >= 2,
        // bits 2c..2c+1 of qh[32 hh + l] on top
        const int j = 4 * hh + c;
        const uint32_t b0 = lds32(xg + 32 * j + 4 * t), b1 = lds32(xg + 32 * j + 16 + 4 * t);
        const float4 r0 = lds128f(xr0 + 16 * j), r1 = lds128f(xr1 + 16 * j);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t a[2][2];
          float A[2][2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint8_t* s6 = sl[mt][h];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint32_t ql = lds32(s6 + 16 + 64 * hh + 32 * (c & 1) + 16 * u + 4 * t);
              const uint32_t qh = lds32(s6 + 144 + 32 * hh + 16 * u + 4 * t);
              a[h][u] = (c < 2 ? lo_nib(ql) : hi_nib(ql)) | (((qh >> (2 * c)) & 0x03030303u) << 4);
              const int si = 2 * j + u;  // scale of values 16u..16u+15 of the block
              const uint32_t sw = si < 4 ? scw[mt][h].x : si < 8 ? scw[mt][h].y : si < 12 ? scw[mt][h].z : scw[mt][h].w;
              A[h][u] = dd[mt][h] * (__int_as_float(__byte_perm(sw, 0x4Bu, 0x4550u | (si & 3))) - 8388736.0f);
            }
          }
          int d0[4], d1[4];
          mma_k16(d0, a[0][0], a[1][0], b0);  // values 0..15 of the block
          mma_k16(d1, a[0][1], a[1][1], b1);  // values 16..31
          // per element: values 0..15 with their scale and -32 * sum, then
          // 16..31; row h's two tokens as one packed pair
          float* ac = acc + 4 * mt;
          const float2 dx = f2(r0.x, r1.x), slo = f2(r0.z, r1.z), shi = f2(r0.w, r1.w);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float n0 = -32.0f * A[h][0], n1 = -32.0f * A[h][1];
            float2 v = fma2(f2(i2f(d0[2 * h]), i2f(d0[2 * h + 1])), mul2(f2(A[h][0], A[h][0]), dx),
                            f2(ac[2 * h], ac[2 * h + 1]));
            v = fma2(f2(n0, n0), slo, v);
            v = fma2(f2(i2f(d1[2 * h]), i2f(d1[2 * h + 1])), mul2(f2(A[h][1], A[h][1]), dx), v);
            v = fma2(f2(n1, n1), shi, v);
            ac[2 * h] = v.x;
            ac[2 * h + 1] = v.y;
          }
        }
      }
    }
  }
}

template <int DT, int MT, bool F32, int RS>
__device__ __forceinline__ void unit(const uint8_t* __restrict__ st, int row, const uint8_t* __restrict__ xs, int M,
                                     float (&acc)[MT]) {
  const uint8_t* sl = st + row * slice_bytes(DT);
  const float tail_d = DT == Q6_K ? h2f((uint16_t)ldsu16(st + UNIT_ROWS * 208 + 2 * row)) : 0.0f;
  if (F32) {
    unit_f32<DT, MT>(sl, tail_d, xs, M, acc);
  } else if (DT == Q4_K) {
    unit_q8_q4k<MT, RS>(sl, xs, M, acc, false);
  } else if (DT == Q5_K) {
    unit_q8_q4k<MT, RS>(sl, xs, M, acc, true);
  } else if (DT == Q6_K) {
    unit_q8_q6k<MT, RS>(sl, tail_d, xs, M, acc);
  } else if (DT == Q8_0) {
    unit_q8_q8_0<MT, RS>(sl, xs, M, acc);
  } else if (DT == Q4_1 || DT == Q5_0 || DT == Q5_1) {
    unit_q8_legacy<DT, MT, RS>(sl, xs, M, acc);
  } else {
    unit_q8_q4_0<MT, RS>(sl, xs, M, acc);
  }
}

// ---------------------------------------------------------------------------
// Cluster helpers (distributed shared memory).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, int rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  return remote;
}
// Asynchronous store into another CTA's shared memory whose completion is
// counted, in bytes, on that CTA's mbarrier (complete-tx): the receiver
// waits on the barrier; the sender needs no fence and no arrival.
__device__ __forceinline__ void st_async_v4(uint32_t remote, float4 v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(remote),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(remote_bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (clock64() - t0 > WAIT_BUDGET_CYCLES) {
      if (err) atomicOr(err, code);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Shared-memory layout of one CTA (offsets in bytes; the host plan holds
// xr_off and ring_off):
//   [0, 512)                mbarriers full[16], empty[16]
//   [512, 520)              reduction mbarrier
//   red   [2][64][MT] fp32  (one-token passes) the two unit-parity sums of
//                           each row
//   part  partials received over distributed shared memory:
//         [C][MT][64] fp32  rank 0 gathers the other ranks' tiles, or
//         [C][MT][64/C]     with the reduce-scatter (pl.rs), every rank the
//                           C partials of its own 64/C rows
//   xr    chunk x MT records of stage_stride(PRE, MT) bytes
//         bytes: staged activations
//   ring  stages x stage_bytes weight units
// Multi-token passes write the two unit-parity sums of each row ([64][MT]
// fp32 each) into ring slots 0 and 1 instead, after a barrier of all
// consumers: every unit has been consumed, so nothing lands there or is read
// there after it (4 KB less shared memory at 8 tokens).
template <int MT>
struct SmemMap {
  static constexpr bool red_in_ring = MT >= 2;
  static constexpr int redbar = 512;
  static constexpr int xbar = 520;  // the consumers' "activation loads issued" barrier
  static constexpr int fuse = 768;  // GemvFuse scratch: rms[MT], partial sums[4][MT]
  static constexpr int red = BAR_BYTES;
  static constexpr int part = red + (red_in_ring ? 0 : 2 * UNIT_ROWS * MT * 4);
  static constexpr int xr(int C, bool rs) {
    return (part + (rs ? 1 : C) * UNIT_ROWS * MT * 4 + 127) / 128 * 128;
  }
};

// One output element: to y, or -- for a row shard -- to every rank's gathered
// buffer (plain stores; peers' buffers are reached over NVLink).
__device__ __forceinline__ float store_out(const GemvArgs& a, int m, int64_t n, float v) {
  if (a.sc.n == 0) {
    float* p = a.y + (int64_t)m * a.N + n;
    const float nv = a.fu.accumulate ? *p + v : v;
    *p = nv;
    return nv;
  }
  const int64_t off = (int64_t)m * a.sc.ld + a.sc.row0 + n;
  for (int p = 0; p < a.sc.n; ++p) a.sc.out[p][off] = v;
  return v;
}

// ssq_out: the squares of this tile's stored values were left at buf[r*rs +
// m*ms]; one thread per token adds the 64 rows in order into slot g.
__device__ __forceinline__ void write_ssq(const GemvArgs& a, const float* buf, int rs, int ms, int g, int G) {
  const int tid = threadIdx.x;
  if (tid < a.M) {
    float s = 0.f;
    for (int r = 0; r < UNIT_ROWS; ++r) s += buf[r * rs + tid * ms];
    a.fu.ssq_out[(int64_t)tid * G + g] = s;
  }
}

// The tile's stored y (fin[r * MT + m]) as records for the next product:
// one warp per 32-row block, lane = row (fu.rec_out).
__device__ __forceinline__ void write_records(const GemvArgs& a, const float* fin, int MTs, int g) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (!a.fu.rec_swiglu) {
    for (int b = warp; b < 2 * a.M; b += NCW) {
      const int m = b >> 1, r = 32 * (b & 1) + lane;
      const int64_t n = (int64_t)g * UNIT_ROWS + r;
      float u = n < a.N ? fin[r * MTs + m] : 0.f;
      if (a.fu.rec_norm_w && n < a.N) u = u * a.fu.rec_norm_w[n];
      q8_block_to_record(u, lane, a.fu.rec_out + ((n >> 8) * a.fu.rec_out_ld + m) * Q8_REC_BYTES,
                         (int)((n & 255) >> 5));
    }
  } else {
    // rows 0-31 of the tile are gate rows, 32-63 the matching up rows: one
    // block of the SwiGLU output, columns 32g .. 32g + 31
    for (int m = warp; m < a.M; m += NCW) {
      const float v = silu_f(fin[lane * MTs + m]) * fin[(32 + lane) * MTs + m];
      const int64_t n = (int64_t)g * 32 + lane;
      q8_block_to_record(v, lane, a.fu.rec_out + ((n >> 8) * a.fu.rec_out_ld + m) * Q8_REC_BYTES,
                         (int)((n & 255) >> 5));
    }
  }
}

// After this CTA's output stores (consumer_sync between), one thread per
// writing CTA: the CTA's stores are ordered before its arrival on the
// launch's local completion count (GPU scope); the last of the
// sc.writers writing CTAs then makes every observed store visible
// system-wide, resets the count for the next launch and adds one arrival to
// this rank's counter on every rank (release, system scope) -- one remote
// signal per launch, not one per CTA.
__device__ __forceinline__ void signal_peers(const GemvArgs& a) {
  if (a.sc.n == 0) return;
  __threadfence();
  const unsigned prev = atomicAdd(a.sc.done, 1u);
  if (prev != (unsigned)a.sc.writers - 1) return;
  __threadfence_system();
  *a.sc.done = 0u;
  for (int p = 0; p < a.sc.n; ++p)
    asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(a.sc.cnt[p] + a.sc.src) : "memory");
}

// ---------------------------------------------------------------------------
// The kernel: grid = G * C CTAs, clusters of C along x.
// ---------------------------------------------------------------------------
template <int DT, int MT, bool F32, bool PRE>
__global__ void __launch_bounds__(NTHREADS, CTAS_PER_SM) qgemv_kernel(const GemvArgs a, const GemvPlan pl) {
  constexpr int RS = stage_stride(PRE, MT);  // bytes per staged (span, token) record
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* redbar = reinterpret_cast<uint64_t*>(smem + SmemMap<MT>::redbar);
  uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + SmemMap<MT>::xbar);
  float* part = reinterpret_cast<float*>(smem + SmemMap<MT>::part);
  uint8_t* xr = smem + SmemMap<MT>::xr(pl.C, pl.rs);
  uint8_t* ring = xr + pl.xq_bytes;
  constexpr int UB = unit_bytes(DT);
  const int S = pl.stages, SB = pl.stage_bytes;
  // the unit-parity row sums, [64][MT] each: their own region, or ring slots
  // 0 and 1 (multi-token passes)
  float* const red0 = SmemMap<MT>::red_in_ring ? reinterpret_cast<float*>(ring)
                                                : reinterpret_cast<float*>(smem + SmemMap<MT>::red);
  float* const red1 = SmemMap<MT>::red_in_ring ? reinterpret_cast<float*>(ring + SB) : red0 + UNIT_ROWS * MT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x / pl.C, rank = blockIdx.x - g * pl.C;
  const int kb0 = rank * pl.chunk;
  const int nsp = min(pl.KB, kb0 + pl.chunk) - kb0;  // >= 1 by construction of the plan
  const uint8_t* wsrc = a.w + ((int64_t)g * pl.KB + kb0) * UB;
#ifdef ODI_GEMV_CHECKS
  if (threadIdx.x == 0) {
    uint32_t hw_rank = 0, hw_n = 1;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(hw_rank));
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(hw_n));
    GCHK(g < pl.G && rank < pl.C && nsp >= 1 && kb0 + nsp <= pl.KB, 1, blockIdx.x, nsp);
    GCHK((int)hw_rank == rank, 2, hw_rank, rank);
    GCHK((int)hw_n == pl.C, 3, hw_n, pl.C);
    GCHK(S >= 2 && S <= MAX_STAGES && (S & 1) == 0 && (ring - smem) + S * SB <= pl.smem_bytes, 4, S,
         (ring - smem) + S * SB);
    GCHK((xr - smem) + nsp * MT * RS <= (ring - smem), 5, nsp, pl.xq_bytes);
  }
#endif

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);  // the two warps of a unit-parity pair
    }
    // Rank 0's reduction barrier: its one arrival is rank 0's own expect-tx
    // of the other ranks' partials (64 rows x M tokens fp32 each), which
    // their st.async pushes count down as they land.
    if (pl.C > 1) mbar_init(redbar, 1);
    mbar_init(xbar, NCW);  // one arrival per consumer warp
    fence_mbar_init();
    if (MT >= 2 && pl.rs)  // every rank receives the other ranks' partials of its 64/C rows
      mbar_arrive_expect_tx(redbar, (uint32_t)((pl.C - 1) * (UNIT_ROWS / pl.C) * a.M * 4));
    else if (pl.C > 1 && rank == 0)
      mbar_arrive_expect_tx(redbar, (uint32_t)((pl.C - 1) * UNIT_ROWS * a.M * 4));
  }
  __syncthreads();
  // Cluster barrier, split: arrive now, wait only before the first remote
  // access (rank 0's reduction mbarrier is initialised before its arrive).
  if (pl.C > 1) cluster_arrive();

  if (warp == NCW) {
    // ---------------- producer: weights only, no dependency on earlier kernels
    if (lane != 0 && a.fu.norm_w) {
      // the RMSNorm weights are constant too: into L2 for the prologue
      const int64_t k0 = (int64_t)kb0 * UNIT_COLS;
      const int64_t kn = min((int64_t)a.K, k0 + (int64_t)nsp * UNIT_COLS);
      for (int64_t k = k0 + 32 * (lane - 1); k < kn; k += 32 * 31)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.fu.norm_w + k));
    }
    if (lane == 0) {
      pdl_launch_dependents();
      const int first = nsp < S ? nsp : S;
      const int early = (PRE || first < EARLY_STAGES) ? first : EARLY_STAGES;
      for (int i = 0; i < first; ++i) {
        // stages past the early ones once the activation loads are issued
        // (a wait that gives up is recorded, and the copies still go out)
        if (i == early) mbar_wait(xbar, 0, a.err, ERR_EMPTY_WAIT);
        mbar_arrive_expect_tx(&full[i], UB);
        bulk_g2s(ring + i * SB, wsrc + (int64_t)i * UB, UB, &full[i]);
      }
      int s = first % S;
      uint32_t par = 0;
      int i = first;
      for (; i < nsp; ++i) {
        if (s == 0) par = (uint32_t)(((i / S) - 1) & 1);
        if (!mbar_wait(&empty[s], par, a.err, ERR_EMPTY_WAIT)) break;
        if (!GCHK(s < S && (int64_t)g * pl.KB + kb0 + i < (int64_t)pl.G * pl.KB, 6, s, i)) break;
        mbar_arrive_expect_tx(&full[s], UB);
        bulk_g2s(ring + s * SB, wsrc + (int64_t)i * UB, UB, &full[s]);
        if (i + S < nsp) bulk_prefetch_l2(wsrc + (int64_t)(i + S) * UB, UB);  // the L2 lookahead
        if (++s == S) s = 0;
      }
      // Drain: every copy issued must land before the CTA may exit.
      for (int t = 0; t < S && t < i; ++t) {
        const int last = t + S * ((i - 1 - t) / S);
        mbar_wait(&full[t], (last / S) & 1, a.err, ERR_DRAIN_WAIT);
      }
    }
    __syncwarp();
    if (pl.C > 1) cluster_wait();
    return;
  }

  // ---------------- consumers
  pdl_wait();  // x is written by earlier kernels on the stream; y may be read by them
  if (PRE)
    stage_records<MT>(a, kb0, nsp, xr, reinterpret_cast<float*>(smem + SmemMap<MT>::fuse), xbar);
  else
    stage_acts<F32, MT>(a, kb0, nsp, xr, reinterpret_cast<float*>(smem + SmemMap<MT>::fuse), xbar);
  // L2 lookahead: the ring holds units 0..S-1; ask L2 for units S..2S-1 now
  // that the activations are staged (asked for earlier, these bytes queue
  // ahead of the activation loads and delay them), so HBM streams them while
  // the first units are consumed.  The producer keeps the lookahead S units
  // ahead of each refill.
  if (threadIdx.x == 0 && nsp > S) bulk_prefetch_l2(wsrc + (int64_t)S * UB, (uint32_t)(min(nsp, 2 * S) - S) * UB);

  const int row = 32 * (warp & 1) + lane;
  const int up = warp >> 1;  // this warp takes units j = up, up + 2, ...
  // 8-token passes of the five main types run their dot products on mma.sync
  constexpr bool TC = !F32 && MT == 8 && (DT == Q4_K || DT == Q5_K || DT == Q6_K || DT == Q8_0 || DT == Q4_0);
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.0f;

  int s = up;  // slot of unit j (S is even: each pair owns the slots of its parity)
  uint32_t par = 0u;
  for (int j = up; j < nsp; j += 2) {
    if (!mbar_wait(&full[s], par, a.err, ERR_FULL_WAIT)) break;
    if (!GCHK(s >= 0 && s < S && j < nsp, 7, s, j)) break;
    if constexpr (TC)
      unit_tc<DT, RS>(ring + s * SB, warp & 1, xr + j * MT * RS, acc);
    else
      unit<DT, MT, F32, RS>(ring + s * SB, row, xr + j * MT * RS, a.M, acc);
    fence_proxy_async_smem();  // this lane's reads of the slot before its refill
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    s += 2;
    if (s >= S) {
      s -= S;
      par ^= 1u;
    }
  }

  // Tile reduction: unit parities (fixed order) -> CTA partial -> ranks (fixed
  // order).  Partials travel as asynchronous float4 stores into the
  // receiver's shared memory, counted on its reduction mbarrier.  Plain
  // multi-token passes (pl.rs) reduce-scatter: rank j receives the C partials
  // of rows [j 64/C, (j+1) 64/C), adds them in rank order and writes those
  // rows.  Otherwise ranks other than 0 push their whole partial to rank 0,
  // which adds in rank order and writes y -- the same sums either way.
  // Ring slots 0 and 1 are free once every consumer is past its last unit
  // (the two warps of a pair share their slots: the barrier keeps one warp's
  // sums off rows its partner may still be reading).
  if (SmemMap<MT>::red_in_ring) consumer_sync();
  float* const redu = up ? red1 : red0;
  if constexpr (TC) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // row 32 (warp & 1) + 16 (i >> 2) + 8 ((i >> 1) & 1) + g, token 2t + (i & 1)
      const int r = 32 * (warp & 1) + 16 * (i >> 2) + 8 * ((i >> 1) & 1) + (lane >> 2), m = 2 * (lane & 3) + (i & 1);
      if (m < a.M) redu[r * MT + m] = acc[i];
    }
  } else {
#pragma unroll
    for (int m = 0; m < MT; ++m)
      if (m < a.M) redu[row * MT + m] = acc[m];
  }
  consumer_sync();
  const int tid = threadIdx.x;
  if (pl.C > 1) cluster_wait();
  if (MT >= 2 && pl.rs) {  // (one-token passes never reduce-scatter: compiled out)
    const int RB = UNIT_ROWS / pl.C, R4 = RB / 4;  // rows per rank; float4s per (rank, token)
    for (int u = tid; u < pl.C * a.M * R4; u += NCW * 32) {
      const int q = u / (a.M * R4), rem = u - q * a.M * R4, m = rem / R4, rq = 4 * (rem - m * R4);
      const int r0 = q * RB + rq;
      float4 v;
      v.x = red0[r0 * MT + m] + red1[r0 * MT + m];
      v.y = red0[(r0 + 1) * MT + m] + red1[(r0 + 1) * MT + m];
      v.z = red0[(r0 + 2) * MT + m] + red1[(r0 + 2) * MT + m];
      v.w = red0[(r0 + 3) * MT + m] + red1[(r0 + 3) * MT + m];
      float* dst = part + (rank * MT + m) * RB + rq;  // slot `rank` of rank q's part
      if (q == rank)
        *reinterpret_cast<float4*>(dst) = v;
      else
        st_async_v4(dsmem_addr(dst, q), v, dsmem_addr(redbar, q));
    }
    mbar_wait_cluster(redbar, 0, a.err, ERR_REDUCE_WAIT);
    consumer_sync();  // this rank's own slot, written by other threads
    for (int t = tid; t < a.M * RB; t += NCW * 32) {
      const int m = t / RB, r = t - m * RB;
      float v = part[m * RB + r];
      for (int q = 1; q < pl.C; ++q) v += part[(q * MT + m) * RB + r];
      const int64_t n = (int64_t)g * UNIT_ROWS + rank * RB + r;
      if (n < a.N) store_out(a, m, n, v);
    }
    return;
  }
  if (pl.C > 1 && rank != 0) {
    for (int u = tid; u < 16 * a.M; u += NCW * 32) {
      const int t0 = 4 * u, m = t0 >> 6, r0 = t0 & 63;
      float4 v;
      v.x = red0[r0 * MT + m] + red1[r0 * MT + m];
      v.y = red0[(r0 + 1) * MT + m] + red1[(r0 + 1) * MT + m];
      v.z = red0[(r0 + 2) * MT + m] + red1[(r0 + 2) * MT + m];
      v.w = red0[(r0 + 3) * MT + m] + red1[(r0 + 3) * MT + m];
      st_async_v4(dsmem_addr(part + rank * UNIT_ROWS * MT + t0, 0), v, dsmem_addr(redbar, 0));
    }
  } else {
    for (int t = tid; t < UNIT_ROWS * a.M; t += NCW * 32) {
      const int m = t >> 6, r = t & 63;
      const float v = red0[r * MT + m] + red1[r * MT + m];
      if (pl.C == 1) {
        const int64_t n = (int64_t)g * UNIT_ROWS + r;
        const float nv = n < a.N ? store_out(a, m, n, v) : 0.f;
        if (a.fu.ssq_out) red0[r * MT + m] = nv * nv;  // the slots this thread just read
        if (a.fu.rec_out) red1[r * MT + m] = nv;
      } else {
        part[t] = v;
      }
    }
  }
  if (pl.C == 1 && a.fu.ssq_out) {
    consumer_sync();
    write_ssq(a, red0, MT, 1, g, pl.G);
  }
  if (pl.C == 1 && a.fu.rec_out) {
    consumer_sync();
    write_records(a, red1, MT, g);
  }
  if (pl.C > 1) {
    if (rank == 0) {
      mbar_wait_cluster(redbar, 0, a.err, ERR_REDUCE_WAIT);
      consumer_sync();  // rank 0's own partial, written by other threads
      for (int t = tid; t < UNIT_ROWS * a.M; t += NCW * 32) {
        const int m = t >> 6, r = t & 63;
        float v = part[t];
        for (int q = 1; q < pl.C; ++q) v += part[q * UNIT_ROWS * MT + t];
        const int64_t n = (int64_t)g * UNIT_ROWS + r;
        const float nv = n < a.N ? store_out(a, m, n, v) : 0.f;
        if (a.fu.ssq_out) part[t] = nv * nv;  // the slot this thread just read
        if (a.fu.rec_out) red1[r * MT + m] = nv;  // red1 is free by now
      }
      if (a.fu.ssq_out) {
        consumer_sync();
        write_ssq(a, part, 1, UNIT_ROWS, g, pl.G);
      }
      if (a.fu.rec_out) {
        consumer_sync();
        write_records(a, red1, MT, g);
      }
      if (a.sc.n) {
        consumer_sync();
        if (tid == 0) signal_peers(a);
      }
    }
  } else if (a.sc.n) {
    consumer_sync();
    if (tid == 0) signal_peers(a);
  }
}

}  // namespace odi_cuda
