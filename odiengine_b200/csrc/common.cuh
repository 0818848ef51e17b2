// common.cuh -- shared device helpers for the sm_100a quantized-matmul backend:
// the tiled weight layout, the activation tile layout, mbarrier / bulk-copy
// PTX wrappers with bounded waits, and the device error word.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace odi_cuda {

// odi_dtype_t ids (include/odi/odi_types.h:32-49).
enum DType : int { Q8_0 = 6, Q4_0 = 7, Q4_1 = 8, Q5_0 = 9, Q5_1 = 10, Q4_K = 11, Q5_K = 12, Q6_K = 13 };

// ----------------------------------------------------------------------------
// Tiled weight layout.  A unit = 64 output rows x 256 input columns.  Each
// unit is 64 row slices of SLICE bytes followed by a tail plane:
//   Q4_0 slice 144 B: d[8] fp16, qs[8][16]           (8 GGUF blocks)
//   Q8_0 slice 272 B: d[8] fp16, qs[8][32]           (8 GGUF blocks)
//   Q4_1 slice 176 B: d[8], m[8] fp16, qs[8][16], 16 B pad
//   Q5_0 slice 176 B: d[8] fp16, qh[8][4], qs[8][16]
//   Q5_1 slice 208 B: d[8], m[8] fp16, qh[8][4], qs[8][16], 16 B pad
//     (the 32-value block types keep their fields field-major over the 8
//     blocks of a span; the pads make every slice stride an odd multiple of
//     16 B, so 128-bit loads of 8 consecutive rows hit distinct banks)
//   Q4_K slice 144 B: the GGUF super-block verbatim  (d, dmin, scales[12], qs[128])
//   Q5_K slice 176 B: the GGUF super-block verbatim  (d, dmin, scales[12], qh[32], qs[128])
//   Q6_K slice 208 B: scales[16], ql[128], qh[64]; tail plane d[64] fp16
// Units are stored tile-major: unit (g, kb) at (g * KB + kb) * UNIT_BYTES.
// Rows >= N and blocks past the end of a row are zero bytes.
// ----------------------------------------------------------------------------
constexpr int UNIT_ROWS = 64;
constexpr int UNIT_COLS = 256;

__host__ __device__ constexpr int slice_bytes(int dt) {
  return dt == Q4_0 ? 144 : dt == Q8_0 ? 272 : dt == Q4_1 ? 176 : dt == Q5_0 ? 176 : dt == Q5_1 ? 208
       : dt == Q4_K ? 144 : dt == Q5_K ? 176 : dt == Q6_K ? 208 : 0;
}
// The 32-value block types: fields of a GGUF block [d][m][qh][qs] (m and qh
// where the type has them) and their field-major places in a slice.
__host__ __device__ constexpr bool is_block32(int dt) {
  return dt == Q4_0 || dt == Q8_0 || dt == Q4_1 || dt == Q5_0 || dt == Q5_1;
}
__host__ __device__ constexpr bool has_min(int dt) { return dt == Q4_1 || dt == Q5_1; }
__host__ __device__ constexpr bool has_qh(int dt) { return dt == Q5_0 || dt == Q5_1; }
__host__ __device__ constexpr int qs_bytes(int dt) { return dt == Q8_0 ? 32 : 16; }
__host__ __device__ constexpr int blk_qh(int dt) { return has_min(dt) ? 4 : 2; }
__host__ __device__ constexpr int blk_qs(int dt) { return 2 + (has_min(dt) ? 2 : 0) + (has_qh(dt) ? 4 : 0); }
__host__ __device__ constexpr int sl_m(int) { return 16; }
__host__ __device__ constexpr int sl_qh(int dt) { return 16 + (has_min(dt) ? 16 : 0); }
__host__ __device__ constexpr int sl_qs(int dt) { return sl_qh(dt) + (has_qh(dt) ? 32 : 0); }
__host__ __device__ constexpr int unit_bytes(int dt) {
  return slice_bytes(dt) * UNIT_ROWS + (dt == Q6_K ? 2 * UNIT_ROWS : 0);
}
__host__ __device__ constexpr int block_elems(int dt) {
  return is_block32(dt) ? 32 : (dt == Q4_K || dt == Q5_K || dt == Q6_K) ? 256 : 0;
}
__host__ __device__ constexpr int block_bytes(int dt) {
  return dt == Q4_0 ? 18 : dt == Q8_0 ? 34 : dt == Q4_1 ? 20 : dt == Q5_0 ? 22 : dt == Q5_1 ? 24
       : dt == Q4_K ? 144 : dt == Q5_K ? 176 : dt == Q6_K ? 210 : 0;
}
inline bool dtype_ok(int dt) { return is_block32(dt) || dt == Q4_K || dt == Q5_K || dt == Q6_K; }

// ----------------------------------------------------------------------------
// Activation tile layout (device scratch written by the activation kernels).
// For span kb and token m, a record of ACT_Q8_BYTES:
//   xq[256] int8  then  8 x {float d; int16 s_lo; int16 s_hi}
// (d = the fp16 Q8_0 scale widened to fp32; s_lo / s_hi = sums of the codes
// of the first / second 16 values of the 32-value block).  Records are
// stored span-major: offset (kb * M + m) * ACT_Q8_BYTES, so the M tokens of
// one span are one contiguous copy.  The fp32 form (ACT_F32_BYTES = 1024)
// holds the 256 fp32 values, zero past K.
// ----------------------------------------------------------------------------
constexpr int ACT_Q8_BYTES = 320;
// The streaming GEMV's Q8 record of one (span, token), as it sits in shared
// memory: 256 int8 codes, then 8 x {dx, sdx, sdx_lo, sdx_hi} fp32.
constexpr int Q8_REC_BYTES = 384;
constexpr int ACT_F32_BYTES = 1024;

struct ActRec {
  float d;
  short s_lo;
  short s_hi;
};

// ----------------------------------------------------------------------------
// Workspace header.  The first 256 bytes of every matmul workspace:
//   int error word (set by kernels whose bounded waits gave up), padding.
// Then the fixup counters (one int per row tile), then fp32 partial sums,
// then the activation tiles.
// ----------------------------------------------------------------------------
constexpr int WS_HEADER = 256;
enum : int { ERR_FULL_WAIT = 1, ERR_EMPTY_WAIT = 2, ERR_DRAIN_WAIT = 4, ERR_REDUCE_WAIT = 8 };

// ~1 s at the B200's clock: far beyond any legitimate wait in these kernels.
constexpr long long WAIT_BUDGET_CYCLES = 2000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the thread may be suspended in hardware for up to
// `hint_ns` while the phase is incomplete, so a waiting warp takes no issue
// slots from the warps doing work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, giving up after
// WAIT_BUDGET_CYCLES.  On give-up, ORs `code` into the error word and
// returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait_sleep(bar, parity, 100000u)) {
    if (clock64() - t0 > WAIT_BUDGET_CYCLES) {
      if (err) atomicOr(err, code);
      return false;
    }
  }
  return true;
}

// One bulk copy global -> this CTA's shared memory, completing on `bar`.
// No multicast.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// The Q8_0 quantiser's three roundings without a division routine.
//  * q8_scale: amax / 127 correctly rounded, as q0 = amax * RN(1/127) and
//    one residual correction q0 + fma(-q0, 127, amax) * RN(1/127) (the
//    correction step of Markstein's division theorem).  Equal to IEEE
//    amax / 127.0f for every non-negative finite fp32 amax, subnormals
//    included (tests/q8_math_check.c walks them all against the host's
//    division).
//  * q8_inv: 1 / d correctly rounded (__frcp_rn), 0 for d == 0.
//  * q8_round: round half away from zero, as trunc(t + copysign(0.5 - 2^-25,
//    t)): the addend is the float below one half, so t + addend reaches the
//    next integer exactly when frac(|t|) >= 1/2.  Equal to roundf(t) for
//    every fp32 |t| < 2^23 (same check); codes are within 128.
__device__ __forceinline__ float q8_scale(float amax) {
  const float r = 0x1.020408p-7f;  // RN(1/127)
  const float q0 = __fmul_rn(amax, r);
  return __fmaf_rn(__fmaf_rn(-q0, 127.0f, amax), r, q0);
}
__device__ __forceinline__ float q8_inv(float d) { return d == 0.0f ? 0.0f : __frcp_rn(d); }
__device__ __forceinline__ int q8_round(float t) {
  return __float2int_rz(__fadd_rn(t, copysignf(0x1.fffffep-2f, t)));
}

// Orders this thread's earlier shared-memory accesses (generic proxy) before
// later async-proxy accesses to shared memory -- a bulk copy that refills a
// ring slot the thread has read.  Each reading thread fences before the slot
// is released; the mbarrier ordering alone does not cover the proxy change
// (reads of a slot still landing after its refill began were observed
// without it).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk prefetch of global bytes into L2 (no shared-memory destination, no
// completion to wait on).  src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// One Q8_0 block of 32 values, one per lane, into a Q8 record: the codes at
// rec + 32 * j + lane, {dx, sdx, sdx_lo, sdx_hi} at rec + 256 + 16 * j.  The
// gguf Q8_0 quantiser in IEEE fp32 (d = amax / 127, id = d ? 1 / d : 0,
// q = round-half-away(v * id), d kept as fp16), then dx = that fp16 widened
// and the block's code sums times dx.  All 32 lanes of the warp take part.
__device__ __forceinline__ void q8_block_to_record(float v, int lane, uint8_t* rec, int j) {
  float am = fabsf(v);
#pragma unroll
  for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  const float d = q8_scale(am);
  const float id = q8_inv(d);
  const int q = q8_round(__fmul_rn(v, id));
  int s = q;
#pragma unroll
  for (int o = 8; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);  // within 16-lane halves
  const int s_lo = __shfl_sync(0xffffffffu, s, 0), s_hi = __shfl_sync(0xffffffffu, s, 16);
  rec[32 * j + lane] = (uint8_t)(int8_t)q;
  if (lane == 0) {
    const float dx = __half2float(__float2half_rn(d));
    *reinterpret_cast<float4*>(rec + 256 + 16 * j) =
        make_float4(dx, __fmul_rn((float)(s_lo + s_hi), dx), __fmul_rn((float)s_lo, dx), __fmul_rn((float)s_hi, dx));
  }
}

// Programmatic dependent launch controls (no-ops when not launched with PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

}  // namespace odi_cuda
