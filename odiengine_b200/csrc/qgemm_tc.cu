// qgemm_tc.cu -- prefill-shaped quantized GEMM on the sm_100a tensor cores
// (tcgen05.mma, fp32 accumulators in tensor memory).
//
// y[M, N] = x[M, K] . dequant(W)^T for many tokens.  The quantized weight is
// decoded on the fly to fp16 in shared memory and multiplied against fp16
// activations; accumulation is fp32 in TMEM.  Per CTA: 128 weight rows (the
// UMMA M) x BN tokens (the UMMA N), the whole K.
//
//   warp 0     producer: one lane streams the raw weight units of the CTA's
//              two 64-row tiles (cp.async.bulk, one 256-column span per
//              stage) and the fp16 activation tiles (one 64-column k-block
//              per stage), each completing on an mbarrier.
//   warp 1     allocates TMEM; one lane issues tcgen05.mma (kind::f16,
//              M=128, N=BN, K=16; four per k-block) and tcgen05.commit
//              releases the shared-memory stages it has read.
//   warps 2-9  decode: thread (h, r) owns half h of weight row r; per
//              k-block it writes 32 of the row's 64 fp16 weights (64 of its
//              128 bytes) into the K-major 128-byte-swizzled operand tile,
//              then fences the writes for the tensor core's async proxy.
//              At the end they read the accumulators back (tcgen05.ld, two
//              warps per 32-lane quarter, half of the columns each) and
//              write y.
//
// Operand tiles (A = weights, B = activations) use the canonical K-major
// SWIZZLE_128B layout: rows of 64 fp16 (128 B), 8-row atoms of 1024 B
// stacked densely, 16-byte chunk c of row r stored at chunk c ^ (r & 7).
// The activations are written in exactly that layout by act_pack_f16 (one
// contiguous block per (k-block, 8 tokens)), so a plain bulk copy lands a
// ready operand tile.
//
// Arithmetic: weights are decoded to fp16 as w = fp16(d*sc) * q - fp16(dmin*m)
// (one fp16 fma, Q4_K), activations rounded to fp16; products are exact in
// the tensor core and summed in fp32.
//
// Every wait is bounded (WAIT_BUDGET_CYCLES); a wait that gives up sets a bit
// in the error word and the roles fall through to the final barrier, where
// the tensor memory is released.
#include "internal.h"

namespace odi_cuda {
namespace tc {

constexpr int BM = 128;            // weight rows per CTA (UMMA M)
constexpr int BK = 64;             // k-block: one 128-byte swizzle row of fp16
constexpr int KBS = UNIT_COLS / BK;  // k-blocks per 256-column span (4)
constexpr int NDEC = 256;          // decode threads: 2 per weight row
constexpr int NTHREADS = 64 + NDEC;
constexpr int A_STAGE = BM * BK * 2;  // 16 KB
constexpr int ERR_TC_WAIT = 16;

template <int DT, int BN>
struct Cfg {
  static constexpr int UB = unit_bytes(DT);
  static constexpr int RAW = 2 * UB;                    // two 64-row units
  static constexpr int RAW_STAGE = (RAW + 1023) / 1024 * 1024;
  static constexpr int B_STAGE = BN * BK * 2;
  static constexpr int SA = 4, SB = BN >= 256 ? 3 : 4;
  static constexpr int RS = (BN >= 256 || UB > 10000) ? 2 : 3;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = A_OFF + SA * A_STAGE;
  static constexpr int R_OFF = B_OFF + SB * B_STAGE;
  static constexpr int BAR_OFF = R_OFF + RS * RAW_STAGE;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
};

__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  // start address >> 4 | LBO (unused for swizzled K-major) = 1 | SBO = 1024 B
  // | descriptor version 1 (bits 46-47) | layout SWIZZLE_128B (2, bits 61-63)
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: D fp32, A and B fp16, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive fp32 columns of the accumulator.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint4 ld128s(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void st128s(uint8_t* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Two 4-bit codes (bytes j, j+1 of w, low or high nibble) as the fp16 pair
// {1024 + q_j, 1024 + q_j+1} (exponent 10: the code sits in the mantissa).
template <int SEL, bool HI>
__device__ __forceinline__ uint32_t nib_pair(uint32_t w) {
  const uint32_t r = __byte_perm(w, 0u, SEL);  // [b_j, 0, b_j+1, 0]
  return ((HI ? (r >> 4) : r) & 0x000F000Fu) | 0x64006400u;
}

// fp16 weights of 4-bit codes: w = q * s + mneg, 8 per 16-byte chunk.
template <bool HI>
__device__ __forceinline__ uint4 chunk_q4(uint32_t w0, uint32_t w1, __half2 s, __half2 mneg) {
  const __half2 k1024 = bits_h2(0x64006400u);
  uint4 o;
  o.x = h2_bits(__hfma2(__hsub2(bits_h2(nib_pair<0x4140, HI>(w0)), k1024), s, mneg));
  o.y = h2_bits(__hfma2(__hsub2(bits_h2(nib_pair<0x4342, HI>(w0)), k1024), s, mneg));
  o.z = h2_bits(__hfma2(__hsub2(bits_h2(nib_pair<0x4140, HI>(w1)), k1024), s, mneg));
  o.w = h2_bits(__hfma2(__hsub2(bits_h2(nib_pair<0x4342, HI>(w1)), k1024), s, mneg));
  return o;
}

// Q4_K: half h of one k-block (64 values = sub-blocks 2j and 2j+1; h = 0 the
// low nibbles = sub-block 2j = chunks 0-3, h = 1 the high nibbles = sub-block
// 2j+1 = chunks 4-7) of one row into its swizzled 128-byte operand row.
__device__ __forceinline__ void decode_q4k_kblock(const uint8_t* sl, int j, int h, uint8_t* arow, int sw) {
  const uint4 hd = ld128s(sl);
  const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
  // 6-bit scales and mins of the 8 sub-blocks, one byte each
  const uint32_t scL = hd.y & 0x3F3F3F3Fu, mnL = hd.z & 0x3F3F3F3Fu;
  const uint32_t scH = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
  const uint32_t mnH = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
  const int b = 2 * j + h;
  const uint32_t sc = ((b < 4 ? scL : scH) >> (8 * (b & 3))) & 0xFFu;
  const uint32_t mn = ((b < 4 ? mnL : mnH) >> (8 * (b & 3))) & 0xFFu;
  const __half2 s = __float2half2_rn(d * (float)sc);
  const __half2 n = __float2half2_rn(-(dmin * (float)mn));
  const uint4 qa = ld128s(sl + 16 + 32 * j), qb = ld128s(sl + 32 + 32 * j);
  const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 o = h ? chunk_q4<true>(q[2 * c], q[2 * c + 1], s, n) : chunk_q4<false>(q[2 * c], q[2 * c + 1], s, n);
    st128s(arow + (((c + 4 * h) ^ sw) << 4), o);
  }
}

// Q6_K: half h of one k-block of one row.  Slice = scales[16], ql[128], qh[64]; d from
// the unit's tail plane.  k-block kb = half (kb >> 1), quarter groups
// g0 = 2*(kb & 1) and g0+1 of that half; group g of a half takes the
// (g >> 1 ? high : low) nibbles of ql[(g & 1) * 32 + l] and bits 2g..2g+1 of
// qh[l], l = 0..31; value = d * sc[8*half + 2g + l/16] * (q - 32).
__device__ __forceinline__ void decode_q6k_kblock(const uint8_t* sl, float d, int kb, int h, uint8_t* arow, int sw) {
  const int half = kb >> 1, g0 = 2 * (kb & 1);
  const uint8_t* ql = sl + 16 + 64 * half;
  const uint8_t* qh = sl + 144 + 32 * half;
  const uint4 scv = ld128s(sl);
  const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
  const __half2 k1056 = __float2half2_rn(1056.0f);
  {
    const int gg = h;  // decode half h = quarter group g0 + h (chunks 4h .. 4h+3)
    const int g = g0 + gg;
    const uint8_t* qlp = ql + (g & 1) * 32;
    const bool hi = (g >> 1) != 0;
#pragma unroll
    for (int part = 0; part < 2; ++part) {  // l = 16*part .. 16*part+15, one scale
      const int si = 8 * half + 2 * g + part;
      const int scb = (int)(int8_t)((scw[si >> 2] >> (8 * (si & 3))) & 0xFFu);
      const __half2 s = __float2half2_rn(d * (float)scb);
      const uint4 lv = ld128s(qlp + 16 * part), hv = ld128s(qh + 16 * part);
      const uint32_t lw[4] = {lv.x, lv.y, lv.z, lv.w}, hw[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {  // two 16-byte output chunks of 8 values
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int wi = 2 * c2 + (e >> 1);
          const uint32_t sel = (e & 1) ? 0x4342u : 0x4140u;
          const uint32_t l2 = __byte_perm(lw[wi], 0u, sel);
          const uint32_t h2 = __byte_perm(hw[wi], 0u, sel);
          const uint32_t lo4 = (hi ? (l2 >> 4) : l2) & 0x000F000Fu;
          const uint32_t hi2 = ((h2 >> (2 * g)) & 0x00030003u) << 4;
          const uint32_t v = lo4 | hi2 | 0x64006400u;  // 1024 + q
          o[e] = h2_bits(__hmul2(__hsub2(bits_h2(v), k1056), s));
        }
        const int chunk = 4 * gg + 2 * part + c2;  // values 8*chunk .. 8*chunk+7 of the k-block
        st128s(arow + ((chunk ^ sw) << 4), make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
  }
}

template <int DT, int BN>
__global__ void __launch_bounds__(NTHREADS, 1)
    qgemm_tc_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ x16, float* __restrict__ y, int* err,
                    int64_t N, int M, int M_pad, int G, int KB) {
  using C = Cfg<DT, BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (base_s & 1023u)) & 1023u);
  uint8_t* a_st = smem + C::A_OFF;
  uint8_t* b_st = smem + C::B_OFF;
  uint8_t* r_st = smem + C::R_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* full_r = bars;
  uint64_t* empty_r = full_r + C::RS;
  uint64_t* full_a = empty_r + C::RS;
  uint64_t* empty_a = full_a + C::SA;
  uint64_t* full_b = empty_a + C::SA;
  uint64_t* empty_b = full_b + C::SB;
  uint64_t* accum = empty_b + C::SB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g0 = 2 * blockIdx.x;
  const bool has_g1 = g0 + 1 < G;
  const int n0 = blockIdx.y * BN;
  const int NKB = KB * KBS;

  if (tid == 0) {
    for (int i = 0; i < C::RS; ++i) {
      mbar_init(&full_r[i], 1);
      mbar_init(&empty_r[i], NDEC);
    }
    for (int i = 0; i < C::SA; ++i) {
      mbar_init(&full_a[i], NDEC);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < C::SB; ++i) {
      mbar_init(&full_b[i], 1);
      mbar_init(&empty_b[i], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int last_r[C::RS], last_b[C::SB];
      for (int i = 0; i < C::RS; ++i) last_r[i] = -1;
      for (int i = 0; i < C::SB; ++i) last_b[i] = -1;
      const uint32_t rbytes = (uint32_t)C::UB * (has_g1 ? 2u : 1u);
      bool ok = true;
      for (int s = 0; s < KB && ok; ++s) {
        const int rs = s % C::RS;
        if (!mbar_wait(&empty_r[rs], ((s / C::RS) & 1) ^ 1, err, ERR_TC_WAIT)) { ok = false; break; }
        mbar_arrive_expect_tx(&full_r[rs], rbytes);
        bulk_g2s(r_st + rs * C::RAW_STAGE, w + ((int64_t)g0 * KB + s) * C::UB, C::UB, &full_r[rs]);
        if (has_g1)
          bulk_g2s(r_st + rs * C::RAW_STAGE + C::UB, w + ((int64_t)(g0 + 1) * KB + s) * C::UB, C::UB, &full_r[rs]);
        last_r[rs] = s;
        for (int q = 0; q < KBS; ++q) {
          const int kk = s * KBS + q, bs = kk % C::SB;
          if (!mbar_wait(&empty_b[bs], ((kk / C::SB) & 1) ^ 1, err, ERR_TC_WAIT)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_b[bs], (uint32_t)C::B_STAGE);
          bulk_g2s(b_st + bs * C::B_STAGE, x16 + ((int64_t)kk * M_pad + n0) * (BK * 2), C::B_STAGE, &full_b[bs]);
          last_b[bs] = kk;
        }
      }
      // drain: every issued copy has landed before the CTA can retire
      for (int i = 0; i < C::RS; ++i)
        if (last_r[i] >= 0) mbar_wait(&full_r[i], (last_r[i] / C::RS) & 1, err, ERR_TC_WAIT);
      for (int i = 0; i < C::SB; ++i)
        if (last_b[i] >= 0) mbar_wait(&full_b[i], (last_b[i] / C::SB) & 1, err, ERR_TC_WAIT);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BN);
      bool ok = true;
      for (int kk = 0; kk < NKB && ok; ++kk) {
        const int as = kk % C::SA, bs = kk % C::SB;
        if (!mbar_wait(&full_a[as], (kk / C::SA) & 1, err, ERR_TC_WAIT)) { ok = false; break; }
        if (!mbar_wait(&full_b[bs], (kk / C::SB) & 1, err, ERR_TC_WAIT)) { ok = false; break; }
        tc_fence_after();
        const uint64_t ad = sw128_kmajor_desc(smem_u32(a_st + as * A_STAGE));
        const uint64_t bd = sw128_kmajor_desc(smem_u32(b_st + bs * C::B_STAGE));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)  // +32 bytes along K per instruction
          mma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc, (kk | k) != 0 ? 1u : 0u);
        mma_commit(&empty_a[as]);
        mma_commit(&empty_b[bs]);
      }
      mma_commit(accum);  // arrives once every MMA issued above has completed
    }
  } else {
    // ---------------- decode + epilogue (warps 2-9) ----------------
    const int r = (tid - 64) & (BM - 1);  // weight row within the CTA
    const int h = (tid - 64) >> 7;        // half of the row's k-block
    const int u = r >> 6, sl_i = r & 63;
    uint8_t* arow0 = a_st + (r >> 3) * 1024 + (r & 7) * 128;
    const int sw = r & 7;
    bool ok = true;
    for (int s = 0; s < KB && ok; ++s) {
      const int rs = s % C::RS;
      if (!mbar_wait(&full_r[rs], (s / C::RS) & 1, err, ERR_TC_WAIT)) { ok = false; break; }
      const uint8_t* unit = r_st + rs * C::RAW_STAGE + u * C::UB;
      const bool live = u == 0 || has_g1;
      const uint8_t* sl = unit + sl_i * slice_bytes(DT);
      float d6 = 0.f;
      if (DT == Q6_K && live) d6 = __half2float(*reinterpret_cast<const __half*>(unit + 64 * 208 + 2 * sl_i));
      for (int q = 0; q < KBS; ++q) {
        const int kk = s * KBS + q, as = kk % C::SA;
        if (!mbar_wait(&empty_a[as], ((kk / C::SA) & 1) ^ 1, err, ERR_TC_WAIT)) { ok = false; break; }
        uint8_t* arow = arow0 + as * A_STAGE;
        if (!live) {
#pragma unroll
          for (int c = 0; c < 4; ++c) st128s(arow + ((c + 4 * h) << 4), make_uint4(0, 0, 0, 0));
        } else if (DT == Q4_K) {
          decode_q4k_kblock(sl, q, h, arow, sw);
        } else if (DT == Q6_K) {
          decode_q6k_kblock(sl, d6, q, h, arow, sw);
        }
        fence_async_smem();
        mbar_arrive(&full_a[as]);
      }
      mbar_arrive(&empty_r[rs]);
    }
    // epilogue: accumulator row = TMEM lane 32 * (warp % 4) + lane; the two
    // warps of a quarter take half of the columns each
    if (mbar_wait(accum, 0, err, ERR_TC_WAIT)) {
      tc_fence_after();
      const int quarter = warp & 3;
      const int chalf = (warp - 2) >> 2;
      const int64_t row = (int64_t)blockIdx.x * BM + quarter * 32 + lane;
#pragma unroll 1
      for (int c = chalf * (BN / 32); c < (chalf + 1) * (BN / 32); ++c) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 16), v);
        if (row < N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tok = n0 + c * 16 + j;
            if (tok < M) y[(int64_t)tok * N + row] = v[j];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// x fp32 [M][K] -> fp16 operand tiles: k-block kb, token m at byte
// (kb * M_pad + m) * 128, 16-byte chunk c (values 8c..8c+7) stored at chunk
// c ^ (m & 7).  Tokens >= M and columns >= K are zero.
__global__ void act_pack_f16_kernel(const float* __restrict__ x, uint8_t* __restrict__ x16, int M, int64_t K,
                                    int M_pad, int NKB) {
  const int64_t total = (int64_t)NKB * M_pad * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i & 7);
    const int64_t rowi = i >> 3;
    const int m = (int)(rowi % M_pad);
    const int64_t kb = rowi / M_pad;
    const int64_t k0 = kb * BK + c * 8;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (m < M && k0 + e < K) ? x[(int64_t)m * K + k0 + e] : 0.f;
    uint4 o;
    o.x = h2_bits(__floats2half2_rn(v[0], v[1]));
    o.y = h2_bits(__floats2half2_rn(v[2], v[3]));
    o.z = h2_bits(__floats2half2_rn(v[4], v[5]));
    o.w = h2_bits(__floats2half2_rn(v[6], v[7]));
    *reinterpret_cast<uint4*>(x16 + rowi * 128 + ((c ^ (m & 7)) << 4)) = o;
  }
}

template <int DT, int BN>
static cudaError_t launch_tc(const TcArgs& a, cudaStream_t s) {
  using C = Cfg<DT, BN>;
  auto kern = qgemm_tc_kernel<DT, BN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int G = (int)((a.N + UNIT_ROWS - 1) / UNIT_ROWS);
  dim3 grid((G + 1) / 2, (a.M + BN - 1) / BN);
  kern<<<grid, NTHREADS, C::SMEM, s>>>(a.w, a.x16, a.y, a.err, a.N, a.M, a.M_pad, G, a.KB);
  return cudaGetLastError();
}

}  // namespace tc

bool tc_supported(int dt) { return dt == Q4_K || dt == Q6_K; }

// Token block (UMMA N) for M tokens against N weight rows on num_sms SMs,
// one CTA per SM: estimated time = waves x per-k-block cost, where a
// k-block costs about max(BN, 160) token-columns (the decode of the
// 128 x 64 weight block bounds small BN).
int tc_block_n(int64_t M, int64_t N, int num_sms) {
  const int64_t rowtiles = (N + tc::BM - 1) / tc::BM;
  const int sms = num_sms > 0 ? num_sms : 148;
  int best = 128;
  double best_t = 1e300;
  for (int bn = 128; bn <= 256; bn *= 2) {
    const int64_t tiles = rowtiles * ((M + bn - 1) / bn);
    const double waves = (double)((tiles + sms - 1) / sms);
    const double t = waves * (bn > 160 ? bn : 160);
    if (t < best_t) {
      best_t = t;
      best = bn;
    }
  }
  return best;
}

// Packed activations: tokens padded to a multiple of 256 (any block), K to
// whole 256-column spans.
int64_t tc_x16_bytes(int64_t M, int64_t K) {
  const int64_t M_pad = (M + 255) / 256 * 256;
  const int64_t nkb = (K + UNIT_COLS - 1) / UNIT_COLS * tc::KBS;
  return nkb * M_pad * tc::BK * 2;
}

cudaError_t launch_act_pack_f16(const float* x, int M, int64_t K, int M_pad, uint8_t* x16, cudaStream_t s) {
  const int nkb = (int)((K + UNIT_COLS - 1) / UNIT_COLS * tc::KBS);
  const int64_t total = (int64_t)nkb * M_pad * 8;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  tc::act_pack_f16_kernel<<<blocks, 256, 0, s>>>(x, x16, M, K, M_pad, nkb);
  return cudaGetLastError();
}

template <int BN>
static cudaError_t launch_bn(int dt, const TcArgs& a, cudaStream_t s) {
  switch (dt) {
    case Q4_K: return tc::launch_tc<Q4_K, BN>(a, s);
    case Q6_K: return tc::launch_tc<Q6_K, BN>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_qgemm_tc(int dt, int bn, const TcArgs& a, cudaStream_t s) {
  return bn == 256 ? launch_bn<256>(dt, a, s) : launch_bn<128>(dt, a, s);
}

}  // namespace odi_cuda
