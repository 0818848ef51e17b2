// qgemm_tc.cu -- prefill-shaped quantized GEMM on the sm_100a tensor cores
// (tcgen05.mma, fp32 accumulators in tensor memory).
//
// y[M, N] = x[M, K] . dequant(W)^T for many tokens.  The quantized weight is
// decoded on the fly to fp16 in shared memory and multiplied against fp16
// activations; accumulation is fp32 in TMEM.  Per CTA: 128 weight rows (the
// UMMA M) x BN tokens (the UMMA N), the whole K.
//
//   warp 0     weight producer: one lane streams the raw weight units of
//              the CTA's two 64-row tiles (cp.async.bulk, one 256-column
//              span per stage, as deep a ring as shared memory allows).
//   warp 2     activation producer: one lane streams the fp16 activation
//              tiles of each operand stage (KSUB 64-column atoms).  Both
//              complete on mbarriers; separate producers let the weight
//              stream run ahead of the tensor core by the whole ring.
//   warp 1     allocates TMEM; one lane issues tcgen05.mma (kind::f16,
//              M=128, N=BN, K=16; 4 * KSUB per operand stage) and one
//              tcgen05.commit per stage, which releases it.  The issuing
//              thread pays a fixed cost per stage (wait + commit) besides
//              about 100 cycles per MMA, so small token blocks, whose MMAs
//              are short, use stages of up to four atoms.
//   warps 3-18 decode: thread (q4, r) owns quarter q4 of weight row r;
//              per 64-column atom it writes 16 of the row's 64 fp16 weights
//              (32 of its 128 bytes) into the K-major 128-byte-swizzled
//              operand tile; per stage each thread fences its writes for the
//              tensor core's async proxy and each warp arrives once on the
//              stage's barrier, with the activation copy.  At the end warps
//              3-10 read the accumulators back (tcgen05.ld, two warps per
//              32-lane quarter, half of the columns each) and the decode
//              warps write y.
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
constexpr int NDEC = 512;          // decode threads: 4 per weight row
constexpr int NTHREADS = 96 + NDEC;
constexpr int SMEM_BUDGET = 225 * 1024;  // one CTA per SM
constexpr int A_STAGE = BM * BK * 2;  // 16 KB
constexpr int ERR_TC_WAIT = 16;

// One operand stage = KSUB 64-column atoms of A (the weights) and of B (the
// activations) = 4 * KSUB MMAs per handshake.  The issuing thread pays a
// fixed cost per stage (barrier wait and commit) on top of each MMA's issue
// time, so small token blocks, whose MMAs are short, use wide stages.
template <int DT, int BN>
struct Cfg {
  static constexpr int UB = unit_bytes(DT);
  static constexpr int RAW = 2 * UB;                    // two 64-row units
  static constexpr int RAW_STAGE = (RAW + 1023) / 1024 * 1024;
  static constexpr int KSUB = BN <= 32 ? 4 : (BN <= 128 ? 2 : 1);
  static constexpr int SPS = KBS / KSUB;                // stages per span
  static constexpr int B_ATOM = BN * BK * 2;
  static constexpr int A_ST = KSUB * A_STAGE, B_ST = KSUB * B_ATOM;
  static constexpr int S = (BN <= 32 || BN == 128) ? 2 : 3;
  // the weight ring takes what the operand stages leave (2..8 spans)
  static constexpr int RS_FIT = (SMEM_BUDGET - 1280 - S * (A_ST + B_ST)) / RAW_STAGE;
  static constexpr int RS = RS_FIT > 8 ? 8 : (RS_FIT < 2 ? 2 : RS_FIT);
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = A_OFF + S * A_ST;
  static constexpr int R_OFF = B_OFF + S * B_ST;
  static constexpr int BAR_OFF = R_OFF + RS * RAW_STAGE;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(BM * (BN + 4) * 4 <= S * (A_ST + B_ST), "reduce-scatter slots must fit the operand stages");
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

// Decode roles.  Four threads share a weight row; thread quarter q4 writes
// two of the row's eight 16-byte chunks (16 fp16 values) per k-block, and
// decodes the scales it needs once per 256-column span.
//
// Q4_K (slice = d, dmin, scales[12], qs[128]): k-block j holds sub-blocks
// 2j (low nibbles of qs[32j .. 32j+31], chunks 0-3) and 2j+1 (high
// nibbles, chunks 4-7).  Quarter q4: nibble half h = q4 >> 1, bytes
// 16 * (q4 & 1) .. +15 of the group, chunks 4h + 2 (q4 & 1) + {0, 1}.
struct Q4kSpan {
  __half2 s[4], n[4];  // fp16(d * sc), -fp16(dmin * m) of sub-blocks 2j + h
};
__device__ __forceinline__ void q4k_span(const uint8_t* sl, int h, Q4kSpan& st) {
  const uint4 hd = ld128s(sl);
  const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
  // 6-bit scales and mins of the 8 sub-blocks, one byte each
  const uint32_t scL = hd.y & 0x3F3F3F3Fu, mnL = hd.z & 0x3F3F3F3Fu;
  const uint32_t scH = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
  const uint32_t mnH = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int b = 2 * j + h;  // sub-block
    const uint32_t sc = ((b < 4 ? scL : scH) >> (8 * (b & 3))) & 0xFFu;
    const uint32_t mn = ((b < 4 ? mnL : mnH) >> (8 * (b & 3))) & 0xFFu;
    st.s[j] = __float2half2_rn(d * (float)sc);
    st.n[j] = __float2half2_rn(-(dmin * (float)mn));
  }
}
template <int J>
__device__ __forceinline__ void q4k_kblock(const uint8_t* sl, int q4, const Q4kSpan& st, uint8_t* arow, int sw) {
  const int h = q4 >> 1, cp = q4 & 1;
  const uint4 q = ld128s(sl + 16 + 32 * J + 16 * cp);
  uint4 o0, o1;
  if (h) {
    o0 = chunk_q4<true>(q.x, q.y, st.s[J], st.n[J]);
    o1 = chunk_q4<true>(q.z, q.w, st.s[J], st.n[J]);
  } else {
    o0 = chunk_q4<false>(q.x, q.y, st.s[J], st.n[J]);
    o1 = chunk_q4<false>(q.z, q.w, st.s[J], st.n[J]);
  }
  const int c = 4 * h + 2 * cp;
  st128s(arow + ((c ^ sw) << 4), o0);
  st128s(arow + (((c + 1) ^ sw) << 4), o1);
}

// Q6_K (slice = scales[16], ql[128], qh[64]; d from the unit's tail plane):
// k-block kb = half (kb >> 1) of the super-block, quarter groups
// g0 = 2 (kb & 1) and g0 + 1; group g takes the (g >> 1 ? high : low)
// nibbles of ql[64 half + 32 (g & 1) + l] and bits 2g, 2g+1 of
// qh[32 half + l], l = 0..31; value = d * sc[8 half + 2g + l / 16] * (q - 32).
// Quarter q4: group g0 + (q4 >> 1), l = 16 (q4 & 1) .. +15 (one scale),
// chunks 4 (q4 >> 1) + 2 (q4 & 1) + {0, 1}.
struct Q6kSpan {
  __half2 s[4];  // fp16(d * sc) for k-blocks 0..3
};
__device__ __forceinline__ void q6k_span(const uint8_t* sl, float d, int q4, Q6kSpan& st) {
  const uint4 scv = ld128s(sl);
  const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
  const int gg = q4 >> 1, part = q4 & 1;
#pragma unroll
  for (int kb = 0; kb < 4; ++kb) {
    const int half = kb >> 1, g = 2 * (kb & 1) + gg;
    const int si = 8 * half + 2 * g + part;
    const int scb = (int)(int8_t)((scw[si >> 2] >> (8 * (si & 3))) & 0xFFu);
    st.s[kb] = __float2half2_rn(d * (float)scb);
  }
}
template <int KBI>
__device__ __forceinline__ void q6k_kblock(const uint8_t* sl, int q4, const Q6kSpan& st, uint8_t* arow, int sw) {
  const int gg = q4 >> 1, part = q4 & 1;
  constexpr int half = KBI >> 1;
  const int g = 2 * (KBI & 1) + gg;
  const uint4 lv = ld128s(sl + 16 + 64 * half + 32 * (g & 1) + 16 * part);
  const uint4 hv = ld128s(sl + 144 + 32 * half + 16 * part);
  const uint32_t lw[4] = {lv.x, lv.y, lv.z, lv.w}, hw[4] = {hv.x, hv.y, hv.z, hv.w};
  const bool hi = (g >> 1) != 0;
  const int sh = 2 * g;
  const __half2 k1056 = __float2half2_rn(1056.0f);
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
      const uint32_t hi2 = ((h2 >> sh) & 0x00030003u) << 4;
      const uint32_t v = lo4 | hi2 | 0x64006400u;  // 1024 + q
      o[e] = h2_bits(__hmul2(__hsub2(bits_h2(v), k1056), st.s[KBI]));
    }
    const int chunk = 4 * gg + 2 * part + c2;  // values 8*chunk .. 8*chunk+7 of the k-block
    st128s(arow + ((chunk ^ sw) << 4), make_uint4(o[0], o[1], o[2], o[3]));
  }
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded mbarrier wait for the pipeline roles: polls the non-blocking
// test_wait (no suspension: the waiter resumes the moment the phase
// completes), checks the clock every 64 polls and gives up after
// WAIT_BUDGET_CYCLES, setting ERR_TC_WAIT in the error word.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (int n = 1;; ++n) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((n & 63) == 0 && clock64() - t0 > WAIT_BUDGET_CYCLES) {
      if (err) atomicOr(err, ERR_TC_WAIT);
      return false;
    }
  }
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}
__device__ __forceinline__ void st_dsmem_v4(uint32_t remote, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}

// One CTA: weight rows [128 * blockIdx.x, +128) x tokens [BN * blockIdx.y, +BN)
// x the spans [rank * chunk, min(KB, (rank + 1) * chunk)) of its cluster
// rank (clusters of C CTAs along z split K).  With C > 1 the C partial
// accumulators are reduce-scattered through distributed shared memory:
// rank r owns rows [r * 128 / C, (r + 1) * 128 / C) of the tile, receives
// every rank's partial rows there, adds them in rank order (deterministic)
// and writes y.
template <int DT, int BN>
__global__ void __launch_bounds__(NTHREADS, 1)
    qgemm_tc_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ x16, float* __restrict__ y, int* err,
                    int64_t N, int M, int M_pad, int G, int KB, int chunk) {
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
  uint64_t* full = empty_r + C::RS;  // operand stage written: decode warps + activation copy
  uint64_t* empty = full + C::S;     // operand stage read by the tensor core
  uint64_t* accum = empty + C::S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g0 = 2 * blockIdx.x;
  const bool has_g1 = g0 + 1 < G;
  const int n0 = blockIdx.y * BN;
  const int csize = (int)cluster_size();
  const int rank = (int)cluster_rank();
  const int s0 = rank * chunk;
  const int s1 = min(KB, s0 + chunk);
  const int nsp = s1 - s0;  // >= 1: the host launches only non-empty ranks
  const int NST = nsp * C::SPS;  // operand stages

  if (tid == 0) {
    for (int i = 0; i < C::RS; ++i) {
      mbar_init(&full_r[i], 1);
      mbar_init(&empty_r[i], NDEC / 32);
    }
    for (int i = 0; i < C::S; ++i) {
      mbar_init(&full[i], NDEC / 32 + 1);
      mbar_init(&empty[i], 1);
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
    // ---------------- weight producer ----------------
    if (lane == 0) {
      int last_r[C::RS];
#pragma unroll
      for (int i = 0; i < C::RS; ++i) last_r[i] = -1;
      const uint32_t rbytes = (uint32_t)C::UB * (has_g1 ? 2u : 1u);
      for (int i = 0; i < nsp; ++i) {
        const int s = s0 + i, rs = i % C::RS;
        if (!tc_wait(&empty_r[rs], ((i / C::RS) & 1) ^ 1, err)) break;
        mbar_arrive_expect_tx(&full_r[rs], rbytes);
        bulk_g2s(r_st + rs * C::RAW_STAGE, w + ((int64_t)g0 * KB + s) * C::UB, C::UB, &full_r[rs]);
        if (has_g1)
          bulk_g2s(r_st + rs * C::RAW_STAGE + C::UB, w + ((int64_t)(g0 + 1) * KB + s) * C::UB, C::UB, &full_r[rs]);
#pragma unroll
        for (int j = 0; j < C::RS; ++j)
          if (j == rs) last_r[j] = i;
      }
      // drain: every issued copy has landed before the CTA can retire
#pragma unroll
      for (int i = 0; i < C::RS; ++i)
        if (last_r[i] >= 0) mbar_wait(&full_r[i], (last_r[i] / C::RS) & 1, err, ERR_TC_WAIT);
    }
  } else if (warp == 2) {
    // ---------------- activation producer ----------------
    if (lane == 0) {
      int last[C::S];
#pragma unroll
      for (int i = 0; i < C::S; ++i) last[i] = -1;
      for (int st = 0; st < NST; ++st) {
        const int slot = st % C::S;
        if (!tc_wait(&empty[slot], ((st / C::S) & 1) ^ 1, err)) break;
        mbar_arrive_expect_tx(&full[slot], (uint32_t)C::B_ST);
#pragma unroll
        for (int j = 0; j < C::KSUB; ++j) {
          const int64_t kb = (int64_t)s0 * KBS + st * C::KSUB + j;  // global k-block
          bulk_g2s(b_st + slot * C::B_ST + j * C::B_ATOM, x16 + (kb * M_pad + n0) * (BK * 2), C::B_ATOM, &full[slot]);
        }
#pragma unroll
        for (int j = 0; j < C::S; ++j)
          if (j == slot) last[j] = st;
      }
      // drain: every issued copy has landed before the CTA can retire
#pragma unroll
      for (int i = 0; i < C::S; ++i)
        if (last[i] >= 0) mbar_wait(&full[i], (last[i] / C::S) & 1, err, ERR_TC_WAIT);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BN);
      for (int st = 0; st < NST; ++st) {
        const int slot = st % C::S;
        if (!tc_wait(&full[slot], (st / C::S) & 1, err)) break;
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < C::KSUB; ++j) {
          const uint64_t ad = sw128_kmajor_desc(smem_u32(a_st + slot * C::A_ST + j * A_STAGE));
          const uint64_t bd = sw128_kmajor_desc(smem_u32(b_st + slot * C::B_ST + j * C::B_ATOM));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // +32 bytes along K per instruction
            mma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc, (st | j | k) != 0 ? 1u : 0u);
        }
        mma_commit(&empty[slot]);
      }
      mma_commit(accum);  // arrives once every MMA issued above has completed
    }
  } else {
    // ---------------- decode (warps 3-18) ----------------
    const int r = (tid - 96) & (BM - 1);  // weight row within the CTA
    const int q4 = (tid - 96) >> 7;       // quarter of the row's k-block
    const int u = r >> 6, sl_i = r & 63;
    uint8_t* arow0 = a_st + (r >> 3) * 1024 + (r & 7) * 128;
    const int sw = r & 7;
    const bool live = u == 0 || has_g1;
    for (int i = 0; i < nsp; ++i) {
      const int rs = i % C::RS;
      if (!mbar_wait(&full_r[rs], (i / C::RS) & 1, err, ERR_TC_WAIT)) break;
      const uint8_t* unit = r_st + rs * C::RAW_STAGE + u * C::UB;
      const uint8_t* sl = unit + sl_i * slice_bytes(DT);
      Q4kSpan s4;
      Q6kSpan s6;
      if (live) {
        if (DT == Q4_K) q4k_span(sl, q4 >> 1, s4);
        if (DT == Q6_K) q6k_span(sl, __half2float(*reinterpret_cast<const __half*>(unit + 64 * 208 + 2 * sl_i)), q4, s6);
      }
      bool ok = true;
#pragma unroll
      for (int q = 0; q < KBS; ++q) {  // k-block q of the span -> atom q % KSUB of stage q / KSUB
        const int st = i * C::SPS + q / C::KSUB, slot = st % C::S;
        if (q % C::KSUB == 0 && ok && !mbar_wait(&empty[slot], ((st / C::S) & 1) ^ 1, err, ERR_TC_WAIT)) ok = false;
        if (ok) {
          uint8_t* arow = arow0 + slot * C::A_ST + (q % C::KSUB) * A_STAGE;
          if (!live) {
            const int c = 2 * q4;  // this quarter's chunk pair, in chunk order 4h + 2cp or 4gg + 2part
            st128s(arow + (((c) ^ sw) << 4), make_uint4(0, 0, 0, 0));
            st128s(arow + (((c + 1) ^ sw) << 4), make_uint4(0, 0, 0, 0));
          } else if (DT == Q4_K) {
            if (q == 0) q4k_kblock<0>(sl, q4, s4, arow, sw);
            if (q == 1) q4k_kblock<1>(sl, q4, s4, arow, sw);
            if (q == 2) q4k_kblock<2>(sl, q4, s4, arow, sw);
            if (q == 3) q4k_kblock<3>(sl, q4, s4, arow, sw);
          } else if (DT == Q6_K) {
            if (q == 0) q6k_kblock<0>(sl, q4, s6, arow, sw);
            if (q == 1) q6k_kblock<1>(sl, q4, s6, arow, sw);
            if (q == 2) q6k_kblock<2>(sl, q4, s6, arow, sw);
            if (q == 3) q6k_kblock<3>(sl, q4, s6, arow, sw);
          }
          if (q % C::KSUB == C::KSUB - 1) {
            // each thread makes its own writes visible to the async proxy;
            // the warp barrier orders the warp's writes before its arrival
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[slot]);
          }
        }
      }
      if (!ok) break;
      fence_async_smem();  // this thread's reads of the raw stage before its refill
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_r[rs]);
    }
  }

  // ---------------- epilogue ----------------
  // Accumulator row = TMEM lane 32 * (warp % 4) + lane; the two decode warps
  // of a quarter take half of the columns each.
  const bool dec = warp >= 3;              // decode threads (all write y)
  const bool epi = warp >= 3 && warp < 11;  // accumulator readers
  bool acc_ok = false;
  if (epi) {
    acc_ok = mbar_wait(accum, 0, err, ERR_TC_WAIT);
    if (acc_ok) tc_fence_after();
  }
  const int quarter = warp & 3;
  const int chalf = (warp - 3) >> 2;
  const int trow = quarter * 32 + lane;  // accumulator row of this thread
  if (csize == 1) {
    if (epi && acc_ok) {
      const int64_t row = (int64_t)blockIdx.x * BM + trow;
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
  } else {
    // Reduce-scatter of the C partial tiles.  Slot (src, lr, col) of the
    // receiving rank, in its (now idle) operand-stage memory:
    //   ((src * RPR + lr) * (BN + 4) + col) * 4 bytes,  RPR = 128 / C rows.
    const int RPR = BM / csize;
    constexpr int SROW = BN + 4;
    float* slots = reinterpret_cast<float*>(smem);
    cluster_sync_all();  // every rank's MMAs are done: its stage memory is free
    if (epi && acc_ok) {
      const int dst = trow / RPR, lr = trow % RPR;
      const uint32_t base = mapa(smem_u32(slots + (rank * RPR + lr) * SROW), (uint32_t)dst);
#pragma unroll 1
      for (int c = chalf * (BN / 32); c < (chalf + 1) * (BN / 32); ++c) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 16), v);
#pragma unroll
        for (int j = 0; j < 16; j += 4) st_dsmem_v4(base + (uint32_t)(c * 16 + j) * 4u, v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
    }
    cluster_sync_all();  // all partial rows have landed
    if (dec) {
      const int64_t row0 = (int64_t)blockIdx.x * BM + rank * RPR;
      for (int idx = tid - 96; idx < RPR * BN; idx += NDEC) {
        const int lr = idx % RPR, col = idx / RPR;
        float v = 0.f;
        for (int src = 0; src < csize; ++src) v += slots[(src * RPR + lr) * SROW + col];
        const int tok = n0 + col;
        const int64_t row = row0 + lr;
        if (tok < M && row < N) y[(int64_t)tok * N + row] = v;
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
static cudaError_t launch_tc(const TcArgs& a, const TcPlan& p, cudaStream_t s) {
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((G + 1) / 2, (a.M + BN - 1) / BN, p.C);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = p.C;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a.w, a.x16, a.y, a.err, a.N, a.M, a.M_pad, G, a.KB, p.chunk);
}

}  // namespace tc

bool tc_supported(int dt) { return dt == Q4_K || dt == Q6_K; }

// Work plan: token block BN (the UMMA N) and the K split C (cluster size).
// Estimated time = the CTAs one SM must run (ceil(tiles / SMs)) x the cost
// of one CTA: (spans + 2 for the prologue and epilogue + BN/64 for the
// reduce-scatter when K is split) x 4 atoms x the cost of one 64-column
// atom in cycles, the larger of the tensor work (about 2.93 * BN at the
// measured rate), the issuing thread (about 95 per MMA, 4 per atom, plus
// about 200 per stage of KSUB atoms) and the decode (about 300).
TcPlan make_tc_plan(int64_t M, int64_t N, int64_t K, int num_sms) {
  const int64_t rowtiles = (N + tc::BM - 1) / tc::BM;
  const int KB = (int)((K + UNIT_COLS - 1) / UNIT_COLS);
  const int sms = num_sms > 0 ? num_sms : 148;
  const int cands[4] = {32, 64, 128, 256};
  TcPlan best{128, 1, KB};
  double best_t = 1e300;
  for (int bn : cands) {
    if (bn < 128 && M > bn) continue;   // small blocks only for small batches
    if (bn >= 128 && M <= 64) continue;
    for (int c = 1; c <= 8 && c <= KB; c *= 2) {
      const int chunk = (KB + c - 1) / c;
      const int ceff = (KB + chunk - 1) / chunk;
      if (ceff != c) continue;  // every rank needs at least one span
      const int64_t tiles = rowtiles * ((M + bn - 1) / bn) * ceff;
      const double per_sm = (double)((tiles + sms - 1) / sms);
      const int ksub = bn <= 32 ? 4 : (bn <= 128 ? 2 : 1);
      double atom = 2.93 * bn;
      if (atom < 380.0 + 200.0 / ksub) atom = 380.0 + 200.0 / ksub;
      if (atom < 300.0) atom = 300.0;
      // a K split adds the reduce-scatter of the 128 x BN partial tile
      const double t = per_sm * (chunk + 2 + (ceff > 1 ? bn / 64.0 : 0.0)) * 4.0 * atom;
      if (t < best_t) {
        best_t = t;
        best = TcPlan{bn, ceff, chunk};
      }
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
static cudaError_t launch_bn(int dt, const TcArgs& a, const TcPlan& p, cudaStream_t s) {
  switch (dt) {
    case Q4_K: return tc::launch_tc<Q4_K, BN>(a, p, s);
    case Q6_K: return tc::launch_tc<Q6_K, BN>(a, p, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_qgemm_tc(int dt, const TcPlan& p, const TcArgs& a, cudaStream_t s) {
  switch (p.BN) {
    case 32: return launch_bn<32>(dt, a, p, s);
    case 64: return launch_bn<64>(dt, a, p, s);
    case 128: return launch_bn<128>(dt, a, p, s);
    case 256: return launch_bn<256>(dt, a, p, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace odi_cuda
