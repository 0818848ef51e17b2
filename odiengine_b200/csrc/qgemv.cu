// qgemv.cu -- host side of the streaming quantized GEMV: work plan and
// launch (the kernel itself is in qgemv_device.cuh).
#include "qgemv_device.cuh"

namespace odi_cuda {

static int tokens_per_pass(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

// Cluster size C per row tile: splitting a tile's spans over C CTAs fills the
// GPU when there are few tiles (decode shapes), at the cost of one
// distributed-shared-memory reduction per tile.  Estimated time in units of
// one span, per CTA slot: waves * (chunk + 1) (+ half a CTA of tail when the
// grid needs more than one wave) (+ the reduction and cluster cost).
GemvPlan make_gemv_plan(int dt, int64_t N, int64_t K, int M, bool f32act, int num_sms, bool pre, bool rs_ok) {
  GemvPlan p{};
  p.G = (int)((N + UNIT_ROWS - 1) / UNIT_ROWS);
  p.KB = (int)((K + UNIT_COLS - 1) / UNIT_COLS);
  const int slots = CTAS_PER_SM * (num_sms > 0 ? num_sms : 148);
  p.pre = (pre && !f32act) ? 1 : 0;
  p.mt = tokens_per_pass(M);
  for (;;) {
    const int rec = stage_stride(p.pre, p.mt);
    double best = 1e30;
    int bestC = 0, bestChunk = 0;
    for (int C = 1; C <= 8; C *= 2) {
      if (C > p.KB) break;
      const int chunk = (p.KB + C - 1) / C;
      const int ceff = (p.KB + chunk - 1) / chunk;
      if ((int64_t)chunk * p.mt * rec > XR_BUDGET) continue;
      const double ctas = (double)p.G * ceff;
      const double waves = ctas / slots;
      double t = (waves > 1.0 ? waves : 1.0) * (chunk + 1);
      if (waves > 1.0) t += 0.5 * (chunk + 1);
      // the cluster reduction, and the scheduling of larger clusters, cost
      // 0.5 + 0.25 * log2(C) spans (fitted to measured C = 1..8 timings of
      // the 7B and 70B decode shapes)
      if (ceff > 1) t += 0.5 + 0.25 * (ceff >= 8 ? 3 : ceff >= 4 ? 2 : 1);
      // With pre-quantized records a CTA's weight streaming is the larger
      // part of its life and each further wave of CTAs adds about two
      // spans of start-up and reduction (fitted the same way)
      if (p.pre) t += 2.0 * (waves > 1.0 ? waves : 1.0);
      if (t < best) {
        best = t;
        bestC = ceff;
        bestChunk = chunk;
      }
    }
    if (bestC) {
      p.C = bestC;
      p.chunk = bestChunk;
      break;
    }
    if (p.mt == 1) {  // activations of one chunk do not fit: signalled by C = 0
      p.C = 0;
      return p;
    }
    p.mt /= 2;
  }
  // Multi-token passes whose epilogue only stores y reduce-scatter across
  // the cluster: each rank receives the partials of 64/C rows only, which
  // keeps the receive buffer at one tile whatever C is (8-token passes with
  // C = 8 needed 16 KB there and ran three CTAs per SM; reduce-scattered,
  // four: Q4_K 4096x11008 M = 8 19.3 -> 14.4 us).  One-token passes keep the
  // gather to rank 0: there the other ranks exit as soon as they have
  // pushed, and the next launch's CTAs take their slots (reduce-scattered,
  // the headline took 7.9 us instead of 7.6).
  p.rs = (rs_ok && p.mt >= 2 && p.C > 1 && (p.C & (p.C - 1)) == 0) ? 1 : 0;
  p.xq_bytes = (p.chunk * p.mt * stage_stride(p.pre, p.mt) + 127) / 128 * 128;
  p.stage_bytes = (unit_bytes(dt) + 127) / 128 * 128;
  const bool rs = p.rs != 0;
  const int xr_off = p.mt == 1 ? SmemMap<1>::xr(p.C, rs)
                     : p.mt == 2 ? SmemMap<2>::xr(p.C, rs)
                     : p.mt == 4 ? SmemMap<4>::xr(p.C, rs)
                                 : SmemMap<8>::xr(p.C, rs);
  const int ring_off = xr_off + p.xq_bytes;
  int st = (SMEM_PER_CTA - ring_off) / p.stage_bytes;
  if (st > MAX_STAGES) st = MAX_STAGES;
  if (st > p.chunk) st = p.chunk;  // never more stages than units
  // The two consumer pairs take alternate units.  With an even ring depth
  // each pair owns its own slots (unit parity = slot parity) and visits them
  // in order, so a parity wait can never be two phases ahead of its slot.
  // An odd depth would let a pair wait on a slot the other pair has not yet
  // released, where the parity test passes a phase early.
  st -= st & 1;
  if (st < 2) st = 2;
  p.stages = st;
  p.smem_bytes = ring_off + p.stages * p.stage_bytes;
  // 228 KB of shared memory per SM, 1 KB of it reserved per resident CTA
  const int fit = (CTAS_PER_SM * (SMEM_MAX_CTA + 1024)) / (p.smem_bytes + 1024);
  p.ctas_per_sm = fit < CTAS_PER_SM ? fit : CTAS_PER_SM;
  return p;
}

template <int DT, int MT, bool F32, bool PRE>
static cudaError_t launch_t(const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
  auto kern = qgemv_kernel<DT, MT, F32, PRE>;
  // The shared-memory opt-in is per function and per device.
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    if (e != cudaSuccess) return e;
    // multi-token passes: the whole unified L1 / shared array as shared
    // memory, four CTAs of up to SMEM_MAX_CTA per SM (the kernel reads
    // nothing through L1)
    if (MT >= 2) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return e;
    }
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.G * pl.C);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = pl.smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pl.C > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = pl.C;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, a, pl);
}

template <int DT, bool F32>
static cudaError_t launch_mt(const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
  if (!F32 && pl.pre) {  // pre-quantized Q8 records
    switch (pl.mt) {
      case 1: return launch_t<DT, 1, F32, !F32>(pl, a, pdl, s);
      case 2: return launch_t<DT, 2, F32, !F32>(pl, a, pdl, s);
      case 4: return launch_t<DT, 4, F32, !F32>(pl, a, pdl, s);
      default: return launch_t<DT, 8, F32, !F32>(pl, a, pdl, s);
    }
  }
  switch (pl.mt) {
    case 1: return launch_t<DT, 1, F32, false>(pl, a, pdl, s);
    case 2: return launch_t<DT, 2, F32, false>(pl, a, pdl, s);
    case 4: return launch_t<DT, 4, F32, false>(pl, a, pdl, s);
    default: return launch_t<DT, 8, F32, false>(pl, a, pdl, s);
  }
}

template <bool F32>
static cudaError_t launch_dt(int dt, const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
  switch (dt) {
    case Q4_0: return launch_mt<Q4_0, F32>(pl, a, pdl, s);
    case Q8_0: return launch_mt<Q8_0, F32>(pl, a, pdl, s);
    case Q4_1: return launch_mt<Q4_1, F32>(pl, a, pdl, s);
    case Q5_0: return launch_mt<Q5_0, F32>(pl, a, pdl, s);
    case Q5_1: return launch_mt<Q5_1, F32>(pl, a, pdl, s);
    case Q4_K: return launch_mt<Q4_K, F32>(pl, a, pdl, s);
    case Q5_K: return launch_mt<Q5_K, F32>(pl, a, pdl, s);
    case Q6_K: return launch_mt<Q6_K, F32>(pl, a, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv(int dt, bool f32act, const GemvPlan& plan, const GemvArgs& a, bool pdl,
                        cudaStream_t s) {
  return f32act ? launch_dt<true>(dt, plan, a, pdl, s) : launch_dt<false>(dt, plan, a, pdl, s);
}

}  // namespace odi_cuda
