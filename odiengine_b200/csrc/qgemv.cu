// qgemv.cu -- host side of the streaming quantized GEMV: work plan and
// launch (the kernel itself is in qgemv_device.cuh).
#include "qgemv_device.cuh"

namespace odi_cuda {

// ---------------------------------------------------------------------------
// Host side: plan and launch.
// ---------------------------------------------------------------------------
static int tokens_per_pass(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

GemvPlan make_gemv_plan(int dt, int64_t N, int64_t K, int M, bool f32act, int num_sms) {
  GemvPlan p{};
  p.mt = tokens_per_pass(M);
  p.G = (int)((N + UNIT_ROWS - 1) / UNIT_ROWS);
  p.KB = (int)((K + UNIT_COLS - 1) / UNIT_COLS);
  p.U = p.G * p.KB;
  const int slots = 2 * (num_sms > 0 ? num_sms : 148);
  p.P = p.U < slots ? p.U : slots;
  if (p.P < 1) p.P = 1;
  const int per = p.U / p.P > 0 ? p.U / p.P : 1;
  p.maxc = (p.KB + per - 1) / per + 1;
  if (p.maxc > p.P) p.maxc = p.P;
  const int xb = f32act ? ACT_F32_BYTES : ACT_Q8_BYTES;
  p.stage_bytes = (unit_bytes(dt) + p.mt * xb + 127) / 128 * 128;
  int st = RING_BUDGET / p.stage_bytes;
  if (st > MAX_STAGES) st = MAX_STAGES;
  if (st < 2) st = 2;
  p.stages = st;
  p.smem_bytes = RING_OFFSET + p.stages * p.stage_bytes;
  return p;
}

size_t gemv_partial_floats(const GemvPlan& p, int /*M*/) {
  return (size_t)p.G * p.maxc * UNIT_ROWS * p.mt;
}

template <int DT, int MT, bool F32>
static cudaError_t launch_t(const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
  auto kern = qgemv_kernel<DT, MT, F32>;
  // The shared-memory opt-in is per function and per device.
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.P);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = pl.smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a, pl);
}

template <int DT, bool F32>
static cudaError_t launch_mt(const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
  switch (pl.mt) {
    case 1: return launch_t<DT, 1, F32>(pl, a, pdl, s);
    case 2: return launch_t<DT, 2, F32>(pl, a, pdl, s);
    case 4: return launch_t<DT, 4, F32>(pl, a, pdl, s);
    default: return launch_t<DT, 8, F32>(pl, a, pdl, s);
  }
}

template <bool F32>
static cudaError_t launch_dt(int dt, const GemvPlan& pl, const GemvArgs& a, bool pdl, cudaStream_t s) {
  switch (dt) {
    case Q4_0: return launch_mt<Q4_0, F32>(pl, a, pdl, s);
    case Q8_0: return launch_mt<Q8_0, F32>(pl, a, pdl, s);
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
