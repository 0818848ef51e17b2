// capi.cu -- the extern "C" boundary (include/odi_cuda.h).
//
// Nothing here throws.  Every entry point returns an odi_error_t code and
// records a thread-local message; CUDA failures are mapped to
// ODI_ERROR_GPU_OUT_OF_MEMORY (allocation) or ODI_ERROR_OPERATION_FAILED.
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/odi_cuda.h"
#include "internal.h"

using namespace odi_cuda;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

}  // namespace

int odi_cuda::set_error(int code, const char* msg) { return fail(code, "%s", msg); }

namespace {

int cuda_fail(cudaError_t e, const char* what) {
  const int code = (e == cudaErrorMemoryAllocation) ? ODI_CUDA_ERR_GPU_OUT_OF_MEMORY
                                                    : ODI_CUDA_ERR_OPERATION_FAILED;
  return fail(code, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// Host-side fault injection for the failure-detection tests: ODI_CUDA_INJECT,
// a comma-separated list read once per process.
//   init  -- odi_cuda_init reports no usable device (BACKEND_UNAVAILABLE);
//   alloc -- every device allocation the library makes fails as out of
//            memory (weight upload, host-call buffers, symmetric buffers);
//   wait  -- the host-buffer products find their error word set, as after a
//            kernel wait that gave up (the word is written on the device by
//            a memset, so the read-back path is the real one);
//   nccl  -- odi_cuda_nccl_init fails as a communicator that cannot form
//            (BACKEND_INIT_FAILED).
// Nothing is made to fail on the GPU itself.
enum { INJ_INIT = 1, INJ_ALLOC = 2, INJ_WAIT = 4, INJ_NCCL = 8 };
int injected() {
  static const int v = [] {
    const char* e = getenv("ODI_CUDA_INJECT");
    if (!e) return 0;
    const std::string s = std::string(",") + e + ",";
    return (s.find(",init,") != std::string::npos ? INJ_INIT : 0) |
           (s.find(",alloc,") != std::string::npos ? INJ_ALLOC : 0) |
           (s.find(",wait,") != std::string::npos ? INJ_WAIT : 0) |
           (s.find(",nccl,") != std::string::npos ? INJ_NCCL : 0);
  }();
  return v;
}

cudaError_t dev_malloc(void** p, size_t n) {
  if (injected() & INJ_ALLOC) {
    *p = nullptr;
    return cudaErrorMemoryAllocation;
  }
  return cudaMalloc(p, n);
}

#define CK(call, what)                         \
  do {                                         \
    cudaError_t e_ = (call);                   \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

int num_sms_current() {
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    sms[dev] = v;
  }
  return sms[dev];
}

// ODI_CUDA_ACT_AUTO resolved for this call; -1 for an unknown mode.
int resolve_act_mode(int dt, int64_t M, int act_mode) {
  switch (act_mode) {
    case ODI_CUDA_ACT_Q8:
    case ODI_CUDA_ACT_F32:
    case ODI_CUDA_ACT_F16:
      return act_mode;
    case ODI_CUDA_ACT_AUTO:
      return (tc_supported(dt) && M >= ODI_CUDA_TC_MIN_TOKENS) ? ODI_CUDA_ACT_F16 : ODI_CUDA_ACT_Q8;
    default:
      return -1;
  }
}

int check_shape(int dt, int64_t N, int64_t K) {
  if (!dtype_ok(dt)) return fail(ODI_CUDA_ERR_UNSUPPORTED_DTYPE, "dtype %d is not supported by the CUDA backend", dt);
  if (N < 1 || K < 1) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid weight shape N=%lld K=%lld", (long long)N, (long long)K);
  if (block_elems(dt) == 256 && K % 256)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "K-quant rows must be whole 256-value super-blocks (K=%lld)", (long long)K);
  if ((N + UNIT_ROWS - 1) / UNIT_ROWS * ((K + UNIT_COLS - 1) / UNIT_COLS) > 0x7FFFFFFFLL / 2)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "weight too large");
  return ODI_CUDA_OK;
}

// Multi-token ACT_Q8 products without an activation prologue quantize the
// tokens once, into Q8 records after the workspace header
// (act_q8_records_kernel), so a pass of up to 8 tokens stages 384 bytes per
// (span, token) instead of the fp32 row and streams the weight once.
size_t q8_records_bytes(int64_t M, int64_t K) { return (size_t)((K + 255) / 256) * (size_t)M * Q8_REC_BYTES; }
bool wants_records(bool f32, int64_t M, const GemvFuse* fu) {
  return !f32 && M >= 2 && !(fu && (fu->norm_w || fu->swiglu));
}

// The streaming GEMV over M tokens: one launch per pass of plan.mt tokens.
// With `sc`, each pass scatters its rows into every rank's gathered buffer.
// ext_recs: the activations already quantized into Q8 records (x unused).
int run_gemv(int dtype, const void* d_w_tiled, const float* d_x, float* d_y, int64_t M, int64_t N, int64_t K,
             bool f32, int* err, size_t ws_bytes, bool pdl, cudaStream_t s, const GemvScatter* sc,
             const GemvFuse* fu = nullptr, const uint8_t* ext_recs = nullptr) {
  const int64_t ldx = (fu && fu->swiglu) ? 2 * K : K;
  const bool pre = ext_recs || (wants_records(f32, M, fu) && ws_bytes >= WS_HEADER + q8_records_bytes(M, K));
  const uint8_t* recs = ext_recs ? ext_recs : reinterpret_cast<uint8_t*>(err) + WS_HEADER;
  if (pre && !ext_recs)
    CK(launch_act_q8_records(d_x, ldx, M, K, reinterpret_cast<uint8_t*>(err) + WS_HEADER, pdl, s),
       "act_q8_records launch");
  // the reduce-scatter serves products whose epilogue only stores y
  const bool rs_ok = !sc && !(fu && (fu->ssq_out || fu->rec_out));
  const GemvPlan plan = make_gemv_plan(dtype, N, K, (int)(M < 8 ? M : 8), f32, num_sms_current(), pre, rs_ok);
  if (plan.C == 0)
    return fail(ODI_CUDA_ERR_NOT_IMPLEMENTED, "K=%lld too large for the on-chip activation stage", (long long)K);
  for (int64_t m0 = 0; m0 < M; m0 += plan.mt) {
    GemvArgs a;
    a.w = (const uint8_t*)d_w_tiled;
    a.x = d_x + m0 * ldx;
    a.y = d_y ? d_y + m0 * N : nullptr;
    a.err = err;
    a.N = N;
    a.K = K;
    a.ldx = ldx;
    a.fu = fu ? *fu : GemvFuse{};
    a.M = (int)((M - m0) < plan.mt ? (M - m0) : plan.mt);
    a.recs = plan.pre ? recs + m0 * Q8_REC_BYTES : nullptr;
    a.rec_ld = M;
    if (a.fu.rec_out) a.fu.rec_out += m0 * Q8_REC_BYTES;
    a.sc = GemvScatter{};
    if (sc) {
      a.sc = *sc;
      for (int p = 0; p < sc->n; ++p) a.sc.out[p] = sc->out[p] + m0 * sc->ld;
      a.sc.done = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(err) + WS_DONE_OFFSET);
      a.sc.writers = plan.G;
    }
    CK(launch_gemv(dtype, f32, plan, a, pdl, s), "qgemv launch");
  }
  return ODI_CUDA_OK;
}

}  // namespace

struct odi_cuda_weight {
  int dtype;
  int64_t N, K;
  void* data;
  int device;
};

extern "C" {

const char* odi_cuda_last_error(void) { return g_err.c_str(); }

int odi_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

static_assert(ODI_CUDA_WS_ERR_FULL_WAIT == ERR_FULL_WAIT && ODI_CUDA_WS_ERR_EMPTY_WAIT == ERR_EMPTY_WAIT &&
                  ODI_CUDA_WS_ERR_DRAIN_WAIT == ERR_DRAIN_WAIT && ODI_CUDA_WS_ERR_REDUCE_WAIT == ERR_REDUCE_WAIT &&
                  ODI_CUDA_WS_ERR_PEER_WAIT == ERR_PEER_WAIT,
              "error word bits");

int odi_cuda_init(int device) {
  if (injected() & INJ_INIT) return fail(ODI_CUDA_ERR_BACKEND_UNAVAILABLE, "no usable CUDA device (ODI_CUDA_INJECT=init)");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return fail(ODI_CUDA_ERR_BACKEND_UNAVAILABLE, "no CUDA device: %s", e == cudaSuccess ? "count is 0" : cudaGetErrorString(e));
  if (device < 0 || device >= n)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "device %d out of range (0..%d)", device, n - 1);
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(ODI_CUDA_ERR_BACKEND_UNAVAILABLE, "device %d is sm_%d%d; this backend is built for sm_100a (B200)",
                device, prop.major, prop.minor);
  CK(cudaSetDevice(device), "cudaSetDevice");
  CK(cudaFree(nullptr), "context init");
  return ODI_CUDA_OK;
}

int odi_cuda_device_info(char* buf, size_t len) {
  if (!buf || !len) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  int dev = 0;
  CK(cudaGetDevice(&dev), "cudaGetDevice");
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
  snprintf(buf, len, "%s (sm_%d%d, %d SMs, %.1f GiB HBM, L2 %d MiB)", prop.name, prop.major, prop.minor,
           prop.multiProcessorCount, prop.totalGlobalMem / 1073741824.0, prop.l2CacheSize >> 20);
  return ODI_CUDA_OK;
}

int odi_cuda_memory_info(size_t* free_bytes, size_t* total_bytes) {
  size_t f = 0, t = 0;
  CK(cudaMemGetInfo(&f, &t), "cudaMemGetInfo");
  if (free_bytes) *free_bytes = f;
  if (total_bytes) *total_bytes = t;
  return ODI_CUDA_OK;
}

int odi_cuda_supports_dtype(int dtype) { return dtype_ok(dtype) ? 1 : 0; }

int odi_cuda_sync(void* stream) {
  CK(cudaStreamSynchronize((cudaStream_t)stream), "cudaStreamSynchronize");
  return ODI_CUDA_OK;
}

int64_t odi_cuda_gguf_bytes(int dtype, int64_t N, int64_t K) {
  if (!dtype_ok(dtype) || N < 0 || K < 0) return -1;
  const int be = block_elems(dtype);
  return N * ((K + be - 1) / be) * block_bytes(dtype);
}

int64_t odi_cuda_tiled_bytes(int dtype, int64_t N, int64_t K) {
  if (!dtype_ok(dtype) || N < 0 || K < 0) return -1;
  return ((N + UNIT_ROWS - 1) / UNIT_ROWS) * ((K + UNIT_COLS - 1) / UNIT_COLS) * unit_bytes(dtype);
}

int odi_cuda_repack(int dtype, const void* d_gguf, void* d_tiled, int64_t N, int64_t K, void* stream) {
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (!d_gguf || !d_tiled) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  CK(launch_repack(dtype, d_gguf, d_tiled, N, K, (cudaStream_t)stream), "repack");
  return ODI_CUDA_OK;
}

int odi_cuda_unpack(int dtype, const void* d_tiled, void* d_gguf, int64_t N, int64_t K, void* stream) {
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (!d_gguf || !d_tiled) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  CK(launch_unpack(dtype, d_tiled, d_gguf, N, K, (cudaStream_t)stream), "unpack");
  return ODI_CUDA_OK;
}

int odi_cuda_weight_upload(const void* host_blocks, int dtype, int64_t N, int64_t K, odi_cuda_weight** out) {
  if (!out || !host_blocks) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  const int64_t gb = odi_cuda_gguf_bytes(dtype, N, K), tb = odi_cuda_tiled_bytes(dtype, N, K);
  void* staging = nullptr;
  void* tiled = nullptr;
  cudaError_t e = dev_malloc(&staging, (size_t)gb);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (upload staging)");
  e = dev_malloc(&tiled, (size_t)tb);
  if (e == cudaSuccess) e = cudaMemcpy(staging, host_blocks, (size_t)gb, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = launch_repack(dtype, staging, tiled, N, K, nullptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(staging);
  if (e != cudaSuccess) {
    if (tiled) cudaFree(tiled);
    return cuda_fail(e, "weight upload");
  }
  odi_cuda_weight* w = new (std::nothrow) odi_cuda_weight;
  if (!w) {
    cudaFree(tiled);
    return fail(ODI_CUDA_ERR_OUT_OF_MEMORY, "host allocation failed");
  }
  w->dtype = dtype;
  w->N = N;
  w->K = K;
  w->data = tiled;
  cudaGetDevice(&w->device);
  *out = w;
  return ODI_CUDA_OK;
}

int odi_cuda_weight_free(odi_cuda_weight* w) {
  if (!w) return ODI_CUDA_OK;
  cudaError_t e = cudaFree(w->data);
  delete w;
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree");
  return ODI_CUDA_OK;
}

const void* odi_cuda_weight_data(const odi_cuda_weight* w) { return w ? w->data : nullptr; }

int odi_cuda_weight_shape(const odi_cuda_weight* w, int* dtype, int64_t* N, int64_t* K) {
  if (!w) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null weight");
  if (dtype) *dtype = w->dtype;
  if (N) *N = w->N;
  if (K) *K = w->K;
  return ODI_CUDA_OK;
}

int odi_cuda_quantize_weight(int dtype, const float* d_w, void* d_blocks, int64_t N, int64_t K, void* stream) {
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (!d_w || !d_blocks) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  CK(launch_quant_weights(dtype, d_w, d_blocks, N, K, (cudaStream_t)stream), "quantize_weight");
  return ODI_CUDA_OK;
}

int odi_cuda_quantize_q8_0(const float* d_x, void* d_blocks, int64_t M, int64_t K, void* stream) {
  if (M < 0 || K < 1) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid shape M=%lld K=%lld", (long long)M, (long long)K);
  if (M == 0) return ODI_CUDA_OK;
  if (!d_x || !d_blocks) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  CK(launch_act_quant(d_x, M, K, nullptr, (uint8_t*)d_blocks, false, (cudaStream_t)stream), "quantize_q8_0");
  return ODI_CUDA_OK;
}

int odi_cuda_tc_supported(int dtype) { return tc_supported(dtype) ? 1 : 0; }

size_t odi_cuda_matmul_workspace_bytes(int dtype, int64_t M, int64_t N, int64_t K, int act_mode) {
  if (!dtype_ok(dtype) || M < 1 || N < 1 || K < 1) return 0;
  const int mode = resolve_act_mode(dtype, M, act_mode);
  if (mode == ODI_CUDA_ACT_F16)
    return (size_t)(TC_X16_OFFSET + tc_x16_bytes(M, K));  // error word + fp16 activation tiles
  if (wants_records(mode == ODI_CUDA_ACT_F32, M, nullptr))
    return WS_HEADER + q8_records_bytes(M, K);  // error word + the tokens' Q8 records
  return WS_HEADER;  // the device error word; one token's activations are staged on chip
}

int odi_cuda_gemv_plan_info(int dtype, int64_t M, int64_t N, int64_t K, int act_mode, odi_cuda_gemv_plan* out) {
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (!out) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null output");
  if (M < 1 || M > (1 << 20)) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid M=%lld", (long long)M);
  const int mode = resolve_act_mode(dtype, M, act_mode);
  if (mode != ODI_CUDA_ACT_Q8 && mode != ODI_CUDA_ACT_F32)
    return fail(ODI_CUDA_ERR_NOT_IMPLEMENTED, "act_mode %d does not run on the streaming GEMV", act_mode);
  const bool f32 = mode == ODI_CUDA_ACT_F32;
  // as run_gemv with the workspace odi_cuda_matmul_workspace_bytes asks for
  const GemvPlan p = make_gemv_plan(dtype, N, K, (int)(M < 8 ? M : 8), f32, num_sms_current(),
                                    wants_records(f32, M, nullptr), true);
  if (p.C == 0)
    return fail(ODI_CUDA_ERR_NOT_IMPLEMENTED, "K=%lld too large for the on-chip activation stage", (long long)K);
  out->tokens_per_pass = p.mt;
  out->passes = (int)((M + p.mt - 1) / p.mt);
  out->cluster = p.C;
  out->spans_per_cta = p.chunk;
  out->stages = p.stages;
  out->reduce_scatter = p.rs;
  out->ctas_per_sm = p.ctas_per_sm;
  out->ctas = (int64_t)p.G * p.C;
  out->shared_bytes = (size_t)p.smem_bytes;
  return ODI_CUDA_OK;
}

int odi_cuda_matmul(int dtype, const void* d_w_tiled, const float* d_x, float* d_y, int64_t M, int64_t N,
                    int64_t K, int act_mode, void* d_workspace, size_t workspace_bytes, int flags,
                    void* stream) {
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (M < 0 || M > (1 << 20)) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid M=%lld", (long long)M);
  if (M == 0) return ODI_CUDA_OK;
  const int mode = resolve_act_mode(dtype, M, act_mode);
  if (mode < 0) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "unknown act_mode %d", act_mode);
  if (mode == ODI_CUDA_ACT_F16 && !tc_supported(dtype))
    return fail(ODI_CUDA_ERR_NOT_IMPLEMENTED, "dtype %d has no tensor-core path (ODI_CUDA_ACT_F16)", dtype);
  if (!d_w_tiled || !d_x || !d_y || !d_workspace) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  if (((uintptr_t)d_w_tiled | (uintptr_t)d_workspace) & 15)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "weight and workspace must be 16-byte aligned");
  const size_t need = odi_cuda_matmul_workspace_bytes(dtype, M, N, K, mode);
  if (workspace_bytes < need)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "workspace too small: %zu < %zu bytes", workspace_bytes, need);
  cudaStream_t s = (cudaStream_t)stream;
  if (mode == ODI_CUDA_ACT_F16) {
    const TcPlan plan = make_tc_plan(M, N, K, num_sms_current());
    TcArgs t;
    t.w = (const uint8_t*)d_w_tiled;
    t.x16 = (const uint8_t*)d_workspace + TC_X16_OFFSET;
    t.y = d_y;
    t.err = (int*)d_workspace;
    t.N = N;
    t.M = (int)M;
    t.M_pad = (int)((M + 255) / 256 * 256);
    t.KB = (int)((K + UNIT_COLS - 1) / UNIT_COLS);
    CK(launch_act_pack_f16(d_x, t.M, K, t.M_pad, (uint8_t*)d_workspace + TC_X16_OFFSET, s), "act_pack_f16 launch");
    CK(launch_qgemm_tc(dtype, plan, t, s), "qgemm_tc launch");
    return ODI_CUDA_OK;
  }
  const bool f32 = mode == ODI_CUDA_ACT_F32;
  const bool pdl = (flags & ODI_CUDA_FLAG_PDL) != 0;
  return run_gemv(dtype, d_w_tiled, d_x, d_y, M, N, K, f32, (int*)d_workspace, workspace_bytes, pdl, s, nullptr);
}

int odi_cuda_matmul_fused(int dtype, const void* d_w_tiled, const float* d_x, float* d_y, int64_t M, int64_t N,
                          int64_t K, int act_mode, void* d_workspace, size_t workspace_bytes, int flags,
                          const odi_cuda_matmul_opts* opts, void* stream) {
  if (!opts) return odi_cuda_matmul(dtype, d_w_tiled, d_x, d_y, M, N, K, act_mode, d_workspace, workspace_bytes,
                                    flags, stream);
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (M < 1 || M > (1 << 20)) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid M=%lld", (long long)M);
  const int mode = resolve_act_mode(dtype, M, act_mode);
  if (mode != ODI_CUDA_ACT_Q8 && mode != ODI_CUDA_ACT_F32)
    return fail(ODI_CUDA_ERR_NOT_IMPLEMENTED, "fused prologues / epilogues run on the streaming GEMV (ACT_Q8 / ACT_F32)");
  if (opts->norm_weight && opts->swiglu)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "norm_weight and swiglu are exclusive");
  if (!d_w_tiled || !d_x || !d_y || !d_workspace) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  if (((uintptr_t)d_w_tiled | (uintptr_t)d_workspace) & 15)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "weight and workspace must be 16-byte aligned");
  if (workspace_bytes < WS_HEADER) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "workspace too small");
  GemvFuse fu{};
  fu.norm_w = opts->norm_weight;
  fu.eps = opts->norm_eps;
  fu.swiglu = opts->swiglu ? 1 : 0;
  fu.accumulate = opts->accumulate ? 1 : 0;
  if (opts->norm_ssq && opts->norm_ssq_count < 1)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "norm_ssq_count must be positive");
  fu.ssq_in = opts->norm_ssq;
  fu.ssq_n = opts->norm_ssq_count;
  fu.ssq_out = opts->out_ssq;
  return run_gemv(dtype, d_w_tiled, d_x, d_y, M, N, K, mode == ODI_CUDA_ACT_F32, (int*)d_workspace, workspace_bytes,
                  (flags & ODI_CUDA_FLAG_PDL) != 0, (cudaStream_t)stream, nullptr, &fu);
}

size_t odi_cuda_q8_records_bytes(int64_t M, int64_t K) {
  if (M < 1 || K < 1) return 0;
  return q8_records_bytes(M, K);
}

// opts -> GemvFuse (norm / swiglu prologue, accumulate / out_ssq epilogue);
// 0 or an error status.
static int fuse_from_opts(const odi_cuda_matmul_opts* opts, GemvFuse* fu) {
  *fu = GemvFuse{};
  if (!opts) return ODI_CUDA_OK;
  if (opts->norm_weight && opts->swiglu)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "norm_weight and swiglu are exclusive");
  if (opts->norm_ssq && opts->norm_ssq_count < 1)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "norm_ssq_count must be positive");
  fu->norm_w = opts->norm_weight;
  fu->eps = opts->norm_eps;
  fu->swiglu = opts->swiglu ? 1 : 0;
  fu->accumulate = opts->accumulate ? 1 : 0;
  fu->ssq_in = opts->norm_ssq;
  fu->ssq_n = opts->norm_ssq_count;
  fu->ssq_out = opts->out_ssq;
  return ODI_CUDA_OK;
}

int odi_cuda_quantize_records(const float* d_x, int64_t M, int64_t K, const odi_cuda_matmul_opts* opts, void* d_recs,
                              int flags, void* stream) {
  if (!d_x || !d_recs) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "quantize_records: null buffer");
  if (M < 1 || K < 1 || M > (1 << 20)) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "quantize_records: bad M or K");
  if ((uintptr_t)d_recs & 15) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "records must be 16-byte aligned");
  GemvFuse fu;
  int rc = fuse_from_opts(opts, &fu);
  if (rc) return rc;
  if (fu.accumulate || fu.ssq_out)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "quantize_records: accumulate / out_ssq belong to the product");
  const int64_t ldx = fu.swiglu ? 2 * K : K;
  const bool pdl = (flags & ODI_CUDA_FLAG_PDL) != 0;
  if (fu.norm_w || fu.swiglu)
    CK(launch_act_records_fused(d_x, ldx, M, K, fu, (uint8_t*)d_recs, pdl, (cudaStream_t)stream),
       "quantize_records launch");
  else
    CK(launch_act_q8_records(d_x, ldx, M, K, (uint8_t*)d_recs, pdl, (cudaStream_t)stream), "quantize_records launch");
  return ODI_CUDA_OK;
}

int odi_cuda_matmul_q8rec(int dtype, const void* d_w_tiled, const void* d_recs, float* d_y, int64_t M, int64_t N,
                          int64_t K, void* d_workspace, size_t workspace_bytes, int flags,
                          const odi_cuda_q8rec_opts* opts, void* stream) {
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (M < 1 || M > (1 << 20)) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid M=%lld", (long long)M);
  if (!d_w_tiled || !d_recs || !d_y || !d_workspace) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  if (((uintptr_t)d_w_tiled | (uintptr_t)d_workspace | (uintptr_t)d_recs) & 15)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "weight, records and workspace must be 16-byte aligned");
  if (workspace_bytes < WS_HEADER) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "workspace too small");
  GemvFuse fu{};
  if (opts) {
    fu.accumulate = opts->accumulate ? 1 : 0;
    fu.ssq_out = opts->out_ssq;
    if (opts->norm_ssq) {
      if (opts->norm_ssq_count < 1) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "norm_ssq_count must be positive");
      fu.rec_scale = 1;
      fu.ssq_in = opts->norm_ssq;
      fu.ssq_n = opts->norm_ssq_count;
      fu.eps = opts->norm_eps;
    }
    if (opts->out_records) {
      if ((uintptr_t)opts->out_records & 15)
        return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "out_records must be 16-byte aligned");
      if (opts->out_swiglu ? (N % 512 != 0) : (N % 256 != 0))
        return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "out_records need N %% 256 == 0 (%% 512 with out_swiglu)");
      if (opts->out_swiglu && opts->out_norm_weight)
        return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "out_swiglu and out_norm_weight are exclusive");
      fu.rec_out = (uint8_t*)opts->out_records;
      fu.rec_out_ld = M;
      fu.rec_norm_w = opts->out_norm_weight;
      fu.rec_swiglu = opts->out_swiglu ? 1 : 0;
    }
  }
  return run_gemv(dtype, d_w_tiled, nullptr, d_y, M, N, K, false, (int*)d_workspace, workspace_bytes,
                  (flags & ODI_CUDA_FLAG_PDL) != 0, (cudaStream_t)stream, nullptr, &fu, (const uint8_t*)d_recs);
}

int odi_cuda_workspace_status(void* d_workspace, int* status, void* stream) {
  if (!d_workspace || !status) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  int v = 0;
  cudaStream_t s = (cudaStream_t)stream;
  CK(cudaMemcpyAsync(&v, d_workspace, sizeof(int), cudaMemcpyDeviceToHost, s), "read error word");
  CK(cudaStreamSynchronize(s), "sync");
  if (v) CK(cudaMemsetAsync(d_workspace, 0, sizeof(int), s), "clear error word");
  CK(cudaStreamSynchronize(s), "sync");
  *status = v;
  return ODI_CUDA_OK;
}

int odi_cuda_dequantize(int dtype, const void* d_w_tiled, float* d_out, int64_t N, int64_t K, void* stream) {
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (!d_w_tiled || !d_out) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  CK(launch_dequant(dtype, d_w_tiled, d_out, N, K, (cudaStream_t)stream), "dequantize");
  return ODI_CUDA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode-step operations (the non-matmul half of Context::forward).
// ---------------------------------------------------------------------------
static_assert(sizeof(odi_cuda_decode_state) == sizeof(DecodeState), "decode state layout");

extern "C" {

int odi_cuda_embed(const float* d_table, int64_t vocab, int64_t E, const odi_cuda_decode_state* d_state, float* d_x,
                   float* d_ssq, const float* d_norm_w, void* d_records, void* stream) {
  if (!d_table || !d_state || !d_x || vocab < 1 || E < 1) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "embed: bad argument");
  if (d_records && (E % 256 || (uintptr_t)d_records & 15))
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "embed: records need E %% 256 == 0 and 16-byte alignment");
  CK(launch_embed(d_table, vocab, E, reinterpret_cast<const DecodeState*>(d_state), d_x, d_ssq, d_norm_w,
                  (uint8_t*)d_records, (cudaStream_t)stream),
     "embed launch");
  return ODI_CUDA_OK;
}

int odi_cuda_rms_norm(const float* d_x, const float* d_w, float* d_y, int64_t rows, int64_t n, float eps,
                      void* stream) {
  if (!d_x || !d_w || !d_y || rows < 1 || rows > 65535 || n < 1)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "rms_norm: bad argument");
  CK(launch_rms_norm(d_x, d_w, d_y, rows, n, eps, (cudaStream_t)stream), "rms_norm launch");
  return ODI_CUDA_OK;
}

int odi_cuda_rope_kv(float* d_q, float* d_k, const float* d_v, void* d_kcache, void* d_vcache,
                     const odi_cuda_decode_state* d_state, int heads, int kv_heads, int head_dim, int ctx,
                     float theta, void* stream) {
  if (!d_q || !d_k || !d_v || !d_kcache || !d_vcache || !d_state)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "rope_kv: null argument");
  if (heads < 1 || kv_heads < 1 || heads % kv_heads || (head_dim != 64 && head_dim != 128) || ctx < 1)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "rope_kv: heads %d / kv_heads %d / head_dim %d / ctx %d", heads,
                kv_heads, head_dim, ctx);
  CK(launch_rope_kv(d_q, d_k, d_v, (__half*)d_kcache, (__half*)d_vcache, reinterpret_cast<const DecodeState*>(d_state),
                    heads, kv_heads, head_dim, ctx, theta, (cudaStream_t)stream),
     "rope_kv launch");
  return ODI_CUDA_OK;
}

size_t odi_cuda_attention_scratch_bytes(int heads, int head_dim, int ctx) {
  if (heads < 1 || head_dim < 1 || ctx < 1) return 0;
  return attention_scratch(heads, head_dim, ctx);
}

}  // extern "C"

namespace {
int attention_common(const float* d_q, const void* d_kcache, const void* d_vcache, float* d_out,
                     const odi_cuda_decode_state* d_state, int heads, int kv_heads, int head_dim, int ctx,
                     float scale, void* d_scratch, size_t scratch_bytes, const AttRope& rp, void* stream) {
  if (!d_q || !d_kcache || !d_vcache || !d_out || !d_state || !d_scratch)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "attention: null argument");
  if (heads < 1 || kv_heads < 1 || heads % kv_heads || (head_dim != 64 && head_dim != 128) || ctx < 1)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "attention: heads %d / kv_heads %d / head_dim %d", heads, kv_heads,
                head_dim);
  {
    const int grp = heads / kv_heads;
    if (grp != 1 && grp != 2 && grp != 4 && grp != 8)
      return fail(ODI_CUDA_ERR_NOT_IMPLEMENTED, "attention: %d query heads per kv head (1, 2, 4 or 8 supported)",
                  grp);
  }
  if (reinterpret_cast<uintptr_t>(d_kcache) & 15 || reinterpret_cast<uintptr_t>(d_vcache) & 15)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "attention: caches must be 16-byte aligned");
  if (scratch_bytes < odi_cuda_attention_scratch_bytes(heads, head_dim, ctx))
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "attention: scratch too small");
  if (reinterpret_cast<uintptr_t>(d_scratch) & 15)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "attention: scratch not 16-byte aligned");
  CK(launch_attention(d_q, (const __half*)d_kcache, (const __half*)d_vcache, d_out, d_scratch,
                      reinterpret_cast<const DecodeState*>(d_state), heads, kv_heads, head_dim, ctx, scale, rp,
                      (cudaStream_t)stream),
     "attention launch");
  return ODI_CUDA_OK;
}
}  // namespace

extern "C" {

int odi_cuda_attention_decode(const float* d_q, const void* d_kcache, const void* d_vcache, float* d_out,
                              const odi_cuda_decode_state* d_state, int heads, int kv_heads, int head_dim, int ctx,
                              float scale, void* d_scratch, size_t scratch_bytes, void* stream) {
  return attention_common(d_q, d_kcache, d_vcache, d_out, d_state, heads, kv_heads, head_dim, ctx, scale, d_scratch,
                          scratch_bytes, AttRope{}, stream);
}

int odi_cuda_rope_attention(const float* d_q, const float* d_k, const float* d_v, void* d_kcache, void* d_vcache,
                            float* d_out, void* d_out_records, const odi_cuda_decode_state* d_state, int heads,
                            int kv_heads, int head_dim, int ctx, float theta, float scale, void* d_scratch,
                            size_t scratch_bytes, void* stream) {
  if (!d_k || !d_v) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "rope_attention: null k or v");
  if ((uintptr_t)d_out_records & 15) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "records must be 16-byte aligned");
  AttRope rp;
  rp.k = d_k;
  rp.v = d_v;
  rp.theta = theta;
  rp.out_recs = (uint8_t*)d_out_records;
  return attention_common(d_q, d_kcache, d_vcache, d_out, d_state, heads, kv_heads, head_dim, ctx, scale, d_scratch,
                          scratch_bytes, rp, stream);
}

int odi_cuda_silu_mul(const float* d_gate_up, float* d_out, int64_t F, void* stream) {
  if (!d_gate_up || !d_out || F < 1) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "silu_mul: bad argument");
  CK(launch_silu_mul(d_gate_up, d_out, F, (cudaStream_t)stream), "silu_mul launch");
  return ODI_CUDA_OK;
}

int odi_cuda_add(float* d_x, const float* d_d, int64_t n, void* stream) {
  if (!d_x || !d_d || n < 1) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "add: bad argument");
  CK(launch_add(d_x, d_d, n, (cudaStream_t)stream), "add launch");
  return ODI_CUDA_OK;
}

int odi_cuda_argmax(const float* d_logits, int64_t V, odi_cuda_decode_state* d_state, int32_t* d_record,
                    int record_len, void* stream) {
  if (!d_logits || !d_state || V < 1 || V > 0x7ffffffe) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "argmax: bad argument");
  CK(launch_argmax(d_logits, V, reinterpret_cast<DecodeState*>(d_state), d_record, d_record ? record_len : 0,
                   (cudaStream_t)stream),
     "argmax launch");
  return ODI_CUDA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Row-shard scatter: the all-gather of a row-sharded product fused into the
// GEMV (peer stores over NVLink), symmetric buffers shared by IPC handles.
// ---------------------------------------------------------------------------
extern "C" {

int64_t odi_cuda_scatter_signals(int dtype, int64_t M, int64_t N, int64_t K, int act_mode) {
  if (!dtype_ok(dtype) || M < 1 || N < 1 || K < 1) return -1;
  const int mode = resolve_act_mode(dtype, M, act_mode);
  if (mode != ODI_CUDA_ACT_Q8 && mode != ODI_CUDA_ACT_F32) return -1;
  const bool f32 = mode == ODI_CUDA_ACT_F32;
  const GemvPlan plan = make_gemv_plan(dtype, N, K, (int)(M < 8 ? M : 8), f32, num_sms_current(),
                                       wants_records(f32, M, nullptr));
  if (plan.C == 0) return -1;
  return (M + plan.mt - 1) / plan.mt;  // one arrival per launch (pass)
}

int odi_cuda_matmul_scatter(int dtype, const void* d_w_tiled, const float* d_x, int64_t M, int64_t N, int64_t K,
                            int act_mode, void* d_workspace, size_t workspace_bytes, int flags,
                            const odi_cuda_scatter* sc, void* stream) {
  int rc = check_shape(dtype, N, K);
  if (rc) return rc;
  if (M < 1 || M > (1 << 20)) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid M=%lld", (long long)M);
  const int mode = resolve_act_mode(dtype, M, act_mode);
  if (mode != ODI_CUDA_ACT_Q8 && mode != ODI_CUDA_ACT_F32)
    return fail(ODI_CUDA_ERR_NOT_IMPLEMENTED, "the fused scatter runs on the streaming GEMV (ACT_Q8 / ACT_F32)");
  if (!sc || sc->nranks < 1 || sc->nranks > MAX_PEERS || sc->rank < 0 || sc->rank >= sc->nranks)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid scatter description");
  if (sc->row0 < 0 || sc->row0 + N > sc->ld)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "shard rows [%lld, %lld) outside the %lld gathered rows",
                (long long)sc->row0, (long long)(sc->row0 + N), (long long)sc->ld);
  for (int p = 0; p < sc->nranks; ++p)
    if (!sc->out[p] || !sc->counters[p]) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null peer buffer %d", p);
  if (!d_w_tiled || !d_x || !d_workspace) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null buffer");
  if (((uintptr_t)d_w_tiled | (uintptr_t)d_workspace) & 15)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "weight and workspace must be 16-byte aligned");
  // the pass count must be the one odi_cuda_scatter_signals reported: the
  // multi-token records need their workspace
  const size_t need = odi_cuda_matmul_workspace_bytes(dtype, M, N, K, mode);
  if (workspace_bytes < need)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "workspace too small: %zu < %zu bytes", workspace_bytes, need);
  GemvScatter g{};
  for (int p = 0; p < sc->nranks; ++p) {
    g.out[p] = sc->out[p];
    g.cnt[p] = sc->counters[p];
  }
  g.n = sc->nranks;
  g.src = sc->rank;
  g.row0 = sc->row0;
  g.ld = sc->ld;
  return run_gemv(dtype, d_w_tiled, d_x, nullptr, M, N, K, mode == ODI_CUDA_ACT_F32, (int*)d_workspace,
                  workspace_bytes, (flags & ODI_CUDA_FLAG_PDL) != 0, (cudaStream_t)stream, &g);
}

int odi_cuda_wait_peers_timeout(const unsigned long long* d_counters, unsigned long long* d_consumed,
                                const unsigned long long* increments, int nranks, uint64_t timeout_us,
                                void* d_workspace, void* stream) {
  if (!d_counters || !d_consumed || !increments || !d_workspace)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  if (nranks < 1 || nranks > MAX_PEERS) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid nranks %d", nranks);
  if (timeout_us < 1 || timeout_us > 60000000ull)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "timeout %llu us outside 1 us .. 60 s", (unsigned long long)timeout_us);
  PeerWait w{};
  for (int p = 0; p < nranks; ++p) w.inc[p] = increments[p];
  w.n = nranks;
  w.timeout_ns = timeout_us * 1000ull;
  CK(launch_wait_peers(d_counters, d_consumed, w, (int*)d_workspace, (cudaStream_t)stream), "wait_peers launch");
  return ODI_CUDA_OK;
}

int odi_cuda_wait_peers(const unsigned long long* d_counters, unsigned long long* d_consumed,
                        const unsigned long long* increments, int nranks, void* d_workspace, void* stream) {
  return odi_cuda_wait_peers_timeout(d_counters, d_consumed, increments, nranks, PEER_WAIT_DEFAULT_NS / 1000,
                                     d_workspace, stream);
}

int odi_cuda_sym_alloc(size_t bytes, void** d_ptr, void* ipc_handle) {
  if (!d_ptr || !ipc_handle || bytes == 0) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  *d_ptr = nullptr;
  void* p = nullptr;
  CK(dev_malloc(&p, bytes), "cudaMalloc (symmetric buffer)");
  cudaError_t e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "symmetric buffer");
  }
  static_assert(sizeof(h) <= ODI_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof h);
  *d_ptr = p;
  return ODI_CUDA_OK;
}

int odi_cuda_buffer_upload(const void* host, size_t bytes, void** d_ptr) {
  if (!host || !d_ptr || bytes == 0) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  *d_ptr = nullptr;
  void* p = nullptr;
  CK(dev_malloc(&p, bytes), "cudaMalloc (buffer)");
  cudaError_t e = cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "buffer upload");
  }
  *d_ptr = p;
  return ODI_CUDA_OK;
}

int odi_cuda_buffer_free(void* d_ptr) {
  if (d_ptr) CK(cudaFree(d_ptr), "cudaFree (buffer)");
  return ODI_CUDA_OK;
}

int odi_cuda_sym_free(void* d_ptr) {
  if (d_ptr) CK(cudaFree(d_ptr), "cudaFree (symmetric buffer)");
  return ODI_CUDA_OK;
}

int odi_cuda_ipc_open(const void* ipc_handle, void** d_ptr) {
  if (!ipc_handle || !d_ptr) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof h);
  *d_ptr = nullptr;
  CK(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return ODI_CUDA_OK;
}

int odi_cuda_ipc_close(void* d_ptr) {
  if (d_ptr) CK(cudaIpcCloseMemHandle(d_ptr), "cudaIpcCloseMemHandle");
  return ODI_CUDA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Row-sharded product over an NCCL communicator (shard.cu).
// ---------------------------------------------------------------------------
struct odi_cuda_comm {
  void* nccl;
  int nranks, rank, device;
};

extern "C" {

int odi_cuda_nccl_unique_id(void* id) {
  if (!id) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null id");
  static_assert(ODI_CUDA_NCCL_ID_BYTES >= 128, "NCCL unique id size");
  const char* why = "";
  if (nccl_unique_id(id, &why))
    return fail(nccl_available() ? ODI_CUDA_ERR_BACKEND_INIT_FAILED : ODI_CUDA_ERR_BACKEND_UNAVAILABLE,
                "ncclGetUniqueId: %s", why);
  return ODI_CUDA_OK;
}

int odi_cuda_nccl_init(const void* id, int nranks, int rank, odi_cuda_comm** comm) {
  if (!id || !comm) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  *comm = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "rank %d outside %d ranks", rank, nranks);
  if (injected() & INJ_NCCL)
    return fail(ODI_CUDA_ERR_BACKEND_INIT_FAILED, "NCCL communicator init failed (ODI_CUDA_INJECT=nccl)");
  int dev = 0;
  CK(cudaGetDevice(&dev), "cudaGetDevice");
  void* c = nullptr;
  const char* why = "";
  if (nccl_comm_init(id, nranks, rank, &c, &why))
    return fail(nccl_available() ? ODI_CUDA_ERR_BACKEND_INIT_FAILED : ODI_CUDA_ERR_BACKEND_UNAVAILABLE,
                "ncclCommInitRank: %s", why);
  odi_cuda_comm* h = new (std::nothrow) odi_cuda_comm{c, nranks, rank, dev};
  if (!h) {
    nccl_comm_destroy(c, &why);
    return fail(ODI_CUDA_ERR_OUT_OF_MEMORY, "host allocation failed");
  }
  *comm = h;
  return ODI_CUDA_OK;
}

int odi_cuda_nccl_free(odi_cuda_comm* comm) {
  if (!comm) return ODI_CUDA_OK;
  const char* why = "";
  const int r = nccl_comm_destroy(comm->nccl, &why);
  delete comm;
  if (r) return fail(ODI_CUDA_ERR_OPERATION_FAILED, "ncclCommDestroy: %s", why);
  return ODI_CUDA_OK;
}

int odi_cuda_comm_ranks(const odi_cuda_comm* comm, int* nranks, int* rank) {
  if (!comm) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null communicator");
  if (nranks) *nranks = comm->nranks;
  if (rank) *rank = comm->rank;
  return ODI_CUDA_OK;
}

size_t odi_cuda_sharded_workspace_bytes(const odi_cuda_comm* comm, int dtype, int64_t M, int64_t S, int64_t K,
                                        int act_mode) {
  if (!comm || M < 1 || S < 1 || K < 1) return 0;
  const size_t pw = odi_cuda_matmul_workspace_bytes(dtype, M, S, K, act_mode);
  if (!pw) return 0;
  return (pw + 255) / 256 * 256 + (size_t)comm->nranks * (size_t)M * (size_t)S * sizeof(float);
}

int odi_cuda_matmul_sharded(odi_cuda_comm* comm, int dtype, const void* d_w_shard, const float* d_x, float* d_y,
                            int64_t M, int64_t N, int64_t S, int64_t K, int act_mode, void* d_workspace,
                            size_t workspace_bytes, int flags, void* stream) {
  if (!comm) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null communicator");
  if (M < 1 || N < 1 || S < 1 || (int64_t)comm->nranks * S < N || (int64_t)(comm->nranks - 1) * S >= N)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "shard of S=%lld rows does not split N=%lld over %d ranks",
                (long long)S, (long long)N, comm->nranks);
  if (!d_y) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null output");
  const size_t need = odi_cuda_sharded_workspace_bytes(comm, dtype, M, S, K, act_mode);
  if (!need) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid sharded product");
  if (workspace_bytes < need)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "workspace too small: %zu < %zu bytes", workspace_bytes, need);
  const size_t pw = (odi_cuda_matmul_workspace_bytes(dtype, M, S, K, act_mode) + 255) / 256 * 256;
  cudaStream_t s = (cudaStream_t)stream;
  // M = 1 with every shard full: the rank-major slices are y itself
  const bool direct = M == 1 && N == (int64_t)comm->nranks * S;
  float* slots = direct ? d_y : reinterpret_cast<float*>(static_cast<uint8_t*>(d_workspace) + pw);
  float* mine = slots + (int64_t)comm->rank * M * S;
  int rc = odi_cuda_matmul(dtype, d_w_shard, d_x, mine, M, S, K, act_mode, d_workspace, pw, flags, stream);
  if (rc) return rc;
  const char* why = "";
  if (nccl_all_gather_f32(mine, slots, (size_t)(M * S), comm->nccl, s, &why))
    return fail(ODI_CUDA_ERR_OPERATION_FAILED, "ncclAllGather: %s", why);
  if (!direct) CK(launch_unshard(slots, d_y, M, N, S, comm->nranks, s), "unshard launch");
  return ODI_CUDA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Host-buffer matmul with a library-owned per-device arena.
// ---------------------------------------------------------------------------
namespace {
struct Arena {
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int* ws_host = nullptr;      // page-locked error-word workspace (WS_HEADER bytes)
  int* ws_host_dev = nullptr;  // its device address
  float* x = nullptr;
  size_t x_bytes = 0;
  float* y = nullptr;
  size_t y_bytes = 0;
  int pending_err = 0;         // error word of a workspace replaced while products were queued
  // Queued products' outputs (odi_cuda_matmul_host_async with page-locked
  // h_y): parked in yring by the products, copied out by one gather launch
  // per batch on the stream they were queued on.
  float* yring = nullptr;
  size_t ring_used = 0;
  GatherTable gt{};
  // The stream of the queued products not yet closed by a sync: the arena's
  // buffers are shared, so work on another stream waits for them first.
  cudaStream_t queue_stream = nullptr;
  bool queued = false;
};
constexpr size_t YRING_BYTES = 64u << 20;
std::mutex g_arena_mu;
Arena g_arena[64];

cudaError_t grow(void** p, size_t* have, size_t need, bool zero) {
  if (*have >= need) return cudaSuccess;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  cudaError_t e = dev_malloc(p, need);
  if (e != cudaSuccess) return e;
  if (zero) {
    e = cudaMemset(*p, 0, need);
    if (e != cudaSuccess) return e;
  }
  *have = need;
  return cudaSuccess;
}

// The device address of page-locked host memory (registered or allocated
// through CUDA), or nullptr for pageable memory.
template <typename T>
T* device_view(T* host) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, host) != cudaSuccess) {
    cudaGetLastError();  // pageable memory on older drivers reports an error; clear it
    return nullptr;
  }
  if (at.type != cudaMemoryTypeHost || !at.devicePointer) return nullptr;
  return static_cast<T*>(at.devicePointer);
}

// End of a synchronous host-buffer call: wait for the stream, then read the
// workspace's error word.  A kernel wait that gave up fails the call (its
// output is not to be trusted); the word is cleared for the next call.
int finish_host_call(Arena& A, cudaStream_t s) {
  int err = 0;
  if (injected() & INJ_WAIT) CK(cudaMemsetAsync(A.ws, 0x01, 1, s), "injected wait failure");
  CK(cudaMemcpyAsync(&err, A.ws, sizeof(int), cudaMemcpyDeviceToHost, s), "read error word");
  CK(cudaStreamSynchronize(s), "sync");
  if (err) {
    CK(cudaMemsetAsync(A.ws, 0, sizeof(int), s), "clear error word");
    CK(cudaStreamSynchronize(s), "sync");
    return fail(ODI_CUDA_ERR_OPERATION_FAILED, "a kernel wait gave up (error word 0x%x); the output is invalid", err);
  }
  return ODI_CUDA_OK;
}

// Launch the gather of the parked outputs (on their stream, after the
// products that wrote them) and start a new batch.
int flush_parked(Arena& A) {
  if (A.gt.n == 0) return ODI_CUDA_OK;
  CK(launch_gather_to_host(A.yring, A.gt, true, A.queue_stream), "y gather launch");
  A.gt.n = 0;
  A.ring_used = 0;
  return ODI_CUDA_OK;
}

// Enqueue one host-buffer product on `s`: x into the arena (pulled by a
// kernel from page-locked memory, or copied from pageable memory), the
// product, y into h_y (stored by the GEMV epilogue when h_y is page-locked,
// else copied back).  Takes the arena lock; *werr_out is the page-locked
// error word the product reports into, or nullptr when the error word is the
// device workspace's.
int enqueue_host_product(const odi_cuda_weight* w, const float* h_x, float* h_y, int64_t M, int mode,
                         cudaStream_t s, bool queued, Arena*& arena, int*& werr_out) {
  int dev = 0;
  CK(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != w->device) return fail(ODI_CUDA_ERR_INVALID_STATE, "weight lives on device %d, current is %d", w->device, dev);
  Arena& A = g_arena[dev & 63];
  arena = &A;
  if (A.queued && A.queue_stream != s) {
    int rc = flush_parked(A);
    if (rc) return rc;
    CK(cudaStreamSynchronize(A.queue_stream), "sync (products queued on another stream)");
    A.queued = false;
  }
  const size_t wsb = odi_cuda_matmul_workspace_bytes(w->dtype, M, w->N, w->K, mode);
  if (A.ws && wsb > A.ws_bytes) {
    // queued products may have reported into the workspace about to be
    // replaced: keep its error word for the next sync
    int old = 0;
    CK(cudaMemcpy(&old, A.ws, sizeof(int), cudaMemcpyDeviceToHost), "read error word");
    A.pending_err |= old;
  }
  CK(grow(&A.ws, &A.ws_bytes, wsb, true), "workspace alloc");
  const size_t xbytes = (size_t)(M * w->K) * sizeof(float);
  CK(grow((void**)&A.x, &A.x_bytes, xbytes, false), "x alloc");
  // A workspace that is only the error word (one-token and fp32 products on
  // the streaming GEMV) lives in page-locked host memory the device writes
  // through, so the host reads the word after the sync without a copy.
  int* werr = nullptr;
  if (wsb <= WS_HEADER) {
    if (!A.ws_host) {
      void* p = nullptr;
      if (injected() & INJ_ALLOC) return cuda_fail(cudaErrorMemoryAllocation, "cudaHostAlloc (error word)");
      CK(cudaHostAlloc(&p, WS_HEADER, cudaHostAllocMapped), "cudaHostAlloc (error word)");
      memset(p, 0, WS_HEADER);
      A.ws_host = static_cast<int*>(p);
      CK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&A.ws_host_dev), p, 0), "error word device address");
    }
    werr = A.ws_host;
  }
  werr_out = werr;
  // y: a page-locked h_y is written by the product itself (its epilogue
  // stores reach host memory directly), saving a copy's latency; the
  // tensor-core path, and pageable buffers, go through the device buffer.
  float* dy = mode == ODI_CUDA_ACT_F16 ? nullptr : device_view(h_y);
  if (!dy) CK(grow((void**)&A.y, &A.y_bytes, (size_t)(M * w->N) * sizeof(float), false), "y alloc");
  // A queued product with page-locked h_y parks its output in the ring (the
  // gather stores it into h_y later); outputs too large for the ring are
  // stored straight into h_y.
  float* ydst = dy;
  const size_t ybytes = (size_t)(M * w->N) * sizeof(float);
  const size_t yslot = (ybytes + 15) / 16 * 16;
  if (queued && dy && yslot <= YRING_BYTES) {
    if (!A.yring) CK(dev_malloc(reinterpret_cast<void**>(&A.yring), YRING_BYTES), "y ring alloc");
    if (A.gt.n == GATHER_MAX || A.ring_used + yslot > YRING_BYTES) {
      int rc = flush_parked(A);
      if (rc) return rc;
    }
    const int e = A.gt.n++;
    A.gt.dst[e] = (unsigned long long)reinterpret_cast<uintptr_t>(dy);
    A.gt.off16[e] = (unsigned)(A.ring_used / 16);
    A.gt.bytes[e] = (unsigned)ybytes;
    ydst = A.yring + A.ring_used / sizeof(float);
    A.ring_used += yslot;
  }
  // x: page-locked h_x is pulled by a kernel whose host loads overlap the
  // previous kernel on the stream; the product then follows it under
  // programmatic dependent launch, so its weight stream starts while x
  // arrives.  Pageable x goes through a copy.
  const float* hxv = device_view(const_cast<float*>(h_x));
  int flags = 0;
  if (hxv && (reinterpret_cast<uintptr_t>(hxv) & 3) == 0) {
    CK(launch_pull_host(hxv, A.x, xbytes, true, s), "x pull launch");
    flags = ODI_CUDA_FLAG_PDL;
  } else {
    CK(cudaMemcpyAsync(A.x, h_x, xbytes, cudaMemcpyHostToDevice, s), "H2D x");
  }
  int rc = odi_cuda_matmul(w->dtype, w->data, A.x, ydst ? ydst : A.y, M, w->N, w->K, mode,
                           werr ? static_cast<void*>(A.ws_host_dev) : A.ws, werr ? (size_t)WS_HEADER : A.ws_bytes,
                           flags, s);
  if (rc) return rc;
  if (!dy) CK(cudaMemcpyAsync(h_y, A.y, (size_t)(M * w->N) * sizeof(float), cudaMemcpyDeviceToHost, s), "D2H y");
  if (queued) {
    A.queued = true;
    A.queue_stream = s;
  }
  return ODI_CUDA_OK;
}

// Error words the host-buffer products of a device report into: the
// page-locked word (read directly) and the device workspace's (copied).
// Both are read after the stream's work is done, and cleared.
int finish_host_products(Arena& A, cudaStream_t s) {
  cudaStream_t qs = A.queue_stream;
  const bool other = A.queued && qs != s;
  int rc = flush_parked(A);
  if (rc) return rc;
  if (other) CK(cudaStreamSynchronize(qs), "sync (queue stream)");
  A.queued = false;
  int err = A.pending_err;
  A.pending_err = 0;
  if (A.ws) {
    if (injected() & INJ_WAIT) CK(cudaMemsetAsync(A.ws, 0x01, 1, s), "injected wait failure");
    CK(cudaMemcpyAsync(&err, A.ws, sizeof(int), cudaMemcpyDeviceToHost, s), "read error word");
  }
  CK(cudaStreamSynchronize(s), "sync");
  if (A.ws_host) {
    if (injected() & INJ_WAIT) *A.ws_host = ERR_FULL_WAIT;
    err |= *reinterpret_cast<volatile int*>(A.ws_host);
    *A.ws_host = 0;
  }
  if (err) {
    if (A.ws) {
      CK(cudaMemsetAsync(A.ws, 0, sizeof(int), s), "clear error word");
      CK(cudaStreamSynchronize(s), "sync");
    }
    return fail(ODI_CUDA_ERR_OPERATION_FAILED, "a kernel wait gave up (error word 0x%x); the output is invalid", err);
  }
  return ODI_CUDA_OK;
}

int check_host_product(const odi_cuda_weight* w, const float* h_x, float* h_y, int64_t M, int act_mode, int* mode) {
  if (!w || !h_x || !h_y) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  if (M < 0) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid M");
  *mode = 0;
  if (M == 0) return ODI_CUDA_OK;
  *mode = resolve_act_mode(w->dtype, M, act_mode);
  if (*mode < 0) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "unknown act_mode %d", act_mode);
  return ODI_CUDA_OK;
}
}  // namespace

extern "C" int odi_cuda_matmul_host(const odi_cuda_weight* w, const float* h_x, float* h_y, int64_t M,
                                    int act_mode, void* stream) {
  int mode = 0;
  int rc = check_host_product(w, h_x, h_y, M, act_mode, &mode);
  if (rc || M == 0) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  std::lock_guard<std::mutex> lk(g_arena_mu);
  Arena* A = nullptr;
  int* werr = nullptr;
  rc = enqueue_host_product(w, h_x, h_y, M, mode, s, false, A, werr);
  if (rc) return rc;
  if (!werr) return finish_host_call(*A, s);
  CK(cudaStreamSynchronize(s), "sync");
  if (injected() & INJ_WAIT) *werr = ERR_FULL_WAIT;
  const int err = *reinterpret_cast<volatile int*>(werr);
  if (err) {
    *werr = 0;
    return fail(ODI_CUDA_ERR_OPERATION_FAILED, "a kernel wait gave up (error word 0x%x); the output is invalid", err);
  }
  return ODI_CUDA_OK;
}

extern "C" int odi_cuda_matmul_host_async(const odi_cuda_weight* w, const float* h_x, float* h_y, int64_t M,
                                          int act_mode, void* stream) {
  int mode = 0;
  int rc = check_host_product(w, h_x, h_y, M, act_mode, &mode);
  if (rc || M == 0) return rc;
  std::lock_guard<std::mutex> lk(g_arena_mu);
  Arena* A = nullptr;
  int* werr = nullptr;
  return enqueue_host_product(w, h_x, h_y, M, mode, (cudaStream_t)stream, true, A, werr);
}

extern "C" int odi_cuda_host_sync(void* stream) {
  int dev = 0;
  CK(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_arena_mu);
  return finish_host_products(g_arena[dev & 63], (cudaStream_t)stream);
}

extern "C" int odi_cuda_dequantize_host(const odi_cuda_weight* w, float* h_out, void* stream) {
  if (!w || !h_out) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  int dev = 0;
  CK(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != w->device) return fail(ODI_CUDA_ERR_INVALID_STATE, "weight lives on device %d, current is %d", w->device, dev);
  const size_t bytes = (size_t)(w->N * w->K) * sizeof(float);
  std::lock_guard<std::mutex> lk(g_arena_mu);
  Arena& A = g_arena[dev & 63];
  // the values land in the arena's output buffer (grown once to the largest
  // weight dequantized), not in a buffer allocated per call
  CK(grow((void**)&A.y, &A.y_bytes, bytes, false), "dequantize output alloc");
  cudaStream_t s = (cudaStream_t)stream;
  CK(launch_dequant(w->dtype, w->data, A.y, w->N, w->K, s), "dequantize launch");
  CK(cudaMemcpyAsync(h_out, A.y, bytes, cudaMemcpyDeviceToHost, s), "D2H dequantized");
  CK(cudaStreamSynchronize(s), "sync");
  return ODI_CUDA_OK;
}

// ---------------------------------------------------------------------------
// Host-buffer matmul that allocates nothing (odi_cuda_matmul_host_noalloc).
//
// For callers that may not allocate device memory while running (HBM
// reserved up front, memory owned by another allocator's pool, or a decode
// loop that cannot take cudaMalloc's synchronisation).  Instead of the
// cudaMalloc-grown arena above, x, y and the error word live in one static
// device array per GPU, held from module load until the process exits:
//   [0, ws)                     the product's workspace: the error word first
//                               (must be zero when a product starts; cleared by
//                               every call), then, on the tensor-core path, the
//                               fp16 activation tiles; ws rounded up to 256 = rw
//   [rw, rw + rx)               x, M*K fp32     (rx = M*K*4 rounded up to 256)
//   [rw + rx, ... + M*N*4)      y, M*N fp32
// Every call shares the array; calls whose GPU work overlaps race on it.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[ODI_CUDA_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_dev[64];  // device address of the array, per device

// The array's name is a host-side stand-in in host code; the device address
// comes from cudaGetSymbolAddress, looked up once per device with that
// device current (the first call on each device does it).
int noalloc_scratch(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_dev[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (static scratch)");
    g_noalloc_dev[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_dev[dev];
  return ODI_CUDA_OK;
}
}  // namespace

extern "C" int odi_cuda_matmul_host_noalloc(const odi_cuda_weight* w, const float* h_x, float* h_y,
                                            int64_t M, int act_mode, void* stream) {
  if (!w || !h_x || !h_y) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "null argument");
  if (M < 0) return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "invalid M");
  if (M == 0) return ODI_CUDA_OK;
  if (resolve_act_mode(w->dtype, M, act_mode) < 0)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT, "unknown act_mode %d", act_mode);
  const int64_t cap = (int64_t)ODI_CUDA_NOALLOC_SCRATCH_BYTES;
  const int64_t per_token = 4 * (w->K + w->N);
  bool fits = M <= (cap - WS_HEADER) / per_token;  // bounds M before any product can overflow
  int64_t ws = 0, x_off = 0, y_off = 0, need = 0;
  if (fits) {
    // the workspace (error word first), then x, then y
    ws = (int64_t)odi_cuda_matmul_workspace_bytes(w->dtype, M, w->N, w->K, act_mode);
    x_off = (ws + 255) / 256 * 256;
    y_off = x_off + (M * w->K * 4 + 255) / 256 * 256;
    need = y_off + M * w->N * 4;
    fits = ws > 0 && need <= cap;
  }
  if (!fits)
    return fail(ODI_CUDA_ERR_INVALID_ARGUMENT,
                "odi_cuda_matmul_host_noalloc: M=%lld tokens of K=%lld inputs and N=%lld outputs exceed its "
                "static scratch of %lld bytes (needs round_up(workspace, 256) + round_up(M*K*4, 256) + M*N*4); "
                "use odi_cuda_matmul_host or fewer tokens per call",
                (long long)M, (long long)w->K, (long long)w->N, (long long)cap);
  int dev = 0;
  CK(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(ODI_CUDA_ERR_INVALID_STATE, "device %d out of range", dev);
  if (dev != w->device) return fail(ODI_CUDA_ERR_INVALID_STATE, "weight lives on device %d, current is %d", w->device, dev);
  unsigned char* scr = nullptr;
  int rc = noalloc_scratch(dev, &scr);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  float* d_x = reinterpret_cast<float*>(scr + x_off);
  float* d_y = reinterpret_cast<float*>(scr + y_off);
  CK(cudaMemsetAsync(scr, 0, sizeof(int), s), "clear error word");
  CK(cudaMemcpyAsync(d_x, h_x, (size_t)(M * w->K) * sizeof(float), cudaMemcpyHostToDevice, s), "H2D x");
  rc = odi_cuda_matmul(w->dtype, w->data, d_x, d_y, M, w->N, w->K, act_mode, scr, (size_t)ws, 0, stream);
  if (rc) return rc;
  CK(cudaMemcpyAsync(h_y, d_y, (size_t)(M * w->N) * sizeof(float), cudaMemcpyDeviceToHost, s), "D2H y");
  int err = 0;
  if (injected() & INJ_WAIT) CK(cudaMemsetAsync(scr, 0x01, 1, s), "injected wait failure");
  CK(cudaMemcpyAsync(&err, scr, sizeof(int), cudaMemcpyDeviceToHost, s), "read error word");
  CK(cudaStreamSynchronize(s), "sync");
  if (err) return fail(ODI_CUDA_ERR_OPERATION_FAILED, "a kernel wait gave up (error word 0x%x)", err);
  return ODI_CUDA_OK;
}
