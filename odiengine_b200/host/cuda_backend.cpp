// cuda_backend.cpp -- odi::CUDABackend (see cuda_backend.hpp).
#include "cuda_backend.hpp"

#include "format/gguf_parser.hpp"

#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

namespace odi {

namespace {

[[noreturn]] void raise(const char* what, int rc) {
  std::string msg = what;
  msg += ": ";
  const char* e = odi_cuda_last_error();
  msg += (e && *e) ? e : "error";
  msg += " (status " + std::to_string(rc) + ")";
  throw std::runtime_error(msg);
}

void ck(int rc, const char* what) {
  if (rc != ODI_CUDA_OK) raise(what, rc);
}

CUDABackend::ActMode act_from_env() {
  const char* v = std::getenv("ODI_CUDA_ACT");
  if (!v) return CUDABackend::ActMode::AUTO;
  if (std::strcmp(v, "f32") == 0 || std::strcmp(v, "F32") == 0) return CUDABackend::ActMode::F32;
  if (std::strcmp(v, "q8") == 0 || std::strcmp(v, "Q8") == 0) return CUDABackend::ActMode::Q8;
  if (std::strcmp(v, "f16") == 0 || std::strcmp(v, "F16") == 0) return CUDABackend::ActMode::F16;
  return CUDABackend::ActMode::AUTO;
}

// The device this host thread last bound; CUDA's current device is per thread.
thread_local int t_bound_device = -1;

}  // namespace

CUDABackend::CUDABackend(int num_threads, int device) : CUDABackend(num_threads, device, act_from_env()) {}

CUDABackend::CUDABackend(int num_threads, int device, ActMode act)
    : CPUBackend(num_threads), device_(device), act_(act) {
  ck(odi_cuda_init(device), "CUDABackend");
  t_bound_device = device;
}

CUDABackend::~CUDABackend() {
  try {
    release_weights();
  } catch (...) {
  }
}

void CUDABackend::bind_device() const {
  if (t_bound_device != device_) {
    ck(odi_cuda_init(device_), "CUDABackend: bind device");
    t_bound_device = device_;
  }
}

std::string CUDABackend::device_info() const {
  bind_device();
  char buf[256] = {};
  ck(odi_cuda_device_info(buf, sizeof buf), "device_info");
  return buf;
}

size_t CUDABackend::available_memory() const {
  bind_device();
  size_t free_b = 0, total_b = 0;
  ck(odi_cuda_memory_info(&free_b, &total_b), "available_memory");
  return free_b;
}

size_t CUDABackend::used_memory() const {
  std::lock_guard<std::mutex> lk(mu_);
  return weight_bytes_;
}

size_t CUDABackend::cached_weights() const {
  std::lock_guard<std::mutex> lk(mu_);
  return weights_.size();
}

bool CUDABackend::supports_dtype(odi_dtype_t dtype) const {
  // Unquantized types run through the inherited CPU element-wise code; of the
  // quantized types only those the GPU computes (odi_cuda_supports_dtype).
  // Q8_K and any other block type the library lacks are refused, never run
  // on the CPU.
  if (dtype_is_quantized(dtype)) return odi_cuda_supports_dtype(dtype) == 1;
  return CPUBackend::supports_dtype(dtype);
}

namespace {
[[noreturn]] void unsupported(const char* op, odi_dtype_t dt) {
  throw std::runtime_error(std::string(op) + ": quantization type " + std::to_string((int)dt) +
                           " is not supported by the CUDA backend");
}

// FNV-1a over the first and last 64 bytes of a weight's blocks: a cached
// device copy whose host bytes no longer match (another tensor now lives at
// the same address) is uploaded again.
uint64_t fingerprint(const void* data, size_t bytes) {
  const unsigned char* p = static_cast<const unsigned char*>(data);
  uint64_t h = 1469598103934665603ull;
  auto mix = [&](const unsigned char* q, size_t n) {
    for (size_t i = 0; i < n; ++i) h = (h ^ q[i]) * 1099511628211ull;
  };
  const size_t n = bytes < 64 ? bytes : 64;
  mix(p, n);
  mix(p + bytes - n, n);
  return h ^ bytes;
}
}  // namespace

odi_cuda_weight* CUDABackend::weight_for(const Tensor& b, int64_t N, int64_t K) {
  const Key key{b.data(), (int)b.dtype(), N, K};
  const int64_t gb = odi_cuda_gguf_bytes((int)b.dtype(), N, K);
  const uint64_t fp = gb > 0 ? fingerprint(b.data(), (size_t)gb) : 0;
  std::lock_guard<std::mutex> lk(mu_);
  auto it = weights_.find(key);
  if (it != weights_.end()) {
    if (it->second.fp == fp) return it->second.w;
    ck(odi_cuda_weight_free(it->second.w), "stale weight free");
    weight_bytes_ -= (size_t)odi_cuda_tiled_bytes((int)b.dtype(), N, K);
    weights_.erase(it);
  }
  odi_cuda_weight* w = nullptr;
  ck(odi_cuda_weight_upload(b.data(), (int)b.dtype(), N, K, &w), "weight upload");
  weights_.emplace(key, Cached{w, fp});
  weight_bytes_ += (size_t)odi_cuda_tiled_bytes((int)b.dtype(), N, K);
  return w;
}

size_t CUDABackend::upload_model(const GGUFFile& file) {
  bind_device();
  size_t n = 0;
  for (const std::string& name : file.tensor_names()) {
    const Tensor t = file.load_tensor(name);
    if (!t.is_valid() || t.ndim() != 2 || !dtype_is_quantized(t.dtype()) || odi_cuda_supports_dtype(t.dtype()) != 1)
      continue;
    // a weight view is [K, N] (GGUF dims, K contiguous), as matmul reads b
    const int64_t K = t.shape(0), N = t.shape(1);
    const size_t before = cached_weights();
    weight_for(t, N, K);
    if (cached_weights() > before) ++n;
  }
  return n;
}

std::unique_ptr<CudaDecoder> CUDABackend::create_decoder(const GGUFFile& file, int ctx, int max_record) {
  bind_device();
  return CudaDecoder::from_gguf(file, ctx, max_record);
}

void CUDABackend::release_weights() {
  std::lock_guard<std::mutex> lk(mu_);
  int first_rc = ODI_CUDA_OK;
  for (auto& kv : weights_) {
    int rc = odi_cuda_weight_free(kv.second.w);
    if (rc != ODI_CUDA_OK && first_rc == ODI_CUDA_OK) first_rc = rc;
  }
  weights_.clear();
  weight_bytes_ = 0;
  ck(first_rc, "release_weights");
}

// Shape rules and messages follow CPUBackend::matmul (cpu_backend.cpp:177-227):
// M = a.shape(-2) (1 for a vector), K = a.shape(-1), N = b.shape(-1), and K
// must equal b.shape(-2) (b.shape(0) for a vector b).  Leading batch
// dimensions of `a` are not iterated, exactly as there.
void CUDABackend::matmul(Tensor& out, const Tensor& a, const Tensor& b) {
  if (!dtype_is_quantized(b.dtype())) {
    // fp32 x fp32 is not the quantized product: the CPU backend's own code.
    CPUBackend::matmul(out, a, b);
    return;
  }
  // Every supported block type runs on the GPU, Q4_1 / Q5_0 / Q5_1 included
  // (the product the block format defines; the CPU backend's fallback for
  // them reads the dequantized weight transposed, cpu_backend.cpp:211-216).
  // A block type the library lacks is refused, not run on the CPU.
  if (odi_cuda_supports_dtype(b.dtype()) != 1) unsupported("matmul", b.dtype());
  if (a.ndim() < 1 || b.ndim() < 1) throw std::runtime_error("matmul: invalid tensor dimensions");
  int64_t M = a.ndim() >= 2 ? a.shape(-2) : 1;
  const int64_t K = a.shape(-1);
  int64_t N = b.shape(-1);
  if (b.ndim() == 1) {
    N = 1;
    if (K != b.shape(0)) throw std::runtime_error("matmul: dimension mismatch");
  } else if (K != b.shape(-2)) {
    throw std::runtime_error("matmul: dimension mismatch");
  }
  if (a.dtype() != ODI_DTYPE_F32) throw std::runtime_error("matmul: quantized weights require F32 activations");
  if (!out.data() || !a.data() || !b.data()) throw std::runtime_error("matmul: null tensor data");
  bind_device();
  odi_cuda_weight* w = weight_for(b, N, K);
  ck(odi_cuda_matmul_host(w, a.data_ptr<float>(), out.data_ptr<float>(), M, (int)act_, nullptr), "matmul");
}

void CUDABackend::quantized_matmul(Tensor& out, const Tensor& a, const Tensor& b_quant) {
  matmul(out, a, b_quant);  // as cpu_backend.cpp:650-653
}

// Block order = element order [N][K], n = x.numel() values (cpu_backend.cpp:625-648).
// A weight tensor has shape [K, N] (K the contiguous dimension); a 1-D
// tensor is one row.
void CUDABackend::dequantize(Tensor& out, const Tensor& x) {
  if (odi_cuda_supports_dtype(x.dtype()) != 1) unsupported("dequantize", x.dtype());
  if (!out.data() || !x.data()) throw std::runtime_error("dequantize: null tensor data");
  const int64_t K = x.ndim() >= 2 ? x.shape(0) : x.numel();
  if (K <= 0 || x.numel() % K) throw std::runtime_error("dequantize: invalid shape");
  const int64_t N = x.numel() / K;
  bind_device();
  odi_cuda_weight* w = weight_for(x, N, K);
  ck(odi_cuda_dequantize_host(w, out.data_ptr<float>(), nullptr), "dequantize");
}

void CUDABackend::sync() {
  bind_device();
  ck(odi_cuda_sync(nullptr), "sync");
}

}  // namespace odi
