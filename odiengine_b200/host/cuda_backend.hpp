// cuda_backend.hpp -- odi::CUDABackend, the reference engine's Backend with
// its quantized matrix product on the B200 (through include/odi_cuda.h).
//
// Drop-in for the factory slot left at src/compute/cpu/cpu_backend.cpp:1011-1013
// (`case ODI_BACKEND_CUDA: // TODO: return std::make_unique<CUDABackend>();`).
// Compiles against the reference tree: it includes its compute/backend.hpp
// and compute/cpu/cpu_backend.hpp.
//
// What runs where:
//   matmul / quantized_matmul with a quantized `b` (backend.hpp:38, 114;
//     cpu_backend.cpp:177-227): on the GPU.  The weight's packed GGUF blocks
//     are uploaded once and kept in HBM in the tiled layout, keyed by the
//     host address of the blocks (the GGUF mmap view, valid while the Model
//     lives, gguf_parser.cpp:614-628), dtype and shape; activations are
//     copied in and the result copied out on every call, so `out` is ready
//     when matmul returns, as Context expects (context.cpp:76-78).
//   dequantize of a supported quantized tensor (backend.hpp:111): on the GPU.
//   A quantized type the library does not compute (e.g. Q8_K) is refused by
//   matmul and dequantize with std::runtime_error and reported unsupported
//   by supports_dtype: the quantized path has no CPU fallback.
//   Everything else (element-wise ops, norms, attention, fp32 x fp32
//   matmul) is the CPU backend's, inherited unchanged.
//
// Errors keep the reference's convention: a failure throws
// std::runtime_error (cpu_backend.cpp:180,192,195,201,226); the message is
// the library's odi_cuda_last_error() text.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>

#include "compute/cpu/cpu_backend.hpp"
#include "cuda_decoder.hpp"
#include "odi_cuda.h"

namespace odi {

class GGUFFile;

class CUDABackend : public CPUBackend {
 public:
  // Activation arithmetic of the quantized product.
  //   Q8   : activations quantised to Q8_0 (the gguf definition), integer
  //          block dots, fp32 scales -- the decode GEMV.
  //   F32  : fp32 activations times the exactly widened codes, fp32 sums --
  //          the reference's own arithmetic.
  //   F16  : tensor cores, fp16-decoded weights and fp16 activations, fp32
  //          sums -- prefill.
  //   AUTO : F16 from ODI_CUDA_TC_MIN_TOKENS tokens on (dtypes with a
  //          tensor-core path), else Q8.
  enum class ActMode { Q8 = ODI_CUDA_ACT_Q8, F32 = ODI_CUDA_ACT_F32, F16 = ODI_CUDA_ACT_F16, AUTO = ODI_CUDA_ACT_AUTO };

  // Throws std::runtime_error when `device` is not a usable sm_100 GPU.
  // Without an explicit mode the environment variable ODI_CUDA_ACT (q8, f32,
  // f16 or auto) selects it; the default is AUTO.
  explicit CUDABackend(int num_threads = 0, int device = 0);
  CUDABackend(int num_threads, int device, ActMode act);
  ~CUDABackend() override;

  CUDABackend(const CUDABackend&) = delete;
  CUDABackend& operator=(const CUDABackend&) = delete;

  odi_backend_type_t type() const override { return ODI_BACKEND_CUDA; }
  std::string name() const override { return "CUDA"; }
  std::string device_info() const override;
  size_t available_memory() const override;
  size_t used_memory() const override;
  bool supports_dtype(odi_dtype_t dtype) const override;

  void matmul(Tensor& out, const Tensor& a, const Tensor& b) override;
  void quantized_matmul(Tensor& out, const Tensor& a, const Tensor& b_quant) override;
  void dequantize(Tensor& out, const Tensor& x) override;
  void sync() override;

  // The loader hook, for Model::Model right after GGUFFile::open
  // (src/core/model.cpp:26-29): every 2-D tensor of the file whose dtype this
  // backend computes on the GPU is uploaded now, once, as its GGUF blocks
  // repacked in HBM, under the key matmul looks up (the GGUF view's host
  // address, dtype and shape; load_tensor returns the same view each time,
  // gguf_parser.cpp:614-628).  The first forward pass then finds every weight
  // resident.  Tensors already resident are skipped.  Returns the number
  // uploaded by this call; throws std::runtime_error if an upload fails.
  // The file must outlive the backend's use of its weights.
  size_t upload_model(const GGUFFile& file);

  // The whole decode step on the device for the Llama model of `file`
  // (cuda_decoder.hpp): one call per token for a Context::forward that hands
  // the step to the backend.  ctx: KV-cache positions (0: the file's).
  std::unique_ptr<CudaDecoder> create_decoder(const GGUFFile& file, int ctx = 0, int max_record = 4096);

  // Drops every cached device copy of a weight.  Call it when a model is
  // unloaded: a later tensor at a reused mmap address is recognised by a
  // fingerprint of its first and last 64 bytes and uploaded again, but only
  // an explicit release frees the HBM of weights no longer used.
  void release_weights();

  // Number of weights currently held in HBM, and their bytes.
  size_t cached_weights() const;

  ActMode act_mode() const { return act_; }

 private:
  using Key = std::tuple<const void*, int, int64_t, int64_t>;
  struct Cached {
    odi_cuda_weight* w;
    uint64_t fp;  // fingerprint of the host bytes it was uploaded from
  };
  odi_cuda_weight* weight_for(const Tensor& b, int64_t N, int64_t K);
  void bind_device() const;

  int device_ = 0;
  ActMode act_ = ActMode::AUTO;
  mutable std::mutex mu_;
  std::map<Key, Cached> weights_;
  size_t weight_bytes_ = 0;
};

// The factory cases for ODI_BACKEND_CUDA (cuda_factory.cpp): the CUDA
// backend, or nullptr with ODI_ERROR_BACKEND_UNAVAILABLE recorded through
// odi_set_error when no usable device exists; never a CPU backend.
std::unique_ptr<Backend> create_cuda_backend(int num_threads);
bool cuda_backend_available();

}  // namespace odi
