// backend_c.cpp -- a C facade over odi::Backend objects: the reference's
// CPUBackend and this project's CUDABackend, driven through the same
// Backend calls (matmul, dequantize, sync, the metadata queries).  Tensors
// are passed as (pointer, dtype, ndim, shape) and wrapped in non-owning
// odi::Tensor views (tensor.hpp:50), the way Context hands the backend its
// scratch and the GGUF weight views.
//
// Every function catches what the backend throws and returns 1 with the
// message in odi_be_last_error(); 0 on success.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include "cuda_backend.hpp"
#include "format/gguf_parser.hpp"

namespace {
thread_local std::string t_err;

int caught(const char* what) {
  t_err = what;
  return 1;
}

std::vector<int64_t> dims(int ndim, const int64_t* shape) { return std::vector<int64_t>(shape, shape + ndim); }

odi::Tensor view(const void* p, int dtype, int ndim, const int64_t* shape) {
  return odi::Tensor(const_cast<void*>(p), dims(ndim, shape), (odi_dtype_t)dtype);
}
}  // namespace

extern "C" {

const char* odi_be_last_error(void) { return t_err.c_str(); }

// kind: ODI_BACKEND_CPU (1) or ODI_BACKEND_CUDA (4).  act_mode (CUDA only):
// an ODI_CUDA_ACT_* value.  NULL on failure.
void* odi_be_create(int kind, int num_threads, int device, int act_mode) {
  try {
    if (kind == ODI_BACKEND_CPU) return static_cast<odi::Backend*>(new odi::CPUBackend(num_threads));
    if (kind == ODI_BACKEND_CUDA)
      return static_cast<odi::Backend*>(
          new odi::CUDABackend(num_threads, device, static_cast<odi::CUDABackend::ActMode>(act_mode)));
    t_err = "unknown backend kind " + std::to_string(kind);
  } catch (const std::exception& e) {
    caught(e.what());
  }
  return nullptr;
}

// The backend the integrated factory (create_backend, cpu_backend.cpp:992-1019
// with the CUDA case patched to create_cuda_backend) returns for `kind`;
// NULL with the C API's last error set when it returns none.
void* odi_be_create_via_factory(int kind, int num_threads) {
  odi_clear_error();
  try {
    if (kind == ODI_BACKEND_CUDA) return odi::create_cuda_backend(num_threads).release();
    if (kind == ODI_BACKEND_CPU) return odi::create_backend(ODI_BACKEND_CPU, num_threads).release();
    odi_set_error(ODI_ERROR_BACKEND_NOT_SUPPORTED, "unknown backend kind");
  } catch (const std::exception& e) {
    odi_set_error(ODI_ERROR_OPERATION_FAILED, e.what());
  }
  return nullptr;
}
int odi_be_factory_error(void) { return (int)odi_get_last_error(); }
const char* odi_be_factory_message(void) { return odi_get_last_error_message(); }
int odi_be_cuda_available(void) { return odi::cuda_backend_available() ? 1 : 0; }

void odi_be_destroy(void* be) { delete static_cast<odi::Backend*>(be); }

int odi_be_matmul(void* be, void* out, int out_ndim, const int64_t* out_shape, const void* a, int a_dtype,
                  int a_ndim, const int64_t* a_shape, const void* b, int b_dtype, int b_ndim,
                  const int64_t* b_shape) {
  try {
    odi::Tensor o = view(out, ODI_DTYPE_F32, out_ndim, out_shape);
    static_cast<odi::Backend*>(be)->matmul(o, view(a, a_dtype, a_ndim, a_shape), view(b, b_dtype, b_ndim, b_shape));
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_quantized_matmul(void* be, void* out, int out_ndim, const int64_t* out_shape, const void* a,
                            int a_ndim, const int64_t* a_shape, const void* b, int b_dtype, int b_ndim,
                            const int64_t* b_shape) {
  try {
    odi::Tensor o = view(out, ODI_DTYPE_F32, out_ndim, out_shape);
    static_cast<odi::Backend*>(be)->quantized_matmul(o, view(a, ODI_DTYPE_F32, a_ndim, a_shape),
                                                    view(b, b_dtype, b_ndim, b_shape));
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_dequantize(void* be, float* out, const void* x, int x_dtype, int x_ndim, const int64_t* x_shape) {
  try {
    odi::Tensor xv = view(x, x_dtype, x_ndim, x_shape);
    const int64_t n = xv.numel();
    odi::Tensor o(out, {n}, ODI_DTYPE_F32);
    static_cast<odi::Backend*>(be)->dequantize(o, xv);
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_sync(void* be) {
  try {
    static_cast<odi::Backend*>(be)->sync();
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_supports_dtype(void* be, int dtype) {
  return static_cast<odi::Backend*>(be)->supports_dtype((odi_dtype_t)dtype) ? 1 : 0;
}

// type(), name(), device_info(), used_memory(), available_memory().
int odi_be_info(void* be, int* type, char* name, size_t name_len, char* info, size_t info_len, size_t* used,
                size_t* avail) {
  try {
    auto* b = static_cast<odi::Backend*>(be);
    if (type) *type = (int)b->type();
    if (name && name_len) std::snprintf(name, name_len, "%s", b->name().c_str());
    if (info && info_len) std::snprintf(info, info_len, "%s", b->device_info().c_str());
    if (used) *used = b->used_memory();
    if (avail) *avail = b->available_memory();
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

// Weights held in HBM by a CUDABackend; -1 for any other backend.
// GGUF files through the reference's own parser (gguf_parser.cpp): open
// (memory-mapped, as Model::Model does), the tensor views Context gets
// from Model::get_tensor, close.  NULL / non-zero on failure.
void* odi_be_gguf_open(const char* path) {
  try {
    std::unique_ptr<odi::GGUFFile> f = odi::GGUFFile::open(path, true);
    if (!f) {
      t_err = std::string("GGUFFile::open failed for ") + (path ? path : "(null)");
      return nullptr;
    }
    return f.release();
  } catch (const std::exception& e) {
    caught(e.what());
  }
  return nullptr;
}

void odi_be_gguf_close(void* f) { delete static_cast<odi::GGUFFile*>(f); }

int64_t odi_be_gguf_tensor_count(void* f) { return (int64_t) static_cast<odi::GGUFFile*>(f)->tensor_count(); }

// The view of tensor `name`: data pointer into the mapping, odi dtype, ndim
// and up to 4 dims (GGUF order).
int odi_be_gguf_tensor(void* f, const char* name, const void** data, int* dtype, int* ndim, int64_t* shape) {
  try {
    const odi::Tensor t = static_cast<odi::GGUFFile*>(f)->load_tensor(name);
    if (!t.is_valid()) return caught((std::string("no tensor ") + name).c_str());
    if (t.ndim() > 4) return caught("tensor has more than 4 dimensions");
    *data = t.data();
    *dtype = (int)t.dtype();
    *ndim = (int)t.ndim();
    for (int i = 0; i < (int)t.ndim(); ++i) shape[i] = t.shape(i);
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

// The loader hook on a CUDA backend: CUDABackend::upload_model(file).
int odi_be_upload_model(void* be, void* f, int64_t* n_uploaded) {
  try {
    auto* cuda = dynamic_cast<odi::CUDABackend*>(static_cast<odi::Backend*>(be));
    if (!cuda) return caught("upload_model: not a CUDA backend");
    const size_t n = cuda->upload_model(*static_cast<odi::GGUFFile*>(f));
    if (n_uploaded) *n_uploaded = (int64_t)n;
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int64_t odi_be_cached_weights(void* be) {
  auto* c = dynamic_cast<odi::CUDABackend*>(static_cast<odi::Backend*>(be));
  return c ? (int64_t)c->cached_weights() : -1;
}

// The decode step of a GGUF Llama model (CUDABackend::create_decoder):
// NULL on failure (message in odi_be_last_error).
void* odi_be_decoder_from_gguf(void* be, void* file, int ctx, int max_record) {
  try {
    auto* cb = dynamic_cast<odi::CUDABackend*>(static_cast<odi::Backend*>(be));
    if (!cb) {
      t_err = "not a CUDA backend";
      return nullptr;
    }
    return cb->create_decoder(*static_cast<odi::GGUFFile*>(file), ctx, max_record).release();
  } catch (const std::exception& e) {
    caught(e.what());
  }
  return nullptr;
}

void odi_be_decoder_free(void* dec) { delete static_cast<odi::CudaDecoder*>(dec); }

int odi_be_decoder_reset(void* dec, int token, int pos, int clear_cache) {
  try {
    static_cast<odi::CudaDecoder*>(dec)->reset(token, pos, clear_cache != 0);
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_decoder_prefill(void* dec, const int32_t* tokens, int n, int pos0) {
  try {
    static_cast<odi::CudaDecoder*>(dec)->prefill(std::vector<int32_t>(tokens, tokens + n), pos0);
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_decoder_generate(void* dec, int n, int32_t* out) {
  try {
    const std::vector<int32_t> t = static_cast<odi::CudaDecoder*>(dec)->generate(n);
    std::copy(t.begin(), t.end(), out);
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_decoder_time(void* dec, int n, float* ms) {
  try {
    *ms = static_cast<odi::CudaDecoder*>(dec)->time_steps(n);
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_decoder_logits(void* dec, float* out) {
  try {
    const std::vector<float> v = static_cast<odi::CudaDecoder*>(dec)->logits();
    std::copy(v.begin(), v.end(), out);
    return 0;
  } catch (const std::exception& e) {
    return caught(e.what());
  }
}

int odi_be_decoder_config(void* dec, int* fields /* layers hidden heads kv_heads head_dim ffn vocab ctx */) {
  const odi_cuda_decoder_config& c = static_cast<odi::CudaDecoder*>(dec)->config();
  const int v[8] = {c.layers, c.hidden, c.heads, c.kv_heads, c.head_dim, c.ffn, c.vocab, c.ctx};
  std::copy(v, v + 8, fields);
  return 0;
}

}  // extern "C"
