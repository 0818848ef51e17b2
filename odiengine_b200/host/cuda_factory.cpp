// cuda_factory.cpp -- what the reference's backend factory returns for
// ODI_BACKEND_CUDA once this backend is integrated.
//
// src/compute/cpu/cpu_backend.cpp:1010-1013 today hands out a CPUBackend for
// ODI_BACKEND_CUDA (a TODO); is_backend_available (cpu_backend.cpp:1040-1063)
// answers true at compile time.  With the integration patch those cases call
// create_cuda_backend / cuda_backend_available instead: a CUDA request gets
// the CUDA backend or nothing -- never a CPU backend in its place.
#include <exception>
#include <memory>

#include "cuda_backend.hpp"

namespace odi {

std::unique_ptr<Backend> create_cuda_backend(int num_threads) {
  try {
    return std::make_unique<CUDABackend>(num_threads, 0);
  } catch (const std::exception& e) {
    // No usable sm_100 device (or its initialisation failed): the engine
    // sees a null backend (engine.cpp:18-21) and the reason is recorded the
    // way the C API records errors (odi_engine.cpp:72-80).
    odi_set_error(ODI_ERROR_BACKEND_UNAVAILABLE, e.what());
    return nullptr;
  }
}

bool cuda_backend_available() {
  return odi_cuda_device_count() > 0 && odi_cuda_init(0) == ODI_CUDA_OK;
}

}  // namespace odi
