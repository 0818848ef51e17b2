// ref_harness.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C-callable wrapper around the UNMODIFIED reference CPU backend
// (src/compute/cpu/cpu_backend.cpp + src/tensor/tensor.cpp of ODIEngine),
// compiled from the reference tree by oracle/Makefile into oracle/_ref/.
// It calls odi::CPUBackend::matmul (cpu_backend.cpp:177-227) exactly as
// Context does (context.cpp:152,188-190): a = fp32 [M,K] view, b = packed
// GGUF weight view of shape [K,N] and the weight dtype, out = fp32 [M,N].
#include "compute/cpu/cpu_backend.hpp"
#include "tensor/tensor.hpp"

#include <cstdio>
#include <cstring>
#include <exception>

static thread_local char g_err[512];

extern "C" {

// The two C symbols the reference backend needs when odi_engine.cpp is not
// linked (declared at include/odi/odi_error.h:58 and odi_types.h:187).
void odi_set_error(odi_error_t, const char* message) {
  std::snprintf(g_err, sizeof g_err, "%s", message ? message : "");
}
const char* odi_dtype_name(odi_dtype_t) { return "?"; }

const char* ref_last_error(void) { return g_err; }

// Returns 0 on success, 1 if the reference threw (message in ref_last_error).
int ref_matmul(int dtype, float* out, const float* a, const void* b, long long M, long long K,
               long long N, int nthreads) {
  try {
    odi::CPUBackend backend(nthreads);
    odi::Tensor ta(const_cast<float*>(a), {M, K}, ODI_DTYPE_F32);
    odi::Tensor tb(const_cast<void*>(b), {K, N}, static_cast<odi_dtype_t>(dtype));
    odi::Tensor to(out, {M, N}, ODI_DTYPE_F32);
    backend.matmul(to, ta, tb);
    return 0;
  } catch (const std::exception& e) {
    std::snprintf(g_err, sizeof g_err, "%s", e.what());
    return 1;
  }
}

// The reference's CPUBackend::dequantize (cpu_backend.cpp:625-648) of n
// values: x a packed block buffer, out fp32 [n].  0 / 1 as ref_matmul.
int ref_dequantize(int dtype, float* out, const void* x, long long n) {
  try {
    odi::CPUBackend backend(1);
    odi::Tensor tx(const_cast<void*>(x), {n}, static_cast<odi_dtype_t>(dtype));
    odi::Tensor to(out, {n}, ODI_DTYPE_F32);
    backend.dequantize(to, tx);
    return 0;
  } catch (const std::exception& e) {
    std::snprintf(g_err, sizeof g_err, "%s", e.what());
    return 1;
  }
}

// Timing helper: runs the reference matmul `reps` times on one backend object
// and returns the total seconds (steady clock), or -1 if it threw.
double ref_matmul_time(int dtype, float* out, const float* a, const void* b, long long M,
                       long long K, long long N, int nthreads, int reps);
}

#include <chrono>
double ref_matmul_time(int dtype, float* out, const float* a, const void* b, long long M,
                       long long K, long long N, int nthreads, int reps) {
  try {
    odi::CPUBackend backend(nthreads);
    odi::Tensor ta(const_cast<float*>(a), {M, K}, ODI_DTYPE_F32);
    odi::Tensor tb(const_cast<void*>(b), {K, N}, static_cast<odi_dtype_t>(dtype));
    odi::Tensor to(out, {M, N}, ODI_DTYPE_F32);
    auto t0 = std::chrono::steady_clock::now();
    for (int r = 0; r < reps; ++r) backend.matmul(to, ta, tb);
    auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(t1 - t0).count();
  } catch (const std::exception& e) {
    std::snprintf(g_err, sizeof g_err, "%s", e.what());
    return -1.0;
  }
}
