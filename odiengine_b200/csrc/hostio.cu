// hostio.cu -- transfers between page-locked host buffers and the device
// for the host-buffer products (odi_cuda_matmul_host, _async): x pulled in
// ahead of its product, queued products' y gathered out in one launch.
#include "internal.h"

namespace odi_cuda {

// Host activations into a device buffer, read by the SMs from page-locked
// host memory through its device address.  Each thread issues its first
// PULL_AHEAD loads before the programmatic dependency wait -- host memory is
// not written by any kernel, so those PCIe round trips overlap the previous
// kernel on the stream -- and stores only after it, since that kernel (or
// an earlier one) may still read the buffer.  The wait also orders every
// earlier kernel before the stores: each product kernel on this path waits
// for its own predecessor, so completion is transitive down the stream.
constexpr int PULL_AHEAD = 2;
constexpr int PULL_BLOCK = 128;

template <typename T>
__global__ void __launch_bounds__(PULL_BLOCK) pull_host_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                               int64_t n) {
  pdl_launch_dependents();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  T v[PULL_AHEAD];
#pragma unroll
  for (int u = 0; u < PULL_AHEAD; ++u)
    if (i0 + u * stride < n) v[u] = src[i0 + u * stride];
  pdl_wait();
#pragma unroll
  for (int u = 0; u < PULL_AHEAD; ++u)
    if (i0 + u * stride < n) dst[i0 + u * stride] = v[u];
  for (int64_t i = i0 + PULL_AHEAD * stride; i < n; i += stride) dst[i] = src[i];
}

cudaError_t launch_pull_host(const void* src_dev_view, void* dst, size_t bytes, bool pdl, cudaStream_t stream) {
  if (bytes == 0) return cudaSuccess;
  if (bytes & 3) return cudaErrorInvalidValue;
  const bool v16 = ((reinterpret_cast<uintptr_t>(src_dev_view) | reinterpret_cast<uintptr_t>(dst) | bytes) & 15) == 0;
  const int64_t n = (int64_t)(bytes / (v16 ? 16 : 4));
  int64_t g = (n + (int64_t)PULL_BLOCK * PULL_AHEAD - 1) / ((int64_t)PULL_BLOCK * PULL_AHEAD);
  if (g > 148 * 4) g = 148 * 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g);
  cfg.blockDim = dim3(PULL_BLOCK);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (v16)
    return cudaLaunchKernelEx(&cfg, pull_host_kernel<uint4>, static_cast<const uint4*>(src_dev_view),
                              static_cast<uint4*>(dst), n);
  return cudaLaunchKernelEx(&cfg, pull_host_kernel<uint32_t>, static_cast<const uint32_t*>(src_dev_view),
                            static_cast<uint32_t*>(dst), n);
}

// Queued products' outputs, parked in a device ring by the products
// themselves, copied to their page-locked host buffers: one CTA per output.
// Kernels that store into host memory cost more per launch in a stream than
// device-only ones, so the products stay device-only and one launch per
// batch does the host stores.  The wait orders the reads of the ring after
// the products that wrote it.
__global__ void __launch_bounds__(256) gather_to_host_kernel(const uint8_t* __restrict__ ring, const GatherTable t) {
  pdl_wait();
  pdl_launch_dependents();
  const int e = blockIdx.x;
  if (e >= t.n) return;
  const uint8_t* src = ring + (size_t)t.off16[e] * 16;
  uint8_t* dst = reinterpret_cast<uint8_t*>(t.dst[e]);
  const uint32_t nb = t.bytes[e];
  if (((reinterpret_cast<uintptr_t>(dst) | nb) & 15) == 0) {
    for (uint32_t i = 16 * threadIdx.x; i < nb; i += 16 * blockDim.x)
      *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + i);
  } else {
    for (uint32_t i = 4 * threadIdx.x; i < nb; i += 4 * blockDim.x)
      *reinterpret_cast<uint32_t*>(dst + i) = *reinterpret_cast<const uint32_t*>(src + i);
  }
}

cudaError_t launch_gather_to_host(const void* ring, const GatherTable& t, bool pdl, cudaStream_t stream) {
  if (t.n <= 0) return cudaSuccess;
  if (t.n > GATHER_MAX) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(t.n);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gather_to_host_kernel, static_cast<const uint8_t*>(ring), t);
}

}  // namespace odi_cuda
