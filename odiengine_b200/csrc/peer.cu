// peer.cu -- arrival counters of the fused row-shard scatter.
//
// Every rank's GEMV stores its slice into all ranks' gathered buffers; the
// launch's last CTA then adds one arrival to its own slot of every rank's
// counter array (release, system scope; qgemv_device.cuh signal_peers).
// Counters only grow.  Before the gathered product is used, wait_peers_kernel on each
// rank waits until counter[src] >= consumed[src] + inc[src] for every source
// rank (acquire, system scope), then advances consumed[src]: the state lives
// on the device, so a CUDA graph replaying the pair stays in step.
//
// The wait is bounded (PeerWait::timeout_ns of the device's global timer, one
// second by default): a rank that never arrives sets ERR_PEER_WAIT in the
// error word and the kernel returns.  The consumed counts advance all the
// same, so the host, which must treat the gathered product as invalid, can
// keep the pair in step once the late rank's arrival lands.
#include "internal.h"

namespace odi_cuda {

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void wait_peers_kernel(const unsigned long long* __restrict__ cnt, unsigned long long* __restrict__ consumed,
                                  const PeerWait w, int* err) {
  // The next kernel may start (and stream its weights) while this one
  // waits; its own griddepcontrol.wait still orders it after this kernel.
  pdl_launch_dependents();
  const int r = threadIdx.x;
  if (r < w.n) {
    const unsigned long long target = consumed[r] + w.inc[r];
    if (ld_acquire_sys(cnt + r) < target) {
      const unsigned long long t0 = global_ns();
      while (ld_acquire_sys(cnt + r) < target) {
        if (global_ns() - t0 > w.timeout_ns) {
          if (err) atomicOr(err, ERR_PEER_WAIT);
          break;
        }
        __nanosleep(64);
      }
    }
    consumed[r] = target;
  }
  __syncthreads();
}

cudaError_t launch_wait_peers(const unsigned long long* cnt, unsigned long long* consumed, const PeerWait& w,
                              int* err, cudaStream_t s) {
  wait_peers_kernel<<<1, 32, 0, s>>>(cnt, consumed, w, err);
  return cudaGetLastError();
}

}  // namespace odi_cuda
