// shard.cu -- the row-sharded product behind the C ABI: an NCCL communicator
// of one process per GPU, and a product whose weight is split by output rows
// across the ranks, its slices all-gathered over NVLink.
//
// NCCL is opened at run time (dlopen of libnccl.so.2, the one the process
// already holds if any), so the library loads and runs single-GPU products
// on machines without it.  The communicator functions are the only users.
//
// The sharded product for rank r of g (shard of S rows, full N):
//   1. the streaming GEMV / tensor-core product of the rank's shard into its
//      slot of the gather buffer: slot r of [g][M][S] fp32;
//   2. ncclAllGather in place over the gather buffer (every rank's slot);
//   3. M = 1 and N = g * S: the buffer is y itself (no copy); otherwise a
//      permute kernel writes y [M][N] from [g][M][S], dropping the padding.
#include <dlfcn.h>

#include <nccl.h>

#include "internal.h"

namespace odi_cuda {

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static const NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_gather && a.error_string;
    return a;
  }();
  return api;
}

// y [M][N] from the rank-major gather buffer [g][M][S] (rows past N dropped).
__global__ void unshard_kernel(const float* __restrict__ src, float* __restrict__ y, int64_t M, int64_t N, int64_t S,
                               int g) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    const int64_t r = n / S, c = n - r * S;
    y[i] = src[(r * M + m) * S + c];
  }
}

}  // namespace

bool nccl_available() { return nccl().ok; }

int nccl_unique_id(void* out, const char** why) {
  const NcclApi& a = nccl();
  if (!a.ok) {
    *why = "libnccl.so.2 could not be loaded";
    return -1;
  }
  ncclUniqueId id;
  const ncclResult_t r = a.get_unique_id(&id);
  if (r != ncclSuccess) {
    *why = a.error_string(r);
    return -1;
  }
  memcpy(out, &id, sizeof id);
  return 0;
}

int nccl_comm_init(const void* id, int nranks, int rank, void** comm, const char** why) {
  const NcclApi& a = nccl();
  if (!a.ok) {
    *why = "libnccl.so.2 could not be loaded";
    return -1;
  }
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  ncclComm_t c = nullptr;
  const ncclResult_t r = a.comm_init_rank(&c, nranks, uid, rank);
  if (r != ncclSuccess) {
    *why = a.error_string(r);
    return -1;
  }
  *comm = c;
  return 0;
}

int nccl_comm_destroy(void* comm, const char** why) {
  const NcclApi& a = nccl();
  if (!a.ok || !comm) return 0;
  const ncclResult_t r = a.comm_destroy(static_cast<ncclComm_t>(comm));
  if (r != ncclSuccess) {
    *why = a.error_string(r);
    return -1;
  }
  return 0;
}

int nccl_all_gather_f32(const float* send, float* recv, size_t count, void* comm, cudaStream_t s, const char** why) {
  const NcclApi& a = nccl();
  const ncclResult_t r = a.all_gather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(comm), s);
  if (r != ncclSuccess) {
    *why = a.error_string(r);
    return -1;
  }
  return 0;
}

cudaError_t launch_unshard(const float* src, float* y, int64_t M, int64_t N, int64_t S, int g, cudaStream_t s) {
  int64_t blocks = (M * N + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  unshard_kernel<<<(unsigned)blocks, 256, 0, s>>>(src, y, M, N, S, g);
  return cudaGetLastError();
}

}  // namespace odi_cuda
