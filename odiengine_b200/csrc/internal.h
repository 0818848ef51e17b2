// internal.h -- launchers shared between the kernel files and the C ABI.
#pragma once

#include "common.cuh"

namespace odi_cuda {

cudaError_t launch_act_quant(const float* x, int64_t M, int64_t K, uint8_t* tiles, uint8_t* blocks,
                             bool pdl, cudaStream_t stream);
cudaError_t launch_act_pack_f32(const float* x, int64_t M, int64_t K, float* tiles, bool pdl,
                                cudaStream_t stream);
cudaError_t launch_repack(int dt, const void* gguf, void* tiled, int64_t N, int64_t K, cudaStream_t s);
cudaError_t launch_unpack(int dt, const void* tiled, void* gguf, int64_t N, int64_t K, cudaStream_t s);
cudaError_t launch_dequant(int dt, const void* tiled, float* out, int64_t N, int64_t K, cudaStream_t s);
cudaError_t launch_quant_weights(int dt, const float* w, void* out, int64_t N, int64_t K, cudaStream_t s);

// Work split of the streaming GEMV: the G*KB units of a weight, in tile-major
// order, are cut into P contiguous ranges, one per CTA (stream-K style).
// Row tiles cut between CTAs are finished by a deterministic fixup: each
// contributor writes its partial sums to a slot, the last to arrive (by an
// atomic counter) adds the slots in CTA order and writes y.
struct GemvPlan {
  int G, KB, U, P;
  int maxc;          // max contributors to one row tile
  int stages;        // ring depth
  int stage_bytes;   // weights unit + activation slice, 128-aligned
  int smem_bytes;    // dynamic shared memory per CTA
  int mt;            // tokens per pass (template instantiation)
};

struct GemvArgs {
  const uint8_t* w;   // tiled weight
  const uint8_t* act; // activation tiles (span-major, M_total tokens)
  float* y;           // output [M_total][N] (already offset to the first token of the pass)
  float* partial;     // fixup slots
  int* counters;      // fixup counters, one per row tile (zero between calls)
  int* err;           // device error word
  int64_t N;
  int M;              // tokens in this pass (<= mt)
  int M_total;        // tokens in the activation tiles
  int m0;             // first token of this pass
};

// Plan for dtype / tokens-per-pass / fp32-activation mode on the current device.
GemvPlan make_gemv_plan(int dt, int64_t N, int64_t K, int M, bool f32act, int num_sms);
size_t gemv_partial_floats(const GemvPlan& p, int M);
cudaError_t launch_gemv(int dt, bool f32act, const GemvPlan& plan, const GemvArgs& a, bool pdl,
                        cudaStream_t s);

}  // namespace odi_cuda
