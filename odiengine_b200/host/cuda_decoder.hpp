// cuda_decoder.hpp -- odi::CudaDecoder: a GGUF Llama model loaded once into
// HBM and decoded one token per call on the device (include/odi_cuda.h,
// odi_cuda_decoder_*), for an engine whose Context::forward
// (src/core/context.cpp:84-282) hands a whole decode step to the backend
// instead of issuing one Backend call per operation.
//
// Loading follows the reference's names and shapes (blk.N.attn_q/k/v/output,
// ffn_gate/up/down, attn_norm, ffn_norm, token_embd, output_norm, output;
// GGUFModelInfo for the hyper-parameters, gguf_parser.hpp:64-87).  Q, K and V
// are stacked into one weight and gate and up interleaved 32 rows each per
// 64-row tile (the layout the decode step's epilogues need), on the host,
// before each stacked weight is uploaded once.  Errors throw
// std::runtime_error, as the reference's backends do.
#pragma once

#include <cstdint>
#include <memory>
#include <vector>

#include "odi_cuda.h"

namespace odi {

class GGUFFile;

class CudaDecoder {
 public:
  // The model of `file` on the current device with a KV cache of `ctx`
  // positions (0: the file's context_length); up to max_record generated
  // tokens are kept on the device between resets.
  static std::unique_ptr<CudaDecoder> from_gguf(const GGUFFile& file, int ctx = 0, int max_record = 4096);
  ~CudaDecoder();
  CudaDecoder(const CudaDecoder&) = delete;
  CudaDecoder& operator=(const CudaDecoder&) = delete;

  const odi_cuda_decoder_config& config() const { return cfg_; }
  // Next step reads `token` at `pos`; clear_cache starts a new sequence.
  void reset(int token, int pos, bool clear_cache);
  // The prompt into the KV cache, one step per token from position pos0.
  void prefill(const std::vector<int32_t>& tokens, int pos0);
  // n greedy steps from the current state.
  std::vector<int32_t> generate(int n);
  // n greedy steps timed on the device, in milliseconds.
  float time_steps(int n);
  std::vector<float> logits();
  int launches_per_step() const;

 private:
  CudaDecoder() = default;
  odi_cuda_decoder_config cfg_{};
  std::vector<odi_cuda_weight*> weights_;
  std::vector<void*> buffers_;
  odi_cuda_decoder* dec_ = nullptr;
};

}  // namespace odi
