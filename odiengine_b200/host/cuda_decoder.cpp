// cuda_decoder.cpp -- odi::CudaDecoder (see cuda_decoder.hpp).
#include "cuda_decoder.hpp"

#include <cstring>
#include <stdexcept>
#include <string>

#include "format/gguf_parser.hpp"

namespace odi {

namespace {

[[noreturn]] void raise(const std::string& what, int rc) {
  const char* e = odi_cuda_last_error();
  throw std::runtime_error(what + ": " + ((e && *e) ? e : "error") + " (status " + std::to_string(rc) + ")");
}

void ck(int rc, const std::string& what) {
  if (rc != ODI_CUDA_OK) raise(what, rc);
}

// A quantized weight view of the file: its GGUF blocks, [K, N] (K contiguous).
struct View {
  const uint8_t* data;
  int dtype;
  int64_t K, N;
  size_t row_bytes;
};

View quant_view(const GGUFFile& f, const std::string& name) {
  const Tensor t = f.load_tensor(name);
  if (!t.is_valid() || t.ndim() != 2 || !dtype_is_quantized(t.dtype()) || odi_cuda_supports_dtype(t.dtype()) != 1)
    throw std::runtime_error("CudaDecoder: " + name + " is missing or not a quantized type the GPU computes");
  const int64_t K = t.shape(0), N = t.shape(1);
  const int64_t bytes = odi_cuda_gguf_bytes((int)t.dtype(), N, K);
  return View{static_cast<const uint8_t*>(t.data()), (int)t.dtype(), K, N, (size_t)(bytes / N)};
}

std::vector<float> f32_values(const GGUFFile& f, const std::string& name, int64_t n) {
  const Tensor t = f.load_tensor(name);
  if (!t.is_valid() || t.dtype() != ODI_DTYPE_F32 || t.numel() != n)
    throw std::runtime_error("CudaDecoder: " + name + " is missing or not fp32 with " + std::to_string(n) + " values");
  std::vector<float> v((size_t)n);
  std::memcpy(v.data(), t.data(), (size_t)n * sizeof(float));
  return v;
}

}  // namespace

std::unique_ptr<CudaDecoder> CudaDecoder::from_gguf(const GGUFFile& file, int ctx, int max_record) {
  const GGUFModelInfo& mi = file.model_info();
  std::unique_ptr<CudaDecoder> d(new CudaDecoder);
  odi_cuda_decoder_config& c = d->cfg_;
  c.layers = (int)mi.block_count;
  c.hidden = (int)mi.embedding_length;
  c.heads = (int)mi.attention_head_count;
  c.kv_heads = (int)(mi.attention_head_count_kv ? mi.attention_head_count_kv : mi.attention_head_count);
  c.head_dim = (int)(mi.rope_dimension_count ? mi.rope_dimension_count : (c.heads ? c.hidden / c.heads : 0));
  c.ffn = (int)mi.feed_forward_length;
  c.ctx = ctx > 0 ? ctx : (int)mi.context_length;
  c.eps = mi.attention_layer_norm_rms_epsilon;
  c.theta = mi.rope_freq_base;
  if (c.layers < 1 || c.hidden < 1 || c.heads < 1 || c.ffn < 1 || c.ctx < 1)
    throw std::runtime_error("CudaDecoder: the file's hyper-parameters are incomplete");
  const View q0 = quant_view(file, "blk.0.attn_q.weight");
  const View d0 = quant_view(file, "blk.0.ffn_down.weight");
  c.attn_dtype = q0.dtype;
  c.down_dtype = d0.dtype;
  const View out = quant_view(file, "output.weight");
  c.vocab = (int)out.N;
  const int64_t E = c.hidden, F = c.ffn, qd = (int64_t)c.heads * c.head_dim, kvd = (int64_t)c.kv_heads * c.head_dim;

  auto upload_buf = [&](const std::vector<float>& v) {
    void* p = nullptr;
    ck(odi_cuda_buffer_upload(v.data(), v.size() * sizeof(float), &p), "CudaDecoder: upload");
    d->buffers_.push_back(p);
    return static_cast<const float*>(p);
  };
  auto upload_weight = [&](const std::vector<uint8_t>& blocks, int dtype, int64_t N, int64_t K) {
    odi_cuda_weight* w = nullptr;
    ck(odi_cuda_weight_upload(blocks.data(), dtype, N, K, &w), "CudaDecoder: weight upload");
    d->weights_.push_back(w);
    return odi_cuda_weight_data(w);
  };
  auto expect = [&](const View& v, const std::string& name, int dtype, int64_t N, int64_t K) {
    if (v.dtype != dtype || v.N != N || v.K != K)
      throw std::runtime_error("CudaDecoder: " + name + " has an unexpected type or shape");
  };
  // weights stacked by GGUF block rows (rows are contiguous runs of blocks)
  auto stacked = [&](const std::vector<std::pair<std::string, int64_t>>& parts, int dtype, int64_t K) {
    std::vector<uint8_t> buf;
    for (const auto& p : parts) {
      const View v = quant_view(file, p.first);
      expect(v, p.first, dtype, p.second, K);
      buf.insert(buf.end(), v.data, v.data + v.row_bytes * (size_t)v.N);
    }
    return buf;
  };

  std::vector<odi_cuda_decoder_layer> layers((size_t)c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    odi_cuda_decoder_layer& L = layers[(size_t)l];
    L.attn_norm = upload_buf(f32_values(file, p + "attn_norm.weight", E));
    L.ffn_norm = upload_buf(f32_values(file, p + "ffn_norm.weight", E));
    L.wqkv = upload_weight(stacked({{p + "attn_q.weight", qd}, {p + "attn_k.weight", kvd}, {p + "attn_v.weight", kvd}},
                                   c.attn_dtype, E),
                           c.attn_dtype, qd + 2 * kvd, E);
    L.wo = upload_weight(stacked({{p + "attn_output.weight", E}}, c.attn_dtype, qd), c.attn_dtype, E, qd);
    // gate|up interleaved: 64-row tile t holds gate rows 32t.. and up rows 32t..
    {
      const View g = quant_view(file, p + "ffn_gate.weight"), u = quant_view(file, p + "ffn_up.weight");
      expect(g, p + "ffn_gate.weight", c.attn_dtype, F, E);
      expect(u, p + "ffn_up.weight", c.attn_dtype, F, E);
      if (F % 32) throw std::runtime_error("CudaDecoder: ffn length must be a multiple of 32");
      std::vector<uint8_t> buf(g.row_bytes * (size_t)(2 * F));
      for (int64_t r = 0; r < 2 * F; ++r) {
        const int64_t t = r / 64, i = r % 64;
        const uint8_t* src = i < 32 ? g.data + (size_t)(32 * t + i) * g.row_bytes
                                    : u.data + (size_t)(32 * t + i - 32) * u.row_bytes;
        std::memcpy(buf.data() + (size_t)r * g.row_bytes, src, g.row_bytes);
      }
      L.wgu = upload_weight(buf, c.attn_dtype, 2 * F, E);
    }
    L.wdown = upload_weight(stacked({{p + "ffn_down.weight", E}}, c.down_dtype, F), c.down_dtype, E, F);
  }
  const float* embd = upload_buf(f32_values(file, "token_embd.weight", (int64_t)c.vocab * E));
  const float* onorm = upload_buf(f32_values(file, "output_norm.weight", E));
  expect(out, "output.weight", c.down_dtype, c.vocab, E);
  const void* ow = upload_weight(stacked({{"output.weight", c.vocab}}, c.down_dtype, E), c.down_dtype, c.vocab, E);
  ck(odi_cuda_decoder_create(&c, embd, layers.data(), onorm, ow, max_record, &d->dec_), "CudaDecoder");
  return d;
}

CudaDecoder::~CudaDecoder() {
  if (dec_) odi_cuda_decoder_free(dec_);
  for (odi_cuda_weight* w : weights_) odi_cuda_weight_free(w);
  for (void* p : buffers_) odi_cuda_buffer_free(p);
}

void CudaDecoder::reset(int token, int pos, bool clear_cache) {
  ck(odi_cuda_decoder_reset(dec_, token, pos, clear_cache ? 1 : 0), "CudaDecoder::reset");
}

void CudaDecoder::prefill(const std::vector<int32_t>& tokens, int pos0) {
  ck(odi_cuda_decoder_prefill(dec_, tokens.data(), (int)tokens.size(), pos0), "CudaDecoder::prefill");
}

std::vector<int32_t> CudaDecoder::generate(int n) {
  std::vector<int32_t> out((size_t)(n > 0 ? n : 0));
  ck(odi_cuda_decoder_generate(dec_, n, out.data()), "CudaDecoder::generate");
  return out;
}

float CudaDecoder::time_steps(int n) {
  float ms = 0.f;
  ck(odi_cuda_decoder_time(dec_, n, &ms), "CudaDecoder::time_steps");
  return ms;
}

std::vector<float> CudaDecoder::logits() {
  std::vector<float> v((size_t)cfg_.vocab);
  ck(odi_cuda_decoder_logits(dec_, v.data()), "CudaDecoder::logits");
  return v;
}

int CudaDecoder::launches_per_step() const { return odi_cuda_decoder_launches_per_step(dec_); }

}  // namespace odi
