// decoder.hpp -- the reference's full decoder forward (LlamaModel with MoE layers,
// server/src/model.cpp) on libflashmoe, with greedy sampling.  One forward call:
//
//   x = embed(ids)                                            model.cpp:490-496
//   per layer:  normed = rms_norm(x)                          813-821
//               q, k, v = quantized_matmul(normed, W{q,k,v})   553-555
//               a = attention(q + bq, k + bk, v + bv)          557-635 (RoPE, cache, SDPA)
//               x = x + quantized_matmul(a, Wo); normed = rms_norm(x)        638-641, 824-827
//               m = moe_block(normed) (or the dense SwiGLU MLP) 829-836
//               x = x + m                                      838
//   logits = lm_head(rms_norm(x[:, -1]))                       499-520
//   next = argmax(logits)                                      sampling.cpp:5-7
//
// Each residual add is fused into the RMSNorm that follows it (fm_rms_norm), with the
// same bf16 rounding as the separate mx::add and mx::fast::rms_norm.  The final norm and
// lm_head run on each sequence's last position only.  All calls are asynchronous on one
// stream; the caches [B, n_kv, max_len, d] per layer live with the decoder.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "device_store.hpp"
#include "flashmoe.hpp"
#include "fmh.h"

namespace flashmoe {

class Checkpoint;
struct TensorView;

// Where a model directory keeps the decoder's tensors (host views into the mapped files),
// checked against its config: what Decoder::open uploads.  MoE layers are read with
// Checkpoint::moe_layer at upload.
struct QView {
  const TensorView* w = nullptr;
  const TensorView* s = nullptr;
  const TensorView* b = nullptr;
};
struct LayerPlan {
  const TensorView* in_norm = nullptr;
  const TensorView* post_norm = nullptr;
  QView q, k, v, o;
  const TensorView* q_bias = nullptr;
  const TensorView* k_bias = nullptr;
  const TensorView* v_bias = nullptr;
  const TensorView* q_norm = nullptr;
  const TensorView* k_norm = nullptr;
  bool is_moe = false;
  QView gate, up, down;
};
struct DecoderPlan {
  fmh_decoder_config cfg{};
  QView embed;                          // quantized embed_tokens, or
  const TensorView* embed_bf16 = nullptr;  // a bf16 table
  const TensorView* norm = nullptr;
  QView lm_head;
  std::vector<LayerPlan> layers;
};
DecoderPlan plan_decoder(const Checkpoint& ck);

class Decoder {
 public:
  // caller-owned device weights (the tables are copied and each layer's q, k and v
  // matrices into one fused matrix; the other weights are read in place)
  Decoder(const fmh_decoder_config& cfg, const fmh_weights& w, int device, int max_batch, int max_len,
          void* stream = nullptr);
  // an MLX-format model directory, loaded, uploaded and owned by the decoder
  static std::unique_ptr<Decoder> open(const std::string& model_dir, int device, int max_batch, int max_len,
                                       void* stream = nullptr);
  ~Decoder();
  Decoder(const Decoder&) = delete;
  Decoder& operator=(const Decoder&) = delete;

  const fmh_decoder_config& config() const { return cfg_; }
  // ids [B, L] device int32 -> next_ids [B] device int32; advances the offset by L
  void forward(const int32_t* ids, int B, int L, int32_t* next_ids);
  const uint16_t* logits() const { return logits_; }
  void copy_logits(uint16_t* dst, int B) const;
  int offset() const { return offset_; }
  void reset() { offset_ = 0; }
  void sync() const { handle_.sync(); }
  Handle& handle() { return handle_; }
  // greedy generation from host memory: prompt [B, L] -> [B, steps]; resets first
  std::vector<int32_t> generate(const int32_t* prompt, int B, int L, int steps);

 private:
  void qmm(const uint16_t* x, int64_t M, int K, const fm_qweight& w, int N, uint16_t* out);
  void validate() const;

  fmh_decoder_config cfg_;
  fmh_weights w_;
  std::vector<fmh_layer> layers_;
  int device_, max_batch_, max_len_;
  int offset_ = 0;
  cudaStream_t stream_ = nullptr;
  fm_attn_config attn_{};
  fm_attn_config attn_qkv_{};            // attn_ on the fused projection's rows (qkv_ld set)
  std::vector<fm_qweight> qkv_;          // per layer: q|k|v rows in one matrix (w == nullptr: separate)
  Handle handle_;
  DeviceStore bufs_;                     // activations, caches, token buffers
  std::unique_ptr<DeviceStore> owned_;   // weights loaded by open()
  uint16_t *x_ = nullptr, *normed_ = nullptr, *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *attn_out_ = nullptr,
           *o_ = nullptr, *mlp_ = nullptr, *gate_ = nullptr, *up_ = nullptr, *last_ = nullptr, *logits_ = nullptr,
           *qkv_out_ = nullptr;
  int32_t* tok_ = nullptr;               // [2][max_batch * max_len] generate()'s token ping-pong
  int32_t* gen_ = nullptr;               // [steps, max_batch] generate()'s output, grown on demand
  int64_t gen_cap_ = 0;
  std::vector<uint16_t*> cache_k_, cache_v_;
};

}  // namespace flashmoe
