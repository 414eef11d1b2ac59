// checkpoint.hpp -- MLX-format model directories (config.json + *.safetensors) read into
// the stacked per-layer arrays libflashmoe's fm_moe_weights points at, in C++ for a C++
// server.  Same rules as the reference's loader for the MoE layers:
//
//   load_config         LlamaModel::load_config (server/src/model.cpp:105-142) and the
//                       Nemotron-H keys (nemotron_h.cpp:244-261), with their defaults
//   Checkpoint          LlamaModel::load_weights (model.cpp:148-184): every *.safetensors
//                       file of the directory in sorted order, later files overriding
//                       earlier keys, a leading "model." (or Nemotron-H's "backbone.",
//                       nemotron_h.cpp:333-337) stripped from every key
//   moe_layer(i)        build_moe_weight_cache (model.cpp:368-470): layers.i.mlp.gate.weight
//                       marks an MoE layer; experts.E.{gate,up,down}_proj.* stacked on a new
//                       leading axis (mlx-lm's pre-stacked switch_mlp.* taken as is), the
//                       shared expert shared_expert.{gate,up,down}_proj.* and its gate
//                       shared_expert_gate.weight
//   sigmoid_moe_layer   NemotronHModel's 'E' layers (pattern nemotron_h.cpp:272-285, weights
//                       444-468): layers.i.mixer.{gate.weight, gate.e_score_correction_bias,
//                       switch_mlp.fc1/fc2, shared_experts.up_proj/down_proj}
//
// Files are memory-mapped; a layer's tensors are copied out when it is stacked.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "flashmoe.h"

namespace flashmoe {

// The ModelConfig fields (server/include/flashmlx/model.h) the decoder uses, with
// LlamaModel::load_config's defaults (server/src/model.cpp:105-142).
struct ModelConfig {
  int hidden_size = 4096;
  int intermediate_size = 14336;
  int num_hidden_layers = 32;
  int num_attention_heads = 32;
  int num_key_value_heads = 8;
  int head_dim = 0;  // 0: hidden_size / num_attention_heads
  int vocab_size = 128256;
  float rms_norm_eps = 1e-5f;
  float rope_theta = 10000.0f;
  bool tie_word_embeddings = true;
  int quant_bits = 0;  // 0 = not quantized
  int quant_group_size = 64;
  int num_experts = 0;
  int num_experts_per_tok = 0;
  int moe_intermediate_size = 0;
  int shared_expert_intermediate_size = 0;
  bool norm_topk_prob = false;
  // Nemotron-H / DeepSeek-style routing
  int n_routed_experts = 0;
  int n_shared_experts = 1;
  int moe_shared_expert_intermediate_size = 0;
  float routed_scaling_factor = 1.0f;
  int n_group = 1;
  int topk_group = 1;
  std::string hybrid_override_pattern;

  // a Nemotron-H model: MoE layers are the 'E' entries of hybrid_override_pattern
  bool sigmoid_routed() const { return hybrid_override_pattern.find('E') != std::string::npos; }
  int experts() const { return num_experts ? num_experts : n_routed_experts; }
  int attn_head_dim() const { return head_dim > 0 ? head_dim : hidden_size / num_attention_heads; }
  int shared_inter() const {
    if (shared_expert_intermediate_size) return shared_expert_intermediate_size;
    return n_shared_experts ? moe_shared_expert_intermediate_size : 0;
  }
  // the libflashmoe description of one MoE layer (bf16 router and shared-expert gate)
  fm_moe_config moe_config() const;
  // the variant description for a sigmoid-routed model (fm_moe_block_variant), without the
  // per-layer correction bias
  fm_moe_variant variant() const;
};

ModelConfig load_config(const std::string& model_dir);

// One tensor of a mapped safetensors file.
struct TensorView {
  std::string dtype;  // safetensors name: "BF16", "U32", "F32", ...
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t numel() const;
};

class SafetensorsFile {
 public:
  explicit SafetensorsFile(const std::string& path);
  ~SafetensorsFile();
  SafetensorsFile(const SafetensorsFile&) = delete;
  SafetensorsFile& operator=(const SafetensorsFile&) = delete;
  const std::map<std::string, TensorView>& tensors() const { return tensors_; }

 private:
  void unmap();
  void* map_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, TensorView> tensors_;
};

// A quantized matrix (or a stack of them) copied out of the checkpoint.
struct HostQ {
  std::vector<uint32_t> w;
  std::vector<uint16_t> s;
  std::vector<uint16_t> b;  // empty: no biases
  std::vector<int64_t> w_shape, s_shape;
  bool has_biases() const { return !b.empty(); }
};

// One MoE layer in host memory, arrays in libflashmoe's layout (bf16 as uint16 bits).
// Sigmoid-routed layers keep fc1 in `up` and fc2 in `down`, as fm_moe_block_variant takes them.
struct HostLayer {
  bool sigmoid = false;
  std::vector<uint16_t> router_w;         // [E, H]
  std::vector<float> correction_bias;     // [E] (sigmoid routing), empty if absent
  HostQ gate, up, down;                   // [E, I, H], [E, I, H], [E, H, I]
  bool has_shared = false;
  HostQ shared_gate, shared_up, shared_down;  // [Is, H], [Is, H], [H, Is]
  std::vector<uint16_t> shared_expert_gate_w;  // [1, H]
};

class Checkpoint {
 public:
  explicit Checkpoint(const std::string& model_dir);
  const ModelConfig& config() const { return config_; }
  bool has(const std::string& key) const { return tensors_.count(key) != 0; }
  // the tensor under a stripped key; throws if absent or (dtype given) of another dtype
  const TensorView& get(const std::string& key, const char* dtype = nullptr) const;
  std::vector<int> moe_layers() const;
  HostLayer moe_layer(int i) const;          // Llama-family layer (softmax routing, SwiGLU)
  HostLayer sigmoid_moe_layer(int i) const;  // Nemotron-H 'E' layer

 private:
  HostQ qmatrix(const std::string& prefix) const;
  HostQ stacked(const std::string& mlp, const std::string& proj) const;
  void check_q(int i, const char* name, const HostQ& q, std::vector<int64_t> lead, int64_t n, int64_t k) const;

  std::string dir_;
  ModelConfig config_;
  std::vector<std::unique_ptr<SafetensorsFile>> files_;
  std::map<std::string, const TensorView*> tensors_;
};

}  // namespace flashmoe
