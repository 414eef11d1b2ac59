// moe_model.hpp -- the MoE layers of an MLX-format checkpoint on one GPU, answering the
// decoder layer's moe_block(x, layer) call through libflashmoe, for a C++ server.
//
// LlamaModel's layer (server/src/model.cpp:825-839) normalises the attention output and
// calls moe_block(normed, layer) when layer_is_moe_[layer] (model.cpp:253-266), else the
// dense MLP; NemotronHModel does the same for its 'E' layers (nemotron_h.cpp:1010-1106).
// MoEModel uploads every MoE layer once (the stacked weights of build_moe_weight_cache,
// model.cpp:368-470, in MLX's packed layout) and runs the call as fm_moe_block, or as
// fm_moe_block_variant (sigmoid routing, relu^2 experts) for a Nemotron-H checkpoint.
// Attention, norms and the dense MLP stay with the caller.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "checkpoint.hpp"
#include "device_store.hpp"
#include "flashmoe.hpp"

namespace flashmoe {

class MoEModel {
 public:
  // device: the CUDA device the weights live on; stream: the cudaStream_t the calls run
  // on (nullptr = legacy default); max_tokens > 0 sizes the workspace once, so calls of
  // up to that many tokens do not allocate; layers: the MoE layers to load (empty = all)
  MoEModel(const std::string& model_dir, int device = 0, void* stream = nullptr, int64_t max_tokens = 0,
           const std::vector<int>& layers = {});
  ~MoEModel();
  MoEModel(const MoEModel&) = delete;
  MoEModel& operator=(const MoEModel&) = delete;

  const ModelConfig& config() const { return config_; }
  const fm_moe_config& moe_config() const { return cfg_; }
  // layer_is_moe_[layer]: the layer has a router and its experts are loaded
  bool is_moe(int layer) const { return layers_.count(layer) != 0; }
  std::vector<int> moe_layers() const;
  Handle& handle() { return handle_; }

  // LlamaModel::moe_block(x, layer) / NemotronHModel::moe_block: x [T, hidden] bf16 on
  // the device -> y [T, hidden] bf16 on the device (16-byte aligned), asynchronous on
  // the handle's stream; throws Error on a rejected call
  void moe_block(const uint16_t* x, int64_t T, uint16_t* y, int layer);

 private:
  struct DeviceLayer {
    fm_moe_weights w{};
    const float* correction_bias = nullptr;
  };

  ModelConfig config_;
  fm_moe_config cfg_{};
  int device_ = 0;
  Handle handle_;
  std::map<int, DeviceLayer> layers_;
  DeviceStore store_;  // declared after handle_: freed first, after the destructor's sync
};

// Uploads one MoE layer into `store` and returns its fm_moe_weights (and, for a
// sigmoid-routed layer, the device correction bias in *correction_bias).
fm_moe_weights upload_moe_layer(DeviceStore& store, const HostLayer& L, const float** correction_bias);

}  // namespace flashmoe
