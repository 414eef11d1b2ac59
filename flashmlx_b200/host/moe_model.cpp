// moe_model.cpp -- see moe_model.hpp.
#include "moe_model.hpp"

#include <algorithm>
#include <stdexcept>

namespace flashmoe {

fm_moe_weights upload_moe_layer(DeviceStore& store, const HostLayer& L, const float** correction_bias) {
  fm_moe_weights w{};
  w.router_w = store.u16(L.router_w);
  if (correction_bias) *correction_bias = nullptr;
  if (L.sigmoid) {
    w.up = store.q(L.up);      // fc1
    w.down = store.q(L.down);  // fc2
    if (L.has_shared) {
      w.shared_up = store.q(L.shared_up);
      w.shared_down = store.q(L.shared_down);
    }
    if (!L.correction_bias.empty() && correction_bias) *correction_bias = store.f32(L.correction_bias);
  } else {
    w.gate = store.q(L.gate);
    w.up = store.q(L.up);
    w.down = store.q(L.down);
    if (L.has_shared) {
      w.shared_gate = store.q(L.shared_gate);
      w.shared_up = store.q(L.shared_up);
      w.shared_down = store.q(L.shared_down);
      w.shared_expert_gate_w = store.u16(L.shared_expert_gate_w);
    }
  }
  return w;
}

MoEModel::MoEModel(const std::string& model_dir, int device, void* stream, int64_t max_tokens,
                   const std::vector<int>& layers)
    : device_(device), store_(device) {
  Checkpoint ck(model_dir);
  config_ = ck.config();
  cfg_ = config_.moe_config();
  std::vector<int> moe = ck.moe_layers();
  if (!layers.empty()) {
    for (int l : layers)
      if (std::find(moe.begin(), moe.end(), l) == moe.end())
        throw std::runtime_error("layer " + std::to_string(l) + " is not an MoE layer of " + model_dir);
    moe = layers;
    std::sort(moe.begin(), moe.end());
  }
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  handle_ = Handle(device_, stream);
  for (int i : moe) {
    const HostLayer L = config_.sigmoid_routed() ? ck.sigmoid_moe_layer(i) : ck.moe_layer(i);
    DeviceLayer d;
    d.w = upload_moe_layer(store_, L, &d.correction_bias);
    layers_[i] = d;
  }
  if (max_tokens > 0 && !layers_.empty()) handle_.reserve(cfg_, max_tokens);
}

MoEModel::~MoEModel() {
  // the handle's stream may still read the weights
  if (handle_) fm_sync_status(handle_.get());
}

std::vector<int> MoEModel::moe_layers() const {
  std::vector<int> out;
  for (const auto& kv : layers_) out.push_back(kv.first);
  return out;
}

void MoEModel::moe_block(const uint16_t* x, int64_t T, uint16_t* y, int layer) {
  auto it = layers_.find(layer);
  if (it == layers_.end()) throw Error(FM_EINVAL, "layer " + std::to_string(layer) + " is not an MoE layer");
  const DeviceLayer& d = it->second;
  if (config_.sigmoid_routed()) {
    fm_moe_variant v = config_.variant();
    v.correction_bias = d.correction_bias;
    handle_.check(fm_moe_block_variant(handle_.get(), &cfg_, &v, &d.w, x, T, y, nullptr));
  } else {
    handle_.check(fm_moe_block(handle_.get(), &cfg_, &d.w, x, T, y, nullptr));
  }
}

}  // namespace flashmoe
