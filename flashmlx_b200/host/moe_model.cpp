// moe_model.cpp -- see moe_model.hpp.  Device memory comes from the CUDA runtime
// (cudaMalloc per tensor: 256-byte aligned, as the tcgen05 path's TMA descriptors need).
#include "moe_model.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>

namespace flashmoe {

namespace {

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(FM_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

MoEModel::MoEModel(const std::string& model_dir, int device, void* stream, int64_t max_tokens,
                   const std::vector<int>& layers)
    : device_(device) {
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
  try {
    for (int i : moe) {
      const HostLayer L = config_.sigmoid_routed() ? ck.sigmoid_moe_layer(i) : ck.moe_layer(i);
      DeviceLayer d;
      d.w.router_w = upload_u16(L.router_w);
      if (L.sigmoid) {
        d.w.up = upload_q(L.up);  // fc1
        d.w.down = upload_q(L.down);  // fc2
        if (L.has_shared) {
          d.w.shared_up = upload_q(L.shared_up);
          d.w.shared_down = upload_q(L.shared_down);
        }
        if (!L.correction_bias.empty()) d.correction_bias = upload_f32(L.correction_bias);
      } else {
        d.w.gate = upload_q(L.gate);
        d.w.up = upload_q(L.up);
        d.w.down = upload_q(L.down);
        if (L.has_shared) {
          d.w.shared_gate = upload_q(L.shared_gate);
          d.w.shared_up = upload_q(L.shared_up);
          d.w.shared_down = upload_q(L.shared_down);
          d.w.shared_expert_gate_w = upload_u16(L.shared_expert_gate_w);
        }
      }
      layers_[i] = d;
    }
    if (max_tokens > 0 && !layers_.empty()) handle_.reserve(cfg_, max_tokens);
  } catch (...) {
    free_all();
    throw;
  }
}

MoEModel::~MoEModel() { free_all(); }

void MoEModel::free_all() noexcept {
  if (allocations_.empty()) return;
  // the handle's stream may still read the weights
  if (handle_) fm_sync_status(handle_.get());
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(device_);
  for (void* p : allocations_) cudaFree(p);
  cudaSetDevice(cur);
  allocations_.clear();
}

std::vector<int> MoEModel::moe_layers() const {
  std::vector<int> out;
  for (const auto& kv : layers_) out.push_back(kv.first);
  return out;
}

void* MoEModel::upload(const void* src, size_t bytes) {
  if (!bytes) return nullptr;
  void* p = nullptr;
  cuda_check(cudaMalloc(&p, bytes), "cudaMalloc");
  allocations_.push_back(p);
  cuda_check(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice), "cudaMemcpy");
  return p;
}

const uint16_t* MoEModel::upload_u16(const std::vector<uint16_t>& v) {
  return static_cast<const uint16_t*>(upload(v.data(), v.size() * sizeof(uint16_t)));
}
const uint32_t* MoEModel::upload_u32(const std::vector<uint32_t>& v) {
  return static_cast<const uint32_t*>(upload(v.data(), v.size() * sizeof(uint32_t)));
}
const float* MoEModel::upload_f32(const std::vector<float>& v) {
  return static_cast<const float*>(upload(v.data(), v.size() * sizeof(float)));
}

fm_qweight MoEModel::upload_q(const HostQ& q) {
  fm_qweight r{};
  r.w = upload_u32(q.w);
  r.scales = upload_u16(q.s);
  r.biases = q.has_biases() ? upload_u16(q.b) : nullptr;
  return r;
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
