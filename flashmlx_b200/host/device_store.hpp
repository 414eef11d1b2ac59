// device_store.hpp -- device copies of host arrays, freed together (the weights a loader
// uploads once).  cudaMalloc per tensor: 256-byte aligned, as the tcgen05 path's TMA
// descriptors need.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "checkpoint.hpp"
#include "flashmoe.hpp"

namespace flashmoe {

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(FM_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

class DeviceStore {
 public:
  explicit DeviceStore(int device) : device_(device) {}
  ~DeviceStore() { release(); }
  DeviceStore(const DeviceStore&) = delete;
  DeviceStore& operator=(const DeviceStore&) = delete;

  // device memory of `bytes` (uninitialized), owned by the store
  void* alloc(size_t bytes) {
    if (!bytes) return nullptr;
    void* p = nullptr;
    cuda_check(cudaMalloc(&p, bytes), "cudaMalloc");
    ptrs_.push_back(p);
    return p;
  }
  void* upload(const void* src, size_t bytes) {
    void* p = alloc(bytes);
    if (p) cuda_check(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice), "cudaMemcpy");
    return p;
  }
  const uint16_t* u16(const std::vector<uint16_t>& v) {
    return static_cast<const uint16_t*>(upload(v.data(), v.size() * sizeof(uint16_t)));
  }
  const uint32_t* u32(const std::vector<uint32_t>& v) {
    return static_cast<const uint32_t*>(upload(v.data(), v.size() * sizeof(uint32_t)));
  }
  const float* f32(const std::vector<float>& v) {
    return static_cast<const float*>(upload(v.data(), v.size() * sizeof(float)));
  }
  fm_qweight q(const HostQ& hq) {
    fm_qweight r{};
    r.w = u32(hq.w);
    r.scales = u16(hq.s);
    r.biases = hq.has_biases() ? u16(hq.b) : nullptr;
    return r;
  }
  // frees everything (callers make sure no stream still reads it)
  void release() noexcept {
    if (ptrs_.empty()) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device_);
    for (void* p : ptrs_) cudaFree(p);
    cudaSetDevice(cur);
    ptrs_.clear();
  }
  int device() const { return device_; }

 private:
  int device_;
  std::vector<void*> ptrs_;
};

}  // namespace flashmoe
