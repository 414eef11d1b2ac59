// flashmoe.hpp -- C++ face of libflashmoe's C ABI for a C++ caller such as FlashMLX's
// server: an owning handle, status codes turned into exceptions, and the two MLX
// operators the model forward calls with MLX's argument order.
//
//   mx::quantized_matmul(x, w, scales, biases, transpose=true, group_size, bits)
//       (server/src/model.cpp:476-480, 741-747)        -> flashmoe::quantized_matmul
//   mx::gather_qmm(x, w, scales, biases, lhs_indices, rhs_indices, transpose=true,
//                  group_size, bits, "affine", sorted_indices)
//       (model.cpp:703-721, nemotron_h.cpp:1074-1092)   -> flashmoe::gather_qmm
//
// Every array is a device pointer on the handle's device; calls are asynchronous on the
// handle's stream, as MLX ops are lazy until mx::eval (scheduler.cpp:204), and
// Handle::sync() is the point where device-side failures surface.  No C++ type crosses
// the library boundary: this header is compiled into the caller.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

#include "flashmoe.h"

namespace flashmoe {

// A libflashmoe status other than FM_OK, with the handle's message.
class Error : public std::runtime_error {
 public:
  Error(int status, const std::string& what)
      : std::runtime_error(std::string(fm_status_string(status)) + ": " + what), status_(status) {}
  int status() const { return status_; }

 private:
  int status_;
};

// A packed MLX quantized tensor on the device: w [.., N, K*bits/32] uint32, scales and
// biases [.., N, K/group_size] bf16 (biases may be null: zero).
struct QTensor {
  const uint32_t* w = nullptr;
  const uint16_t* scales = nullptr;
  const uint16_t* biases = nullptr;
  fm_qweight c() const { return fm_qweight{w, scales, biases}; }
};

// One libflashmoe handle: a device, a stream and the workspace the calls reuse.
class Handle {
 public:
  Handle() = default;
  // stream: a cudaStream_t (nullptr = the legacy default stream)
  explicit Handle(int device, void* stream = nullptr) {
    const int rc = fm_create(&h_, device, stream);
    if (rc != FM_OK) {
      const std::string msg = h_ ? fm_last_error(h_) : "fm_create failed";
      if (h_) fm_destroy(h_);
      h_ = nullptr;
      throw Error(rc, msg);
    }
  }
  ~Handle() { reset(); }
  Handle(const Handle&) = delete;
  Handle& operator=(const Handle&) = delete;
  Handle(Handle&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
  Handle& operator=(Handle&& o) noexcept {
    if (this != &o) {
      reset();
      h_ = std::exchange(o.h_, nullptr);
    }
    return *this;
  }

  fm_handle* get() const { return h_; }
  explicit operator bool() const { return h_ != nullptr; }

  // throws Error(rc, the handle's last message) unless rc is FM_OK
  void check(int rc) const {
    if (rc != FM_OK) throw Error(rc, h_ ? fm_last_error(h_) : "no handle");
  }
  // sizes the workspace for up to max_tokens tokens of cfg, so later calls do not allocate
  void reserve(const fm_moe_config& cfg, int64_t max_tokens) { check(fm_reserve(h_, &cfg, max_tokens)); }
  void set_stream(void* stream) { check(fm_set_stream(h_, stream)); }
  // expert-product path (FM_PATH_*) and routing-kernel form (FM_ROUTE_*) of later calls
  void set_path(int path) { check(fm_set_path(h_, path)); }
  void set_route_mode(int mode) { check(fm_set_route_mode(h_, mode)); }
  // waits for the handle's stream; a device-side failure (bounded wait, bounds check) throws
  void sync() const { check(fm_sync_status(h_)); }

 private:
  void reset() {
    if (h_) fm_destroy(h_);
    h_ = nullptr;
  }
  fm_handle* h_ = nullptr;
};

// out [M, N] = x [M, K] . dequant(w)^T  (transpose = true, the only form the model uses)
inline void quantized_matmul(const Handle& h, const uint16_t* x, int64_t M, int K, const QTensor& w, int N,
                             int group_size, int bits, uint16_t* out, bool transpose = true) {
  h.check(fm_quantized_matmul(h.get(), x, M, K, w.w, w.scales, w.biases, N, transpose ? 1 : 0, group_size, bits,
                              out));
}

// out [B, M, N]: batch b multiplies x[lhs_indices ? lhs_indices[b] : b % x_batches] [M, K]
// by expert rhs_indices[b] of w [E, N, K]; sorted_indices is MLX's hint (accepted, the
// expert-major order is rebuilt either way).
inline void gather_qmm(const Handle& h, const uint16_t* x, int64_t x_batches, int M, int K, const QTensor& w, int E,
                       int N, const uint32_t* lhs_indices, const uint32_t* rhs_indices, int64_t B, int group_size,
                       int bits, bool sorted_indices, uint16_t* out, bool transpose = true) {
  h.check(fm_gather_qmm(h.get(), x, x_batches, M, K, w.w, w.scales, w.biases, E, N, lhs_indices, rhs_indices, B,
                        transpose ? 1 : 0, group_size, bits, sorted_indices ? 1 : 0, out));
}

}  // namespace flashmoe
