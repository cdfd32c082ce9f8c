// C++ host API of the B200 Gated DeltaNet recurrence, shaped like the
// reference's delta namespace (cpp/src/delta.hpp:49-76): available(), a Result
// with o, s_out and the per-step states, run() for head-expanded fp32 inputs
// with precomputed gates, and run_gated() for the north-star form with raw
// gates and 16 key heads.  Arrays are device buffers owned by DeviceArray
// (the reference uses MLX arrays); errors are thrown as std::runtime_error
// (the reference throws from MLX).  Everything goes through the C ABI in
// gdn_b200.h; there is no CPU path.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <numeric>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "gdn_b200.h"

namespace gdn {

enum class DType { F32, BF16, I32 };

inline size_t dtype_size(DType t) { return t == DType::BF16 ? 2 : 4; }

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

inline void check_gdn(int rc) {
  if (rc != GDN_OK) throw std::runtime_error(std::string("gdn: ") + gdn_last_error());
}

// Owning, contiguous device array with a shape.
class DeviceArray {
 public:
  DeviceArray() = default;
  DeviceArray(std::vector<int64_t> shape, DType dtype) : shape_(std::move(shape)), dtype_(dtype) {
    const size_t n = bytes();
    if (n) check_cuda(cudaMalloc(&ptr_, n), "cudaMalloc");
  }
  ~DeviceArray() { reset(); }
  DeviceArray(const DeviceArray&) = delete;
  DeviceArray& operator=(const DeviceArray&) = delete;
  DeviceArray(DeviceArray&& o) noexcept { *this = std::move(o); }
  DeviceArray& operator=(DeviceArray&& o) noexcept {
    if (this != &o) {
      reset();
      ptr_ = std::exchange(o.ptr_, nullptr);
      shape_ = std::move(o.shape_);
      dtype_ = o.dtype_;
    }
    return *this;
  }

  void* data() const { return ptr_; }
  template <class T>
  T* as() const { return static_cast<T*>(ptr_); }
  const std::vector<int64_t>& shape() const { return shape_; }
  int64_t shape(int i) const { return shape_.at(static_cast<size_t>(i < 0 ? i + ndim() : i)); }
  int ndim() const { return static_cast<int>(shape_.size()); }
  DType dtype() const { return dtype_; }
  size_t size() const {
    return std::accumulate(shape_.begin(), shape_.end(), size_t{1},
                           [](size_t a, int64_t b) { return a * static_cast<size_t>(b); });
  }
  size_t bytes() const { return size() * dtype_size(dtype_); }

  void upload(const void* host, cudaStream_t st = nullptr) {
    check_cuda(cudaMemcpyAsync(ptr_, host, bytes(), cudaMemcpyHostToDevice, st), "upload");
  }
  void download(void* host, cudaStream_t st = nullptr) const {
    check_cuda(cudaMemcpyAsync(host, ptr_, bytes(), cudaMemcpyDeviceToHost, st), "download");
    check_cuda(cudaStreamSynchronize(st), "download sync");
  }

 private:
  void reset() {
    if (ptr_) cudaFree(ptr_);
    ptr_ = nullptr;
  }
  void* ptr_ = nullptr;
  std::vector<int64_t> shape_;
  DType dtype_ = DType::F32;
};

namespace delta {

// True when a CUDA device is present (the reference: Metal is available).
inline bool available() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

struct Result {
  DeviceArray o;                    // (B, L, H, Dv) fp32
  DeviceArray s_out;                // (B, H, Dv, Dk) fp32
  DeviceArray states;               // (B, H, L, Dv, Dk) fp32, only when collect = true
};

// Drop-in for delta::run (cpp/src/delta.hpp:66-68): q, k (B,L,H,Dk) fp32
// already l2-normalised and head-expanded; v (B,L,H,Dv); alpha, beta (B,L,H);
// S (B,H,Dv,Dk) or nullptr for zeros.
inline Result run(const DeviceArray& q, const DeviceArray& k, const DeviceArray& v, const DeviceArray& alpha,
                  const DeviceArray& beta, const DeviceArray* S, bool collect = false,
                  cudaStream_t stream = nullptr) {
  const int B = static_cast<int>(q.shape(0)), L = static_cast<int>(q.shape(1)), H = static_cast<int>(q.shape(2)),
            Dk = static_cast<int>(q.shape(3)), Dv = static_cast<int>(v.shape(3));
  Result r{DeviceArray({B, L, H, Dv}, DType::F32), DeviceArray({B, H, Dv, Dk}, DType::F32), {}};
  if (collect) r.states = DeviceArray({B, H, L, Dv, Dk}, DType::F32);
  check_gdn(gdn_delta_run(q.as<float>(), k.as<float>(), v.as<float>(), alpha.as<float>(), beta.as<float>(),
                          S ? S->as<float>() : nullptr, r.o.as<float>(), r.s_out.as<float>(),
                          collect ? r.states.as<float>() : nullptr, B, L, H, Dk, Dv, stream));
  return r;
}

// North-star form: q, k (B,L,Hk,Dk) and v (B,L,Hv,Dv) bf16 as they leave the
// conv (l2norm applied in-kernel when `l2norm`), a, b (B,L,Hv) fp32 raw gate
// inputs, A_log, dt_bias (Hv) fp32.
inline Result run_gated(const DeviceArray& q, const DeviceArray& k, const DeviceArray& v, const DeviceArray& a,
                        const DeviceArray& b, const DeviceArray& A_log, const DeviceArray& dt_bias,
                        const DeviceArray* S, bool collect = false, bool l2norm = false,
                        cudaStream_t stream = nullptr) {
  const int B = static_cast<int>(q.shape(0)), L = static_cast<int>(q.shape(1)), Hk = static_cast<int>(q.shape(2)),
            Dk = static_cast<int>(q.shape(3)), Hv = static_cast<int>(v.shape(2)), Dv = static_cast<int>(v.shape(3));
  unsigned flags = (q.dtype() == DType::F32 ? GDN_F_QKV_F32 : 0u) | (l2norm ? GDN_F_QK_L2NORM : 0u);
  Result r{DeviceArray({B, L, Hv, Dv}, DType::F32), DeviceArray({B, Hv, Dv, Dk}, DType::F32), {}};
  if (collect) r.states = DeviceArray({B, Hv, L, Dv, Dk}, DType::F32);
  check_gdn(gdn_recurrent_fwd(q.data(), k.data(), v.data(), a.as<float>(), b.as<float>(), A_log.as<float>(),
                              dt_bias.as<float>(), S ? S->as<float>() : nullptr, r.s_out.as<float>(), r.o.data(),
                              collect ? r.states.as<float>() : nullptr, B, L, Hk, Hv, Dk, Dv, flags, stream));
  return r;
}

// The states of a serving batch in slots of a pool (gdn_recurrent_fwd_pool):
// the layout of DeltaCache::state across a batch (cpp/src/model.hpp:211-227),
// where admitting or retiring a sequence only rewrites the slot indices.
class StatePool {
 public:
  StatePool(int n_slots, int Hv, int D = 128)
      : pool_({n_slots, Hv, D, D}, DType::F32), n_slots_(n_slots), Hv_(Hv) {}
  DeviceArray& states() { return pool_; }
  int n_slots() const { return n_slots_; }

  // One decode / verify step of the sequences in `slots` (B int32 on the
  // device): the north-star inputs of run_gated; the new states are written
  // back to the slots (GDN_POOL_FINAL), or left alone with per-position
  // checkpoints returned (record mode, GDN_POOL_KEEP).
  Result step(const DeviceArray& q, const DeviceArray& k, const DeviceArray& v, const DeviceArray& a,
              const DeviceArray& b, const DeviceArray& A_log, const DeviceArray& dt_bias, const DeviceArray& slots,
              bool record = false, bool l2norm = false, cudaStream_t stream = nullptr) {
    const int B = static_cast<int>(q.shape(0)), L = static_cast<int>(q.shape(1)), Hk = static_cast<int>(q.shape(2)),
              Dk = static_cast<int>(q.shape(3)), Hv = static_cast<int>(v.shape(2)), Dv = static_cast<int>(v.shape(3));
    if (Hv != Hv_) throw std::runtime_error("gdn: value heads do not match the pool");
    unsigned flags = (q.dtype() == DType::F32 ? GDN_F_QKV_F32 : 0u) | (l2norm ? GDN_F_QK_L2NORM : 0u);
    Result r{DeviceArray({B, L, Hv, Dv}, DType::F32), {}, {}};
    if (record) r.states = DeviceArray({B, Hv, L, Dv, Dk}, DType::F32);
    check_gdn(gdn_recurrent_fwd_pool(q.data(), k.data(), v.data(), a.as<float>(), b.as<float>(), A_log.as<float>(),
                                     dt_bias.as<float>(), pool_.as<float>(), slots.as<int32_t>(), n_slots_, nullptr,
                                     nullptr, 0, record ? GDN_POOL_KEEP : GDN_POOL_FINAL, r.o.data(),
                                     record ? r.states.as<float>() : nullptr, nullptr, B, L, Hk, Hv, Dk, Dv, flags,
                                     stream));
    return r;
  }

 private:
  DeviceArray pool_;
  int n_slots_, Hv_;
};

}  // namespace delta
}  // namespace gdn
