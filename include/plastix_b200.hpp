// plastix_b200.hpp -- C++ host layer over the C ABI in plastix_b200.h.
//
// For C++ programs that drive the device path directly (no Python): RAII
// device arrays and contexts, exceptions carrying plx_last_error(), and
// network classes whose stepping methods follow the reference's
// Network<Traits> (include/plastix/plastix.hpp:101-463): DoForwardPass,
// DoStep, GetOutput, GetStep. Each class runs one of the rule families the
// device library implements:
//
//   HebbianLayerNetwork  one sparse layer, Pipeline propagation, identity
//                        Apply, per-connection trace rule
//                        e = decay*e + pre*post; w += rate*e (the single-layer
//                        sweep workload), forward and update fused
//   SwiftTDNetwork       the SwiftTD learner of examples/swifttd/swifttd.cpp
//
// Header only; link with libplastix_b200.so and the CUDA runtime.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <memory>
#include <span>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "plastix_b200.h"

namespace plastix_b200 {

class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& where)
      : std::runtime_error(where + ": " + plx_last_error()), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

inline void check(int rc, const char* where) {
  if (rc != PLX_OK) throw Error(rc, where);
}

inline void check_cuda(cudaError_t e, const char* where) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(where) + ": " + cudaGetErrorString(e));
}

// A device array owned by this object (cudaMalloc / cudaFree).
template <class T>
class DeviceArray {
 public:
  DeviceArray() = default;
  explicit DeviceArray(size_t n) : n_(n) {
    if (n) check_cuda(cudaMalloc(&p_, n * sizeof(T)), "cudaMalloc");
  }
  DeviceArray(std::span<const T> host) : DeviceArray(host.size()) { upload(host); }
  ~DeviceArray() {
    if (p_) cudaFree(p_);
  }
  DeviceArray(const DeviceArray&) = delete;
  DeviceArray& operator=(const DeviceArray&) = delete;
  DeviceArray(DeviceArray&& o) noexcept : p_(std::exchange(o.p_, nullptr)), n_(o.n_) {}
  DeviceArray& operator=(DeviceArray&& o) noexcept {
    std::swap(p_, o.p_);
    std::swap(n_, o.n_);
    return *this;
  }
  void upload(std::span<const T> host, cudaStream_t s = nullptr) {
    if (host.size() > n_) throw std::length_error("DeviceArray::upload: too many elements");
    if (!host.empty())
      check_cuda(cudaMemcpyAsync(p_, host.data(), host.size() * sizeof(T),
                                 cudaMemcpyHostToDevice, s),
                 "cudaMemcpyAsync");
  }
  std::vector<T> download(cudaStream_t s = nullptr) const {
    std::vector<T> out(n_);
    if (n_) {
      check_cuda(cudaMemcpyAsync(out.data(), p_, n_ * sizeof(T), cudaMemcpyDeviceToHost, s),
                 "cudaMemcpyAsync");
      check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    }
    return out;
  }
  void fill_zero(cudaStream_t s = nullptr) {
    if (n_) check_cuda(cudaMemsetAsync(p_, 0, n_ * sizeof(T), s), "cudaMemsetAsync");
  }
  T* data() { return p_; }
  const T* data() const { return p_; }
  size_t size() const { return n_; }

 private:
  T* p_ = nullptr;
  size_t n_ = 0;
};

// One device and the stream every call of this context is enqueued on.
class Context {
 public:
  explicit Context(int device = 0, cudaStream_t stream = nullptr) : stream_(stream) {
    check(plx_ctx_create(device, stream, &ctx_), "plx_ctx_create");
  }
  ~Context() {
    if (ctx_) plx_ctx_destroy(ctx_);
  }
  Context(const Context&) = delete;
  Context& operator=(const Context&) = delete;
  plx_ctx* get() const { return ctx_; }
  cudaStream_t stream() const { return stream_; }
  // Waits for the stream; throws if a kernel reported an error.
  void sync() const { check(plx_ctx_sync(ctx_), "plx_ctx_sync"); }

 private:
  plx_ctx* ctx_ = nullptr;
  cudaStream_t stream_;
};

// CSR index over destination-sorted connections (rows = destination units
// [row_base, row_base + n_rows)).
class DstCsr {
 public:
  DstCsr(Context& ctx, const DeviceArray<uint32_t>& to_id, uint32_t row_base, uint32_t n_rows)
      : row_ptr_(n_rows + 1),
        plan_(plx_csr_plan_words(to_id.size(), n_rows)) {
    check(plx_csr_row_ptr(ctx.get(), to_id.data(), to_id.size(), row_base, n_rows,
                          row_ptr_.data()),
          "plx_csr_row_ptr");
    check(plx_csr_plan(ctx.get(), row_ptr_.data(), n_rows, to_id.size(), plan_.data(),
                       plan_.size(), &csr_),
          "plx_csr_plan");
    csr_.to_id = to_id.data();  // the warp fast path reads the sorted ToId
    csr_.row_base = row_base;
  }
  const plx_csr* get() const { return &csr_; }

 private:
  DeviceArray<uint32_t> row_ptr_, plan_;
  plx_csr csr_{};
};

// One sparse layer of num_output units fed by num_input units through an
// explicit connection list (absolute unit ids; ToId sorted ascending, the
// reference's FullyConnected / LayerBuilder order), stepped like
// Network::DoStep in Pipeline mode with the per-connection trace rule.
class HebbianLayerNetwork {
 public:
  HebbianLayerNetwork(Context& ctx, uint32_t num_input, uint32_t num_output,
                      std::span<const uint32_t> from_id, std::span<const uint32_t> to_id,
                      std::span<const float> weight, float decay, float rate)
      : ctx_(ctx),
        num_input_(num_input),
        num_output_(num_output),
        from_(from_id),
        to_(to_id),
        act_in_(num_input),
        act_out_(num_output),
        decay_(decay),
        rate_(rate) {
    if (from_id.size() != to_id.size() || weight.size() != to_id.size())
      throw std::invalid_argument("from_id, to_id and weight must have the same length");
    for (int i = 0; i < 2; ++i) {
      w_[i] = DeviceArray<float>(weight.size());
      e_[i] = DeviceArray<float>(weight.size());
      e_[i].fill_zero(ctx.stream());
    }
    w_[0].upload(weight, ctx.stream());
    // Destination units follow the inputs: rows [num_input, num_input + num_output).
    csr_ = std::make_unique<DstCsr>(ctx, to_, num_input, num_output);
  }

  // DoForwardPass + DoUpdateConnectionState of the trace rule, as one fused
  // sweep (plastix.hpp:132-149, :232-256).
  void DoStep(std::span<const float> inputs) {
    act_in_.upload(inputs.first(num_input_), ctx_.stream());
    check(plx_sweep_forward_hebbian(ctx_.get(), csr_->get(), from_.data(), nullptr,
                                    act_in_.data(), num_input_, w_[cur_].data(),
                                    w_[cur_ ^ 1].data(), e_[cur_].data(), e_[cur_ ^ 1].data(),
                                    decay_, rate_, act_out_.data()),
          "plx_sweep_forward_hebbian");
    cur_ ^= 1;
    ++step_;
  }

  // DoForwardPass alone (identity Apply).
  void DoForwardPass(std::span<const float> inputs) {
    act_in_.upload(inputs.first(num_input_), ctx_.stream());
    check(plx_sweep_forward(ctx_.get(), csr_->get(), from_.data(), w_[cur_].data(), nullptr,
                            act_in_.data(), num_input_, PLX_APPLY_IDENTITY, act_out_.data(),
                            nullptr, nullptr),
          "plx_sweep_forward");
    ++step_;
  }

  // Activations of the output units (synchronises, downloads).
  std::vector<float> GetOutput() const {
    ctx_.sync();
    return act_out_.download(ctx_.stream());
  }
  std::vector<float> GetWeights() const {
    ctx_.sync();
    return w_[cur_].download(ctx_.stream());
  }
  std::vector<float> GetTraces() const {
    ctx_.sync();
    return e_[cur_].download(ctx_.stream());
  }
  size_t GetStep() const { return step_; }

 private:
  Context& ctx_;
  uint32_t num_input_, num_output_;
  DeviceArray<uint32_t> from_, to_;
  DeviceArray<float> act_in_, act_out_;
  DeviceArray<float> w_[2], e_[2];
  std::unique_ptr<DstCsr> csr_;
  float decay_, rate_;
  int cur_ = 0;
  size_t step_ = 0;
};

// The SwiftTD network of examples/swifttd/swifttd.cpp: n features -> one
// value unit, the ten per-connection fields in SoA, the globals record
// (swifttd.cpp:47-62) in device memory. DoStep takes the active features
// (sorted, strictly increasing; value 1 unless values are given) and the
// reward, as the example's DoStep(features, {reward}) does with the dense
// feature vector.
class SwiftTDNetwork {
 public:
  struct Params {
    float gamma = 0.99f, lambda = 0.9f, eta = 0.05f, eta_min = 1e-7f, decay = 0.999f,
          meta = 1e-3f, alpha_init = 0.05f;
  };

  SwiftTDNetwork(Context& ctx, uint32_t n_features, uint32_t max_active, Params p)
      : ctx_(ctx),
        n_(n_features),
        stride_((n_features + 3u) & ~3u),
        state_((size_t)PLX_TD_NUM_FIELDS * stride_),
        globals_(sizeof(plx_td_globals) / sizeof(float)),
        v_(1),
        reward_(1),
        idx_(max_active ? max_active : 1),
        val_(max_active ? max_active : 1),
        max_active_(max_active),
        scratch_(plx_swifttd_scratch_bytes(n_features, max_active)) {
    state_.fill_zero(ctx.stream());
    scratch_.fill_zero(ctx.stream());
    // Beta = log(alpha_init) (SwiftTDConnInit, swifttd.cpp:66-72), computed on
    // the host in single precision like std::log on a float.
    std::vector<float> beta(stride_, std::log(p.alpha_init));
    check_cuda(cudaMemcpyAsync(state_.data() + (size_t)9 * stride_, beta.data(),
                               stride_ * sizeof(float), cudaMemcpyHostToDevice, ctx.stream()),
               "cudaMemcpyAsync");
    const plx_td_globals g{p.gamma, p.lambda, p.eta, p.eta_min, p.decay, p.meta,
                           0, 0, 0, 0, 0, 0, 0};
    check_cuda(cudaMemcpyAsync(globals_.data(), &g, sizeof(g), cudaMemcpyHostToDevice,
                               ctx.stream()),
               "cudaMemcpyAsync");
    for (int j = 0; j < PLX_TD_NUM_FIELDS; ++j) fields_[j] = state_.data() + (size_t)j * stride_;
    ctx.sync();  // the host staging vectors above go out of scope
  }

  void DoStep(std::span<const uint32_t> active, float reward,
              std::span<const float> values = {}) {
    if (active.size() > max_active_) throw std::length_error("more active features than max_active");
    host_reward_ = reward;
    idx_.upload(active, ctx_.stream());
    if (!values.empty()) val_.upload(values, ctx_.stream());
    reward_.upload(std::span<const float>(&host_reward_, 1), ctx_.stream());
    check(plx_swifttd_step(ctx_.get(), n_, fields_, active.empty() ? nullptr : idx_.data(),
                           values.empty() ? nullptr : val_.data(), (uint32_t)active.size(),
                           reward_.data(), reinterpret_cast<plx_td_globals*>(globals_.data()),
                           v_.data(), scratch_.data(), scratch_.size()),
          "plx_swifttd_step");
    ctx_.sync();  // the reward and index uploads read host memory of this call
    ++step_;
  }

  float GetOutput() const { return v_.download(ctx_.stream())[0]; }
  std::vector<float> GetField(int j) const {
    std::vector<float> all = state_.download(ctx_.stream());
    return std::vector<float>(all.begin() + (size_t)j * stride_,
                              all.begin() + (size_t)j * stride_ + n_);
  }
  size_t GetStep() const { return step_; }

 private:
  Context& ctx_;
  uint32_t n_, stride_;
  DeviceArray<float> state_, globals_, v_, reward_;
  DeviceArray<uint32_t> idx_;
  DeviceArray<float> val_;
  uint32_t max_active_;
  DeviceArray<uint8_t> scratch_;
  float* fields_[PLX_TD_NUM_FIELDS];
  float host_reward_ = 0.0f;
  size_t step_ = 0;
};

}  // namespace plastix_b200
