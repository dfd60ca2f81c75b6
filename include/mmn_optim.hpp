/*
 * mmn_optim.hpp — C++17 mirror of the reference's Rust optimizer API
 * (crates/mmn-optim/src/lib.rs), header-only, over the C ABI of mmn_optim.h.
 *
 * Names, argument meaning and call semantics follow the Rust items:
 *   AdamWConfig / AdamW::step_param          lib.rs:6-61
 *   MuonConfig / Muon::step_matrix           lib.rs:63-80, 128-176
 *   newton_schulz5                           lib.rs:82-126
 *   ParamKind / HybridOptimizer              lib.rs:178-210
 *   GradAccumulator                          lib.rs:212-262
 *   cuda::is_available, require_cuda         crates/mmn-cuda/src/lib.rs:5-12,
 *                                            crates/mmn-core/src/device.rs:29-37
 *   OptimizerStep (the whole model's step)   crates/mmn-models/src/chatbot.rs:208-227,
 *                                            crates/mmn-train/src/lib.rs:367-378
 * Parameters and grads are host arrays (ArrayD, the role of ndarray's
 * ArrayD<f32>); the optimizer state lives on the GPU, keyed by the caller's id
 * like the reference's HashMaps. Where the reference panics (a shape that
 * differs from the state of an id, lib.rs:148,161) these calls throw
 * mmn::Error; cuda requested without a usable GPU throws mmn::CudaError.
 *
 * Configs are fixed when an optimizer is created (the C ABI copies them), so
 * the `config` members are read-only here, unlike the Rust public fields.
 */
#ifndef MMN_OPTIM_HPP
#define MMN_OPTIM_HPP

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "mmn_optim.h"

namespace mmn {

// ------------------------------------------------------------------ errors
class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

// MmnError::Cuda (crates/mmn-core/src/error.rs:84-90): CUDA requested but unusable.
class CudaError : public Error {
 public:
  using Error::Error;
};

inline void check(int rc) {
  if (rc == MMN_OK) return;
  std::string msg = mmn_last_error();
  if (rc == MMN_E_NO_DEVICE) throw CudaError(rc, msg);
  throw Error(rc, msg);
}

namespace cuda {
// crates/mmn-cuda/src/lib.rs:5-12
inline bool is_available() { return mmn_cuda_is_available() != 0; }
}  // namespace cuda

// Device::require_cuda_available_checked (crates/mmn-core/src/device.rs:29-37).
inline void require_cuda(bool cuda_requested) { check(mmn_require_cuda(cuda_requested ? 1 : 0)); }

// ------------------------------------------------------------------ arrays
// An owned row-major f32 array with a dynamic shape.
struct ArrayD {
  std::vector<int64_t> shape;
  std::vector<float> data;

  ArrayD() = default;
  explicit ArrayD(std::vector<int64_t> s, float fill = 0.0f) : shape(std::move(s)) {
    data.assign(numel(shape), fill);
  }
  ArrayD(std::vector<int64_t> s, std::vector<float> values) : shape(std::move(s)), data(std::move(values)) {
    if ((int64_t)data.size() != numel(shape)) throw Error(MMN_E_SHAPE, "values do not fill the shape");
  }
  // Array2::from_shape_fn((rows, cols), f) .into_dyn()
  static ArrayD from_shape_fn(int64_t rows, int64_t cols, const std::function<float(int64_t, int64_t)>& f) {
    ArrayD a({rows, cols});
    for (int64_t i = 0; i < rows; ++i)
      for (int64_t j = 0; j < cols; ++j) a.data[(size_t)(i * cols + j)] = f(i, j);
    return a;
  }
  static int64_t numel(const std::vector<int64_t>& s) {
    int64_t n = 1;
    for (int64_t d : s) n *= d;
    return n;
  }
  size_t len() const { return data.size(); }
  int ndim() const { return (int)shape.size(); }
  float& at(int64_t i, int64_t j) { return data[(size_t)(i * shape[1] + j)]; }
  float at(int64_t i, int64_t j) const { return data[(size_t)(i * shape[1] + j)]; }
  bool operator==(const ArrayD& o) const { return shape == o.shape && data == o.data; }
  bool operator!=(const ArrayD& o) const { return !(*this == o); }
};

// ------------------------------------------------------------------ AdamW
// AdamWConfig and its Default (lib.rs:6-22).
struct AdamWConfig {
  float lr = 3e-4f;
  std::pair<float, float> betas{0.9f, 0.95f};
  float eps = 1e-8f;
  float weight_decay = 0.01f;

  mmn_adamw_config c() const { return {lr, betas.first, betas.second, eps, weight_decay}; }
};

class HybridOptimizer;

// AdamW (lib.rs:24-61): one step counter per instance, zero m/v per new id.
class AdamW {
 public:
  const AdamWConfig config;

  explicit AdamW(AdamWConfig cfg = {}, int device = 0) : config(cfg), own_(true) {
    const mmn_adamw_config c = cfg.c();
    check(mmn_adamw_create(&c, device, nullptr, &h_));
  }
  AdamW(const AdamW&) = delete;
  AdamW& operator=(const AdamW&) = delete;
  ~AdamW() {
    if (own_ && h_) mmn_adamw_destroy(h_);
  }

  // AdamW::step_param (lib.rs:41-60): param updated in place.
  void step_param(size_t id, ArrayD& param, const ArrayD& grad, float grad_divisor = 1.0f) {
    if (param.shape != grad.shape) throw Error(MMN_E_SHAPE, "param and grad shapes differ");
    check(mmn_adamw_step_param(h_, id, param.data.data(), grad.data.data(), param.shape.data(),
                               param.ndim(), grad_divisor, MMN_MEM_HOST));
  }

  // The instance step counter (lib.rs:26).
  uint64_t step() const {
    uint64_t s = 0;
    check(mmn_adamw_get_step(h_, &s));
    return s;
  }

  mmn_adamw_t* handle() const { return h_; }

 private:
  friend class HybridOptimizer;
  AdamW(mmn_adamw_t* h, AdamWConfig cfg) : config(cfg), h_(h), own_(false) {}
  mmn_adamw_t* h_ = nullptr;
  bool own_ = false;
};

// ------------------------------------------------------------------- Muon
// MuonConfig and its Default (lib.rs:63-80).
struct MuonConfig {
  float lr = 0.02f;
  float momentum = 0.95f;
  bool nesterov = true;
  size_t ns_steps = 5;

  mmn_muon_config c() const { return {lr, momentum, nesterov ? 1 : 0, (int32_t)ns_steps}; }
};

// Muon (lib.rs:128-176) with the Newton-Schulz arithmetic mode (MMN_NS_*).
class Muon {
 public:
  const MuonConfig config;

  explicit Muon(MuonConfig cfg = {}, int ns_mode = MMN_NS_REFERENCE, int device = 0)
      : config(cfg), own_(true) {
    const mmn_muon_config c = cfg.c();
    check(mmn_muon_create(&c, ns_mode, device, nullptr, &h_));
  }
  Muon(const Muon&) = delete;
  Muon& operator=(const Muon&) = delete;
  ~Muon() {
    if (own_ && h_) mmn_muon_destroy(h_);
  }

  // Muon::step_matrix (lib.rs:141-175): p -= lr * sqrt(rows/cols) * NS(momentum(g)).
  void step_matrix(size_t id, ArrayD& param, const ArrayD& grad, float grad_divisor = 1.0f) {
    if (param.shape != grad.shape) throw Error(MMN_E_SHAPE, "param and grad shapes differ");
    check(mmn_muon_step_matrix(h_, id, param.data.data(), grad.data.data(), param.shape.data(),
                               param.ndim(), grad_divisor, MMN_MEM_HOST));
  }

  // The velocity of an id (rows*cols values).
  std::vector<float> velocity(size_t id, int64_t numel) const {
    std::vector<float> v((size_t)numel);
    check(mmn_muon_export_velocity(h_, id, v.data(), numel, MMN_MEM_HOST));
    return v;
  }

  mmn_muon_t* handle() const { return h_; }

 private:
  friend class HybridOptimizer;
  Muon(mmn_muon_t* h, MuonConfig cfg) : config(cfg), h_(h), own_(false) {}
  mmn_muon_t* h_ = nullptr;
  bool own_ = false;
};

// newton_schulz5 (lib.rs:82-126): a non-2-D input of n elements is zero-padded
// row-major into side x side, side = ceil(sqrt(n)); the result has the 2-D
// shape.
inline ArrayD newton_schulz5(const ArrayD& g, size_t steps, int ns_mode = MMN_NS_REFERENCE,
                             int device = 0) {
  std::vector<int64_t> out_shape = g.shape;
  if (g.ndim() != 2) {
    const int64_t side = (int64_t)std::ceil(std::sqrt((float)g.len()));
    out_shape = {side, side};
  }
  ArrayD out(out_shape);
  check(mmn_newton_schulz5(g.data.data(), g.shape.data(), g.ndim(), (int)steps, ns_mode,
                           out.data.data(), device, nullptr, MMN_MEM_HOST));
  return out;
}

// ---------------------------------------------------------------- Hybrid
enum class ParamKind { Matrix, Other };  // lib.rs:178-181

// HybridOptimizer (lib.rs:183-210): Muon for 2-D matrices with both dims > 1,
// AdamW for everything else; the public members are the two optimizers.
class HybridOptimizer {
 public:
  explicit HybridOptimizer(MuonConfig muon_cfg = {}, AdamWConfig adamw_cfg = {},
                           int ns_mode = MMN_NS_REFERENCE, int device = 0)
      : h_(create(muon_cfg, adamw_cfg, ns_mode, device)),
        muon(mmn_hybrid_muon(h_), muon_cfg),
        adamw(mmn_hybrid_adamw(h_), adamw_cfg) {}
  HybridOptimizer(const HybridOptimizer&) = delete;
  HybridOptimizer& operator=(const HybridOptimizer&) = delete;
  ~HybridOptimizer() { mmn_hybrid_destroy(h_); }

  // HybridOptimizer::classify_param (lib.rs:196-202).
  static ParamKind classify_param(const std::vector<int64_t>& shape) {
    return (shape.size() == 2 && shape[0] > 1 && shape[1] > 1) ? ParamKind::Matrix
                                                                : ParamKind::Other;
  }

  // HybridOptimizer::step (lib.rs:204-209). `route` MMN_ROUTE_MUON / _ADAMW
  // overrides the shape rule (embeddings and lm_head to AdamW).
  void step(size_t id, ArrayD& param, const ArrayD& grad, int route = MMN_ROUTE_AUTO,
            float grad_divisor = 1.0f) {
    if (param.shape != grad.shape) throw Error(MMN_E_SHAPE, "param and grad shapes differ");
    check(mmn_hybrid_step(h_, id, param.data.data(), grad.data.data(), param.shape.data(),
                          param.ndim(), route, grad_divisor, MMN_MEM_HOST));
  }

 private:
  static mmn_hybrid_t* create(const MuonConfig& m, const AdamWConfig& a, int ns_mode, int device) {
    const mmn_muon_config mc = m.c();
    const mmn_adamw_config ac = a.c();
    mmn_hybrid_t* h = nullptr;
    check(mmn_hybrid_create(&mc, &ac, ns_mode, device, nullptr, &h));
    return h;
  }
  mmn_hybrid_t* h_;

 public:
  Muon muon;
  AdamW adamw;
};

// ------------------------------------------------------------ accumulator
// GradAccumulator (lib.rs:212-262): sums each parameter's grad over
// micro-batches in call order; averaged_grad divides by max(micro_batches, 1).
// Host-side only: the batched GPU step folds the divisor into its kernels
// (grad_divisor) instead.
class GradAccumulator {
 public:
  void clear() {
    grads_.clear();
    micro_batches_ = 0;
    param_index_ = 0;
  }
  size_t micro_batches() const { return micro_batches_; }
  void begin_micro_batch() { param_index_ = 0; }
  void finish_micro_batch() {
    ++micro_batches_;
    param_index_ = 0;
  }
  void add_param_grad(const ArrayD& grad) {
    if (param_index_ < grads_.size()) {
      ArrayD& acc = grads_[param_index_];
      if (acc.shape != grad.shape) throw Error(MMN_E_SHAPE, "grad shape differs from the sum");
      for (size_t i = 0; i < acc.data.size(); ++i) acc.data[i] += grad.data[i];
    } else {
      grads_.push_back(grad);
    }
    ++param_index_;
  }
  // The plain sum of a tensor's grads (no reference counterpart): the batched
  // GPU step takes the sum and the micro-batch count and divides itself.
  const ArrayD& sum(size_t index) const { return grads_.at(index); }
  ArrayD averaged_grad(size_t index) const {
    const float n = (float)(micro_batches_ > 0 ? micro_batches_ : 1);
    ArrayD out = grads_.at(index);
    for (float& x : out.data) x = x / n;
    return out;
  }
  size_t len() const { return grads_.size(); }

 private:
  std::vector<ArrayD> grads_;
  size_t micro_batches_ = 0;
  size_t param_index_ = 0;
};

// ------------------------------------------------------------ batched step
// The whole model's step as one device-resident operation: the trainer's call
// that replaces the per-tensor optim_step_weight loop of a training step
// (crates/mmn-models/src/chatbot.rs:208-227, call order :1104-1196) and the
// optimizer construction of crates/mmn-train/src/lib.rs:367-378. Tensors are
// registered in the reference's call order, which fixes each AdamW tensor's
// step count.
class OptimizerStep {
 public:
  struct Tensor {
    uint64_t id;
    std::vector<int64_t> shape;
    int route = MMN_ROUTE_AUTO;
  };

  OptimizerStep(const std::vector<Tensor>& tensors, const mmn_optim_config& cfg, int device = 0)
      : shapes_() {
    check(mmn_optim_create(&cfg, device, nullptr, &h_));
    try {
      for (const Tensor& t : tensors) {
        int slot = -1;
        check(mmn_optim_add_param(h_, t.id, t.shape.data(), (int)t.shape.size(), t.route, &slot));
        shapes_.push_back(t.shape);
      }
      check(mmn_optim_finalize(h_));
    } catch (...) {
      mmn_optim_destroy(h_);
      throw;
    }
  }
  OptimizerStep(const OptimizerStep&) = delete;
  OptimizerStep& operator=(const OptimizerStep&) = delete;
  ~OptimizerStep() { mmn_optim_destroy(h_); }

  static mmn_optim_config default_config() { return mmn_optim_config_default(); }

  size_t size() const { return shapes_.size(); }

  void set_param(int slot, const ArrayD& p) {
    expect(slot, p);
    check(mmn_optim_set_param(h_, slot, p.data.data(), MMN_MEM_HOST));
  }
  ArrayD get_param(int slot) {
    ArrayD p(shapes_.at((size_t)slot));
    check(mmn_optim_get_param(h_, slot, p.data.data(), MMN_MEM_HOST));
    return p;
  }
  // fp32 grads (config.grad_dtype == MMN_DTYPE_F32)
  void set_grad(int slot, const ArrayD& g) {
    expect(slot, g);
    check(mmn_optim_set_grad(h_, slot, g.data.data(), MMN_MEM_HOST));
  }

  // One step over every registered tensor; grad_divisor is the accumulator's
  // micro-batch count (GradAccumulator::averaged_grad, lib.rs:254-257).
  void step(float grad_divisor = 1.0f) { check(mmn_optim_step(h_, grad_divisor)); }
  void sync() { check(mmn_optim_sync(h_)); }

  // One step from host memory: grads in, updated params out (slot order; an
  // empty array skips that slot's copy). Returns when params hold the result.
  void step_host(const std::vector<ArrayD>& grads, std::vector<ArrayD>& params,
                 float grad_divisor = 1.0f) {
    if (grads.size() != size() || params.size() != size())
      throw Error(MMN_E_INVALID, "need one grad and one param array per slot");
    std::vector<const void*> gp(size());
    std::vector<float*> pp(size());
    for (size_t k = 0; k < size(); ++k) {
      gp[k] = grads[k].len() ? grads[k].data.data() : nullptr;
      if (params[k].len() && params[k].shape != shapes_[k]) params[k] = ArrayD(shapes_[k]);
      pp[k] = params[k].len() ? params[k].data.data() : nullptr;
      if (gp[k]) expect((int)k, grads[k]);
    }
    check(mmn_optim_step_host(h_, gp.data(), pp.data(), grad_divisor));
  }

  uint64_t adamw_step() const {
    uint64_t s = 0;
    check(mmn_optim_get_adamw_step(h_, &s));
    return s;
  }

  mmn_optim_t* handle() const { return h_; }

 private:
  void expect(int slot, const ArrayD& a) const {
    if (slot < 0 || (size_t)slot >= shapes_.size() || a.shape != shapes_[(size_t)slot])
      throw Error(MMN_E_SHAPE, "array shape differs from the registered tensor");
  }
  mmn_optim_t* h_ = nullptr;
  std::vector<std::vector<int64_t>> shapes_;
};

}  // namespace mmn

#endif  // MMN_OPTIM_HPP
