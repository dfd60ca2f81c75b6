/*
 * mmn_train.hpp — C++17 mirror of the optimizer plumbing of the reference's
 * trainer, header-only, over the batched GPU step of mmn_optim.hpp.
 *
 *   TrainConfig                  crates/mmn-train/src/lib.rs:22-41 (defaults and
 *                                the Python repr of crates/mmn-py/src/train_config.rs:37-44)
 *   optimizer construction       crates/mmn-train/src/lib.rs:360-380
 *   the step loop                crates/mmn-train/src/lib.rs:382-442 (train_with_encoder)
 *   one step's calls             crates/mmn-models/src/chatbot.rs:935-1075
 *                                (train_step_lm, apply_accumulated_lm_grads)
 *
 * The reference builds a HybridOptimizer (MuonConfig::default(), AdamW with
 * lr = learning_rate and default betas) and a separate AdamW with the same lr;
 * optimizer == "hybrid" routes through the first, anything else (including
 * "muon") through the second. Every optimizer call gets a new id (param_id is
 * incremented per tensor and never reset), so m, v and velocity start at zero
 * on every step while the AdamW instance's step counter keeps counting. With
 * batch_size == 1 each sample's grads are stepped at once; otherwise grads
 * are summed per tensor over the micro-batches of a batch
 * (GradAccumulator, lib.rs:212-262) and averaged on the flush that comes after
 * batch_size micro-batches or at the last sample of the epoch.
 *
 * Here the model's forward/backward stays where the caller runs it (a
 * callback fills one sample's grads on the host), the accumulation is the
 * same fp32 sum in micro-batch order, and each flush is one batched step on
 * the GPU (mmn_optim_step_host) that divides by the micro-batch count inside
 * its kernels and writes the updated fp32 weights back to the caller's
 * arrays. The stepper is a template parameter, so the same loop drives a
 * per-call CPU replay in the tests.
 */
#ifndef MMN_TRAIN_HPP
#define MMN_TRAIN_HPP

#include <cstddef>
#include <cstdint>
#include <functional>
#include <sstream>
#include <string>
#include <vector>

#include "mmn_optim.hpp"

namespace mmn {

// TrainConfig (crates/mmn-train/src/lib.rs:22-41; Python defaults
// crates/mmn-py/src/train_config.rs:21).
struct TrainConfig {
  size_t epochs = 1;
  size_t batch_size = 8;
  bool cuda = false;
  std::string optimizer = "hybrid";
  float learning_rate = 3e-4f;

  // The Python repr (crates/mmn-py/src/train_config.rs:37-44).
  std::string repr() const {
    std::ostringstream s;
    s << "TrainConfig(epochs=" << epochs << ", batch_size=" << batch_size
      << ", cuda=" << (cuda ? "true" : "false") << ", optimizer=\"" << optimizer
      << "\", learning_rate=" << learning_rate << ")";
    return s.str();
  }
};

// The batched step's configuration for the optimizer the trainer builds
// (crates/mmn-train/src/lib.rs:367-380): Muon with MuonConfig::default()
// (learning_rate never reaches Muon), AdamW with lr = learning_rate and
// default betas, eps and decay, hybrid routing only for "hybrid", and fresh
// state every step because the trainer's ids are never reused.
inline mmn_optim_config optim_config_for(const TrainConfig& c) {
  mmn_optim_config cfg = mmn_optim_config_default();
  cfg.adamw = mmn_adamw_config_default();
  cfg.adamw.lr = c.learning_rate;
  cfg.muon = mmn_muon_config_default();
  cfg.use_hybrid = c.optimizer == "hybrid" ? 1 : 0;
  cfg.fresh_state = 1;
  return cfg;
}

// One training run's optimizer loop (train_with_encoder, lib.rs:382-442).
// Step needs size(), and step_host(grads, params, grad_divisor) that steps
// every tensor once from host grads and writes the updated params.
template <class Step>
class TrainLoop {
 public:
  // Fills grads[k] (the shape of tensor k) with one sample's gradients.
  using Backward = std::function<void(size_t sample, std::vector<ArrayD>& grads)>;
  // The sample order of an epoch (the reference shuffles with thread_rng).
  using Order = std::function<std::vector<size_t>(size_t epoch)>;

  TrainLoop(const TrainConfig& cfg, Step& step) : cfg_(cfg), step_(step) {}

  // Runs config.epochs epochs over n_samples samples; params (one array per
  // tensor, in the optimizer's call order) are updated in place at every step.
  void train(size_t n_samples, const Order& order, const Backward& backward,
             std::vector<ArrayD>& params) {
    const size_t n = step_.size();
    if (params.size() != n) throw Error(MMN_E_INVALID, "need one param array per tensor");
    const size_t batch_size = cfg_.batch_size > 0 ? cfg_.batch_size : 1;  // lib.rs:381
    std::vector<ArrayD> grads(n);
    for (size_t k = 0; k < n; ++k) grads[k] = ArrayD(params[k].shape);
    for (size_t epoch = 0; epoch < cfg_.epochs; ++epoch) {
      const std::vector<size_t> idx = order(epoch);
      if (idx.size() != n_samples) throw Error(MMN_E_INVALID, "order must list every sample");
      GradAccumulator accum;  // a new one per epoch (lib.rs:390)
      size_t micro = 0;
      for (size_t i = 0; i < idx.size(); ++i) {
        backward(idx[i], grads);
        if (batch_size == 1) {
          // train_step_lm without an accumulator: backward_lm steps at once
          step_.step_host(grads, params, 1.0f);
          param_id_ += n;
          ++steps_;
          continue;
        }
        ++micro;
        accum.begin_micro_batch();
        for (const ArrayD& g : grads) accum.add_param_grad(g);
        accum.finish_micro_batch();
        if (micro >= batch_size || i + 1 == idx.size()) {  // lib.rs:431
          // apply_accumulated_lm_grads: averaged_grad divides each sum by the
          // micro-batch count; the GPU step does that division itself
          sums_.resize(n);
          for (size_t k = 0; k < n; ++k) sums_[k] = accum.sum(k);
          step_.step_host(sums_, params, (float)accum.micro_batches());
          param_id_ += n;
          ++steps_;
          accum.clear();
          micro = 0;
        }
      }
    }
  }

  // The reference's param_id after the run: one id per tensor per step.
  size_t param_id() const { return param_id_; }
  size_t steps() const { return steps_; }

 private:
  TrainConfig cfg_;
  Step& step_;
  std::vector<ArrayD> sums_;
  size_t param_id_ = 0;
  size_t steps_ = 0;
};

// The trainer's device optimizer for tensors in call order, with the CUDA
// gate of crates/mmn-train/src/lib.rs:360-361 (cuda without a usable GPU
// throws CudaError). The product path is the GPU: a configuration without
// cuda belongs to the reference's own CPU optimizer, and is refused.
class Trainer {
 public:
  Trainer(const TrainConfig& cfg, const std::vector<OptimizerStep::Tensor>& tensors,
          const std::vector<ArrayD>& params, int device = 0)
      : cfg_(gate(cfg)), step_(tensors, optim_config_for(cfg_), device), loop_(cfg_, step_) {
    if (params.size() != step_.size()) throw Error(MMN_E_INVALID, "need one param per tensor");
    for (size_t k = 0; k < params.size(); ++k) step_.set_param((int)k, params[k]);
  }

  void train(size_t n_samples, const TrainLoop<OptimizerStep>::Order& order,
             const TrainLoop<OptimizerStep>::Backward& backward, std::vector<ArrayD>& params) {
    loop_.train(n_samples, order, backward, params);
  }

  size_t param_id() const { return loop_.param_id(); }
  size_t steps() const { return loop_.steps(); }
  OptimizerStep& optimizer() { return step_; }

 private:
  static const TrainConfig& gate(const TrainConfig& c) {
    require_cuda(c.cuda);
    if (!c.cuda)
      throw Error(MMN_E_UNSUPPORTED,
                  "cuda=false trains with the reference's CPU optimizer; this library "
                  "steps on the GPU (TrainConfig.cuda = true)");
    return c;
  }
  TrainConfig cfg_;
  OptimizerStep step_;
  TrainLoop<OptimizerStep> loop_;
};

}  // namespace mmn

#endif  // MMN_TRAIN_HPP
