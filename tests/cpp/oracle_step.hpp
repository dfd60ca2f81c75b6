// The reference's per-call optimizer step, on the CPU oracle (test
// infrastructure only): one training step's optim_step_weight calls
// (crates/mmn-models/src/chatbot.rs:208-227) for every tensor in call order,
// each with a new id, through HybridOptimizer::step (routing by shape,
// crates/mmn-optim/src/lib.rs:204-209) or the trainer's separate AdamW
// (crates/mmn-train/src/lib.rs:371-378), with GradAccumulator::averaged_grad
// (lib.rs:254-257) applied first. The stepper interface of mmn::TrainLoop.
#ifndef MMN_TEST_ORACLE_STEP_HPP
#define MMN_TEST_ORACLE_STEP_HPP

#include <cmath>
#include <cstdint>
#include <vector>

#include "mmn_optim_ref.h"
#include "mmn_train.hpp"

namespace mmn_test {

class OracleStep {
 public:
  OracleStep(const mmn::TrainConfig& cfg, const std::vector<std::vector<int64_t>>& shapes,
             int gemm_order = REF_GEMM_F64)
      : cfg_(cfg), shapes_(shapes), order_(gemm_order) {}

  size_t size() const { return shapes_.size(); }

  void step_host(const std::vector<mmn::ArrayD>& grads, std::vector<mmn::ArrayD>& params,
                 float divisor) {
    const bool hybrid = cfg_.optimizer == "hybrid";
    const mmn_adamw_config ad = adamw_cfg();
    const mmn_muon_config mu = mmn_muon_config_default();
    for (size_t k = 0; k < shapes_.size(); ++k) {
      mmn::ArrayD g = grads[k];
      // GradAccumulator::averaged_grad; x / 1 is x (batch_size 1 steps raw grads)
      ref_grad_average(grads[k].data.data(), g.data.data(), g.len(), (int64_t)divisor);
      float* p = params[k].data.data();
      const int64_t n = g.len();
      const auto& s = shapes_[k];
      const bool matrix = s.size() == 2 && s[0] > 1 && s[1] > 1;  // lib.rs:196-202
      if (hybrid && matrix) {
        // Muon::step_matrix with a new id: zero velocity
        std::vector<float> vel((size_t)n, 0.0f), u((size_t)n), o((size_t)n);
        ref_muon_momentum(vel.data(), g.data.data(), u.data(), n, mu.momentum, mu.nesterov, 1.0f);
        ref_newton_schulz5(u.data(), s[0], s[1], mu.ns_steps, o.data(), order_, REF_NS_REFERENCE,
                           nullptr, 0);
        ref_muon_apply(p, o.data(), s[0], s[1], mu.lr);
      } else {
        // AdamW::step_param with a new id: zero m and v, the instance's next t
        std::vector<float> m((size_t)n, 0.0f), v((size_t)n, 0.0f);
        int64_t& t = hybrid ? t_hybrid_ : t_adamw_;
        ++t;
        ref_adamw_step(p, m.data(), v.data(), g.data.data(), n, ad.lr, ad.beta1, ad.beta2, ad.eps,
                       ad.weight_decay, t, 1.0f);
      }
    }
  }

 private:
  mmn_adamw_config adamw_cfg() const {
    mmn_adamw_config c = mmn_adamw_config_default();
    c.lr = cfg_.learning_rate;
    return c;
  }
  mmn::TrainConfig cfg_;
  std::vector<std::vector<int64_t>> shapes_;
  int order_;
  int64_t t_hybrid_ = 0;  // HybridOptimizer.adamw's step counter
  int64_t t_adamw_ = 0;   // the trainer's separate AdamW
};

}  // namespace mmn_test

#endif
