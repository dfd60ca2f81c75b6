// The trainer's optimizer plumbing (crates/mmn-train/src/lib.rs:354-448) driven
// through the GPU step (include/mmn_train.hpp) and checked against the
// reference's per-call step on the CPU oracle.
//
// Usage: test_train_loop [--cpu-only]
//   --cpu-only: the loop itself against a literal restatement of
//   train_with_encoder on the oracle (flush points, the ragged last batch,
//   averaging, ids and step counters), the config mapping and the CUDA gate.
//   Without it, also the GPU trainer against the oracle replay on the
//   Chatbot(vocab 512, 2 layers, d_model 64) tensors: AdamW tensors bit for
//   bit, Muon tensors within 2e-2 relative Frobenius of their total update.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

#include "mmn_train.hpp"
#include "oracle_step.hpp"

namespace {

int failures = 0, passed = 0;

#define EXPECT(cond)                                                             \
  do {                                                                           \
    if (!(cond)) {                                                               \
      std::fprintf(stderr, "  FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);   \
      throw std::runtime_error("expectation failed");                           \
    }                                                                            \
  } while (0)

void run(const char* name, const std::function<void()>& fn) {
  try {
    fn();
    ++passed;
    std::printf("ok   %s\n", name);
  } catch (const std::exception& e) {
    ++failures;
    std::printf("FAIL %s: %s\n", name, e.what());
  }
}

using mmn::ArrayD;

// Chatbot tensors in optimizer call order (crates/mmn-models/src/chatbot.rs:
// 1104-1196): lm_head; blocks last..first as ffn2, ffn, out, q, k, v,
// ln2.gamma, ln2.beta, ln1.gamma, ln1.beta; embed.
std::vector<std::vector<int64_t>> chatbot_shapes(int64_t vocab, int n_layer, int64_t d) {
  std::vector<std::vector<int64_t>> s{{vocab, d}};
  for (int l = n_layer - 1; l >= 0; --l) {
    s.push_back({d, 4 * d});
    s.push_back({4 * d, d});
    for (int k = 0; k < 4; ++k) s.push_back({d, d});
    for (int k = 0; k < 4; ++k) s.push_back({d});
  }
  s.push_back({vocab, d});
  return s;
}

// Seeded values: Linear U(-s/2, s/2) with s = sqrt(2/(in+out))
// (crates/mmn-nn/src/lib.rs:300-304), embeddings U(-1, 1), LayerNorm gamma 1
// and beta 0; a sample's grads N(0, 1e-3) from a seed of (sample, tensor).
std::vector<ArrayD> init_params(const std::vector<std::vector<int64_t>>& shapes) {
  std::mt19937 rng(0);
  std::vector<ArrayD> p;
  for (size_t k = 0; k < shapes.size(); ++k) {
    ArrayD a(shapes[k]);
    if (shapes[k].size() == 1) {
      const bool gamma = (k % 10) == 7 || (k % 10) == 9;  // ln2.gamma, ln1.gamma positions
      for (float& x : a.data) x = gamma ? 1.0f : 0.0f;
    } else if (k + 1 == shapes.size()) {  // embed (crates/mmn-core/src/tensor.rs:50-57)
      std::uniform_real_distribution<float> u(-1.0f, 1.0f);
      for (float& x : a.data) x = u(rng);
    } else {
      const float s = std::sqrt(2.0f / (float)(shapes[k][0] + shapes[k][1]));
      std::uniform_real_distribution<float> u(-s / 2, s / 2);
      for (float& x : a.data) x = u(rng);
    }
    p.push_back(std::move(a));
  }
  return p;
}

void sample_grads(size_t sample, std::vector<ArrayD>& grads) {
  for (size_t k = 0; k < grads.size(); ++k) {
    std::mt19937 rng((uint32_t)(1000003u * sample + 7919u * k + 17u));
    std::normal_distribution<float> nd(0.0f, 1e-3f);
    for (float& x : grads[k].data) x = nd(rng);
  }
}

std::vector<size_t> shuffled(size_t n, size_t epoch) {
  std::vector<size_t> idx(n);
  for (size_t i = 0; i < n; ++i) idx[i] = i;
  std::mt19937 rng((uint32_t)(42 + epoch));
  for (size_t i = 0; i < n; ++i) std::swap(idx[i], idx[(size_t)(rng() % n)]);  // lib.rs:385-389
  return idx;
}

bool same_bits(const ArrayD& a, const ArrayD& b) {
  return a.data.size() == b.data.size() &&
         std::memcmp(a.data.data(), b.data.data(), a.data.size() * 4) == 0;
}

double rel_update(const ArrayD& got, const ArrayD& want, const ArrayD& p0) {
  double d = 0, n = 0;
  for (size_t i = 0; i < p0.data.size(); ++i) {
    const double a = (double)got.data[i] - p0.data[i], b = (double)want.data[i] - p0.data[i];
    d += (a - b) * (a - b);
    n += b * b;
  }
  return std::sqrt(d) / (n > 0 ? std::sqrt(n) : 1.0);
}

// train_with_encoder's loop (crates/mmn-train/src/lib.rs:382-442) written out
// literally on the oracle, one optim_step_weight call per tensor with its own
// id, for the loop under test to be compared against.
struct LiteralRun {
  std::vector<ArrayD> params;
  size_t param_id = 0;
};

LiteralRun literal_train(const mmn::TrainConfig& cfg,
                         const std::vector<std::vector<int64_t>>& shapes, size_t n_samples) {
  LiteralRun r;
  r.params = init_params(shapes);
  const bool use_hybrid = cfg.optimizer == "hybrid";
  const mmn_adamw_config ad = [&] {
    mmn_adamw_config c = mmn_adamw_config_default();
    c.lr = cfg.learning_rate;
    return c;
  }();
  const mmn_muon_config mu = mmn_muon_config_default();
  int64_t t_hybrid = 0, t_adamw = 0;
  // optim_step_weight (chatbot.rs:208-227) for one tensor and its averaged grad
  auto optim_step_weight = [&](size_t k, const ArrayD& g) {
    const auto& s = shapes[k];
    float* p = r.params[k].data.data();
    const int64_t n = g.len();
    if (use_hybrid && s.size() == 2 && s[0] > 1 && s[1] > 1) {
      std::vector<float> vel((size_t)n, 0.0f), u((size_t)n), o((size_t)n);  // id is new
      ref_muon_momentum(vel.data(), g.data.data(), u.data(), n, mu.momentum, mu.nesterov, 1.0f);
      ref_newton_schulz5(u.data(), s[0], s[1], mu.ns_steps, o.data(), REF_GEMM_F64,
                         REF_NS_REFERENCE, nullptr, 0);
      ref_muon_apply(p, o.data(), s[0], s[1], mu.lr);
    } else {
      std::vector<float> m((size_t)n, 0.0f), v((size_t)n, 0.0f);
      int64_t& t = use_hybrid ? t_hybrid : t_adamw;
      ++t;
      ref_adamw_step(p, m.data(), v.data(), g.data.data(), n, ad.lr, ad.beta1, ad.beta2,
                     ad.eps, ad.weight_decay, t, 1.0f);
    }
    ++r.param_id;
  };
  const size_t batch_size = cfg.batch_size > 0 ? cfg.batch_size : 1;
  std::vector<ArrayD> grads;
  for (const auto& s : shapes) grads.emplace_back(s);
  for (size_t epoch = 0; epoch < cfg.epochs; ++epoch) {
    const std::vector<size_t> idx = shuffled(n_samples, epoch);
    mmn::GradAccumulator accum;
    size_t micro = 0;
    for (size_t i = 0; i < idx.size(); ++i) {
      sample_grads(idx[i], grads);
      if (batch_size == 1) {
        for (size_t k = 0; k < shapes.size(); ++k) optim_step_weight(k, grads[k]);
        continue;
      }
      ++micro;
      accum.begin_micro_batch();
      for (const ArrayD& g : grads) accum.add_param_grad(g);
      accum.finish_micro_batch();
      if (micro >= batch_size || i + 1 == idx.size()) {
        for (size_t k = 0; k < shapes.size(); ++k) optim_step_weight(k, accum.averaged_grad(k));
        accum.clear();
        micro = 0;
      }
    }
  }
  return r;
}

mmn::TrainConfig config(const std::string& optimizer, size_t batch_size, size_t epochs) {
  mmn::TrainConfig c;
  c.cuda = true;
  c.optimizer = optimizer;
  c.batch_size = batch_size;
  c.epochs = epochs;
  c.learning_rate = 1e-3f;
  return c;
}

const size_t kSamples = 10;  // with batch_size 3: batches of 3, 3, 3 and a ragged 1

}  // namespace

int main(int argc, char** argv) {
  const bool cpu_only = argc > 1 && std::strcmp(argv[1], "--cpu-only") == 0;
  const auto shapes = chatbot_shapes(512, 2, 64);

  run("train_config_defaults_and_repr", [] {
    mmn::TrainConfig c;
    EXPECT(c.epochs == 1 && c.batch_size == 8 && !c.cuda && c.optimizer == "hybrid");
    EXPECT(std::fabs(c.learning_rate - 3e-4f) == 0.0f);
    EXPECT(c.repr() == "TrainConfig(epochs=1, batch_size=8, cuda=false, optimizer=\"hybrid\", "
                       "learning_rate=0.0003)");
  });

  run("optimizer_construction", [] {
    // lib.rs:367-380: hybrid only for "hybrid" ("muon" falls back to AdamW),
    // AdamW lr from the config with default betas, Muon defaults, new ids
    mmn::TrainConfig c = config("muon", 4, 1);
    c.learning_rate = 5e-4f;
    const mmn_optim_config o = mmn::optim_config_for(c);
    EXPECT(o.use_hybrid == 0 && o.fresh_state == 1);
    EXPECT(o.adamw.lr == 5e-4f && o.adamw.beta1 == 0.9f && o.adamw.beta2 == 0.95f);
    EXPECT(o.muon.lr == 0.02f && o.muon.ns_steps == 5);
    EXPECT(mmn::optim_config_for(config("hybrid", 4, 1)).use_hybrid == 1);
  });

  run("cpu_config_is_refused", [&] {
    mmn::TrainConfig c = config("hybrid", 3, 1);
    c.cuda = false;
    try {
      mmn::Trainer t(c, {}, {});
      EXPECT(false);
    } catch (const mmn::Error& e) {
      EXPECT(e.code() == MMN_E_UNSUPPORTED);
    }
  });

  // The loop under test on the oracle stepper against the literal restatement:
  // identical parameters bit for bit and the same ids.
  for (const auto& opt : {std::string("hybrid"), std::string("adamw")}) {
    for (size_t bs : {(size_t)3, (size_t)1}) {
      const std::string name = "loop_matches_literal_" + opt + "_bs" + std::to_string(bs);
      run(name.c_str(), [&] {
        const mmn::TrainConfig c = config(opt, bs, 2);
        const LiteralRun lit = literal_train(c, shapes, kSamples);
        mmn_test::OracleStep step(c, shapes);
        mmn::TrainLoop<mmn_test::OracleStep> loop(c, step);
        std::vector<ArrayD> params = init_params(shapes);
        loop.train(kSamples, [](size_t e) { return shuffled(kSamples, e); }, sample_grads, params);
        const size_t per_epoch = bs == 1 ? kSamples : (kSamples + bs - 1) / bs;
        EXPECT(loop.steps() == 2 * per_epoch);
        EXPECT(loop.param_id() == lit.param_id && lit.param_id == 2 * per_epoch * shapes.size());
        for (size_t k = 0; k < shapes.size(); ++k) EXPECT(same_bits(params[k], lit.params[k]));
      });
    }
  }

  if (!cpu_only) {
    // The GPU trainer against the oracle replay of the same run.
    for (const auto& opt : {std::string("hybrid"), std::string("adamw"), std::string("muon")}) {
      for (size_t bs : {(size_t)3, (size_t)1}) {
        const std::string name = "gpu_trainer_matches_oracle_" + opt + "_bs" + std::to_string(bs);
        run(name.c_str(), [&] {
          const mmn::TrainConfig c = config(opt, bs, 2);
          const std::vector<ArrayD> p0 = init_params(shapes);
          std::vector<mmn::OptimizerStep::Tensor> tensors;
          for (size_t k = 0; k < shapes.size(); ++k) tensors.push_back({k, shapes[k]});
          std::vector<ArrayD> gpu = p0;
          mmn::Trainer trainer(c, tensors, gpu);
          trainer.train(kSamples, [](size_t e) { return shuffled(kSamples, e); }, sample_grads,
                        gpu);
          mmn_test::OracleStep step(c, shapes);
          mmn::TrainLoop<mmn_test::OracleStep> loop(c, step);
          std::vector<ArrayD> ref = p0;
          loop.train(kSamples, [](size_t e) { return shuffled(kSamples, e); }, sample_grads, ref);
          EXPECT(trainer.steps() == loop.steps() && trainer.param_id() == loop.param_id());
          const bool hybrid = opt == "hybrid";
          for (size_t k = 0; k < shapes.size(); ++k) {
            const bool matrix = hybrid && shapes[k].size() == 2;
            if (matrix) {
              const double rel = rel_update(gpu[k], ref[k], p0[k]);
              if (rel > 2e-2) std::fprintf(stderr, "  tensor %zu: %.3e\n", k, rel);
              EXPECT(rel <= 2e-2);
            } else {
              EXPECT(same_bits(gpu[k], ref[k]));
            }
          }
          // the device AdamW counter: one call per AdamW tensor per step
          size_t adamw_tensors = 0;
          for (const auto& s : shapes) adamw_tensors += (!hybrid || s.size() != 2) ? 1 : 0;
          EXPECT(trainer.optimizer().adamw_step() == adamw_tensors * trainer.steps());
        });
      }
    }
  }

  std::printf("%d passed, %d failed\n", passed, failures);
  return failures ? 1 : 0;
}
