// The reference's own unit tests of crates/mmn-optim/src/lib.rs:264-382,
// restated against the C++ mirror of its API (include/mmn_optim.hpp), plus
// parity checks of the same calls against the CPU oracle (oracle/, which only
// this test program links).
//
// Usage: test_optim_api [--cpu-only]
//   --cpu-only runs the tests that need no GPU (routing table, accumulator,
//   the CUDA gate); without it every test runs and a B200 is required.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

#include "mmn_optim.hpp"
#include "mmn_optim_ref.h"

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

ArrayD arr2(std::vector<std::vector<float>> rows) {
  std::vector<float> v;
  for (auto& r : rows) v.insert(v.end(), r.begin(), r.end());
  return ArrayD({(int64_t)rows.size(), (int64_t)rows[0].size()}, v);
}

double rel_fro(const std::vector<float>& a, const std::vector<float>& b) {
  double d = 0, n = 0;
  for (size_t i = 0; i < a.size(); ++i) {
    d += ((double)a[i] - b[i]) * ((double)a[i] - b[i]);
    n += (double)b[i] * b[i];
  }
  return std::sqrt(d) / (n > 0 ? std::sqrt(n) : 1.0);
}

ArrayD normal(std::mt19937& rng, std::vector<int64_t> shape, float sigma) {
  std::normal_distribution<float> d(0.0f, sigma);
  ArrayD a(std::move(shape));
  for (float& x : a.data) x = d(rng);
  return a;
}

// ------------------------------------------------------ CPU (no GPU) tests
void cpu_tests() {
  // lib.rs:283-293
  run("grad_accumulator_averages_two_micro_batches", [] {
    mmn::GradAccumulator acc;
    acc.begin_micro_batch();
    acc.add_param_grad(arr2({{1.0f}}));
    acc.finish_micro_batch();
    acc.begin_micro_batch();
    acc.add_param_grad(arr2({{3.0f}}));
    acc.finish_micro_batch();
    EXPECT(std::fabs(acc.averaged_grad(0).at(0, 0) - 2.0f) < 1e-6f);
  });
  // lib.rs:303-320
  run("classify_param_matrix_vs_other", [] {
    using H = mmn::HybridOptimizer;
    EXPECT(H::classify_param({64, 32}) == mmn::ParamKind::Matrix);
    EXPECT(H::classify_param({16}) == mmn::ParamKind::Other);
    EXPECT(H::classify_param({16, 1}) == mmn::ParamKind::Other);
    EXPECT(H::classify_param({1, 3, 3, 3}) == mmn::ParamKind::Other);
  });
  // lib.rs:371-381
  run("grad_accumulator_clear_resets_state", [] {
    mmn::GradAccumulator acc;
    acc.begin_micro_batch();
    acc.add_param_grad(arr2({{1.0f}}));
    acc.finish_micro_batch();
    EXPECT(acc.micro_batches() == 1);
    acc.clear();
    EXPECT(acc.micro_batches() == 0);
    EXPECT(acc.len() == 0);
  });
  // crates/mmn-core/src/device.rs:29-37: cuda=True without a GPU is CUDAError
  run("cuda_gate", [] {
    mmn::require_cuda(false);
    if (mmn::cuda::is_available()) {
      mmn::require_cuda(true);
      return;
    }
    bool threw = false;
    try {
      mmn::require_cuda(true);
    } catch (const mmn::CudaError& e) {
      threw = e.code() == MMN_E_NO_DEVICE;
    }
    EXPECT(threw);
    threw = false;
    try {
      mmn::AdamW opt;
    } catch (const mmn::CudaError&) {
      threw = true;
    }
    EXPECT(threw);
  });
  // the defaults of lib.rs:13-21 and lib.rs:71-80
  run("config_defaults", [] {
    const mmn::AdamWConfig a;
    const mmn_adamw_config c = mmn_adamw_config_default();
    EXPECT(a.lr == c.lr && a.betas.first == c.beta1 && a.betas.second == c.beta2 &&
           a.eps == c.eps && a.weight_decay == c.weight_decay);
    const mmn::MuonConfig m;
    const mmn_muon_config mc = mmn_muon_config_default();
    EXPECT(m.lr == mc.lr && m.momentum == mc.momentum && (int)m.nesterov == mc.nesterov &&
           (int)m.ns_steps == mc.ns_steps);
  });
}

// ------------------------------------------------------------- GPU tests
ArrayD muon_p() {
  return ArrayD::from_shape_fn(4, 4, [](int64_t i, int64_t j) { return 1.0f + (float)(i + j) * 0.01f; });
}
ArrayD muon_g() {
  return ArrayD::from_shape_fn(4, 4, [](int64_t i, int64_t j) {
    return 0.1f + (float)i * 0.02f + (float)j * 0.03f;
  });
}

void gpu_tests() {
  // lib.rs:269-281
  run("adamw_changes_weights", [] {
    ArrayD p = arr2({{1.0f}});
    const ArrayD g = arr2({{0.5f}});
    mmn::AdamWConfig cfg;
    cfg.lr = 0.1f;
    mmn::AdamW opt(cfg);
    const float before = p.at(0, 0);
    opt.step_param(0, p, g);
    EXPECT(p.at(0, 0) != before);
  });
  // lib.rs:295-300
  run("newton_schulz_output_finite", [] {
    const ArrayD o = mmn::newton_schulz5(arr2({{1.0f, 0.0f}, {0.0f, 1.0f}}), 5);
    for (float x : o.data) EXPECT(std::isfinite(x));
  });
  // lib.rs:322-328
  run("newton_schulz_output_nonzero", [] {
    const ArrayD g = ArrayD::from_shape_fn(4, 4, [](int64_t i, int64_t j) { return (float)(i + j) * 0.1f; });
    const ArrayD o = mmn::newton_schulz5(g, 5);
    float s = 0;
    for (float x : o.data) s += std::fabs(x);
    EXPECT(s > 1e-6f);
  });
  // lib.rs:330-342
  run("muon_step_matrix_changes_weights", [] {
    mmn::MuonConfig cfg;
    cfg.lr = 0.1f;
    mmn::Muon opt(cfg);
    ArrayD p = muon_p();
    const ArrayD before = p;
    opt.step_matrix(0, p, muon_g());
    EXPECT(p != before);
  });
  // lib.rs:344-359
  run("hybrid_routes_matrix_to_muon", [] {
    mmn::MuonConfig mc;
    mc.lr = 0.1f;
    mmn::HybridOptimizer opt(mc, mmn::AdamWConfig{});
    ArrayD p = muon_p();
    const ArrayD before = p;
    opt.step(0, p, muon_g());
    EXPECT(p != before);
    EXPECT(opt.adamw.step() == 0);  // the matrix did not touch AdamW
  });
  // lib.rs:361-369
  run("hybrid_vector_step_uses_adamw", [] {
    mmn::HybridOptimizer opt;
    ArrayD p = arr2({{1.0f}, {2.0f}, {3.0f}});
    const ArrayD g = arr2({{0.5f}, {0.5f}, {0.5f}});
    const float before = p.at(0, 0);
    opt.step(1, p, g);
    EXPECT(p.at(0, 0) != before);
    EXPECT(opt.adamw.step() == 1);
  });
  // lib.rs:148,161 panic on a shape that differs from an id's state: an error here
  run("shape_mismatch_is_an_error", [] {
    mmn::AdamW opt;
    ArrayD p({8}), g({8});
    opt.step_param(3, p, g);
    ArrayD p2({4}), g2({4});
    bool threw = false;
    try {
      opt.step_param(3, p2, g2);
    } catch (const mmn::Error& e) {
      threw = e.code() == MMN_E_SHAPE;
    }
    EXPECT(threw);
  });

  // ---- parity with the CPU oracle
  run("adamw_parity_bit_exact_three_steps", [] {
    std::mt19937 rng(1);
    mmn::AdamWConfig cfg;
    cfg.lr = 1e-3f;
    cfg.betas = {0.9f, 0.999f};
    mmn::AdamW opt(cfg);
    std::vector<std::vector<int64_t>> shapes = {{64}, {33, 5}, {1000}};
    std::vector<ArrayD> ps, rs, ms, vs;
    for (auto& s : shapes) {
      ps.push_back(normal(rng, s, 0.02f));
      rs.push_back(ps.back());
      ms.emplace_back(s);
      vs.emplace_back(s);
    }
    int64_t t = 0;
    for (int step = 0; step < 3; ++step)
      for (size_t k = 0; k < shapes.size(); ++k) {
        const ArrayD g = normal(rng, shapes[k], 1e-3f);
        opt.step_param(k, ps[k], g);
        ref_adamw_step(rs[k].data.data(), ms[k].data.data(), vs[k].data.data(), g.data.data(),
                       (int64_t)g.len(), cfg.lr, cfg.betas.first, cfg.betas.second, cfg.eps,
                       cfg.weight_decay, ++t, 1.0f);  // one counter per instance
        EXPECT(std::memcmp(ps[k].data.data(), rs[k].data.data(), g.len() * 4) == 0);
      }
  });
  auto muon_parity = [](int ns_mode, int variant, double tol) {
    std::mt19937 rng(2);
    const mmn::MuonConfig cfg;
    mmn::Muon opt(cfg, ns_mode);
    for (auto shape : std::vector<std::vector<int64_t>>{{64, 256}, {256, 64}, {96, 96}}) {
      ArrayD p = normal(rng, shape, 0.02f);
      const ArrayD before = p;
      const ArrayD g = normal(rng, shape, 1e-3f);
      static size_t id = 0;
      opt.step_matrix(++id, p, g);
      std::vector<float> vel(g.len(), 0.0f), u(g.len()), o(g.len());
      std::vector<float> want = before.data;
      ref_muon_momentum(vel.data(), g.data.data(), u.data(), (int64_t)g.len(), cfg.momentum,
                        cfg.nesterov, 1.0f);
      ref_newton_schulz5(u.data(), shape[0], shape[1], (int)cfg.ns_steps, o.data(),
                         REF_GEMM_F64, variant, nullptr, 0);
      ref_muon_apply(want.data(), o.data(), shape[0], shape[1], cfg.lr);
      std::vector<float> du(g.len()), dw(g.len());
      for (size_t i = 0; i < g.len(); ++i) {
        du[i] = p.data[i] - before.data[i];
        dw[i] = want[i] - before.data[i];
      }
      const double r = rel_fro(du, dw);
      if (!(r <= tol)) std::fprintf(stderr, "  update differs by %.3e (bar %.1e)\n", r, tol);
      EXPECT(r <= tol);
    }
  };
  // The whole-model step (the trainer's call) on the Chatbot(vocab 512, 2
  // layers, d_model 64) tensors in the reference's call order
  // (crates/mmn-models/src/chatbot.rs:1104-1196), routed by the shape rule:
  // AdamW tensors bit-exact with the per-call counter, Muon within 2e-2; the
  // step from host memory equals the device-resident step bit for bit.
  run("optimizer_step_chatbot_vs_oracle", [] {
    std::vector<std::vector<int64_t>> shapes = {{512, 64}};
    for (int layer = 1; layer >= 0; --layer) {
      (void)layer;
      for (auto s : std::vector<std::vector<int64_t>>{{64, 256}, {256, 64}, {64, 64}, {64, 64},
                                                      {64, 64}, {64, 64}, {64}, {64}, {64}, {64}})
        shapes.push_back(s);
    }
    shapes.push_back({512, 64});
    EXPECT(shapes.size() == 22);
    std::vector<mmn::OptimizerStep::Tensor> ts;
    for (size_t k = 0; k < shapes.size(); ++k) ts.push_back({k, shapes[k], MMN_ROUTE_AUTO});
    mmn_optim_config cfg = mmn::OptimizerStep::default_config();
    cfg.adamw.lr = 1e-3f;
    cfg.adamw.beta2 = 0.999f;
    cfg.use_graph = 0;
    mmn::OptimizerStep dev(ts, cfg), host(ts, cfg);
    std::mt19937 rng(7);
    std::vector<ArrayD> p, g;
    for (auto& s : shapes) {
      p.push_back(normal(rng, s, 0.02f));
      g.push_back(normal(rng, s, 1e-3f));
    }
    for (size_t k = 0; k < shapes.size(); ++k) {
      dev.set_param((int)k, p[k]);
      host.set_param((int)k, p[k]);
      dev.set_grad((int)k, g[k]);
    }
    dev.step();
    dev.sync();
    std::vector<ArrayD> out_host(shapes.size());
    for (size_t k = 0; k < shapes.size(); ++k) out_host[k] = ArrayD(shapes[k]);
    host.step_host(g, out_host);
    int64_t t = 0;
    const mmn::MuonConfig mc;
    for (size_t k = 0; k < shapes.size(); ++k) {
      const ArrayD got = dev.get_param((int)k);
      EXPECT(std::memcmp(got.data.data(), out_host[k].data.data(), got.len() * 4) == 0);
      std::vector<float> want = p[k].data;
      const int64_t n = (int64_t)want.size();
      if (mmn::HybridOptimizer::classify_param(shapes[k]) == mmn::ParamKind::Other) {
        std::vector<float> m((size_t)n, 0.0f), v((size_t)n, 0.0f);
        ref_adamw_step(want.data(), m.data(), v.data(), g[k].data.data(), n, cfg.adamw.lr,
                       cfg.adamw.beta1, cfg.adamw.beta2, cfg.adamw.eps, cfg.adamw.weight_decay,
                       ++t, 1.0f);
        EXPECT(std::memcmp(got.data.data(), want.data(), (size_t)n * 4) == 0);
      } else {
        std::vector<float> vel((size_t)n, 0.0f), u((size_t)n), o((size_t)n);
        ref_muon_momentum(vel.data(), g[k].data.data(), u.data(), n, mc.momentum, 1, 1.0f);
        ref_newton_schulz5(u.data(), shapes[k][0], shapes[k][1], (int)mc.ns_steps, o.data(),
                           REF_GEMM_F64, REF_NS_REFERENCE, nullptr, 0);
        ref_muon_apply(want.data(), o.data(), shapes[k][0], shapes[k][1], mc.lr);
        std::vector<float> du((size_t)n), dw((size_t)n);
        for (int64_t i = 0; i < n; ++i) {
          du[(size_t)i] = got.data[(size_t)i] - p[k].data[(size_t)i];
          dw[(size_t)i] = want[(size_t)i] - p[k].data[(size_t)i];
        }
        EXPECT(rel_fro(du, dw) <= 2e-2);
      }
    }
    EXPECT(dev.adamw_step() == (uint64_t)t);  // one count per AdamW tensor
  });
  run("muon_parity_reference_mode_2e-2", [&] { muon_parity(MMN_NS_REFERENCE, REF_NS_REFERENCE, 2e-2); });
  run("muon_parity_tf32_mode_3e-3", [&] { muon_parity(MMN_NS_TF32, REF_NS_TF32, 3e-3); });
  run("muon_parity_fp32_mode_1e-4", [&] { muon_parity(MMN_NS_FP32, REF_NS_FP32, 1e-4); });
}

}  // namespace

int main(int argc, char** argv) {
  const bool cpu_only = argc > 1 && std::strcmp(argv[1], "--cpu-only") == 0;
  cpu_tests();
  if (!cpu_only) gpu_tests();
  std::printf("%d passed, %d failed\n", passed, failures);
  return failures ? 1 : 0;
}
