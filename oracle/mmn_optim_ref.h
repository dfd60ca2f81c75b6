/*
 * CPU oracle for the MagicMindNet optimizer step — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of crates/mmn-optim/src/lib.rs (AdamW, Muon,
 * newton_schulz5, GradAccumulator averaging). Only tests/, the smoke check and
 * bench.py's CPU-baseline leg may load this library; the CUDA product path never
 * links or calls it.
 *
 * Parity pinning: the reference is Rust and no Rust toolchain exists on either
 * machine, so the reference cannot be run to produce golden outputs, and its own
 * tests pin only the GradAccumulator average (lib.rs:283-293) and the routing
 * table (lib.rs:303-320). Everything else here is pinned by known-answer tests
 * derived from the arithmetic: tests/golden/known_answers.json, written by
 * tests/golden/make_golden.py from a numpy restatement of the reference's
 * operation order that does not use this library, and the closed forms of
 * tests/test_oracle.py. Parity is therefore "partially
 * pinned": AdamW/momentum/update arithmetic is a literal restatement of the
 * reference's operation order; the Newton-Schulz GEMM summation order of the
 * reference (matrixmultiply 0.3.10 sgemm) is not reproduced.
 *
 * Floating-point rules: compiled with -ffp-contract=off so every a*b+c rounds
 * twice, as Rust does (Rust never contracts to FMA). bf16 rounding is
 * round-to-nearest-even on the f32 bit pattern, the behaviour of
 * half 2.7.1 bf16::from_f32 (Cargo.lock:521-524).
 */
#ifndef MMN_OPTIM_REF_H
#define MMN_OPTIM_REF_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GEMM summation order used inside the Newton-Schulz restatement. */
enum {
    REF_GEMM_F32_SEQ = 0, /* fp32 accumulator, k in order, separate mul and add */
    REF_GEMM_F32_FMA = 1, /* fp32 accumulator, k in order, fused multiply-add   */
    REF_GEMM_F64 = 2      /* fp64 accumulator, one rounding to fp32 at the end  */
};

/* Newton-Schulz recipe variants. */
enum {
    REF_NS_REFERENCE = 0, /* lib.rs:112-120 exactly: B = b*A_bf + c*A2_bf kept fp32 */
    REF_NS_BF16 = 1,      /* fast variant (no reference counterpart): B rounded to bf16 */
    REF_NS_TF32 = 2,      /* TF32 mode (no reference counterpart): the REF_NS_REFERENCE
                             recipe with every bf16 rounding point of lib.rs:104,115,116,119
                             replaced by a tf32 rounding (10-bit mantissa, nearest-even),
                             and the norm's sum of squares rounded to fp32 once, as in
                             REF_NS_FP32 */
    REF_NS_FP32 = 3       /* fp32 mode (no reference counterpart): the same recipe with no
                             rounding points at all, every value kept in fp32, and the
                             norm's sum of squares rounded to fp32 once */
};

float ref_bf16_round(float x);
float ref_tf32_round(float x);

/* AdamW::step_param (lib.rs:41-60) for one tensor whose step counter is already t. */
void ref_adamw_step(float *p, float *m, float *v, const float *g, int64_t n,
                    float lr, float beta1, float beta2, float eps, float weight_decay,
                    int64_t t, float grad_divisor);

/* Muon momentum (lib.rs:154-165): updates vel in place, writes the NS input to u. */
void ref_muon_momentum(float *vel, const float *g, float *u, int64_t n,
                       float momentum, int nesterov, float grad_divisor);

/* newton_schulz5 (lib.rs:83-126) for a rows x cols matrix. out is rows x cols.
 * norm_out (optional) receives the clamped Frobenius norm. n_threads <= 0 uses
 * every OpenMP thread. Returns 0. */
int ref_newton_schulz5(const float *g, int64_t rows, int64_t cols, int steps,
                       float *out, int gemm_order, int variant, float *norm_out,
                       int n_threads);

/* One Newton-Schulz iteration on an n x m (n <= m) fp32 matrix x (bf16-valued
 * or pre-normalised), writing the next x. Exposed for per-iteration parity. */
void ref_ns_iteration(const float *x, int64_t n, int64_t m, float *x_next,
                      int gemm_order, int variant, int n_threads);

/* C = A * B, A is M x K, B is K x N, all row-major. */
void ref_gemm(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K,
              int gemm_order, int n_threads);

/* Muon::step_matrix tail (lib.rs:169-174): p -= lr * sqrt(rows/cols) * o. */
void ref_muon_apply(float *p, const float *o, int64_t rows, int64_t cols, float lr);

/* The scalar sqrt(rows/cols) the reference computes in f32. */
float ref_muon_scale(int64_t rows, int64_t cols);

/* 1 - powf(beta, t), the AdamW bias-correction divisor for step t. */
float ref_bias_correction(float beta, int64_t t);

/* GradAccumulator::averaged_grad (lib.rs:254-257). */
void ref_grad_average(const float *sum, float *out, int64_t n, int64_t micro_batches);

/* Elementwise AdamW over an arena with all the OpenMP threads; returns seconds
 * of wall time (used only as the CPU baseline timing). */
double ref_adamw_step_timed(float *p, float *m, float *v, const float *g, int64_t n,
                            float lr, float beta1, float beta2, float eps,
                            float weight_decay, int64_t t, float grad_divisor,
                            int n_threads);

int ref_max_threads(void);

/* ns_round of the variant (bf16, tf32 or none) over n elements; out may equal in. */
void ref_ns_round_array(const float *in, float *out, int64_t n, int variant);

#ifdef __cplusplus
}
#endif
#endif
