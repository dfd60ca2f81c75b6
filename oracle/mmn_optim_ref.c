/*
 * CPU oracle for the MagicMindNet optimizer step — TEST INFRASTRUCTURE ONLY.
 * See mmn_optim_ref.h for the scope, the pinning status and the rounding rules.
 * Every function cites the reference line it restates (paths are relative to the
 * MagicMindNet repository root).
 */
#include "mmn_optim_ref.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int ref_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int pick_threads(int n_threads) {
    int mx = ref_max_threads();
    if (n_threads <= 0 || n_threads > mx) return mx;
    return n_threads;
}

static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/*
 * bf16 round-to-nearest-even, written from the IEEE-754 definition: keep the
 * upper 16 bits of the f32 pattern and round on the discarded 16 bits, ties to
 * the even upper half. A NaN stays a NaN (quiet bit set). This is the rounding
 * half::bf16::from_f32 performs at lib.rs:104,106,115,116,119.
 */
float ref_bf16_round(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return u2f((u | 0x00400000u) & 0xFFFF0000u);
    uint32_t hi = u >> 16, lo = u & 0xFFFFu;
    if (lo > 0x8000u || (lo == 0x8000u && (hi & 1u))) hi += 1u;
    return u2f(hi << 16);
}

/* lib.rs:53-54: the divisor (1 - beta^t) with t the instance step count as f32. */
float ref_bias_correction(float beta, int64_t t) {
    return 1.0f - powf(beta, (float)t);
}

/*
 * AdamW::step_param, lib.rs:41-60, for one tensor after the caller advanced the
 * instance counter to t. Operation order is the reference's:
 *   m = b1*m + (1-b1)*g                     (:47-49)
 *   v = b2*v + (1-b2)*g*g                   (:50-52)  ((1-b2)*g)*g, left to right
 *   m_hat = m / (1-b1^t); v_hat = v / (1-b2^t)   (:53-54)
 *   p = p - lr * (m_hat / (sqrt(v_hat) + eps))   (:55-57)
 *   p = p * (1 - lr*wd)                     (:58-59)
 * grad_divisor folds GradAccumulator::averaged_grad (lib.rs:254-257: sum / n)
 * into the read of g; a divisor of 1 is the identity.
 */
static void adamw_range(float *p, float *m, float *v, const float *g, int64_t lo, int64_t hi,
                        float lr, float b1, float b2, float eps, float wd, float bc1,
                        float bc2, float grad_divisor) {
    const float one_m_b1 = 1.0f - b1;
    const float one_m_b2 = 1.0f - b2;
    const float decay = 1.0f - lr * wd;
    for (int64_t i = lo; i < hi; ++i) {
        float gi = g[i];
        if (grad_divisor != 1.0f) gi = gi / grad_divisor;
        float mi = b1 * m[i] + one_m_b1 * gi;
        float vi = b2 * v[i] + one_m_b2 * gi * gi;
        m[i] = mi;
        v[i] = vi;
        float mh = mi / bc1;
        float vh = vi / bc2;
        float upd = mh / (sqrtf(vh) + eps);
        float pi = p[i] - lr * upd;
        p[i] = pi * decay;
    }
}

void ref_adamw_step(float *p, float *m, float *v, const float *g, int64_t n, float lr,
                    float beta1, float beta2, float eps, float weight_decay, int64_t t,
                    float grad_divisor) {
    float bc1 = ref_bias_correction(beta1, t);
    float bc2 = ref_bias_correction(beta2, t);
    adamw_range(p, m, v, g, 0, n, lr, beta1, beta2, eps, weight_decay, bc1, bc2, grad_divisor);
}

double ref_adamw_step_timed(float *p, float *m, float *v, const float *g, int64_t n, float lr,
                            float beta1, float beta2, float eps, float weight_decay, int64_t t,
                            float grad_divisor, int n_threads) {
    float bc1 = ref_bias_correction(beta1, t);
    float bc2 = ref_bias_correction(beta2, t);
    int nt = pick_threads(n_threads);
    struct timespec a, b;
    clock_gettime(CLOCK_MONOTONIC, &a);
#pragma omp parallel num_threads(nt)
    {
        int tid = 0, cnt = 1;
#ifdef _OPENMP
        tid = omp_get_thread_num();
        cnt = omp_get_num_threads();
#endif
        int64_t per = (n + cnt - 1) / cnt;
        int64_t lo = (int64_t)tid * per, hi = lo + per;
        if (hi > n) hi = n;
        if (lo < hi)
            adamw_range(p, m, v, g, lo, hi, lr, beta1, beta2, eps, weight_decay, bc1, bc2,
                        grad_divisor);
    }
    clock_gettime(CLOCK_MONOTONIC, &b);
    return (double)(b.tv_sec - a.tv_sec) + 1e-9 * (double)(b.tv_nsec - a.tv_nsec);
}

/*
 * Muon momentum, lib.rs:154-165:
 *   vel = mu*vel + (1-mu)*g
 *   nesterov: u = g*(1-mu) + vel*mu   else u = vel
 */
void ref_muon_momentum(float *vel, const float *g, float *u, int64_t n, float momentum,
                       int nesterov, float grad_divisor) {
    const float one_m = 1.0f - momentum;
    for (int64_t i = 0; i < n; ++i) {
        float gi = g[i];
        if (grad_divisor != 1.0f) gi = gi / grad_divisor;
        float vi = momentum * vel[i] + one_m * gi;
        vel[i] = vi;
        u[i] = nesterov ? (gi * one_m + vi * momentum) : vi;
    }
}

/* lib.rs:169-171: scale = sqrt(shape[0] / shape[1]) in f32. */
float ref_muon_scale(int64_t rows, int64_t cols) {
    return sqrtf((float)rows / (float)cols);
}

/* lib.rs:172-174: p -= lr * scale * u, evaluated (lr*scale)*u. */
void ref_muon_apply(float *p, const float *o, int64_t rows, int64_t cols, float lr) {
    const float ls = lr * ref_muon_scale(rows, cols);
    for (int64_t i = 0; i < rows * cols; ++i) p[i] = p[i] - ls * o[i];
}

/* lib.rs:254-257: sum / max(n, 1). */
void ref_grad_average(const float *sum, float *out, int64_t n, int64_t micro_batches) {
    float d = (float)(micro_batches > 1 ? micro_batches : 1);
    for (int64_t i = 0; i < n; ++i) out[i] = sum[i] / d;
}

/* ---------------------------------------------------------------- GEMMs -- */
/*
 * C = A * B with every C[i][j] accumulated over k in ascending order. The
 * outer-product loop order (i block, j block, k, j) keeps that per-element
 * order while letting the compiler vectorise over j, so the result does not
 * depend on the thread count.
 */
#define GI 4
#define GJ 64

__attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))
static void gemm_block_f32(const float *A, const float *B, float *C, int64_t N, int64_t K,
                           int64_t i0, int64_t im, int64_t j0, int64_t jn, int fma_mode) {
    float acc[GI][GJ];
    for (int ii = 0; ii < GI; ++ii)
        for (int jj = 0; jj < GJ; ++jj) acc[ii][jj] = 0.0f;
    if (jn == GJ && im == GI) {
        for (int64_t k = 0; k < K; ++k) {
            const float *b = B + k * N + j0;
            for (int ii = 0; ii < GI; ++ii) {
                const float a = A[(i0 + ii) * K + k];
                if (fma_mode)
                    for (int jj = 0; jj < GJ; ++jj) acc[ii][jj] = fmaf(a, b[jj], acc[ii][jj]);
                else
                    for (int jj = 0; jj < GJ; ++jj) acc[ii][jj] = acc[ii][jj] + a * b[jj];
            }
        }
    } else {
        for (int64_t k = 0; k < K; ++k) {
            const float *b = B + k * N + j0;
            for (int ii = 0; ii < im; ++ii) {
                const float a = A[(i0 + ii) * K + k];
                for (int jj = 0; jj < jn; ++jj)
                    acc[ii][jj] = fma_mode ? fmaf(a, b[jj], acc[ii][jj]) : acc[ii][jj] + a * b[jj];
            }
        }
    }
    for (int ii = 0; ii < im; ++ii)
        for (int jj = 0; jj < jn; ++jj) C[(i0 + ii) * N + j0 + jj] = acc[ii][jj];
}

__attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))
static void gemm_block_f64(const float *A, const float *B, float *C, int64_t N, int64_t K,
                           int64_t i0, int64_t im, int64_t j0, int64_t jn) {
    double acc[GI][GJ];
    for (int ii = 0; ii < GI; ++ii)
        for (int jj = 0; jj < GJ; ++jj) acc[ii][jj] = 0.0;
    for (int64_t k = 0; k < K; ++k) {
        const float *b = B + k * N + j0;
        for (int ii = 0; ii < im; ++ii) {
            const double a = (double)A[(i0 + ii) * K + k];
            for (int jj = 0; jj < jn; ++jj) acc[ii][jj] += a * (double)b[jj];
        }
    }
    for (int ii = 0; ii < im; ++ii)
        for (int jj = 0; jj < jn; ++jj) C[(i0 + ii) * N + j0 + jj] = (float)acc[ii][jj];
}

void ref_gemm(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K,
              int gemm_order, int n_threads) {
    int nt = pick_threads(n_threads);
    int64_t ib = (M + GI - 1) / GI, jb = (N + GJ - 1) / GJ;
#pragma omp parallel for schedule(dynamic, 4) num_threads(nt)
    for (int64_t blk = 0; blk < ib * jb; ++blk) {
        int64_t i0 = (blk / jb) * GI, j0 = (blk % jb) * GJ;
        int64_t im = M - i0 < GI ? M - i0 : GI;
        int64_t jn = N - j0 < GJ ? N - j0 : GJ;
        if (gemm_order == REF_GEMM_F64)
            gemm_block_f64(A, B, C, N, K, i0, im, j0, jn);
        else
            gemm_block_f32(A, B, C, N, K, i0, im, j0, jn, gemm_order == REF_GEMM_F32_FMA);
    }
}

/*
 * tf32 round-to-nearest-even on the f32 bit pattern: keep the sign, the
 * exponent and the 10 leading mantissa bits, round on the 13 discarded bits,
 * ties to the even kept value. Inf and NaN pass through. The rounding point of
 * the TF32 Newton-Schulz mode (REF_NS_TF32), which has no reference
 * counterpart.
 */
float ref_tf32_round(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

/* The rounding point of a Newton-Schulz variant: bf16, tf32 for REF_NS_TF32,
 * none for REF_NS_FP32. */
static float ns_round(float x, int variant) {
    if (variant == REF_NS_FP32) return x;
    return variant == REF_NS_TF32 ? ref_tf32_round(x) : ref_bf16_round(x);
}

/* The rounding point of a variant over an array (out may equal in), on all
 * threads: the elementwise part of the full-size Newton-Schulz checks. */
void ref_ns_round_array(const float *in, float *out, int64_t n, int variant) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = ns_round(in[i], variant);
}

/* --------------------------------------------------------- Newton-Schulz -- */
static const float NS_A = 3.4445f, NS_B = -4.7750f, NS_C = 2.0315f; /* lib.rs:84-86 */
static const float NS_EPS = 1e-7f;                                  /* lib.rs:87 */

/*
 * One loop body of lib.rs:112-120 on x (n x m):
 *   A    = x * x^T                       (:114)
 *   A_bf = bf16(A)                       (:115)
 *   A2   = bf16(A_bf * A_bf)             (:116)
 *   B    = A_bf*b + A2*c                 (:117, kept fp32)
 *   x'   = bf16(x*a + B*x)               (:118-119)
 * REF_NS_BF16 additionally rounds B to bf16 (no reference counterpart).
 * REF_NS_TF32 rounds to tf32 wherever the reference rounds to bf16;
 * REF_NS_FP32 does not round at all.
 */
void ref_ns_iteration(const float *x, int64_t n, int64_t m, float *x_next, int gemm_order,
                      int variant, int n_threads) {
    float *xt = (float *)calloc((size_t)(n * m), sizeof(float));
    float *a = (float *)malloc(sizeof(float) * (size_t)(n * n));
    float *a2 = (float *)malloc(sizeof(float) * (size_t)(n * n));
    float *bx = (float *)malloc(sizeof(float) * (size_t)(n * m));
    for (int64_t i = 0; i < n; ++i)
        for (int64_t j = 0; j < m; ++j) xt[j * n + i] = x[i * m + j];
    ref_gemm(x, xt, a, n, n, m, gemm_order, n_threads);
    for (int64_t i = 0; i < n * n; ++i) a[i] = ns_round(a[i], variant);
    ref_gemm(a, a, a2, n, n, n, gemm_order, n_threads);
    for (int64_t i = 0; i < n * n; ++i) {
        float sq = ns_round(a2[i], variant);
        float b = a[i] * NS_B + sq * NS_C;
        a2[i] = variant == REF_NS_BF16 ? ref_bf16_round(b) : b;
    }
    ref_gemm(a2, x, bx, n, m, n, gemm_order, n_threads);
    for (int64_t i = 0; i < n * m; ++i) x_next[i] = ns_round(x[i] * NS_A + bx[i], variant);
    free(xt);
    free(a);
    free(a2);
    free(bx);
}

/*
 * newton_schulz5, lib.rs:83-126, for a 2-D rows x cols input (the non-2-D
 * zero-padding branch at :93-99 is applied by the caller before this point).
 * Transposes when rows > cols (:101-107, :122-124); the Frobenius norm is a
 * sequential fp32 sum over the transposed matrix in row-major order, clamped
 * with max(1e-7) (:109), and the input is divided by it (:110). REF_NS_TF32
 * and REF_NS_FP32 (modes with no reference counterpart, meant to sit close to
 * exact Newton-Schulz) sum in fp64 and round the sum to fp32 once: at large
 * sizes the sequential fp32 sum stagnates (about 17% low at 4096 x 14336).
 */
int ref_newton_schulz5(const float *g, int64_t rows, int64_t cols, int steps, float *out,
                       int gemm_order, int variant, float *norm_out, int n_threads) {
    const int transposed = rows > cols;
    const int64_t n = transposed ? cols : rows, m = transposed ? rows : cols;
    float *x = (float *)malloc(sizeof(float) * (size_t)(n * m));
    float *y = (float *)malloc(sizeof(float) * (size_t)(n * m));
    for (int64_t i = 0; i < n; ++i)
        for (int64_t j = 0; j < m; ++j)
            x[i * m + j] = ns_round(transposed ? g[j * cols + i] : g[i * cols + j], variant);
    float s = 0.0f;
    if (variant == REF_NS_FP32 || variant == REF_NS_TF32) {
        /* fp32 and TF32 modes (no reference counterpart): the correctly rounded
         * fp32 sum of squares, so that the norm carries no summation-order error */
        double d = 0.0;
        for (int64_t i = 0; i < n * m; ++i) d += (double)x[i] * (double)x[i];
        s = (float)d;
    } else {
        for (int64_t i = 0; i < n * m; ++i) s = s + x[i] * x[i];
    }
    float norm = fmaxf(sqrtf(s), NS_EPS);
    if (norm_out) *norm_out = norm;
    for (int64_t i = 0; i < n * m; ++i) x[i] = x[i] / norm;
    for (int it = 0; it < steps; ++it) {
        ref_ns_iteration(x, n, m, y, gemm_order, variant, n_threads);
        float *t = x;
        x = y;
        y = t;
    }
    for (int64_t i = 0; i < n; ++i)
        for (int64_t j = 0; j < m; ++j) {
            if (transposed)
                out[j * n + i] = x[i * m + j];
            else
                out[i * m + j] = x[i * m + j];
        }
    free(x);
    free(y);
    return 0;
}
