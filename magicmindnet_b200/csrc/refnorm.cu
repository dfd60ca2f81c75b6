// The reference's Frobenius norm of the Newton-Schulz input, bit for bit.
//
// newton_schulz5 (crates/mmn-optim/src/lib.rs:109) computes
//   x.iter().map(|v| v * v).sum::<f32>()
// over the oriented matrix x (bf16 values, row-major): one fp32 accumulator,
// one element after another. At the sizes of large models this sum drifts far
// from the exact one (the running sum grows until most squares are smaller
// than half its last-place unit and vanish; at 4096 x 14336 it ends about 17%
// low), and Newton-Schulz is sensitive to the input scale, so matching the
// reference needs this exact sum, not an accurate one.
//
// The sum is sequential, but it has structure that a GPU can use. Every term
// t = fl(x * x) is >= 0, so the running sum s never decreases. While s stays in
// one binade [2^E, 2^(E+1)), every value s can take lies on the grid
// u = 2^(E-23), and fl(s + t) = s + RN_u(t) as long as s + t stays below
// 2^(E+1) - u/2: the add rounds the term alone to the grid. In units of u,
// with S = s/u an integer and k = t/u:
//   - k not an odd multiple of 1/2: S += rint(k), whatever S is;
//   - k = q + 1/2 (a tie): S = rue(S + q), rounded up to even, because ties go
//     to the neighbour with an even last bit.
// So inside a binade the sum is an integer sum, and only ties depend on the
// order. The maps S -> S + A and S -> S + A + ((S + B) & 1) are closed under
// composition (after a tie the running value is even, so a later tie's parity
// no longer depends on S), which makes the per-element maps an associative
// monoid: a block reduces (or scans) the maps of its elements in order.
//
// The kernel gives each matrix one CTA, which walks the sequence in tiles of
// kRnThreads x kRnEpt elements, each thread a run of kRnEpt consecutive ones:
//   - fast path: compose the tile's element maps in order (thread, warp,
//     block); if no term was marked for exact handling and the composed map
//     leaves S <= 2^24 - 1, no add in the tile left the binade (S_i + k_i <=
//     S_end + 1/2 for every element), and S takes the composed value;
//   - slow path (a binade change or a term of at least 2^22 units): an
//     ordered block scan gives every thread the S at its first element;
//     threads walk their elements to the first one whose add can leave the
//     binade, that add is done as an fp32 add, and the tile resumes after it
//     with the new binade.
// A binade change happens about log2(N) times per matrix, so nearly every
// tile takes the fast path; ties (about 1% of the terms of bf16 squares) stay
// on it. The element arithmetic runs on pairs with the packed fp32x2
// instructions of sm_100. A non-finite running sum ends the walk: fp32
// addition of the remaining terms (all >= 0 or NaN) then gives NaN if any of
// them is NaN, else the infinity already reached.
//
// The TF32 and fp32 Newton-Schulz modes have no reference counterpart; they
// aim at exact Newton-Schulz and keep an accurate fixed-order tile sum
// (muon_norm_kernel).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cooperative_groups.h>

#include <climits>
#include <cstdint>

#include "elementwise.cuh"

namespace mmn {
namespace {

constexpr int kRnThreads = 512;
constexpr int kRnWarps = kRnThreads / 32;
constexpr int kRnGroups = 3;                 // 16-byte groups (8 bf16) per thread per tile
constexpr int kRnEpt = kRnGroups * 8;        // elements per thread per tile
constexpr int kRnSat = 1 << 25;              // integers at or above 2^24 mean "left the binade"
constexpr float kRnBig = 4194304.0f;         // 2^22: larger terms take the exact add
constexpr uint32_t kRnBigBits = 0x4A800000u; // its bit pattern (NaNs compare above it)
constexpr float kRnMagic = 12582912.0f;      // 1.5 * 2^23: k + M - M = rint(k) for k < 2^22

__device__ __forceinline__ int rn_sat(int x) { return x < kRnSat ? x : kRnSat; }

// S -> S + A (tie = 0) or S -> S + A + ((S + B) & 1) (tie = 1). An element's
// map is S -> S + rint(k), or for a tie k = q + 1/2, S -> rue(S + q) with
// rue(y) = y + (y & 1), i.e. A = B = q. After a tie the running value's
// parity no longer depends on S (it is A + B mod 2), so maps compose into
// maps of the same form.
struct RnMap {
  int tie, A, B;
};

__device__ __forceinline__ RnMap rn_compose(const RnMap a, const RnMap b) {  // a, then b
  RnMap r;
  if (!b.tie) {
    r.tie = a.tie;
    r.A = rn_sat(a.A + b.A);
    r.B = a.B;
  } else if (!a.tie) {
    r.tie = 1;
    r.A = rn_sat(a.A + b.A);
    r.B = rn_sat(a.A + b.B);
  } else {
    r.tie = 1;
    r.A = rn_sat(a.A + b.A + ((a.A + a.B + b.B) & 1));
    r.B = a.B;
  }
  return r;
}

__device__ __forceinline__ int rn_apply(const RnMap m, int s) {
  return rn_sat(s + m.A + (m.tie ? ((s + m.B) & 1) : 0));
}

__device__ __forceinline__ RnMap rn_shfl_down(const RnMap m, int off) {
  return {__shfl_down_sync(0xffffffffu, m.tie, off), __shfl_down_sync(0xffffffffu, m.A, off),
          __shfl_down_sync(0xffffffffu, m.B, off)};
}

__device__ __forceinline__ RnMap rn_shfl_up(const RnMap m, int off) {
  return {__shfl_up_sync(0xffffffffu, m.tie, off), __shfl_up_sync(0xffffffffu, m.A, off),
          __shfl_up_sync(0xffffffffu, m.B, off)};
}

// The binade of the running sum: s = S * 2^(E-23) with S < 2^24 an integer,
// E >= -126 (the subnormals share the grid of the first normal binade). From
// the fp32 bit pattern: bits = ((E + 126) << 23) + S.
struct RnState {
  int E;       // binade exponent (>= -126)
  int S;       // running sum in grid units
  float scf;   // 2^(23-E) when E >= -100
  double scd;  // 2^(23-E)
  bool tiny;   // E < -100: the scale is applied in double (2^(23-E) is beyond
               // the fp32 range); k = t * 2^(23-E) is exact either way
  int parity;  // shared-slot set of the next fast-path reduction
};

__device__ __forceinline__ void rn_set(RnState& st, float s) {
  const uint32_t b = __float_as_uint(s);
  const int ex = (int)(b >> 23);
  st.E = ex == 0 ? -126 : ex - 127;
  st.S = (int)(b - ((uint32_t)(st.E + 126) << 23));
  st.tiny = st.E < -100;
  st.scd = ldexp(1.0, 23 - st.E);
  st.scf = st.tiny ? 0.0f : ldexpf(1.0f, 23 - st.E);
}

__device__ __forceinline__ float rn_value(const RnState& st, int S) {
  return __uint_as_float(((uint32_t)(st.E + 126) << 23) + (uint32_t)S);
}

// Terms x*x of two elements in grid units: k = x*x * 2^(23-E), exact wherever
// it matters (a power-of-two scale of the product; a k that loses bits to the
// fp32 subnormal range is far below 1/2, adds nothing and is no tie). kbits is
// k's bit pattern (unsigned: NaNs and k >= 2^22 compare at or above
// kRnBigBits and need the exact add). val = rint(k) for k < 2^22, ties to
// even; a tie k = q + 1/2 has q = val - neg.
struct RnPair {
  uint32_t kbits[2];
  int val[2];
  bool tie[2];
  bool neg[2];
};

template <bool TINY>
__device__ __forceinline__ RnPair rn_pair(uint32_t w, const RnState& st) {
  const float2 x = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  const float2 t = __fmul2_rn(x, x);
  float2 k;
  if constexpr (!TINY) {
    k = __fmul2_rn(t, make_float2(st.scf, st.scf));  // the scale is exact
  } else {
    const double a = (double)t.x * st.scd, b = (double)t.y * st.scd;
    k = make_float2(a < (double)kRnBig ? (float)a : kRnBig, b < (double)kRnBig ? (float)b : kRnBig);
  }
  const float2 y = __fadd2_rn(k, make_float2(kRnMagic, kRnMagic));  // M + rint(k), ties to even
  const float2 kr = __fadd2_rn(y, make_float2(-kRnMagic, -kRnMagic));
  const float2 d = __ffma2_rn(kr, make_float2(-1.0f, -1.0f), k);  // k - rint(k), exact
  RnPair p;
  p.kbits[0] = __float_as_uint(k.x);
  p.kbits[1] = __float_as_uint(k.y);
  p.val[0] = __float_as_int(y.x) - 0x4B400000;  // rint(k): the low mantissa bits of y
  p.val[1] = __float_as_int(y.y) - 0x4B400000;
  p.tie[0] = fabsf(d.x) == 0.5f;
  p.tie[1] = fabsf(d.y) == 0.5f;
  p.neg[0] = d.x < 0.0f;
  p.neg[1] = d.y < 0.0f;
  return p;
}

// Appends an element to a thread's running map (at most kRnEpt elements of at
// most 2^22 units each, so no value reaches 2^31 before rn_fold_sat). Ties are
// about 1% of bf16 squares: they take the branch.
__device__ __forceinline__ void rn_fold(RnMap& m, int val, bool tie, bool neg) {
  if (!tie) {
    m.A += val;
  } else {
    const int q = val - (neg ? 1 : 0);
    if (!m.tie) {
      m.tie = 1;
      m.A += q;
      m.B = m.A;
    } else {
      m.A += q + ((m.A + m.B + q) & 1);
    }
  }
}

__device__ __forceinline__ RnMap rn_fold_sat(RnMap m) {
  m.A = rn_sat(m.A);
  m.B = rn_sat(m.B);
  return m;
}

// The new S after one element from S (no binade change).
__device__ __forceinline__ int rn_step(int val, bool tie, bool neg, int S) {
  if (!tie) return S + val;
  const int y = S + val - (neg ? 1 : 0);
  return y + (y & 1);
}

// One tile's run of a thread: kRnGroups 16-byte groups of consecutive bf16
// elements (elements past the end of the matrix read as 0, which adds
// nothing).
struct RnRun {
  uint4 g[kRnGroups];

  __device__ __forceinline__ uint32_t word(int i) const {  // elements 2i, 2i + 1
    const uint4& v = g[i / 4];
    const int j = i % 4;
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
  }
};

// Where a thread's run starts, advanced one tile at a time without division.
struct RnCursor {
  long long e;    // first element of the run
  long long row;  // its row of the oriented matrix
  int col;
};

// Loads a run of consecutive elements starting at c. Rows hold whole groups
// (m % 8 == 0) and start 16-byte aligned: vector loads.
__device__ __forceinline__ void rn_load_vec(RnRun& r, const __nv_bfloat16* X, int ld, int m,
                                            long long total, RnCursor c) {
#pragma unroll
  for (int u = 0; u < kRnGroups; ++u) {
    if (c.e < total)
      r.g[u] = __ldg(reinterpret_cast<const uint4*>(X + c.row * ld + c.col));
    else
      r.g[u] = make_uint4(0u, 0u, 0u, 0u);
    c.e += 8;
    c.col += 8;
    if (c.col >= m) {
      c.col -= m;
      ++c.row;
    }
  }
}

// The same for rows of any length: element by element.
__device__ __forceinline__ void rn_load_scalar(RnRun& r, const __nv_bfloat16* X, int ld, int m,
                                               long long total, RnCursor c) {
  const unsigned short* xs = reinterpret_cast<const unsigned short*>(X);
#pragma unroll
  for (int u = 0; u < kRnGroups; ++u) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t lo = 0, hi = 0;
      if (c.e < total) lo = xs[c.row * ld + c.col];
      ++c.e;
      if (++c.col >= m) {
        c.col = 0;
        ++c.row;
      }
      if (c.e < total) hi = xs[c.row * ld + c.col];
      ++c.e;
      if (++c.col >= m) {
        c.col = 0;
        ++c.row;
      }
      w[j] = lo | (hi << 16);
    }
    r.g[u] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

struct RnShared {
  uint4 run[kRnGroups][kRnThreads];  // the tile's runs, for the slow path
  RnMap warp[kRnWarps];
  RnMap total;
  int stop;          // first tile-local element needing the exact add
  uint32_t s_bits;   // running sum after that add
  // fast-path reduction, double-buffered by tile parity so that a tile needs
  // two barriers: warp results in, block result out
  RnMap fwarp[2][kRnWarps];
  uint32_t fmax[2][kRnWarps];
  RnMap ftotal[2];
  uint32_t ftmax[2];
};

// Fast path: ordered composition of the block's per-thread maps and the max of
// their k bit patterns, in two barriers (shared slots alternate by tile).
__device__ __forceinline__ RnMap rn_block_reduce_fast(RnMap m, uint32_t kmax, RnShared& sh,
                                                      int p, uint32_t* kmax_out) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const RnMap o = rn_shfl_down(m, off);
    const uint32_t ko = __shfl_down_sync(0xffffffffu, kmax, off);
    if (lane + off < 32) {
      m = rn_compose(m, o);
      kmax = max(kmax, ko);
    }
  }
  if (lane == 0) {
    sh.fwarp[p][w] = m;
    sh.fmax[p][w] = kmax;
  }
  __syncthreads();
  if (w == 0) {
    RnMap t = lane < kRnWarps ? sh.fwarp[p][lane] : RnMap{0, 0, 0};
    uint32_t km = lane < kRnWarps ? sh.fmax[p][lane] : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const RnMap o = rn_shfl_down(t, off);
      const uint32_t ko = __shfl_down_sync(0xffffffffu, km, off);
      if (lane + off < 32) {
        t = rn_compose(t, o);
        km = max(km, ko);
      }
    }
    if (lane == 0) {
      sh.ftotal[p] = t;
      sh.ftmax[p] = km;
    }
  }
  __syncthreads();
  *kmax_out = sh.ftmax[p];
  return sh.ftotal[p];
}

// Ordered exclusive scan of the per-thread maps (prefix of the threads before
// this one) and the block total.
__device__ __forceinline__ RnMap rn_block_scan(RnMap m, RnShared& sh, RnMap* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  RnMap inc = m;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const RnMap o = rn_shfl_up(inc, off);
    if (lane >= off) inc = rn_compose(o, inc);
  }
  RnMap exc = rn_shfl_up(inc, 1);
  if (lane == 0) exc = RnMap{0, 0, 0};
  if (lane == 31) sh.warp[w] = inc;
  __syncthreads();
  if (w == 0) {
    RnMap t = lane < kRnWarps ? sh.warp[lane] : RnMap{0, 0, 0};
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const RnMap o = rn_shfl_up(t, off);
      if (lane >= off) t = rn_compose(o, t);
    }
    RnMap te = rn_shfl_up(t, 1);
    if (lane == 0) te = RnMap{0, 0, 0};
    if (lane < kRnWarps) sh.warp[lane] = te;  // exclusive prefix of warp `lane`
    if (lane == kRnWarps - 1) sh.total = t;
  }
  __syncthreads();
  const RnMap r = rn_compose(sh.warp[w], exc);
  *total = sh.total;
  __syncthreads();
  return r;
}

// The composed map of the run's elements and the max of their k bit patterns.
// A pair without a tie (98% of pairs) adds its two values at once; the branch
// is taken per pair.
template <bool TINY>
__device__ __forceinline__ RnMap rn_run_fold(const RnRun& r, const RnState& st,
                                             uint32_t* kmax_out) {
  RnMap m{0, 0, 0};
  uint32_t kmax = 0;
#pragma unroll
  for (int i = 0; i < kRnEpt / 2; ++i) {
    const RnPair p = rn_pair<TINY>(r.word(i), st);
    kmax = max(kmax, max(p.kbits[0], p.kbits[1]));
    if (!(p.tie[0] | p.tie[1])) {
      m.A += p.val[0] + p.val[1];
    } else {
      rn_fold(m, p.val[0], p.tie[0], p.neg[0]);
      rn_fold(m, p.val[1], p.tie[1], p.neg[1]);
    }
  }
  *kmax_out = kmax;
  return m;
}

// The word of elements 2i, 2i + 1 of this thread's run, from its shared copy.
__device__ __forceinline__ uint32_t rn_shared_word(const RnShared& sh, int i) {
  const uint4 v = sh.run[i / 4][threadIdx.x];
  const int j = i % 4;
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// Slow-path form of rn_run_fold: the run from its shared copy, one pair at a
// time.
template <bool TINY>
__device__ __noinline__ RnMap rn_shared_fold(const RnShared& sh, const RnState& st, int start,
                                             int base) {
  RnMap m{0, 0, 0};
#pragma unroll 1
  for (int i = 0; i < kRnEpt / 2; ++i) {
    const RnPair p = rn_pair<TINY>(rn_shared_word(sh, i), st);
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (base + 2 * i + h >= start) rn_fold(m, p.val[h], p.tie[h], p.neg[h]);
  }
  return m;
}

// Runs the sequential sum over one tile (this thread's run r), starting from
// `st`; returns false when the sum became non-finite (s_out holds it; the
// caller finishes the NaN check).
__device__ __forceinline__ bool rn_tile(const RnRun& r, RnState& st, RnShared& sh, float& s_out) {
  const int base = threadIdx.x * kRnEpt;
  // fast path: the composed map of the whole tile
  {
    uint32_t kmax;
    const RnMap m = st.tiny ? rn_run_fold<true>(r, st, &kmax) : rn_run_fold<false>(r, st, &kmax);
    const RnMap tot = rn_block_reduce_fast(rn_fold_sat(m), kmax, sh, st.parity, &kmax);
    st.parity ^= 1;  // the next tile reduces through the other slots
    if (kmax < kRnBigBits) {
      const int s_end = rn_apply(tot, st.S);
      if (s_end <= (1 << 24) - 1) {
        st.S = s_end;
        return true;
      }
    }
  }
  // slow path: walk to each add that can leave the binade (or has a term of
  // 2^22 units or more), do it as an fp32 add, resume after it. The runs go
  // to shared memory so that the rarely taken walk needs no registers of its
  // own.
#pragma unroll
  for (int u = 0; u < kRnGroups; ++u) sh.run[u][threadIdx.x] = r.g[u];
  int start = 0;
  while (true) {
    const RnMap m = st.tiny ? rn_shared_fold<true>(sh, st, start, base)
                            : rn_shared_fold<false>(sh, st, start, base);
    RnMap total;
    const RnMap pre = rn_block_scan(rn_fold_sat(m), sh, &total);
    if (threadIdx.x == 0) sh.stop = INT_MAX;
    __syncthreads();
    int S = rn_apply(pre, st.S);
    int cand = INT_MAX;
    uint32_t cand_bits = 0;
#pragma unroll 1
    for (int i = 0; i < kRnEpt / 2; ++i) {
      if (cand == INT_MAX) {
        const uint32_t w = rn_shared_word(sh, i);
        const RnPair p = st.tiny ? rn_pair<true>(w, st) : rn_pair<false>(w, st);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (cand == INT_MAX && base + 2 * i + h >= start) {
            // room below the binade's top, less 1/2 (exact where k can reach it)
            const float room = __fsub_rn((float)((1 << 24) - S), 0.5f);
            if (p.kbits[h] >= kRnBigBits || !(__uint_as_float(p.kbits[h]) < room)) {
              const float xv = __uint_as_float(h ? (w & 0xFFFF0000u) : (w << 16));
              cand = base + 2 * i + h;
              cand_bits = __float_as_uint(__fadd_rn(rn_value(st, S), __fmul_rn(xv, xv)));
            } else {
              S = rn_step(p.val[h], p.tie[h], p.neg[h], S);
            }
          }
        }
      }
    }
    if (cand != INT_MAX) atomicMin(&sh.stop, cand);
    __syncthreads();
    const int stop = sh.stop;
    if (stop == INT_MAX) {
      st.S = rn_apply(total, st.S);
      __syncthreads();
      return true;
    }
    if (cand == stop) sh.s_bits = cand_bits;
    __syncthreads();
    const float s = __uint_as_float(sh.s_bits);
    __syncthreads();
    if (!isfinite(s)) {
      s_out = s;
      return false;
    }
    rn_set(st, s);
    start = stop + 1;
  }
}

// Cluster-level slots: one composed map per CTA and exchange parity, and the
// state a CTA publishes after walking its part of a slow cluster step.
constexpr int kRnTilesPerExchange = 8;  // CTA tiles folded between cluster exchanges

struct RnClusterSlots {
  RnMap map[2];
  uint32_t kmax[2];
  RnMap all;        // the cluster step's composed map (thread 0's result)
  uint32_t all_kmax;
  RnMap tmap[kRnTilesPerExchange];    // this CTA's tile maps of the current step
  uint32_t tkmax[kRnTilesPerExchange];
  int bad;            // first tile of this CTA's part whose adds leave the binade
  int bad_S;          // the running sum (grid units) at that tile's start
  int first_bad;      // the cluster's first such tile (thread 0's result)
  uint32_t pub_bits;  // running sum after the exactly walked tile
  int pub_ok;         // 0: the sum became non-finite there
};

template <bool VEC>
__device__ __forceinline__ void rn_load(RnRun& r, const __nv_bfloat16* X, int ld, int m,
                                        long long total, const RnCursor& c) {
  if (VEC)
    rn_load_vec(r, X, ld, m, total, c);
  else
    rn_load_scalar(r, X, ld, m, total, c);
}

__device__ __forceinline__ RnCursor rn_cursor_at(long long e, int m) {
  RnCursor c;
  c.e = e;
  c.row = e / m;
  c.col = (int)(e - c.row * m);
  return c;
}

__device__ __forceinline__ void rn_advance(RnCursor& c, long long d, long long d_rows, int d_cols,
                                           int m) {
  c.e += d;
  c.row += d_rows;
  c.col += d_cols;
  if (c.col >= m) {
    c.col -= m;
    ++c.row;
  }
}

// The sequential sum over the whole oriented matrix X (n x m, row stride ld),
// computed by the C CTAs of a cluster (C = 1: one CTA). A cluster step is C
// parts of up to K = kRnTilesPerExchange consecutive CTA tiles; CTA r folds
// the r-th part, composing its tiles' maps in order. The CTAs then exchange their
// parts' maps through distributed shared memory, and each composes all of
// them in order, so every CTA holds the same running state. A cluster step
// whose composed map leaves the binade (or holds a term of 2^22 grid units or
// more) is walked part after part and tile after tile, each part starting
// from the state its predecessor published.
template <bool VEC>
__device__ __forceinline__ float rn_matrix_sum(const __nv_bfloat16* X, int ld, int m,
                                               long long total, RnShared& sh,
                                               RnClusterSlots& cs, int C, int crank) {
  namespace cg = cooperative_groups;
  constexpr int K = kRnTilesPerExchange;
  constexpr long long T = (long long)kRnThreads * kRnEpt;  // elements per CTA tile
  RnState st;
  rn_set(st, 0.0f);
  st.parity = 0;
  float s_nf = 0.0f;
  long long done = -1;  // first element of the cluster step where the sum stopped being finite
  const long long own = (long long)threadIdx.x * kRnEpt;
  // Tiles per part: a restart refolds at most one cluster step, and early on
  // the sum changes binade whenever it doubles, so parts grow with the
  // distance covered (one tile at first, K once the sum is past C K tiles).
  auto tiles_at = [&](long long e) {
    const long long k = e / (T * C);
    return (int)(k < 1 ? 1 : (k > K ? K : k));
  };
  // this thread's run: one tile further (T) inside the part
  const long long t_rows = T / m;
  const int t_cols = (int)(T - t_rows * m);
  long long e0 = 0;
  int kt = tiles_at(0);
  RnCursor c = rn_cursor_at((long long)crank * kt * T + own, m);
  RnRun cur, nxt;
  rn_load<VEC>(cur, X, ld, m, total, c);
  int cp = 0;
  while (e0 < total) {
    const long long part = kt * T, step = part * C;
    const long long part0 = e0 + (long long)crank * part;  // this CTA's part
    const int kt_next = tiles_at(e0 + step);
    RnMap acc{0, 0, 0};
    uint32_t kacc = 0;
    for (int j = 0; j < kt; ++j) {
      // the next tile's loads fly while this one folds (zeros past the end)
      if (j + 1 < kt)
        rn_advance(c, T, t_rows, t_cols, m);
      else
        c = rn_cursor_at(e0 + step + (long long)crank * kt_next * T + own, m);
      rn_load<VEC>(nxt, X, ld, m, total, c);
      RnMap tot{0, 0, 0};
      uint32_t kmax = 0;
      if (part0 + j * T < total) {  // a tile past the end adds nothing
        const RnMap mm =
            st.tiny ? rn_run_fold<true>(cur, st, &kmax) : rn_run_fold<false>(cur, st, &kmax);
        tot = rn_block_reduce_fast(rn_fold_sat(mm), kmax, sh, st.parity, &kmax);
        st.parity ^= 1;
        acc = rn_compose(acc, tot);
        kacc = max(kacc, kmax);
      }
      if (threadIdx.x == 0) {
        cs.tmap[j] = tot;
        cs.tkmax[j] = kmax;
      }
      cur = nxt;
    }
    RnMap all = acc;
    uint32_t all_kmax = kacc;
    const int cp_step = cp;
    if (C > 1) {
      cg::cluster_group cluster = cg::this_cluster();
      if (threadIdx.x == 0) {
        cs.map[cp] = acc;
        cs.kmax[cp] = kacc;
      }
      cluster.sync();
      if (threadIdx.x == 0) {
        RnMap t{0, 0, 0};
        uint32_t km = 0;
        for (int r = 0; r < C; ++r) {
          const RnClusterSlots* rem = cluster.map_shared_rank(&cs, r);
          t = rn_compose(t, rem->map[cp]);
          km = max(km, rem->kmax[cp]);
        }
        cs.all = t;
        cs.all_kmax = km;
      }
      __syncthreads();
      all = cs.all;
      all_kmax = cs.all_kmax;
      __syncthreads();
      cp ^= 1;
    }
    if (all_kmax < kRnBigBits) {
      const int s_end = rn_apply(all, st.S);
      if (s_end <= (1 << 24) - 1) {
        st.S = s_end;
        e0 += step;
        kt = kt_next;
        continue;
      }
    }
    // slow: find the cluster's first tile whose adds leave the binade (or hold
    // a term of 2^22 units or more), walk that tile exactly, and restart the
    // cluster step after it (the tiles behind it were folded for the old
    // binade). Each CTA starts from the composed maps of the parts before its
    // own and applies its tile maps in order.
    if (threadIdx.x == 0) {
      RnMap pre{0, 0, 0};
      if (C > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        for (int r = 0; r < crank; ++r)
          pre = rn_compose(pre, cluster.map_shared_rank(&cs, r)->map[cp_step]);
      }
      int S = rn_apply(pre, st.S);
      int bad = INT_MAX;
      for (int j = 0; j < kt; ++j) {
        if (part0 + j * T >= total) break;
        const int next = cs.tkmax[j] >= kRnBigBits ? (1 << 24) : rn_apply(cs.tmap[j], S);
        if (next >= (1 << 24)) {
          bad = crank * kt + j;
          break;
        }
        S = next;
      }
      cs.bad = bad;
      cs.bad_S = S;
    }
    int first = INT_MAX;
    if (C > 1) {
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();
      if (threadIdx.x == 0) {
        int b = INT_MAX;
        for (int r = 0; r < C; ++r) b = min(b, cluster.map_shared_rank(&cs, r)->bad);
        cs.first_bad = b;
      }
      __syncthreads();
      first = cs.first_bad;
    } else {
      __syncthreads();
      first = cs.bad;
    }
    if (first == INT_MAX) first = C * kt - 1;  // not expected: the composed check failed
    const int r_bad = first / kt, j_bad = first % kt;
    const long long t_bad = e0 + (long long)r_bad * part + (long long)j_bad * T;
    if (crank == r_bad) {
      RnState sb = st;
      sb.S = cs.bad_S;
      RnRun tile;
      rn_load<VEC>(tile, X, ld, m, total, rn_cursor_at(t_bad + own, m));
      float snf = 0.0f;
      const bool ok = rn_tile(tile, sb, sh, snf);
      st.parity = sb.parity;
      if (threadIdx.x == 0) {
        cs.pub_ok = ok ? 1 : 0;
        cs.pub_bits = ok ? __float_as_uint(rn_value(sb, sb.S)) : __float_as_uint(snf);
      }
    }
    const RnClusterSlots* pub = &cs;
    if (C > 1) {
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();
      pub = cluster.map_shared_rank(&cs, r_bad);
    } else {
      __syncthreads();
    }
    const int ok = pub->pub_ok;
    const float sv = __uint_as_float(pub->pub_bits);
    // every read of this step's slots precedes the next step's writes
    if (C > 1)
      cg::this_cluster().sync();
    else
      __syncthreads();
    if (!ok) {
      s_nf = sv;
      done = t_bad;
      break;
    }
    rn_set(st, sv);
    e0 = t_bad + T;
    kt = tiles_at(e0);
    c = rn_cursor_at(e0 + (long long)crank * kt * T + own, m);
    rn_load<VEC>(cur, X, ld, m, total, c);
  }
  // the cluster's CTAs stay resident until every remote read is done
  if (C > 1) cg::this_cluster().sync();
  if (done < 0) return rn_value(st, st.S);
  if (isnan(s_nf)) return s_nf;
  // +inf reached: adding the remaining terms keeps it, unless one is NaN
  bool nan = false;
  for (long long e = done + threadIdx.x; e < total; e += kRnThreads) {
    const long long row = e / m, col = e - row * m;
    nan |= isnan(__bfloat162float(X[row * ld + col]));
  }
  return __syncthreads_or(nan) ? __int_as_float(0x7fffffff) : s_nf;
}

// One cluster of C CTAs per matrix (grid = clusters x C), the clusters striding
// over the launch's matrices. VEC: the matrices whose rows hold whole 16-byte
// groups (16-byte loads; rows start 16-byte aligned since the class row stride
// is a multiple of 8 elements); otherwise the others, element by element.
template <bool VEC>
__global__ void __launch_bounds__(kRnThreads) refnorm_kernel(const MuonArgs a, int C) {
  __shared__ RnShared sh;
  __shared__ RnClusterSlots cs;
  if (a.skip && *a.skip) return;
  const int crank = C > 1 ? (int)cooperative_groups::this_cluster().block_rank() : 0;
  const int nclusters = gridDim.x / C;
  for (int k = blockIdx.x / C; k < a.nmat; k += nclusters) {
    const MuonMat mm = a.mats[k];
    const MuonClassPtr cp = a.cls[mm.xcls];
    const __nv_bfloat16* X =
        static_cast<const __nv_bfloat16*>(cp.x) + (long long)mm.xbatch * cp.bstride;
    const int n = mm.transposed ? mm.cols : mm.rows;
    const int m = mm.transposed ? mm.rows : mm.cols;
    if ((m % 8 == 0) != VEC) continue;  // the other instantiation's matrix
    const float s = rn_matrix_sum<VEC>(X, cp.ld, m, (long long)n * m, sh, cs, C, crank);
    if (crank == 0 && threadIdx.x == 0)
      a.norms[mm.norm_idx] = fmaxf(__fsqrt_rn(s), 1e-7f);  // lib.rs:109
    __syncthreads();
  }
}

}  // namespace

int ref_norm_cluster(long long max_elems, long long total_elems, int nmat, int num_sms) {
  // Split the largest matrix until its share is no larger than 1.5 times an
  // even spread of all the launch's elements over the SMs (at most 8 CTAs,
  // the portable cluster size): the long sequential sums then no longer set
  // the launch's length.
  const long long even = total_elems / (num_sms > 0 ? num_sms : 1) + 1;
  int c = 1;
  while (c < 8 && max_elems / c > even + even / 2) c *= 2;
  (void)nmat;
  return c;
}

void launch_ref_norms(const MuonArgs& a, int cluster, cudaStream_t stream) {
  if (a.nmat <= 0) return;
  const int C = cluster == 2 || cluster == 4 || cluster == 8 ? cluster : 1;
  // clusters stride over the matrices (largest first)
  const int clusters = a.nmat < 4096 ? a.nmat : 4096;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * C));
  cfg.blockDim = dim3(kRnThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, refnorm_kernel<true>, a, C);
  if (a.norm_scalar_rows) cudaLaunchKernelEx(&cfg, refnorm_kernel<false>, a, C);
}

}  // namespace mmn
