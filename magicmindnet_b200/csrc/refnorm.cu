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
// monoid: a warp reduces (or scans) the maps of its elements in order.
//
// The kernel gives each matrix a cluster of C CTAs, which walks the sequence
// in cluster steps of consecutive parts, one per CTA; inside a part each warp
// owns a run of consecutive warp tiles (32 lanes x kRnEpt elements, each lane
// a run of kRnEpt consecutive ones):
//   - fast path: compose the element maps in order (lane, warp tile by
//     shuffles, warp segment, CTA part, cluster step); if no term was marked
//     for exact handling and the composed map leaves S <= 2^24 - 1, no add in
//     the step left the binade (S_i + k_i <= S_end + 1/2 for every element),
//     and S takes the composed value;
//   - slow path (a binade change or a term of at least 2^22 units): the first
//     warp tile whose map leaves the binade is walked by its warp: an ordered
//     warp scan gives every lane the S at its first element, lanes walk their
//     elements to the first one whose add can leave the binade, that add is
//     done as an fp32 add, and the walk resumes after it with the new binade;
//     the cluster step restarts after that warp tile.
// A binade change happens about log2(N) times per matrix, so nearly every
// step takes the fast path; ties (about 1% of the terms of bf16 squares) stay
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
constexpr uint32_t kRnMagicBits = 0x4B400000u;  // its bit pattern

__device__ __forceinline__ int rn_sat(int x) { return x < kRnSat ? x : kRnSat; }

// S -> S + A (tie = 0) or S -> S + A + ((S + B) & 1) (tie = 1). An element's
// map is S -> S + rint(k), or for a tie k = q + 1/2, S -> rue(S + q) with
// rue(y) = y + (y & 1), i.e. A = B = q. After a tie the running value's
// parity no longer depends on S (it is A + B mod 2), so maps compose into
// maps of the same form.
struct RnMap {
  int tie, A, B;
};

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
  uint32_t ybits[2];  // bit patterns of M + rint(k): val + kRnMagicBits
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
  p.ybits[0] = __float_as_uint(y.x);
  p.ybits[1] = __float_as_uint(y.y);
  p.val[0] = (int)(p.ybits[0] - kRnMagicBits);  // rint(k): the low mantissa bits of y
  p.val[1] = (int)(p.ybits[1] - kRnMagicBits);
  p.tie[0] = fabsf(d.x) == 0.5f;
  p.tie[1] = fabsf(d.y) == 0.5f;
  p.neg[0] = d.x < 0.0f;
  p.neg[1] = d.y < 0.0f;
  return p;
}

// Appends an element to a thread's running map. The sums wrap modulo 2^32:
// with terms below 2^22 units (at most kRnEpt of them) nothing wraps, and a
// run holding a larger term or a NaN leaves A meaningless, its k bit patterns
// sending it to the exact walk. Ties are about 1% of bf16 squares: they take
// the branch.
__device__ __forceinline__ void rn_fold(RnMap& m, int val, bool tie, bool neg) {
  const uint32_t a = (uint32_t)m.A, v = (uint32_t)val;
  if (!tie) {
    m.A = (int)(a + v);
  } else {
    const uint32_t q = v - (neg ? 1u : 0u);
    if (!m.tie) {
      m.tie = 1;
      m.A = (int)(a + q);
      m.B = m.A;
    } else {
      m.A = (int)(a + q + ((a + (uint32_t)m.B + q) & 1u));
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

// Warp form of a map: B < 0 when the map holds no tie (B >= 0 otherwise), so a
// map crosses a shuffle as two words and composes without branches.
struct RnWMap {
  int A, B;
};

__device__ __forceinline__ RnWMap rn_wmap(const RnMap m) {
  return {rn_sat(m.A), m.tie ? rn_sat(m.B) : -1};
}

__device__ __forceinline__ RnWMap rn_wcompose(const RnWMap a, const RnWMap b) {  // a, then b
  const bool at = a.B >= 0, bt = b.B >= 0;
  int A = a.A + b.A;
  if (at && bt) A += (a.A + a.B + b.B) & 1;
  const int B = at ? a.B : (bt ? a.A + b.B : -1);
  return {rn_sat(A), rn_sat(B)};
}

__device__ __forceinline__ int rn_wapply(const RnWMap m, int s) {
  return rn_sat(s + m.A + (m.B >= 0 ? ((s + m.B) & 1) : 0));
}

constexpr int kRnWarpTile = 32 * kRnEpt;  // elements of a warp tile: its lanes' runs in order

// Ordered composition of the lanes' maps; lane 0 receives lanes 0..31 in order
// (the other lanes' results are partial and unused).
__device__ __forceinline__ RnWMap rn_warp_reduce(RnWMap m) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const RnWMap o{__shfl_down_sync(0xffffffffu, m.A, off),
                   __shfl_down_sync(0xffffffffu, m.B, off)};
    m = rn_wcompose(m, o);
  }
  return m;
}

// Ordered inclusive scan of the lanes' maps.
__device__ __forceinline__ RnWMap rn_warp_scan(RnWMap m) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const RnWMap o{__shfl_up_sync(0xffffffffu, m.A, off), __shfl_up_sync(0xffffffffu, m.B, off)};
    if (lane >= off) m = rn_wcompose(o, m);
  }
  return m;
}

// The composed map of the run's elements and the max of their k bit patterns.
// A pair without a tie (98% of pairs) adds the bit patterns of its two M +
// rint(k) at once (one three-input add); the sum carries kRnMagicBits per
// element folded so far, modulo 2^32, and loses it at the end. The branch is
// taken per pair. (A term of 2^22 units or more, or a NaN, leaves A
// meaningless; kmax sends such a run to the exact walk.)
template <bool TINY>
__device__ __forceinline__ RnMap rn_run_fold(const RnRun& r, const RnState& st,
                                             uint32_t* kmax_out) {
  RnMap m{0, 0, 0};
  uint32_t biased = 0;  // A + (elements folded) * kRnMagicBits, modulo 2^32
  uint32_t kmax = 0;
#pragma unroll
  for (int i = 0; i < kRnEpt / 2; ++i) {
    const RnPair p = rn_pair<TINY>(r.word(i), st);
    kmax = max(kmax, max(p.kbits[0], p.kbits[1]));
    if (!(p.tie[0] | p.tie[1])) {
      biased += p.ybits[0] + p.ybits[1];
    } else {
      RnMap t{m.tie, (int)(biased - (uint32_t)(2 * i) * kRnMagicBits), m.B};
      rn_fold(t, p.val[0], p.tie[0], p.neg[0]);
      rn_fold(t, p.val[1], p.tie[1], p.neg[1]);
      m.tie = t.tie;
      m.B = t.B;
      biased = (uint32_t)t.A + (uint32_t)(2 * i + 2) * kRnMagicBits;
    }
  }
  m.A = (int)(biased - (uint32_t)kRnEpt * kRnMagicBits);
  *kmax_out = kmax;
  return m;
}

// The fold while the sum is below 2^-100 (its scale applied in double): out of
// line, so that its registers stay out of the main loop's.
__device__ __noinline__ RnMap rn_run_fold_tiny(const RnRun& r, const RnState& st,
                                               uint32_t* kmax_out) {
  return rn_run_fold<true>(r, st, kmax_out);
}

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

// Walks one warp tile (the 32 runs from element t0) exactly, on one warp: an
// ordered warp scan gives every lane the running sum at its first element, the
// lanes walk their elements to the first add that can leave the binade (or has
// a term of 2^22 units or more), that add is done as an fp32 add, and the walk
// resumes after it in the new binade. Returns false when the sum became
// non-finite (s_out holds it). Taken about log2(length) times per matrix, so
// it reloads its elements rather than holding registers for them.
template <bool VEC>
__device__ __forceinline__ bool rn_warp_walk(const __nv_bfloat16* X, int ld, int m, long long total,
                                          long long t0, RnState& st, float& s_out) {
  const int lane = threadIdx.x & 31;
  const int base = lane * kRnEpt;
  RnRun r;
  rn_load<VEC>(r, X, ld, m, total, rn_cursor_at(t0 + base, m));
  int start = 0;
  while (true) {
    // this lane's map over its elements from `start` on (values clamped so a
    // non-finite or huge term cannot overflow it; the walk stops there anyway)
    RnMap mm{0, 0, 0};
#pragma unroll
    for (int i = 0; i < kRnEpt / 2; ++i) {
      const RnPair p = st.tiny ? rn_pair<true>(r.word(i), st) : rn_pair<false>(r.word(i), st);
#pragma unroll
      for (int h = 0; h < 2; ++h)
        if (base + 2 * i + h >= start) rn_fold(mm, min(p.val[h], kRnSat), p.tie[h], p.neg[h]);
    }
    const RnWMap inc = rn_warp_scan(rn_wmap(rn_fold_sat(mm)));
    RnWMap exc{__shfl_up_sync(0xffffffffu, inc.A, 1), __shfl_up_sync(0xffffffffu, inc.B, 1)};
    if (lane == 0) exc = RnWMap{0, -1};
    const RnWMap all{__shfl_sync(0xffffffffu, inc.A, 31), __shfl_sync(0xffffffffu, inc.B, 31)};
    int S = rn_wapply(exc, st.S);
    int cand = INT_MAX;
    uint32_t cand_bits = 0;
#pragma unroll
    for (int i = 0; i < kRnEpt / 2; ++i) {
      const uint32_t w = r.word(i);
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
    // lanes after a stop may hold a meaningless S; their candidates come later
    const int stop = __reduce_min_sync(0xffffffffu, cand);
    if (stop == INT_MAX) {
      st.S = rn_wapply(all, st.S);
      return true;
    }
    const float s = __uint_as_float(__shfl_sync(0xffffffffu, cand_bits, stop / kRnEpt));
    if (!isfinite(s)) {
      s_out = s;
      return false;
    }
    rn_set(st, s);
    start = stop + 1;
  }
}

// Warp tiles a warp folds between cluster exchanges (at most).
constexpr int kRnTilesPerExchange = 16;

// Per-CTA slots: each warp's tile maps of the current cluster step and the
// composed map of its segment.
struct RnWarpSlots {
  RnWMap tile[kRnWarps][kRnTilesPerExchange];
  uint32_t tkmax[kRnWarps][kRnTilesPerExchange];
  RnWMap seg[kRnWarps];
  uint32_t skmax[kRnWarps];
};

// Cluster-level slots: one composed map per CTA and exchange parity, and the
// state a CTA publishes after walking the cluster step's first bad warp tile.
struct RnClusterSlots {
  RnWMap map[2];
  uint32_t kmax[2];
  RnWMap all;         // the cluster step's composed map (thread 0's result)
  uint32_t all_kmax;
  int bad;            // first warp tile of this CTA's part whose adds leave the binade
  int bad_S;          // the running sum (grid units) at that warp tile's start
  int first_bad;      // the cluster's first such warp tile (thread 0's result)
  uint32_t pub_bits;  // running sum after the exactly walked warp tile
  int pub_ok;         // 0: the sum became non-finite there
};

// The sequential sum over the whole oriented matrix X (n x m, row stride ld),
// computed by the C CTAs of a cluster (C = 1: one CTA). A cluster step is C
// consecutive parts of kt CTA tiles each (kt <= kRnTilesPerExchange); inside
// CTA r's part, warp w owns the w-th of kRnWarps consecutive segments of kt
// warp tiles and composes its tiles' maps in order with shuffles alone, so
// the warps run independently between exchanges. At the end of the step the
// CTA composes its warps' maps, the CTAs exchange their parts' maps through
// distributed shared memory, and each composes all of them in order, so every
// CTA holds the same running state. A cluster step whose composed map leaves
// the binade (or holds a term of 2^22 grid units or more) is resolved at warp
// tile granularity: its first bad warp tile is walked exactly by one warp, and
// the cluster restarts after that warp tile (the tiles behind it were folded
// for the old binade).
template <bool VEC>
__device__ __forceinline__ float rn_matrix_sum(const __nv_bfloat16* X, int ld, int m,
                                               long long total, RnWarpSlots& ws,
                                               RnClusterSlots& cs, int C, int crank) {
  namespace cg = cooperative_groups;
  constexpr int K = kRnTilesPerExchange;
  constexpr long long T = (long long)kRnThreads * kRnEpt;  // elements per CTA tile
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  RnState st;
  rn_set(st, 0.0f);
  float s_nf = 0.0f;
  long long done = -1;  // first element of the warp tile where the sum stopped being finite
  // Tiles per part. A step that leaves the binade is refolded from the warp
  // tile after the change, so steps are sized to end before the binade's top:
  // early on the sum changes binade whenever it doubles, so parts grow with
  // the distance covered (one tile at first, K once the sum is past C K
  // tiles); after that, with the growth per element of the last fast step
  // (rate, in value units), a step covers at most 3/4 of the elements expected
  // to fit in the room left above S (one tile per part near the top). Every
  // CTA of the cluster computes the same sizes from the same state.
  float rate = 0.0f;
  auto tiles_for = [&](long long e, float s_at) {
    const long long k0 = e / (T * C);
    int k = (int)(k0 < 1 ? 1 : (k0 > K ? K : k0));
    if (rate > 0.0f && !st.tiny) {
      const float fit = 0.75f * ((float)((1 << 24) - 1) - s_at) / (rate * st.scf) /
                        (float)(T * C);
      if (fit < (float)k) k = fit < 1.0f ? 1 : (int)fit;
    }
    return k;
  };
  // this thread's first run in the cluster step that starts at e
  auto run_at = [&](long long e, int kt) {
    return rn_cursor_at(e + ((long long)crank * kRnWarps + w) * kt * kRnWarpTile +
                            (long long)lane * kRnEpt,
                        m);
  };
  // one warp tile further inside the warp's segment
  const long long wt_rows = kRnWarpTile / m;
  const int wt_cols = (int)(kRnWarpTile - wt_rows * m);
  long long e0 = 0;
  int kt = tiles_for(0, 0.0f);
  RnCursor c = run_at(0, kt);
  RnRun cur, nxt;
  rn_load<VEC>(cur, X, ld, m, total, c);
  int cp = 0;
  while (e0 < total) {
    const long long part = kt * T, step = part * C;
    const long long seg0 = e0 + ((long long)crank * kRnWarps + w) * kt * kRnWarpTile;
    // the next step's first loads are issued before this step's sum is known:
    // it is sized from the sum this step is expected to reach
    const float s_pred = (float)st.S + (st.tiny ? 0.0f : rate * st.scf * (float)step);
    const int kt_next = tiles_for(e0 + step, s_pred);
    RnWMap acc{0, -1};
    uint32_t kacc = 0;
    for (int j = 0; j < kt; ++j) {
      // the next warp tile's loads fly while this one folds (zeros past the end)
      if (j + 1 < kt)
        rn_advance(c, kRnWarpTile, wt_rows, wt_cols, m);
      else
        c = run_at(e0 + step, kt_next);
      rn_load<VEC>(nxt, X, ld, m, total, c);
      RnWMap tot{0, -1};
      uint32_t kmax = 0;
      if (seg0 + (long long)j * kRnWarpTile < total) {  // warp-uniform: past the end adds nothing
        const RnMap mm =
            st.tiny ? rn_run_fold_tiny(cur, st, &kmax) : rn_run_fold<false>(cur, st, &kmax);
        tot = rn_warp_reduce(rn_wmap(mm));
        kmax = __reduce_max_sync(0xffffffffu, kmax);
        acc = rn_wcompose(acc, tot);
        kacc = max(kacc, kmax);
      }
      if (lane == 0) {
        ws.tile[w][j] = tot;
        ws.tkmax[w][j] = kmax;
      }
      cur = nxt;
    }
    if (lane == 0) {
      ws.seg[w] = acc;
      ws.skmax[w] = kacc;
    }
    __syncthreads();
    if (w == 0) {  // the CTA's part: its warps' segments in order
      RnWMap t = lane < kRnWarps ? ws.seg[lane] : RnWMap{0, -1};
      uint32_t km = lane < kRnWarps ? ws.skmax[lane] : 0u;
      t = rn_warp_reduce(t);
      km = __reduce_max_sync(0xffffffffu, km);
      if (lane == 0) {
        cs.map[cp] = t;
        cs.kmax[cp] = km;
      }
    }
    RnWMap all;
    uint32_t all_kmax;
    const int cp_step = cp;
    if (C > 1) {
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();
      if (w == 0) {  // lane r reads CTA r's part; the lanes compose them in order
        RnWMap t{0, -1};
        uint32_t km = 0;
        if (lane < C) {
          const RnClusterSlots* rem = cluster.map_shared_rank(&cs, lane);
          t = rem->map[cp];
          km = rem->kmax[cp];
        }
        t = rn_warp_reduce(t);
        km = __reduce_max_sync(0xffffffffu, km);
        if (lane == 0) {
          cs.all = t;
          cs.all_kmax = km;
        }
      }
      __syncthreads();
      all = cs.all;
      all_kmax = cs.all_kmax;
      cp ^= 1;
    } else {
      __syncthreads();
      all = cs.map[0];
      all_kmax = cs.kmax[0];
    }
    if (all_kmax < kRnBigBits) {
      const int s_end = rn_wapply(all, st.S);
      if (s_end <= (1 << 24) - 1) {
        if (!st.tiny) rate = (float)(s_end - st.S) / (st.scf * (float)step);
        st.S = s_end;
        e0 += step;
        kt = kt_next;
        continue;
      }
    }
    // slow: the cluster's first warp tile whose adds leave the binade (or hold
    // a term of 2^22 units or more). Each CTA starts from the composed maps of
    // the parts before its own and applies its warps' segment maps, then the
    // failing segment's tile maps, in order.
    const int units = kRnWarps * kt;  // warp tiles per part
    RnWMap pre{0, -1};
    if (C > 1 && w == 0) {  // the parts before this CTA's, composed across lanes
      if (lane < crank) pre = cg::this_cluster().map_shared_rank(&cs, lane)->map[cp_step];
      pre = rn_warp_reduce(pre);
    }
    if (threadIdx.x == 0) {
      int S = rn_wapply(pre, st.S);
      int bad = INT_MAX;
      const long long p0 = e0 + (long long)crank * part;
      for (int ww = 0; ww < kRnWarps && bad == INT_MAX; ++ww) {
        if (ws.skmax[ww] < kRnBigBits) {
          const int nx = rn_wapply(ws.seg[ww], S);
          if (nx < (1 << 24)) {
            S = nx;
            continue;
          }
        }
        for (int j = 0; j < kt; ++j) {
          if (p0 + ((long long)ww * kt + j) * kRnWarpTile >= total) break;
          const int next = ws.tkmax[ww][j] >= kRnBigBits ? (1 << 24) : rn_wapply(ws.tile[ww][j], S);
          if (next >= (1 << 24)) {
            bad = crank * units + ww * kt + j;
            break;
          }
          S = next;
        }
      }
      cs.bad = bad;
      cs.bad_S = S;
    }
    int first = INT_MAX;
    if (C > 1) {
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();
      if (w == 0) {
        const int b = __reduce_min_sync(
            0xffffffffu, lane < C ? cluster.map_shared_rank(&cs, lane)->bad : INT_MAX);
        if (lane == 0) cs.first_bad = b;
      }
      __syncthreads();
      first = cs.first_bad;
    } else {
      __syncthreads();
      first = cs.bad;
    }
    if (first == INT_MAX) first = C * units - 1;  // not expected: the composed check failed
    const int r_bad = first / units, u_bad = first % units;
    const long long t_bad = e0 + (long long)r_bad * part + (long long)u_bad * kRnWarpTile;
    if (crank == r_bad && w == u_bad / kt) {
      RnState sb = st;
      sb.S = cs.bad_S;
      float snf = 0.0f;
      const bool ok = rn_warp_walk<VEC>(X, ld, m, total, t_bad, sb, snf);
      if (lane == 0) {
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
    e0 = t_bad + kRnWarpTile;
    kt = tiles_for(e0, (float)st.S);
    c = run_at(e0, kt);
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
  __shared__ RnWarpSlots ws;
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
    const float s = rn_matrix_sum<VEC>(X, cp.ld, m, (long long)n * m, ws, cs, C, crank);
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
