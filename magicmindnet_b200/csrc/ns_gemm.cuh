// Newton-Schulz GEMMs on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One persistent, warp-specialised kernel template covers the three products of
// one Newton-Schulz iteration of crates/mmn-optim/src/lib.rs:112-120 over a batch
// of same-shaped matrices X[b] (n x m, n <= m, bf16-valued, row-major):
//
//   Gram   : A   = bf16((X X^T) / s / s)          M=N=n, K=m, symmetric
//   Square : A2  = bf16(A A)                      M=N=n, K=n, symmetric (A = A^T)
//            (bf16 mode: Bm = bf16(b*A + c*bf16(A A)))
//   Poly   : X'  = bf16((X/s)*a + (b*(A X) + c*(A2 X))/s)   M=n, N=m, K=n
//            two TMEM accumulators share each X tile, so the reference's fp32
//            B = b*A + c*A2 never has to be rounded to feed the tensor cores
//            (bf16 mode: X' = bf16((X/s)*a + (Bm X)/s), one accumulator).
//            On CTA pairs the product is computed transposed, X'^T = X^T [A | A2]
//            (A and A2 are symmetric): X^T is the MN-major A operand (a
//            256-column strip of X), and 64 rows of A stacked on the same 64
//            rows of A2 form each CTA's half of one N = 256 K-major B operand,
//            so both accumulators come from one MMA per K step and sit side by
//            side in TMEM. A stage holds 32 KB per 512 tensor clocks instead of
//            40 KB, with half the MMA instructions.
//
// s is the per-matrix Frobenius norm in the first iteration (lib.rs:109-110)
// and 1 afterwards. All operand values are exactly bf16, so the tensor-core
// products are exact and only the fp32 summation order differs from the CPU.
//
// F32 = true instantiates the TF32 mode: the same three products and the same
// rounding points, with every stored matrix (X, A, A2) held in fp32 words
// rounded to tf32 (10-bit mantissa, round-to-nearest-even) instead of bf16,
// and the MMAs issued as kind::tf32. A 128-byte swizzle row then holds 32
// elements, so a stage covers K = 32 and one MMA K = 8; stage byte sizes and
// the TMEM layout are the same as in bf16. MN-major tf32 operands use the
// 128-byte swizzle with 32-byte atoms, the only layout tcgen05 reads them in.
//
// SPLIT = true (with F32) instantiates the fp32 mode: no rounding points at
// all. Every stored matrix is kept as two tf32 planes, hi = tf32(v) and
// lo = tf32(v - hi) (batch items 2b and 2b + 1 of the same buffer), and every
// product is the three-pass hi*hi + hi*lo + lo*hi, which carries about 21
// mantissa bits instead of tf32's 11: hi*hi into the main accumulator, the two
// corrections into a second one, summed in the epilogue. Stages hold both
// planes of each operand; the symmetric outputs are stored from registers.
//
// In the last iteration the Poly epilogue can apply the Muon update
// p -= lr*sqrt(rows/cols) * X' (lib.rs:169-174) directly instead of storing X'.
//
// Roles (320 threads per CTA): warp 0 issues TMA loads, warp 1 owns TMEM and
// one lane issues tcgen05.mma, warps 2-9 drain TMEM and run the epilogue.
// PAIR=true runs one 256-row tile on a CTA pair (cluster of 2, cta_group::2):
// each CTA loads its 128 rows of A and half of B's columns, the leader CTA
// issues the MMAs for both and commits to both CTAs' barriers. No TMA load
// uses cluster multicast. Every mbarrier wait is time-bounded; on timeout the
// kernel records a status, drains what it issued, frees TMEM and returns.
#pragma once
#include <cuda.h>

#include "mmn_ptx.cuh"

namespace mmn {

enum NsEpilogue : int {
  kEpiGram = 0,
  kEpiSquare = 1,
  kEpiSquareBf16 = 2,
  kEpiPolyDual = 3,
  kEpiPolySingle = 4,
  kEpiPolyDualT = 5,  // PolyDual computed as X'^T = X^T [A | A2] (pairs only)
};

constexpr int kBM = 128;  // rows per CTA (TMEM lanes)

// Where the last iteration writes when it is fused with the Muon update.
struct NsApply {
  long long off;   // element offset of the parameter in the fp32 arena
  float lr_scale;  // lr * sqrt(rows / cols), f32 as the reference computes it
  int transposed;  // parameter is m x n and X holds its transpose
};

struct NsGemmArgs {
  void* out;                 // output matrices (bf16, or tf32-valued fp32 for F32)
  long long out_bstride;     // elements between batch items
  int out_ld;                // elements between rows
  const void* aux;           // epilogue input: X (Poly) or A (SquareBf16), as out
  long long aux_bstride;
  int aux_ld;
  const float* norms;        // per-matrix divisor s (nullptr means 1)
  int M, N, K;               // output rows, output cols, reduction length
  int tiles_n;               // column tiles per matrix (dense schedule)
  int tiles_per_matrix;      // tiles of one matrix
  int num_tiles;             // tiles_per_matrix * batch
  const int2* tile_list;     // symmetric schedule: (tm, tn) per tile, or nullptr
  int* status;               // device status word (0 = ok)
  float coef_a, coef_b, coef_c;
  float* p;                  // Poly, last iteration: fp32 params to update (or nullptr)
  __nv_bfloat16* p_bf16;     // optional bf16 copy of the updated params
  const NsApply* apply;      // per batch item, used when p is set
  const int* skip;           // device non-finite flag: when set the launch does nothing
};

template <int BN, bool DUAL, bool B_MN, bool PAIR, int EPI, bool F32 = false,
          bool SPLIT = false>
struct NsGemmShape {
  static constexpr int kPlanes = SPLIT ? 2 : 1;  // hi and lo tf32 planes per operand
  static constexpr int kEsz = F32 ? 4 : 2;  // bytes per stored operand element
  static constexpr int kBKe = 128 / kEsz;   // K per stage: one 128-byte swizzle row
  static constexpr int kKi = 32 / kEsz;     // K per MMA instruction (32 bytes)
  static constexpr int kMNe = 128 / kEsz;   // MN elements per 128-byte row of an MN-major box
  // transposed Poly: one A operand (X^T, MN-major) and a B operand of stacked
  // A and A2 rows
  static constexpr bool SWAP = EPI == kEpiPolyDualT;
  static constexpr bool SYM = EPI == kEpiGram || EPI == kEpiSquare || EPI == kEpiSquareBf16;
  static constexpr int kCtas = PAIR ? 2 : 1;
  static constexpr int kTileM = kBM * kCtas;        // output rows per tile
  static constexpr int kBNc = BN / kCtas;           // B columns loaded by one CTA
  static constexpr int kABytes = kBM * 128;         // 16 KB per A operand
  static constexpr int kBBytes = kBNc * 128;
  static constexpr int kStageBytes =
      kPlanes * (SWAP ? kABytes + 2 * kBBytes : kABytes * (DUAL ? 2 : 1) + kBBytes);
  // per epilogue warp: two 32 x 32 blocks of the symmetric output (direct and
  // mirrored, staged for TMA stores), or (SWAP) a 32 x 33 fp32 tile that turns
  // lane-per-column values into lane-per-row ones
  // (SPLIT symmetric outputs are stored directly from registers: their MMA phase
  // is three tf32 products per step, so the epilogue has time to spare)
  static constexpr int kEpiWarpBytes =
      SWAP ? 32 * 33 * 4 : ((SYM && !SPLIT) ? 2 * 32 * 32 * kEsz : 0);
  // bf16: at most 200 KB of stages; tf32: whatever the larger fp32 epilogue
  // stage leaves of the 227 KB
  static constexpr int kStageBudget =
      F32 ? 232448 - 2048 - 8 * kEpiWarpBytes : 204800;
  static constexpr int kStages =
      (kStageBudget / kStageBytes) < 8 ? (kStageBudget / kStageBytes) : 8;
  // SPLIT: the hi*hi products and the small hi*lo + lo*hi corrections go to two
  // accumulators (the corrections kSmallOff columns further), summed in the
  // epilogue. The tensor cores round each accumulator update toward zero, so
  // keeping the corrections apart leaves the main accumulator one update per K
  // step, as in the TF32 mode, and makes the corrections' own bias 2^-11 smaller.
  static constexpr int kSmallOff = SPLIT ? BN * (DUAL ? 2 : 1) : 0;
  static constexpr int kAccCols = BN * (DUAL ? 2 : 1) * (SPLIT ? 2 : 1);  // per buffer
  // two accumulator buffers when they fit in TMEM's 512 columns, else one
  // (the MMA of the next tile then waits for the epilogue)
  static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kAccBufs * kAccCols;
  static constexpr int kBarBytes = 1024;
  // Eight epilogue warps: two per TMEM lane quarter, each finishing half of a
  // tile's column chunks, so that the epilogue keeps pace with short K loops.
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kEpiBytes = kEpiWarps * kEpiWarpBytes;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + kEpiBytes + 1024;
  static_assert(kTmemCols <= 512, "TMEM has 512 columns");
  static_assert(kStages >= 2, "pipeline needs two stages");
  static_assert(!B_MN || kBNc % kMNe == 0, "MN-major B is loaded in 128-byte-wide boxes");
  static_assert(kEpiWarps == 8, "the stage budget counts eight epilogue warps");
  static_assert(!F32 || (EPI != kEpiSquareBf16 && EPI != kEpiPolySingle),
                "the bf16 mode has no tf32 form");
  static_assert(!SPLIT || F32, "split planes are tf32");
  static_assert(!SWAP || (DUAL && !B_MN && PAIR && kBNc == 64), "transposed Poly: pairs, dual");
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Round an fp32 value to tf32 (the 10 leading mantissa bits), to nearest with
// ties to even on the 13 discarded bits, written from the IEEE-754 definition.
// Inf and NaN pass through unchanged.
__device__ __forceinline__ float tf32r(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
  return __uint_as_float(u);
}

// The rounding point of the stored matrices: bf16, or tf32 in the TF32 mode.
template <bool F32>
__device__ __forceinline__ float op_round(float x) {
  if constexpr (F32)
    return tf32r(x);
  else
    return bf16r(x);
}

// 32 consecutive fp32 <-> float[32] (16-byte aligned).
__device__ __forceinline__ void load_f32x32(const float* src, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 u = *reinterpret_cast<const float4*>(src + q * 4);
    v[q * 4 + 0] = u.x;
    v[q * 4 + 1] = u.y;
    v[q * 4 + 2] = u.z;
    v[q * 4 + 3] = u.w;
  }
}
__device__ __forceinline__ void store_f32x32(float* dst, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<float4*>(dst + q * 4) =
        make_float4(v[q * 4 + 0], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
}

// 32 consecutive bf16 -> float (16-byte aligned source).
__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + q * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      v[q * 8 + e * 2] = f.x;
      v[q * 8 + e * 2 + 1] = f.y;
    }
  }
}

// 32 floats -> 32 consecutive bf16 (16-byte aligned destination).
__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
    u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
    u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
    u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
    *reinterpret_cast<uint4*>(dst + q * 8) = u;
  }
}

// Last step of every Poly epilogue for one row r and 32 columns c0..c0+31,
// given bx = (b*A X + c*A2 X) or Bm X: o = round((X/s)*a + bx/s) (bf16, or tf32
// for F32), stored as X' or, in the last iteration, applied as
// p -= lr*scale*o in the parameter's orientation (lib.rs:169-174). bx is
// overwritten with o.
template <bool F32, bool SPLIT = false>
__device__ __forceinline__ void poly_finish(const NsGemmArgs& args, int b, int r, int c0,
                                            bool row_ok, bool cols_full, float s,
                                            float (&v)[32]) {
  const long long xoff = (long long)b * args.aux_bstride * (SPLIT ? 2 : 1) +
                         (long long)r * args.aux_ld + c0;
  float xv[32];
  if constexpr (SPLIT) {
    // X = hi + lo (planes 2b and 2b + 1); no rounding point: the sum is X's
    // fp32 value up to the bits below the lo plane's tf32 precision
    const float* xh = static_cast<const float*>(args.aux) + xoff;
    const float* xl = xh + args.aux_bstride;
    if (row_ok && cols_full) {
      float lo[32];
      load_f32x32(xh, xv);
      load_f32x32(xl, lo);
#pragma unroll
      for (int j = 0; j < 32; ++j) xv[j] = __fadd_rn(xv[j], lo[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        xv[j] = (row_ok && c0 + j < args.N) ? __fadd_rn(xh[j], xl[j]) : 0.0f;
    }
  } else if constexpr (F32) {
    const float* xrow = static_cast<const float*>(args.aux) + xoff;
    if (row_ok && cols_full) {
      load_f32x32(xrow, xv);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) xv[j] = (row_ok && c0 + j < args.N) ? xrow[j] : 0.0f;
    }
  } else {
    const __nv_bfloat16* xrow = static_cast<const __nv_bfloat16*>(args.aux) + xoff;
    if (row_ok && cols_full) {
      load_bf16x32(xrow, xv);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        xv[j] = (row_ok && c0 + j < args.N) ? __bfloat162float(xrow[j]) : 0.0f;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float x0 = s != 1.0f ? __fdiv_rn(xv[j], s) : xv[j];
    const float bs = s != 1.0f ? __fdiv_rn(v[j], s) : v[j];
    const float o = __fadd_rn(__fmul_rn(x0, args.coef_a), bs);
    v[j] = SPLIT ? o : op_round<F32>(o);
  }
  if (!args.p) {
    const long long ooff = (long long)b * args.out_bstride * (SPLIT ? 2 : 1) +
                           (long long)r * args.out_ld + c0;
    if constexpr (SPLIT) {
      // X' as its hi and lo tf32 planes
      float hi[32], lo[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        hi[j] = tf32r(v[j]);
        lo[j] = tf32r(__fsub_rn(v[j], hi[j]));
      }
      float* oh = static_cast<float*>(args.out) + ooff;
      float* ol = oh + args.out_bstride;
      if (row_ok && cols_full) {
        store_f32x32(oh, hi);
        store_f32x32(ol, lo);
      } else if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < args.N) {
            oh[j] = hi[j];
            ol[j] = lo[j];
          }
      }
    } else if constexpr (F32) {
      float* orow = static_cast<float*>(args.out) + ooff;
      if (row_ok && cols_full) {
        store_f32x32(orow, v);
      } else if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < args.N) orow[j] = v[j];
      }
    } else {
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(args.out) + ooff;
      if (row_ok && cols_full) {
        store_bf16x32(orow, v);
      } else if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < args.N) orow[j] = __float2bfloat16_rn(v[j]);
      }
    }
    return;
  }
  // The parameters are read in full before the first store: a store through
  // args.p (or args.p_bf16) may alias a later load as far as the compiler can
  // tell, so interleaved loads and stores would wait out one memory round trip
  // each.
  const NsApply ap = args.apply[b];
  const float ls = ap.lr_scale;
  if (!ap.transposed) {
    const long long base = ap.off + (long long)r * args.N + c0;
    float* prow = args.p + base;
    if (row_ok && cols_full && (base & 3) == 0) {
      float4 pin[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) pin[q] = *reinterpret_cast<const float4*>(prow + q * 4);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 pv = pin[q];
        pv.x = __fsub_rn(pv.x, __fmul_rn(ls, v[q * 4 + 0]));
        pv.y = __fsub_rn(pv.y, __fmul_rn(ls, v[q * 4 + 1]));
        pv.z = __fsub_rn(pv.z, __fmul_rn(ls, v[q * 4 + 2]));
        pv.w = __fsub_rn(pv.w, __fmul_rn(ls, v[q * 4 + 3]));
        *reinterpret_cast<float4*>(prow + q * 4) = pv;
        if (args.p_bf16) {
          uint2 u;
          u.x = pack_bf16x2(pv.x, pv.y);
          u.y = pack_bf16x2(pv.z, pv.w);
          *reinterpret_cast<uint2*>(args.p_bf16 + base + q * 4) = u;
        }
      }
    } else if (row_ok) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < args.N) {
          const float pn = __fsub_rn(prow[j], __fmul_rn(ls, v[j]));
          prow[j] = pn;
          if (args.p_bf16) args.p_bf16[base + j] = __float2bfloat16_rn(pn);
        }
    }
  } else if (row_ok) {
    // Parameter element (c, r): consecutive lanes touch consecutive r.
    float pin[32];
#pragma unroll
    for (int j = 0; j < 32; ++j)
      pin[j] = c0 + j < args.N ? args.p[ap.off + (long long)(c0 + j) * args.M + r] : 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (c0 + j < args.N) {
        const long long idx = ap.off + (long long)(c0 + j) * args.M + r;
        const float pn = __fsub_rn(pin[j], __fmul_rn(ls, v[j]));
        args.p[idx] = pn;
        if (args.p_bf16) args.p_bf16[idx] = __float2bfloat16_rn(pn);
      }
  }
}

// One MMA of the tile's element type, on one CTA or on the pair.
template <bool F32, bool PAIR>
__device__ __forceinline__ void ns_mma(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc,
                                       uint32_t accum) {
  if constexpr (F32) {
    if constexpr (PAIR)
      tc_mma_tf32_pair(d, da, db, idesc, accum);
    else
      tc_mma_tf32(d, da, db, idesc, accum);
  } else {
    if constexpr (PAIR)
      tc_mma_bf16_pair(d, da, db, idesc, accum);
    else
      tc_mma_bf16(d, da, db, idesc, accum);
  }
}

// The fused Muon update of the transposed bf16 Poly for a parameter laid out
// like X' (not transposed). v[j] is X' element (c0 + j, rw + lane); the warp's
// 32 x 32 block goes through its shared-memory stage so that eight lanes cover
// one row, four consecutive columns each: every load and store of X (4 bf16)
// and of the fp32 parameters (a float4) is then vectorised, and one warp
// instruction touches four whole 128-byte lines. Same arithmetic as
// poly_finish. Only full, 16-byte-aligned blocks come here.
// The caller has staged the block (tst[j * 33 + lane] = v[j]) and passes the
// fields it needs by value; out of line, so that its registers stay out of the
// epilogue's. xb: X of this batch item; p: the parameter's first element.
static __device__ __noinline__ void poly_update_rows(const __nv_bfloat16* xb, int aux_ld, float* p,
                                              __nv_bfloat16* p_bf16, int N, float coef_a,
                                              float ls, int c0, int rw, float s,
                                              const float* tst) {
  const int lane = threadIdx.x & 31;
  const int rsub = lane >> 3, c4 = (lane & 7) * 4;
  // Two halves of four rounds; in each, every load comes before the first
  // store (a store may alias a later load as far as the compiler can tell).
#pragma unroll
  for (int h = 0; h < 8; h += 4) {
    uint2 xin[4];
    float4 pin[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int row = c0 + (h + q) * 4 + rsub;
      xin[q] = *reinterpret_cast<const uint2*>(xb + (long long)row * aux_ld + rw + c4);
      pin[q] =
          *reinterpret_cast<const float4*>(p + (long long)row * N + rw + c4);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int rl = (h + q) * 4 + rsub;  // row in the block
      const long long base = (long long)(c0 + rl) * N + rw + c4;
      const __nv_bfloat162 x01 = *reinterpret_cast<const __nv_bfloat162*>(&xin[q].x);
      const __nv_bfloat162 x23 = *reinterpret_cast<const __nv_bfloat162*>(&xin[q].y);
      const float xv[4] = {__low2float(x01), __high2float(x01), __low2float(x23),
                           __high2float(x23)};
      float pv[4] = {pin[q].x, pin[q].y, pin[q].z, pin[q].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float vv = tst[rl * 33 + c4 + i];
        const float x0 = s != 1.0f ? __fdiv_rn(xv[i], s) : xv[i];
        const float bs = s != 1.0f ? __fdiv_rn(vv, s) : vv;
        const float o = op_round<false>(__fadd_rn(__fmul_rn(x0, coef_a), bs));
        pv[i] = __fsub_rn(pv[i], __fmul_rn(ls, o));
      }
      *reinterpret_cast<float4*>(p + base) = make_float4(pv[0], pv[1], pv[2], pv[3]);
      if (p_bf16) {
        uint2 u;
        u.x = pack_bf16x2(pv[0], pv[1]);
        u.y = pack_bf16x2(pv[2], pv[3]);
        *reinterpret_cast<uint2*>(p_bf16 + base) = u;
      }
    }
  }
  __syncwarp();  // the stage is rewritten by the next chunk
}

// X' of a full block of the transposed bf16 Poly (no fused update), from the
// warp's stage (tst[j * 33 + lane] = v[j], v[j] being X' element (c0 + j, rw +
// lane)): four lanes cover one row, eight consecutive columns each, so X is
// read and X' written as 16-byte vectors, eight whole rows per instruction.
// Same arithmetic as poly_finish.
static __device__ __noinline__ void poly_store_rows(const __nv_bfloat16* xb, __nv_bfloat16* ob,
                                                    int ld, float coef_a, int c0, int rw, float s,
                                                    const float* tst) {
  const int lane = threadIdx.x & 31;
  const int rsub = lane >> 2, c8 = (lane & 3) * 8;
  uint4 xin[4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
    xin[q] = *reinterpret_cast<const uint4*>(xb + (long long)(c0 + q * 8 + rsub) * ld + rw + c8);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int rl = q * 8 + rsub;
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xin[q]);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __nv_bfloat162 x2 = *reinterpret_cast<const __nv_bfloat162*>(&xw[i / 2]);
      const float xv = (i & 1) ? __high2float(x2) : __low2float(x2);
      const float vv = tst[rl * 33 + c8 + i];
      const float x0 = s != 1.0f ? __fdiv_rn(xv, s) : xv;
      const float bs = s != 1.0f ? __fdiv_rn(vv, s) : vv;
      o[i] = op_round<false>(__fadd_rn(__fmul_rn(x0, coef_a), bs));
    }
    uint4 u;
    u.x = pack_bf16x2(o[0], o[1]);
    u.y = pack_bf16x2(o[2], o[3]);
    u.z = pack_bf16x2(o[4], o[5]);
    u.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4*>(ob + (long long)(c0 + rl) * ld + rw + c8) = u;
  }
  __syncwarp();  // the stage is rewritten by the next chunk
}

template <int BN, bool DUAL, bool B_MN, int EPI, bool PAIR, bool F32 = false, bool SPLIT = false>
__global__ void __launch_bounds__(320, 1)
    ns_gemm_kernel(const __grid_constant__ CUtensorMap tm_a1,
                   const __grid_constant__ CUtensorMap tm_a2,
                   const __grid_constant__ CUtensorMap tm_b, const NsGemmArgs args) {
  constexpr bool kSwap = EPI == kEpiPolyDualT;
  using S = NsGemmShape<BN, DUAL, B_MN, PAIR, EPI, F32, SPLIT>;
  constexpr int kBK = S::kBKe;  // K per stage
  constexpr int STAGES = S::kStages;
  constexpr bool kSym = EPI == kEpiGram || EPI == kEpiSquare || EPI == kEpiSquareBf16;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* full = bars;                     // [STAGES] TMA -> MMA
  uint64_t* empty = bars + STAGES;           // [STAGES] MMA -> TMA
  uint64_t* tfull = bars + 2 * STAGES;       // [2] MMA -> epilogue
  uint64_t* tempty = bars + 2 * STAGES + 2;  // [2] epilogue -> MMA
  uint64_t* drain = bars + 2 * STAGES + 4;   // abort path: MMA completion
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 6);
  uint8_t* epi_stage = smem + STAGES * S::kStageBytes + S::kBarBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int group = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int groups = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 32 * S::kEpiWarps * S::kCtas);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a1);
    if (DUAL || kSym) tma_prefetch_desc(&tm_a2);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, S::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, S::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // peer barriers initialised, both TMEM allocations done
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Launched as a programmatic dependent: the setup above touches only this
  // CTA's shared memory, its TMEM and the tensor-map parameters, so it overlaps
  // the previous kernel's last tiles (a CTA is placed on an SM only once the
  // previous kernel's CTA there has left, shared memory and TMEM included).
  // Nothing in global memory is read or written before the previous kernel has
  // completed. The next kernel may then be scheduled; it waits the same way.
  griddep_wait();
  griddep_launch_dependents();
  // A skipped step (non-finite grads) leaves every buffer untouched. The flag
  // is the same for every CTA, so both CTAs of a pair take this path together.
  if (args.skip && *args.skip) {
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync_all();
    if (warp == 1) {
      tc_fence_after();
      if (PAIR)
        tmem_dealloc_pair(tmem_base, S::kTmemCols);
      else
        tmem_dealloc(tmem_base, S::kTmemCols);
    }
    return;
  }
  const int num_kb = (args.K + kBK - 1) / kBK;

  auto decode = [&](int tile, int& b, int& tm, int& tn) {
    b = tile / args.tiles_per_matrix;
    const int r = tile - b * args.tiles_per_matrix;
    if (args.tile_list) {
      const int2 t = args.tile_list[r];
      tm = t.x;
      tn = t.y;
    } else {
      tm = r / args.tiles_n;
      tn = r - tm * args.tiles_n;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_parity = 0;
      bool ok = true;
      for (int tile = group; ok && tile < args.num_tiles; tile += groups) {
        int b, tm, tn;
        decode(tile, b, tm, tn);
        const int row0 = tm * S::kTileM + (int)rank * kBM;
        const int col0 = tn * BN + (int)rank * S::kBNc;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = tiles + stage * S::kStageBytes;
          if (leader) mbar_arrive_expect_tx(&full[stage], S::kStageBytes * S::kCtas);
          const int k0 = kb * kBK;
          // One load of a box into st_dst, on the pair's leader barrier or this CTA's.
          const uint32_t fb = PAIR ? mapa_shared(smem_u32(&full[stage]), 0) : 0u;
          auto load = [&](uint8_t* dst, const CUtensorMap* map, int x, int y, int z) {
            if constexpr (PAIR)
              tma_load_3d_pair(dst, map, fb, x, y, z);
            else
              tma_load_3d(dst, map, &full[stage], x, y, z);
          };
          // SPLIT: every operand comes as two planes (hi at batch index 2b, lo
          // at 2b + 1), stored one after the other in the stage.
#pragma unroll
          for (int pl = 0; pl < S::kPlanes; ++pl) {
            const int z = b * S::kPlanes + pl;
            if (kSwap) {
              // A side: X^T rows row0.. = X columns, 128-byte-wide MN-major
              // boxes; B side: rows col0.. of A (tm_b) and of A2 (tm_a2), K-major.
              uint8_t* sa = st + pl * S::kABytes;
              uint8_t* sbp = st + S::kPlanes * S::kABytes + pl * 2 * S::kBBytes;
#pragma unroll
              for (int g = 0; g < kBM / S::kMNe; ++g)  // 2 (bf16) or 4 (tf32) boxes
                load(sa + g * (kBK * 128), &tm_a1, row0 + g * S::kMNe, k0, z);
              load(sbp, &tm_b, k0, col0, z);
              load(sbp + S::kBBytes, &tm_a2, k0, col0, z);
            } else {
              load(st + pl * S::kABytes, &tm_a1, k0, row0, z);
              if (DUAL) load(st + (S::kPlanes + pl) * S::kABytes, &tm_a2, k0, row0, z);
              uint8_t* sbp = st + S::kPlanes * S::kABytes * (DUAL ? 2 : 1) + pl * S::kBBytes;
              if (B_MN) {
#pragma unroll
                for (int g = 0; g < S::kBNc / S::kMNe; ++g)
                  load(sbp + g * (kBK * 128), &tm_b, col0 + g * S::kMNe, k0, z);
              } else {
                load(sbp, &tm_b, k0, col0, z);
              }
            }
          }
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every load must land before the CTA may exit. The leader's full
      // barriers count both CTAs' bytes; the peer is held by the final
      // cluster barrier until the leader has seen them complete.
      if (leader) {
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s)) {
            const uint64_t t0 = global_timer_ns();
            while (!mbar_try_wait(&full[s], (last_parity >> s) & 1u)) {
              if (global_timer_ns() - t0 > kWaitLimitNs) {
                *abort_flag = 1;
                break;
              }
            }
          }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue
    if (lane == 0 && leader) {
      // (transposed Poly: one N = 2*BN MMA over the stacked [A rows | A2 rows])
      constexpr uint32_t idesc =
          F32 ? umma_idesc_tf32(S::kTileM, kSwap ? 2 * BN : BN, kSwap, B_MN)
              : umma_idesc_bf16(S::kTileM, kSwap ? 2 * BN : BN, kSwap, B_MN);
      constexpr int kKSteps = kBK / S::kKi;  // MMAs per stage (4)
      constexpr uint32_t kMnStep = S::kKi * 128;  // MN-major operand: bytes per MMA K
      // MN-major operand descriptor: bf16 in the 128-byte swizzle (8-row
      // pattern), tf32 in the 32-byte-atom 128-byte swizzle (4-row pattern)
      auto mn_desc = [](uint32_t addr) -> uint64_t {
        if constexpr (F32)
          return umma_desc_sw128_32b(addr, kBK * 128, 512);
        else
          return umma_desc_sw128(addr, kBK * 128, 1024);
      };
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = group; ok && tile < args.num_tiles; tile += groups) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d1 = tmem_base + acc * S::kAccCols;
        const uint32_t d2 = d1 + BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a1 = smem_u32(tiles + stage * S::kStageBytes);
          // SPLIT: products hi*hi + hi*lo + lo*hi of the two planes (plane pa of
          // the A operand, pb of the B operand), the three-pass tf32 product that
          // carries about 21 mantissa bits; hi*hi into the main accumulator, the
          // two corrections into the one kSmallOff columns further.
          constexpr int kCombos = SPLIT ? 3 : 1;
          if (kSwap) {
            // The CTA's A box and A2 box lie back to back: one 128-row K-major B
            // operand per CTA, 256 rows for the pair. Accumulator columns:
            // [A X | A2 X] for the leader's 64 rows of A, then the same for the
            // peer's 64 rows.
            const uint32_t b1 = a1 + S::kPlanes * S::kABytes;
#pragma unroll
            for (int kk = 0; kk < kKSteps; ++kk) {
#pragma unroll
              for (int cmb = 0; cmb < kCombos; ++cmb) {
                const uint32_t pa = cmb == 2, pb = cmb == 1;
                const uint64_t da = mn_desc(a1 + pa * S::kABytes + kk * kMnStep);
                const uint64_t db = umma_desc_sw128(b1 + pb * 2 * S::kBBytes + kk * 32, 16, 1024);
                ns_mma<F32, true>(d1 + (cmb ? S::kSmallOff : 0), da, db, idesc,
                                  cmb == 2 || (kb | kk) != 0);
              }
            }
          }
          const uint32_t a2 = a1 + S::kPlanes * S::kABytes;
          const uint32_t bb = a1 + S::kPlanes * S::kABytes * (DUAL ? 2 : 1);
#pragma unroll
          for (int kk = 0; kk < (kSwap ? 0 : kKSteps); ++kk) {
#pragma unroll
            for (int cmb = 0; cmb < kCombos; ++cmb) {
              const uint32_t pa = cmb == 2, pb = cmb == 1;
              const uint64_t da1 = umma_desc_sw128(a1 + pa * S::kABytes + kk * 32, 16, 1024);
              const uint32_t bp = bb + pb * S::kBBytes;
              const uint64_t db = B_MN ? mn_desc(bp + kk * kMnStep)
                                       : umma_desc_sw128(bp + kk * 32, 16, 1024);
              const uint32_t accum = cmb == 2 || (kb | kk) != 0;
              const uint32_t off = cmb ? S::kSmallOff : 0;
              ns_mma<F32, PAIR>(d1 + off, da1, db, idesc, accum);
              if (DUAL) {
                const uint64_t da2 = umma_desc_sw128(a2 + pa * S::kABytes + kk * 32, 16, 1024);
                ns_mma<F32, PAIR>(d2 + off, da2, db, idesc, accum);
              }
            }
          }
          issued_any = true;
          if (PAIR)
            tc_commit_pair_mc(&empty[stage], 0x3);
          else
            tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (PAIR)
          tc_commit_pair_mc(&tfull[acc], 0x3);
        else
          tc_commit(&tfull[acc]);
        if (++acc == S::kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (*abort_flag && issued_any) {
        // Let every MMA this thread issued finish before TMEM is freed.
        if (PAIR)
          tc_commit_pair_mc(drain, 0x1);
        else
          tc_commit(drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (global_timer_ns() - t0 > kWaitLimitNs) break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;  // TMEM lane quarter this warp may access
    // column chunks of a tile this warp finishes: [ch_lo, ch_hi)
    constexpr int kChunksPerWarp = (BN / 32) / (S::kEpiWarps / 4);
    const int ch_lo = ((warp - 2) >> 2) * kChunksPerWarp, ch_hi = ch_lo + kChunksPerWarp;
    // symmetric outputs: two 32 x 32 blocks per warp (direct, mirror)
    uint8_t* stg = epi_stage + (warp - 2) * S::kEpiWarpBytes;
    const uint32_t tempty_leader0 = PAIR ? mapa_shared(smem_u32(&tempty[0]), 0) : 0u;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = group; tile < args.num_tiles; tile += groups) {
      int b, tm, tn;
      decode(tile, b, tm, tn);
      if (kSwap && args.p) {
        // Last iteration: the epilogue reads and writes the fp32 parameters,
        // which sit in DRAM. Their lines for this tile go to L2 while the MMAs
        // still run (one 128-byte line per lane and chunk).
        const NsApply ap = args.apply[b];
        const int rw0 = tm * S::kTileM + (int)rank * kBM + sub * 32;
#pragma unroll
        for (int ch = ch_lo; ch < ch_hi; ++ch) {
          const int n0 = tn * BN + ch * 32;
          if (!ap.transposed) {
            const int n = n0 + lane;
            if (n < args.M && rw0 < args.N)
              prefetch_l2(args.p + ap.off + (long long)n * args.N + rw0);
          } else {
            const int m = rw0 + lane;
            if (m < args.N && n0 < args.M)
              prefetch_l2(args.p + ap.off + (long long)m * args.M + n0);
          }
        }
      }
      // tcgen05.ld is warp-collective: the warp proceeds only if every lane saw
      // the accumulator become ready.
      const bool ready = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int rw = tm * S::kTileM + (int)rank * kBM + sub * 32;  // first row of this warp
      const int r = rw + lane;
      const uint32_t tbase = tmem_base + acc * S::kAccCols + ((uint32_t)(sub * 32) << 16);
      const float s = args.norms ? args.norms[b] : 1.0f;
      // SquareBf16 epilogue input (bf16 A of this batch item)
      const __nv_bfloat16* aux =
          (!F32 && args.aux)
              ? static_cast<const __nv_bfloat16*>(args.aux) + (long long)b * args.aux_bstride
              : nullptr;
      // (transposed Poly: the TMEM lanes run along X' columns, the
      // accumulator columns along X' rows)
      const int lane_dim = kSwap ? args.N : args.M, col_dim = kSwap ? args.M : args.N;
      const bool row_ok = r < lane_dim;
#pragma unroll 1
      for (int ch = ch_lo; ch < ch_hi; ++ch) {
        const int c0 = tn * BN + ch * 32;
        if (c0 >= col_dim) break;  // whole chunk beyond the matrix (uniform over the warp)
        const bool cols_full = c0 + 32 <= col_dim;
        float v[32];
        float w[32];
        // rows tn*BN + ch*32 .. +31 of A X at column (ch/2)*128 + (ch%2)*32 and
        // of A2 X 64 columns further (transposed Poly), or columns ch*32.. of
        // the first accumulator and BN further of the second
        const uint32_t col_v = kSwap ? (uint32_t)((ch >> 1) * 128 + (ch & 1) * 32) : ch * 32;
        const uint32_t col_w = kSwap ? col_v + 64 : BN + ch * 32;
        tmem_ld_32x32b_x32(tbase + col_v, v);
        if constexpr (SPLIT) {
          // main + corrections, rounded once
          float t[32];
          tmem_ld_32x32b_x32(tbase + S::kSmallOff + col_v, t);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], t[j]);
          if (DUAL) {
            tmem_ld_32x32b_x32(tbase + col_w, w);
            tmem_ld_32x32b_x32(tbase + S::kSmallOff + col_w, t);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = __fadd_rn(w[j], t[j]);
          }
        } else {
          if (DUAL) tmem_ld_32x32b_x32(tbase + col_w, w);
          tmem_ld_wait();
        }
        if (kSym) {
          // This tile owns the symmetric entries with col >= row and writes each
          // at (r, c) and, through a transposing smem stage, at (c, r).
          if (c0 + 31 < rw) continue;  // block entirely below the diagonal
          if constexpr (EPI == kEpiSquareBf16) {
            float a_in[32];
            const __nv_bfloat16* arow =
                static_cast<const __nv_bfloat16*>(aux) + (long long)r * args.aux_ld + c0;
            if (row_ok && cols_full) {
              load_bf16x32(arow, a_in);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                a_in[j] = (row_ok && c0 + j < args.N) ? __bfloat162float(arow[j]) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j)
              v[j] = __fadd_rn(__fmul_rn(a_in[j], args.coef_b), __fmul_rn(bf16r(v[j]), args.coef_c));
          } else if (EPI == kEpiGram) {
            if (s != 1.0f) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fdiv_rn(__fdiv_rn(v[j], s), s);
            }
          }
          // The warp's 32 x 32 block (rows rw.., columns c0..; c0 and rw are
          // multiples of 32, so it lies on or above the diagonal) is staged
          // row-major in shared memory and written by one TMA store, and its
          // transpose, the block (c0.., rw..), by a second. A diagonal block
          // takes its lower triangle from the mirrored values so that the
          // output is exactly symmetric. The stores clip at the matrix edge.
          const bool diag = c0 == rw;
          if constexpr (SPLIT) {
            // The fp32 result as its hi and lo tf32 planes (batch items 2b and
            // 2b + 1), stored from registers: the direct entries (r, c0 + j) and
            // the mirrored ones (c0 + j, r); on a diagonal block the lower
            // triangle comes from the mirrored values only.
#pragma unroll
            for (int pl = 0; pl < 2; ++pl) {
              float* o = static_cast<float*>(args.out) + (long long)(b * 2 + pl) * args.out_bstride;
              float pv[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float hi = tf32r(v[j]);
                pv[j] = pl == 0 ? hi : tf32r(__fsub_rn(v[j], hi));
              }
              if (row_ok) {
                float* orow = o + (long long)r * args.out_ld + c0;
                if (!diag && cols_full) {
                  store_f32x32(orow, pv);
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if ((!diag || j >= lane) && c0 + j < args.N) orow[j] = pv[j];
                }
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if ((!diag || j > lane) && c0 + j < args.N)
                    o[(long long)(c0 + j) * args.out_ld + r] = pv[j];
              }
            }
            continue;
          }
          if (lane == 0) bulk_wait_read_all();  // this warp's previous stores read their stage
          __syncwarp();
          uint8_t* mir_base = stg + 32 * 32 * S::kEsz;
          if constexpr (F32) {
            float* drow = reinterpret_cast<float*>(stg) + lane * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = tf32r(v[j]);
            store_f32x32(drow, v);
            float* mir = reinterpret_cast<float*>(diag ? stg : mir_base);
            if (diag) __syncwarp();  // the lower triangle overwrites direct values
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (!diag || j > lane) mir[j * 32 + lane] = v[j];
          } else {
            uint4* drow = reinterpret_cast<uint4*>(stg) + lane * 4;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 u;
              u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
              u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
              u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
              u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
              drow[q] = u;
            }
            __nv_bfloat16* mir = reinterpret_cast<__nv_bfloat16*>(diag ? stg : mir_base);
            if (diag) __syncwarp();  // the lower triangle overwrites direct values
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (!diag || j > lane) mir[j * 32 + lane] = __float2bfloat16_rn(v[j]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tm_a2, stg, c0, rw, b);
            if (!diag) tma_store_3d(&tm_a2, mir_base, rw, c0, b);
            bulk_commit();
          }
        } else {
          // Poly: bx = b*D1 + c*D2 (reference mode) or D (bf16 mode)
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (DUAL) v[j] = __fadd_rn(__fmul_rn(args.coef_b, v[j]), __fmul_rn(args.coef_c, w[j]));
          if (kSwap) {
            if constexpr (!F32) {
              if (args.p && !args.apply[b].transposed && c0 + 32 <= args.M &&
                  rw + 32 <= args.N && ((args.apply[b].off | args.N) & 3) == 0) {
                float* tst = reinterpret_cast<float*>(epi_stage) + (warp - 2) * 32 * 33;
#pragma unroll
                for (int j = 0; j < 32; ++j) tst[j * 33 + lane] = v[j];
                __syncwarp();
                const NsApply ap = args.apply[b];
                poly_update_rows(static_cast<const __nv_bfloat16*>(args.aux) +
                                     (long long)b * args.aux_bstride,
                                 args.aux_ld, args.p + ap.off,
                                 args.p_bf16 ? args.p_bf16 + ap.off : nullptr, args.N,
                                 args.coef_a, ap.lr_scale, c0, rw, s, tst);
                continue;
              }
              if (!args.p && c0 + 32 <= args.M && rw + 32 <= args.N &&
                  args.aux_ld == args.out_ld && args.aux_bstride == args.out_bstride) {
                float* tst = reinterpret_cast<float*>(epi_stage) + (warp - 2) * 32 * 33;
#pragma unroll
                for (int j = 0; j < 32; ++j) tst[j * 33 + lane] = v[j];
                __syncwarp();
                poly_store_rows(static_cast<const __nv_bfloat16*>(args.aux) +
                                    (long long)b * args.aux_bstride,
                                static_cast<__nv_bfloat16*>(args.out) +
                                    (long long)b * args.out_bstride,
                                args.out_ld, args.coef_a, c0, rw, s, tst);
                continue;
              }
            }
            // v[j] is X' element (c0 + j, r): transpose the warp's 32 x 32 block
            // through shared memory so that lane L holds row c0 + L, columns
            // rw .. rw + 31, and finish it like the row-major Poly.
            float* tst = reinterpret_cast<float*>(epi_stage) + (warp - 2) * 32 * 33;
#pragma unroll
            for (int j = 0; j < 32; ++j) tst[j * 33 + lane] = v[j];
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = tst[lane * 33 + j];
            __syncwarp();
            const int xr = c0 + lane;
            poly_finish<F32, SPLIT>(args, b, xr, rw, xr < args.M, rw + 32 <= args.N, s, v);
          } else {
            poly_finish<F32, SPLIT>(args, b, r, c0, row_ok, cols_full, s, v);
          }
        }
      }
      tc_fence_before();
      if (PAIR && !leader)
        mbar_arrive_cluster(tempty_leader0 + acc * 8);
      else
        mbar_arrive(&tempty[acc]);
      if (++acc == S::kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // the stage must outlive the TMA stores that read it
    if (kSym && lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // peer loads landed, remote arrivals done, MMAs retired
  if (*abort_flag && threadIdx.x == 0) atomicExch(args.status, kDevWaitTimeout);
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, S::kTmemCols);
    else
      tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace mmn
