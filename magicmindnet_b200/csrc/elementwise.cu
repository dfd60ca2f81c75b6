// Memory-bound kernels of the optimizer step. Every arithmetic step uses an
// explicitly rounded intrinsic (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn) so
// the compiler cannot contract a*b+c into an FMA: the reference (Rust, no FMA
// contraction) rounds after every operation, and so do these kernels.
#include "elementwise.cuh"
#include "mmn_ptx.cuh"

namespace mmn {

namespace {

__device__ __forceinline__ float load_grad(const float* g32, const __nv_bfloat16* g16,
                                           long long i) {
  return g16 ? __bfloat162float(g16[i]) : g32[i];
}

// AdamW::step_param arithmetic (crates/mmn-optim/src/lib.rs:47-59) for one element.
struct AdamwConst {
  float lr, b1, b2, one_m_b1, one_m_b2, eps, decay;
};

__device__ __forceinline__ void adamw_elem(float& p, float& m, float& v, float g, float bc1,
                                           float bc2, const AdamwConst& c) {
  m = __fadd_rn(__fmul_rn(c.b1, m), __fmul_rn(c.one_m_b1, g));
  v = __fadd_rn(__fmul_rn(c.b2, v), __fmul_rn(__fmul_rn(c.one_m_b2, g), g));
  const float mh = __fdiv_rn(m, bc1);
  const float vh = __fdiv_rn(v, bc2);
  const float upd = __fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), c.eps));
  p = __fsub_rn(p, __fmul_rn(c.lr, upd));
  p = __fmul_rn(p, c.decay);
}

// Division of a grad by the loss scale or the accumulation divisor. A power
// of two divides exactly as a multiplication by its reciprocal (both round
// the same real value), which saves the division sequence.
struct GradScaler {
  float d;
  float inv;
  int mode;  // 0: identity, 1: multiply by inv, 2: IEEE division by d
};

__device__ __forceinline__ GradScaler make_scaler(float d) {
  GradScaler s;
  s.d = d;
  s.inv = 1.0f;
  const uint32_t u = __float_as_uint(d);
  const uint32_t ex = (u >> 23) & 0xFFu;
  if (d == 1.0f) {
    s.mode = 0;
  } else if ((u & 0x007FFFFFu) == 0 && ex > 1 && ex < 253) {
    s.mode = 1;
    s.inv = __uint_as_float((254u - ex) << 23 | (u & 0x80000000u));  // exactly 1/d
  } else {
    s.mode = 2;
  }
  return s;
}

__device__ __forceinline__ float apply_scaler(float g, const GradScaler& s) {
  return s.mode == 0 ? g : (s.mode == 1 ? __fmul_rn(g, s.inv) : __fdiv_rn(g, s.d));
}

struct AdamwVec {
  float4 p, m, v;
  float g[4];
};

template <bool BF16G, bool FRESH>
__device__ __forceinline__ void adamw_load(const AdamwArgs& a, long long i, AdamwVec& q) {
  q.p = __ldcs(reinterpret_cast<const float4*>(a.p) + i);
  if (BF16G) {
    const uint2 raw = __ldcs(reinterpret_cast<const uint2*>(a.g_bf16) + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
    q.g[0] = f0.x;
    q.g[1] = f0.y;
    q.g[2] = f1.x;
    q.g[3] = f1.y;
  } else {
    const float4 g4 = __ldcs(reinterpret_cast<const float4*>(a.g) + i);
    q.g[0] = g4.x;
    q.g[1] = g4.y;
    q.g[2] = g4.z;
    q.g[3] = g4.w;
  }
  if (FRESH) {
    q.m = make_float4(0.f, 0.f, 0.f, 0.f);
    q.v = make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
    q.m = __ldcs(reinterpret_cast<const float4*>(a.m) + i);
    q.v = __ldcs(reinterpret_cast<const float4*>(a.v) + i);
  }
}

template <bool FRESH, bool SHADOW>
__device__ __forceinline__ void adamw_store(const AdamwArgs& a, long long i, const AdamwVec& q) {
  __stcs(reinterpret_cast<float4*>(a.p) + i, q.p);
  if (!FRESH) {
    __stcs(reinterpret_cast<float4*>(a.m) + i, q.m);
    __stcs(reinterpret_cast<float4*>(a.v) + i, q.v);
  }
  if (SHADOW) {
    uint2 out;
    __nv_bfloat162 h0 = __floats2bfloat162_rn(q.p.x, q.p.y);
    __nv_bfloat162 h1 = __floats2bfloat162_rn(q.p.z, q.p.w);
    out.x = *reinterpret_cast<uint32_t*>(&h0);
    out.y = *reinterpret_cast<uint32_t*>(&h1);
    __stcs(reinterpret_cast<uint2*>(a.p_bf16) + i, out);
  }
}

__device__ __forceinline__ void adamw_math(const AdamwArgs& a, long long i, long long base,
                                           const GradScaler& sc_scale, const GradScaler& sc_div,
                                           const AdamwConst& c, AdamwVec& q) {
  int t_off = a.seg0.t_offset;
  if (a.segs) {
    int s = __ldg(&a.chunk_seg[i / kAdamwChunk4]);
    while (i >= a.segs[s].end4) ++s;
    t_off = a.segs[s].t_offset;
  }
  long long t = base + t_off;
  if (t > a.t_sat) t = a.t_sat;
  const float2 bc = __ldg(&a.bc_table[t]);
#pragma unroll
  for (int e = 0; e < 4; ++e) q.g[e] = apply_scaler(apply_scaler(q.g[e], sc_scale), sc_div);
  adamw_elem(q.p.x, q.m.x, q.v.x, q.g[0], bc.x, bc.y, c);
  adamw_elem(q.p.y, q.m.y, q.v.y, q.g[1], bc.x, bc.y, c);
  adamw_elem(q.p.z, q.m.z, q.v.z, q.g[2], bc.x, bc.y, c);
  adamw_elem(q.p.w, q.m.w, q.v.w, q.g[3], bc.x, bc.y, c);
}

template <bool BF16G, bool FRESH, bool SHADOW>
__global__ void __launch_bounds__(256) adamw_kernel(const AdamwArgs a) {
  if (a.skip && *a.skip) return;
  const long long base = a.step_base ? *a.step_base : a.step_base_value;
  const float scale = a.grad_scale ? *a.grad_scale : 1.0f;
  AdamwConst c;
  c.lr = a.lr;
  c.b1 = a.b1;
  c.b2 = a.b2;
  c.one_m_b1 = __fsub_rn(1.0f, a.b1);
  c.one_m_b2 = __fsub_rn(1.0f, a.b2);
  c.eps = a.eps;
  c.decay = __fsub_rn(1.0f, __fmul_rn(a.lr, a.wd));
  const GradScaler sc_scale = make_scaler(scale);
  const GradScaler sc_div = make_scaler(a.grad_divisor);
  // Two float4 groups per thread and iteration: all eight loads are issued
  // before any arithmetic, doubling the bytes each thread keeps in flight.
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = a.begin4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i0 < a.end4;
       i0 += 2 * stride) {
    const long long i1 = i0 + stride;
    const bool has1 = i1 < a.end4;
    AdamwVec q0, q1;
    adamw_load<BF16G, FRESH>(a, i0, q0);
    if (has1) adamw_load<BF16G, FRESH>(a, i1, q1);
    adamw_math(a, i0, base, sc_scale, sc_div, c, q0);
    adamw_store<FRESH, SHADOW>(a, i0, q0);
    if (has1) {
      adamw_math(a, i1, base, sc_scale, sc_div, c, q1);
      adamw_store<FRESH, SHADOW>(a, i1, q1);
    }
  }
}

// Index of the matrix owning tile t: the last k with mats[k].tile0 <= t.
__device__ __forceinline__ int find_mat(const MuonMat* mats, int nmat, int t) {
  int lo = 0, hi = nmat - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (mats[mid].tile0 <= t)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

constexpr int kTile = 64;  // Muon elementwise kernels work on 64 x 64 tiles

__device__ __forceinline__ float block_sum_256(float x, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, o));
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = x;
  __syncthreads();
  float r = 0.0f;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) r = __fadd_rn(r, red[i]);
  }
  __syncthreads();
  return r;
}

// Round to tf32 (10 leading mantissa bits), to nearest with ties to even on
// the 13 discarded bits; Inf and NaN pass through.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
  return __uint_as_float(u);
}

// How the Newton-Schulz input X is stored (MuonArgs::x_mode): 0 bf16(u), the
// rounding of lib.rs:104; 1 tf32(u) in fp32 words (TF32 mode); 2 u itself as
// two tf32 planes, hi = tf32(u) at item 2b and lo = tf32(u - hi) at item
// 2b + 1 (fp32 mode). x_value() is the value the norm and the iteration see.
template <int XM>
__device__ __forceinline__ float x_value(float u) {
  if constexpr (XM == 0)
    return __bfloat162float(__float2bfloat16_rn(u));
  else if constexpr (XM == 1)
    return tf32_round(u);
  else
    return u;
}

// Stores 4 consecutive X values y (already x_value) at element i of the
// matrix item(s) starting at X; plane_stride separates the split planes.
template <int XM>
__device__ __forceinline__ void x_store4(void* X, long long i, long long plane_stride,
                                         const float (&y)[4]) {
  if constexpr (XM == 0) {
    uint2 o;
    __nv_bfloat162 h0 = __floats2bfloat162_rn(y[0], y[1]);
    __nv_bfloat162 h1 = __floats2bfloat162_rn(y[2], y[3]);
    o.x = *reinterpret_cast<uint32_t*>(&h0);
    o.y = *reinterpret_cast<uint32_t*>(&h1);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(X) + i) = o;
  } else if constexpr (XM == 1) {
    *reinterpret_cast<float4*>(static_cast<float*>(X) + i) = make_float4(y[0], y[1], y[2], y[3]);
  } else {
    float hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      hi[e] = tf32_round(y[e]);
      lo[e] = tf32_round(__fsub_rn(y[e], hi[e]));
    }
    float* xf = static_cast<float*>(X) + i;
    *reinterpret_cast<float4*>(xf) = make_float4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<float4*>(xf + plane_stride) = make_float4(lo[0], lo[1], lo[2], lo[3]);
  }
}

template <int XM>
__device__ __forceinline__ void x_store1(void* X, long long i, long long plane_stride, float y) {
  if constexpr (XM == 0) {
    static_cast<__nv_bfloat16*>(X)[i] = __float2bfloat16_rn(y);
  } else if constexpr (XM == 1) {
    static_cast<float*>(X)[i] = y;
  } else {
    const float hi = tf32_round(y);
    static_cast<float*>(X)[i] = hi;
    static_cast<float*>(X)[i + plane_stride] = tf32_round(__fsub_rn(y, hi));
  }
}

template <int XM>
__device__ __forceinline__ float x_load1(const void* X, long long i, long long plane_stride) {
  if constexpr (XM == 0)
    return __bfloat162float(static_cast<const __nv_bfloat16*>(X)[i]);
  else if constexpr (XM == 1)
    return static_cast<const float*>(X)[i];
  else
    return __fadd_rn(static_cast<const float*>(X)[i], static_cast<const float*>(X)[i + plane_stride]);
}

// The first X element of a matrix: item xbatch (2 * xbatch with split planes).
template <int XM>
__device__ __forceinline__ void* x_matrix(const MuonClassPtr& cp, int xbatch) {
  if constexpr (XM == 0)
    return static_cast<__nv_bfloat16*>(cp.x) + (long long)xbatch * cp.bstride;
  else
    return static_cast<float*>(cp.x) + (long long)xbatch * (XM == 2 ? 2 : 1) * cp.bstride;
}

// Momentum arithmetic of lib.rs:154-165 for one element; returns x_value(u).
template <int XM>
__device__ __forceinline__ float momentum_elem(float g, float& vel, float mu, float one_m,
                                               int nesterov) {
  const float v1 = __fadd_rn(__fmul_rn(mu, vel), __fmul_rn(one_m, g));
  vel = v1;
  const float u = nesterov ? __fadd_rn(__fmul_rn(g, one_m), __fmul_rn(v1, mu)) : v1;
  return x_value<XM>(u);
}

// 128-bit variant of one 64 x 64 momentum tile: thread t covers 4 consecutive
// columns; a transposed X is written through `tile` in groups of 4 rows.
template <bool BF16G, bool FRESH, int XM>
__device__ __forceinline__ float momentum_tile_vec(const MuonArgs& a, const MuonMat& mm, int r0,
                                                   int c0, void* Xv, int ld, long long pstride,
                                                   float (*tile)[kTile + 1], float scale,
                                                   float mu, float one_m) {
  const int cq = (threadIdx.x & 15) * 4;
  const int rs = threadIdx.x >> 4;
  constexpr int kRounds = kTile / 16;  // rows rs, rs + 16, rs + 32, rs + 48
  // All of the thread's loads are issued before any store, so that 8 x 16 B
  // (fp32 grads) per thread are in flight at once.
  float g[kRounds][4];
  float vv[kRounds][4];
  bool ok[kRounds];
#pragma unroll
  for (int q = 0; q < kRounds; ++q) {
    const int r = r0 + rs + 16 * q, c = c0 + cq;
    ok[q] = r < mm.rows && c < mm.cols;
    const long long idx = mm.off + (long long)r * mm.cols + c;
    if (ok[q]) {
      if (BF16G) {
        const uint2 raw = *reinterpret_cast<const uint2*>(a.g_bf16 + idx);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
        const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
        g[q][0] = f0.x;
        g[q][1] = f0.y;
        g[q][2] = f1.x;
        g[q][3] = f1.y;
      } else {
        const float4 g4 = __ldcs(reinterpret_cast<const float4*>(a.g + idx));
        g[q][0] = g4.x;
        g[q][1] = g4.y;
        g[q][2] = g4.z;
        g[q][3] = g4.w;
      }
      const float4 v4 = FRESH ? make_float4(0.f, 0.f, 0.f, 0.f)
                              : __ldcs(reinterpret_cast<const float4*>(a.vel + idx));
      vv[q][0] = v4.x;
      vv[q][1] = v4.y;
      vv[q][2] = v4.z;
      vv[q][3] = v4.w;
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int q = 0; q < kRounds; ++q) {
    const int rr = rs + 16 * q;
    const int r = r0 + rr, c = c0 + cq;
    float y[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (ok[q]) {
      const long long idx = mm.off + (long long)r * mm.cols + c;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float ge = g[q][e];
        if (scale != 1.0f) ge = __fdiv_rn(ge, scale);
        if (a.grad_divisor != 1.0f) ge = __fdiv_rn(ge, a.grad_divisor);
        y[e] = momentum_elem<XM>(ge, vv[q][e], mu, one_m, a.nesterov);
      }
      __stcs(reinterpret_cast<float4*>(a.vel + idx),
             make_float4(vv[q][0], vv[q][1], vv[q][2], vv[q][3]));
      if (!mm.transposed) x_store4<XM>(Xv, (long long)r * ld + c, pstride, y);
    }
    if (mm.transposed) {
#pragma unroll
      for (int e = 0; e < 4; ++e) tile[rr][cq + e] = y[e];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) ss = __fadd_rn(ss, __fmul_rn(y[e], y[e]));
  }
  if (mm.transposed) {
    __syncthreads();
    // X row c = c0 + cl holds u[r0 .. r0+63][c]; thread writes 4 consecutive r.
    const int rq = (threadIdx.x & 15) * 4;
    for (int cl = rs; cl < kTile; cl += 16) {
      const int c = c0 + cl, r = r0 + rq;
      if (c < mm.cols && r < mm.rows) {
        const long long i = (long long)c * ld + r;
        if (r + 3 < mm.rows) {
          const float y4[4] = {tile[rq][cl], tile[rq + 1][cl], tile[rq + 2][cl], tile[rq + 3][cl]};
          x_store4<XM>(Xv, i, pstride, y4);
        } else {
          for (int e = 0; e < 4 && r + e < mm.rows; ++e)
            x_store1<XM>(Xv, i + e, pstride, tile[rq + e][cl]);
        }
      }
    }
  }
  return ss;
}

// Muon momentum (lib.rs:154-165) + the bf16 cast and orientation of
// newton_schulz5 (lib.rs:101-107) + per-tile sums of squares of the bf16
// values (lib.rs:109), all in one pass over g and vel. XM selects the X
// storage of the TF32 and fp32 modes instead of bf16 (x_value).
// Four 256-thread blocks per SM (at most 64 registers a thread, 16.6 KB of
// shared memory a block), launched as one wave that strides over the tiles.
constexpr int kMomentumBlocksPerSm = 4;
template <bool BF16G, bool FRESH, int XM>
__global__ void __launch_bounds__(256, kMomentumBlocksPerSm) muon_momentum_kernel(const MuonArgs a) {
  __shared__ float tile[kTile][kTile + 1];
  __shared__ float red[8];
  if (a.skip && *a.skip) return;
  const float scale = a.grad_scale ? *a.grad_scale : 1.0f;
  const float mu = a.momentum;
  const float one_m = __fsub_rn(1.0f, mu);
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  for (int t = a.tile_begin + blockIdx.x; t < a.tile_begin + a.total_tiles; t += gridDim.x) {
    const int k = find_mat(a.mats, a.nmat, t);
    const MuonMat mm = a.mats[k];
    const int tiles_c = (mm.cols + kTile - 1) / kTile;
    const int lt = t - mm.tile0;
    const int r0 = (lt / tiles_c) * kTile, c0 = (lt % tiles_c) * kTile;
    const MuonClassPtr cp = a.cls[mm.xcls];
    void* Xv = x_matrix<XM>(cp, mm.xbatch);
    if (a.vec_ok && (mm.cols & 3) == 0 && (mm.off & 3) == 0) {
      const float ssv = momentum_tile_vec<BF16G, FRESH, XM>(a, mm, r0, c0, Xv, cp.ld, cp.bstride,
                                                            tile, scale, mu, one_m);
      if constexpr (XM != 0) {
        const float totv = block_sum_256(ssv, red);
        if (threadIdx.x == 0) a.partials[t] = totv;
      } else if (mm.transposed) {
        __syncthreads();  // the next tile may overwrite `tile`
      }
      continue;
    }
    float ss = 0.0f;
    for (int rr = ty; rr < kTile; rr += 4) {
      const int r = r0 + rr, c = c0 + tx;
      float y = 0.0f;
      if (r < mm.rows && c < mm.cols) {
        const long long idx = mm.off + (long long)r * mm.cols + c;
        float g = load_grad(a.g, a.g_bf16, idx);
        if (scale != 1.0f) g = __fdiv_rn(g, scale);
        if (a.grad_divisor != 1.0f) g = __fdiv_rn(g, a.grad_divisor);
        const float v0 = FRESH ? 0.0f : a.vel[idx];
        const float v1 = __fadd_rn(__fmul_rn(mu, v0), __fmul_rn(one_m, g));
        a.vel[idx] = v1;
        const float u = a.nesterov ? __fadd_rn(__fmul_rn(g, one_m), __fmul_rn(v1, mu)) : v1;
        y = x_value<XM>(u);
        if (!mm.transposed) x_store1<XM>(Xv, (long long)r * cp.ld + c, cp.bstride, y);
      }
      if (mm.transposed) tile[rr][tx] = y;
      ss = __fadd_rn(ss, __fmul_rn(y, y));
    }
    if (mm.transposed) {
      __syncthreads();
      // X[c][r] = tile[r - r0][c - c0]; consecutive threads write consecutive r.
      for (int cc = ty; cc < kTile; cc += 4) {
        const int c = c0 + cc, r = r0 + tx;
        if (c < mm.cols && r < mm.rows)
          x_store1<XM>(Xv, (long long)c * cp.ld + r, cp.bstride, tile[tx][cc]);
      }
    }
    if constexpr (XM != 0) {
      const float tot = block_sum_256(ss, red);
      if (threadIdx.x == 0) a.partials[t] = tot;
    } else if (mm.transposed) {
      __syncthreads();  // the next tile may overwrite `tile`
    }
  }
}

// Deterministic per-matrix total of the tile partials: norm = max(sqrt(sum), 1e-7).
__global__ void __launch_bounds__(256) muon_norm_kernel(const MuonArgs a) {
  __shared__ float red[8];
  if (a.skip && *a.skip) return;
  for (int k = blockIdx.x; k < a.nmat; k += gridDim.x) {
    const MuonMat mm = a.mats[k];
    const int ntiles = ((mm.rows + kTile - 1) / kTile) * ((mm.cols + kTile - 1) / kTile);
    float s = 0.0f;
    for (int i = threadIdx.x; i < ntiles; i += 256) s = __fadd_rn(s, a.partials[mm.tile0 + i]);
    const float tot = block_sum_256(s, red);
    if (threadIdx.x == 0) a.norms[mm.norm_idx] = fmaxf(__fsqrt_rn(tot), 1e-7f);
  }
}

// Muon::step_matrix tail (lib.rs:169-174): p -= (lr*scale) * O, O read back in
// the parameter's orientation from the final Newton-Schulz X.
template <bool SHADOW, int XM>
__global__ void __launch_bounds__(256) muon_apply_kernel(const MuonArgs a) {
  __shared__ float tile[kTile][kTile + 1];
  if (a.skip && *a.skip) return;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  for (int t = a.tile_begin + blockIdx.x; t < a.tile_begin + a.total_tiles; t += gridDim.x) {
    const int k = find_mat(a.mats, a.nmat, t);
    const MuonMat mm = a.mats[k];
    const int tiles_c = (mm.cols + kTile - 1) / kTile;
    const int lt = t - mm.tile0;
    const int r0 = (lt / tiles_c) * kTile, c0 = (lt % tiles_c) * kTile;
    const MuonClassPtr cp = a.cls[mm.xcls];
    const void* X = x_matrix<XM>(cp, mm.xbatch);
    if (mm.transposed) {
      __syncthreads();
      for (int cc = ty; cc < kTile; cc += 4) {
        const int c = c0 + cc, r = r0 + tx;
        tile[cc][tx] = (c < mm.cols && r < mm.rows)
                           ? x_load1<XM>(X, (long long)c * cp.ld + r, cp.bstride)
                           : 0.0f;
      }
      __syncthreads();
    }
    for (int rr = ty; rr < kTile; rr += 4) {
      const int r = r0 + rr, c = c0 + tx;
      if (r < mm.rows && c < mm.cols) {
        const long long idx = mm.off + (long long)r * mm.cols + c;
        float o = mm.transposed ? tile[tx][rr] : x_load1<XM>(X, (long long)r * cp.ld + c, cp.bstride);
        if (a.apply_divides_norm) o = __fdiv_rn(o, a.norms[mm.norm_idx]);
        const float pn = __fsub_rn(a.p[idx], __fmul_rn(mm.lr_scale, o));
        a.p[idx] = pn;
        if (SHADOW) a.p_bf16[idx] = __float2bfloat16_rn(pn);
      }
    }
  }
}

__device__ __forceinline__ bool nonfinite_bits(uint32_t u) {
  return (u & 0x7F800000u) == 0x7F800000u;
}

// This thread's share of a non-finite scan of g32[0, n32) and g16[0, n16).
__device__ __forceinline__ bool scan_nonfinite(const float* g32, long long n32,
                                               const __nv_bfloat16* g16, long long n16) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  bool bad = false;
  if (g32) {
    const long long n4 = n32 / 4;
    const float4* p = reinterpret_cast<const float4*>(g32);
    for (long long i = tid; i < n4; i += stride) {
      const float4 x = __ldcs(p + i);
      bad |= nonfinite_bits(__float_as_uint(x.x)) | nonfinite_bits(__float_as_uint(x.y)) |
             nonfinite_bits(__float_as_uint(x.z)) | nonfinite_bits(__float_as_uint(x.w));
    }
    for (long long i = n4 * 4 + tid; i < n32; i += stride) bad |= nonfinite_bits(__float_as_uint(g32[i]));
  }
  if (g16) {
    const long long n8 = n16 / 8;
    const uint4* p = reinterpret_cast<const uint4*>(g16);
    for (long long i = tid; i < n8; i += stride) {
      const uint4 x = __ldcs(p + i);
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        bad |= ((w[e] & 0x7F80u) == 0x7F80u) | ((w[e] & 0x7F800000u) == 0x7F800000u);
    }
    for (long long i = n8 * 8 + tid; i < n16; i += stride) {
      const uint32_t u = (uint32_t)__bfloat16_as_ushort(g16[i]) << 16;
      bad |= nonfinite_bits(u);
    }
  }
  return bad;
}

__global__ void __launch_bounds__(256) nonfinite_kernel(const float* g32, long long n32,
                                                        const __nv_bfloat16* g16, long long n16,
                                                        int* flag) {
  const bool bad = scan_nonfinite(g32, n32, g16, n16);
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1);
}

// The scan of one rank's part, its verdict stored into every rank's flag.
__global__ void __launch_bounds__(256) nonfinite_ranks_kernel(const float* g32, long long n32,
                                                              const __nv_bfloat16* g16,
                                                              long long n16, const RankFlags f) {
  const bool bad = scan_nonfinite(g32, n32, g16, n16);
  if (__syncthreads_or(bad) && threadIdx.x == 0) {
    for (int r = 0; r < f.n; ++r) *(volatile int*)f.flag[r] = 1;
    __threadfence_system();
  }
}

// fp32: four elements per vector; every rank's vector is loaded before the
// rank-ordered sum, so the NVLink loads of one thread are in flight together.
template <int W>
__global__ void __launch_bounds__(256) grad_reduce_f32_kernel(const GradReduceArgs a) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long b4 = a.begin / 4, e4 = a.end / 4;
  bool bad = false;
  float4* dst = reinterpret_cast<float4*>(a.dst);
  for (long long i = b4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < e4; i += stride) {
    float4 v[W];
#pragma unroll
    for (int r = 0; r < W; ++r) v[r] = __ldcs(reinterpret_cast<const float4*>(a.src[r]) + i);
    float4 s = v[0];
#pragma unroll
    for (int r = 1; r < W; ++r) {
      s.x = __fadd_rn(s.x, v[r].x);
      s.y = __fadd_rn(s.y, v[r].y);
      s.z = __fadd_rn(s.z, v[r].z);
      s.w = __fadd_rn(s.w, v[r].w);
    }
    bad |= nonfinite_bits(__float_as_uint(s.x)) | nonfinite_bits(__float_as_uint(s.y)) |
           nonfinite_bits(__float_as_uint(s.z)) | nonfinite_bits(__float_as_uint(s.w));
    dst[i] = s;
  }
  // scalar tail (end not a multiple of 4)
  for (long long i = e4 * 4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < a.end;
       i += stride) {
    float s = reinterpret_cast<const float*>(a.src[0])[i];
    for (int r = 1; r < W; ++r) s = __fadd_rn(s, reinterpret_cast<const float*>(a.src[r])[i]);
    bad |= nonfinite_bits(__float_as_uint(s));
    reinterpret_cast<float*>(a.dst)[i] = s;
  }
  if (__syncthreads_or(bad) && a.scan && threadIdx.x == 0) {
    for (int r = 0; r < a.world; ++r) *(volatile int*)a.skip_flags[r] = 1;
    __threadfence_system();
  }
}

// bf16: eight elements per vector, summed in fp32, rounded once.
template <int W>
__global__ void __launch_bounds__(256) grad_reduce_bf16_kernel(const GradReduceArgs a) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long b8 = a.begin / 8, e8 = a.end / 8;
  bool bad = false;
  uint4* dst = reinterpret_cast<uint4*>(a.dst);
  for (long long i = b8 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < e8; i += stride) {
    uint4 v[W];
#pragma unroll
    for (int r = 0; r < W; ++r) v[r] = __ldcs(reinterpret_cast<const uint4*>(a.src[r]) + i);
    float s[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&v[0])[e]);
      s[2 * e] = f.x;
      s[2 * e + 1] = f.y;
    }
#pragma unroll
    for (int r = 1; r < W; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&v[r])[e]);
        s[2 * e] = __fadd_rn(s[2 * e], f.x);
        s[2 * e + 1] = __fadd_rn(s[2 * e + 1], f.y);
      }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 h = __floats2bfloat162_rn(s[2 * e], s[2 * e + 1]);
      ow[e] = *reinterpret_cast<uint32_t*>(&h);
      bad |= ((ow[e] & 0x7F80u) == 0x7F80u) | ((ow[e] & 0x7F800000u) == 0x7F800000u);
    }
    dst[i] = o;
  }
  for (long long i = e8 * 8 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < a.end;
       i += stride) {
    float s = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.src[0])[i]);
    for (int r = 1; r < W; ++r)
      s = __fadd_rn(s, __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.src[r])[i]));
    const __nv_bfloat16 h = __float2bfloat16_rn(s);
    bad |= nonfinite_bits((uint32_t)__bfloat16_as_ushort(h) << 16);
    reinterpret_cast<__nv_bfloat16*>(a.dst)[i] = h;
  }
  if (__syncthreads_or(bad) && a.scan && threadIdx.x == 0) {
    for (int r = 0; r < a.world; ++r) *(volatile int*)a.skip_flags[r] = 1;
    __threadfence_system();
  }
}

__global__ void step_tail_kernel(const StepTail t) {
  const bool skipped = t.skip && *t.skip;
  if (!skipped) *t.step_counter += t.adamw_calls;
  if (skipped && t.skipped_total) *t.skipped_total += 1;
  if (t.grad_scale) {
    if (skipped) {
      *t.grad_scale = *t.grad_scale * 0.5f;
      *t.good_steps = 0;
    } else if (++*t.good_steps >= t.growth_interval) {
      *t.grad_scale = *t.grad_scale * 2.0f;
      *t.good_steps = 0;
    }
  }
  if (t.reset_skip && t.skip) *t.skip = 0;
}

int grid_for(long long work_items, int threads, int num_sms, int per_sm) {
  long long blocks = (work_items + threads - 1) / threads;
  const long long cap = (long long)num_sms * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

}  // namespace

void launch_adamw(const AdamwArgs& a, int num_sms, cudaStream_t stream) {
  if (a.end4 <= a.begin4) return;
  const int grid = grid_for(a.end4 - a.begin4, 256, num_sms, 8);
  const bool bf = a.g_bf16 != nullptr, fresh = a.fresh_state != 0, sh = a.p_bf16 != nullptr;
#define MMN_ADAMW(B, F, S) \
  if (bf == B && fresh == F && sh == S) adamw_kernel<B, F, S><<<grid, 256, 0, stream>>>(a);
  MMN_ADAMW(false, false, false)
  MMN_ADAMW(false, false, true)
  MMN_ADAMW(false, true, false)
  MMN_ADAMW(false, true, true)
  MMN_ADAMW(true, false, false)
  MMN_ADAMW(true, false, true)
  MMN_ADAMW(true, true, false)
  MMN_ADAMW(true, true, true)
#undef MMN_ADAMW
}

void launch_muon_momentum(const MuonArgs& a, int num_sms, cudaStream_t stream) {
  if (a.total_tiles <= 0) return;
  const int grid = grid_for(a.total_tiles, 1, num_sms, kMomentumBlocksPerSm);
  const bool bf = a.g_bf16 != nullptr, fresh = a.fresh_state != 0;
#define MMN_MOM(XM)                                                                  \
  if (bf && fresh) muon_momentum_kernel<true, true, XM><<<grid, 256, 0, stream>>>(a);   \
  if (bf && !fresh) muon_momentum_kernel<true, false, XM><<<grid, 256, 0, stream>>>(a); \
  if (!bf && fresh) muon_momentum_kernel<false, true, XM><<<grid, 256, 0, stream>>>(a); \
  if (!bf && !fresh) muon_momentum_kernel<false, false, XM><<<grid, 256, 0, stream>>>(a);
  if (a.x_mode == 2) {
    MMN_MOM(2)
  } else if (a.x_mode == 1) {
    MMN_MOM(1)
  } else {
    MMN_MOM(0)
  }
#undef MMN_MOM
}

void launch_muon_norms(const MuonArgs& a, cudaStream_t stream, int cluster) {
  if (a.nmat <= 0) return;
  if (a.x_mode == 0) {
    launch_ref_norms(a, cluster, stream);
    return;
  }
  muon_norm_kernel<<<a.nmat < 1024 ? a.nmat : 1024, 256, 0, stream>>>(a);
}

void launch_muon_apply(const MuonArgs& a, int num_sms, cudaStream_t stream) {
  if (a.total_tiles <= 0) return;
  const int grid = grid_for(a.total_tiles, 1, num_sms, 8);
#define MMN_APPLY(XM)                                                   \
  if (a.p_bf16)                                                         \
    muon_apply_kernel<true, XM><<<grid, 256, 0, stream>>>(a);           \
  else                                                                  \
    muon_apply_kernel<false, XM><<<grid, 256, 0, stream>>>(a);
  if (a.x_mode == 2) {
    MMN_APPLY(2)
  } else if (a.x_mode == 1) {
    MMN_APPLY(1)
  } else {
    MMN_APPLY(0)
  }
#undef MMN_APPLY
}

void launch_grad_reduce(const GradReduceArgs& a, int num_sms, cudaStream_t stream) {
  if (a.end <= a.begin || a.world < 2 || a.world > kMaxRanks) return;
  const long long vecs = (a.end - a.begin) / (a.bf16 ? 8 : 4) + 1;
  const int grid = grid_for(vecs, 256, num_sms, 8);
#define MMN_GR(W)                                                                 \
  case W:                                                                         \
    if (a.bf16)                                                                   \
      grad_reduce_bf16_kernel<W><<<grid, 256, 0, stream>>>(a);                    \
    else                                                                          \
      grad_reduce_f32_kernel<W><<<grid, 256, 0, stream>>>(a);                     \
    break;
  switch (a.world) {
    MMN_GR(2)
    MMN_GR(3)
    MMN_GR(4)
    MMN_GR(5)
    MMN_GR(6)
    MMN_GR(7)
    MMN_GR(8)
  }
#undef MMN_GR
}

void launch_nonfinite_scan(const float* g32, long long n32, const __nv_bfloat16* g16,
                           long long n16, int* flag, int num_sms, cudaStream_t stream) {
  const long long work = (n32 / 4 > n16 / 8 ? n32 / 4 : n16 / 8) + 1;
  nonfinite_kernel<<<grid_for(work, 256, num_sms, 8), 256, 0, stream>>>(g32, n32, g16, n16, flag);
}

void launch_nonfinite_scan_ranks(const float* g32, long long n32, const __nv_bfloat16* g16,
                                 long long n16, const RankFlags& f, int num_sms,
                                 cudaStream_t stream) {
  if (f.n < 1 || f.n > kMaxRanks || (n32 <= 0 && n16 <= 0)) return;
  const long long work = (n32 / 4 > n16 / 8 ? n32 / 4 : n16 / 8) + 1;
  nonfinite_ranks_kernel<<<grid_for(work, 256, num_sms, 8), 256, 0, stream>>>(g32, n32, g16, n16,
                                                                              f);
}

void launch_step_tail(const StepTail& t, cudaStream_t stream) {
  step_tail_kernel<<<1, 1, 0, stream>>>(t);
}

}  // namespace mmn
