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
//            (bf16 mode: X' = bf16((X/s)*a + (Bm X)/s), one accumulator)
//
// s is the per-matrix Frobenius norm in the first iteration (lib.rs:109-110)
// and 1 afterwards. All operand values are exactly bf16, so the tensor-core
// products are exact and only the fp32 summation order differs from the CPU.
//
// Roles (192 threads): warp 0 issues TMA loads, warp 1 owns TMEM and one lane
// issues tcgen05.mma, warps 2-5 drain TMEM and run the fused epilogue. Every
// mbarrier wait is time-bounded; on timeout the kernel records a status,
// drains what it issued, frees TMEM and returns.
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
};

constexpr int kBM = 128;  // tile rows (TMEM lanes)
constexpr int kBK = 64;   // K per stage: one 128-byte swizzle row of bf16

struct NsGemmArgs {
  __nv_bfloat16* out;        // output matrices (bf16)
  long long out_bstride;     // elements between batch items
  int out_ld;                // elements between rows
  const __nv_bfloat16* aux;  // epilogue input: X (Poly) or A (SquareBf16)
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
};

template <int BN, bool DUAL, bool B_MN>
struct NsGemmShape {
  static constexpr int kABytes = kBM * kBK * 2;             // 16 KB
  static constexpr int kBBytes = BN * kBK * 2;              // BN*128 B
  static constexpr int kStageBytes = kABytes * (DUAL ? 2 : 1) + kBBytes;
  static constexpr int kStages = (196608 / kStageBytes) < 8 ? (196608 / kStageBytes) : 8;
  static constexpr int kAccCols = BN * (DUAL ? 2 : 1);      // per accumulator buffer
  static constexpr int kTmemCols = 2 * kAccCols;            // double-buffered
  static constexpr int kBarBytes = 1024;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;  // +align slack
  static_assert(kTmemCols <= 512, "TMEM has 512 columns");
  static_assert(kStages >= 2, "pipeline needs two stages");
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int BN, bool DUAL, bool B_MN, int EPI>
__global__ void __launch_bounds__(192, 1)
    ns_gemm_kernel(const __grid_constant__ CUtensorMap tm_a1,
                   const __grid_constant__ CUtensorMap tm_a2,
                   const __grid_constant__ CUtensorMap tm_b, const NsGemmArgs args) {
  using S = NsGemmShape<BN, DUAL, B_MN>;
  constexpr int STAGES = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* full = bars;                  // [STAGES] TMA -> MMA
  uint64_t* empty = bars + STAGES;        // [STAGES] MMA -> TMA
  uint64_t* tfull = bars + 2 * STAGES;    // [2] MMA -> epilogue
  uint64_t* tempty = bars + 2 * STAGES + 2;  // [2] epilogue -> MMA
  uint64_t* drain = bars + 2 * STAGES + 4;   // abort path: MMA completion
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 6);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a1);
    if (DUAL) tma_prefetch_desc(&tm_a2);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
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
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
        int b, tm, tn;
        decode(tile, b, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = tiles + stage * S::kStageBytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          const int k0 = kb * kBK;
          tma_load_3d(st, &tm_a1, &full[stage], k0, tm * kBM, b);
          if (DUAL) tma_load_3d(st + S::kABytes, &tm_a2, &full[stage], k0, tm * kBM, b);
          uint8_t* sb = st + S::kABytes * (DUAL ? 2 : 1);
          if (B_MN) {
#pragma unroll
            for (int g = 0; g < BN / 64; ++g)
              tma_load_3d(sb + g * (kBK * 128), &tm_b, &full[stage], tn * BN + g * 64, k0, b);
          } else {
            tma_load_3d(sb, &tm_b, &full[stage], k0, tn * BN, b);
          }
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every load this thread issued must land before the CTA may exit.
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
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN, false, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
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
          const uint32_t a2 = a1 + S::kABytes;
          const uint32_t bb = a1 + S::kABytes * (DUAL ? 2 : 1);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t da1 = umma_desc_sw128(a1 + kk * 32, 16, 1024);
            const uint64_t db = B_MN ? umma_desc_sw128(bb + kk * 2048, kBK * 128, 1024)
                                     : umma_desc_sw128(bb + kk * 32, 16, 1024);
            const uint32_t accum = (kb | kk) != 0;
            tc_mma_bf16(d1, da1, db, idesc, accum);
            if (DUAL) {
              const uint64_t da2 = umma_desc_sw128(a2 + kk * 32, 16, 1024);
              tc_mma_bf16(d2, da2, db, idesc, accum);
            }
          }
          issued_any = true;
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (*abort_flag && issued_any) {
        // Let every MMA this thread issued finish before TMEM is freed.
        tc_commit(drain);
        uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (global_timer_ns() - t0 > kWaitLimitNs) break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x) {
      int b, tm, tn;
      decode(tile, b, tm, tn);
      // tcgen05.ld is warp-collective: the warp proceeds only if every lane saw
      // the accumulator become ready.
      const bool ready = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int r = tm * kBM + sub * 32 + lane;
      const uint32_t tbase = tmem_base + acc * S::kAccCols + ((uint32_t)(sub * 32) << 16);
      const float s = args.norms ? args.norms[b] : 1.0f;
      __nv_bfloat16* out = args.out + (long long)b * args.out_bstride;
      const __nv_bfloat16* aux = args.aux ? args.aux + (long long)b * args.aux_bstride : nullptr;
      const bool row_ok = r < args.M;
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        const int c0 = tn * BN + ch * 32;
        float v[32];
        tmem_ld_32x32b_x32(tbase + ch * 32, v);
        float w[32];
        if (DUAL) tmem_ld_32x32b_x32(tbase + BN + ch * 32, w);
        tmem_ld_wait();
        if (EPI == kEpiGram || EPI == kEpiSquare || EPI == kEpiSquareBf16) {
          // Symmetric output: this tile owns the elements with col >= row and
          // writes each one twice, at (r, c) and at (c, r).
          float a_in[32];
          if (EPI == kEpiSquareBf16) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int c = c0 + j;
              a_in[j] = (row_ok && c < args.N)
                            ? __bfloat162float(aux[(long long)r * args.aux_ld + c])
                            : 0.0f;
            }
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = v[j];
            if (EPI == kEpiGram) x = __fdiv_rn(__fdiv_rn(x, s), s);
            if (EPI == kEpiSquareBf16) {
              const float sq = __bfloat162float(__float2bfloat16_rn(x));
              x = __fadd_rn(__fmul_rn(a_in[j], args.coef_b), __fmul_rn(sq, args.coef_c));
            }
            v[j] = x;
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int c = c0 + j;
            if (row_ok && c < args.N && c >= r) {
              const __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
              out[(long long)r * args.out_ld + c] = h;
              out[(long long)c * args.out_ld + r] = h;
            }
          }
        } else {
          // Poly: X' = bf16((X/s)*a + (b*D1 + c*D2)/s)  or  bf16((X/s)*a + D/s).
          const __nv_bfloat16* xrow = aux + (long long)r * args.aux_ld + c0;
          __nv_bfloat16* orow = out + (long long)r * args.out_ld + c0;
          const bool full_chunk = row_ok && (c0 + 32 <= args.N);
          float xv[32];
          if (full_chunk) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 u = *reinterpret_cast<const uint4*>(xrow + q * 8);
              const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(h[e]);
                xv[q * 8 + e * 2] = f.x;
                xv[q * 8 + e * 2 + 1] = f.y;
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              xv[j] = (row_ok && c0 + j < args.N) ? __bfloat162float(xrow[j]) : 0.0f;
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float bx = DUAL ? __fadd_rn(__fmul_rn(args.coef_b, v[j]), __fmul_rn(args.coef_c, w[j]))
                            : v[j];
            const float x0 = __fdiv_rn(xv[j], s);
            v[j] = __fadd_rn(__fmul_rn(x0, args.coef_a), __fdiv_rn(bx, s));
          }
          if (full_chunk) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 u;
              u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
              u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
              u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
              u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
              *reinterpret_cast<uint4*>(orow + q * 8) = u;
            }
          } else if (row_ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (c0 + j < args.N) orow[j] = __float2bfloat16_rn(v[j]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) atomicExch(args.status, kDevWaitTimeout);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace mmn
