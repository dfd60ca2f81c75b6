// Memory-bound kernels of the optimizer step (sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mmn {

// One tensor of the flat AdamW arena, in float4 units. Segments tile the arena
// contiguously: seg[k].end4 == seg[k+1].start4.
struct AdamwSeg {
  long long start4;
  long long end4;
  int t_offset;  // 1-based position of this tensor among one step's AdamW calls
  int pad;
};

struct AdamwArgs {
  float* p;                   // fp32 params (master copy)
  const float* g;             // fp32 grads, or nullptr when g_bf16 is used
  const __nv_bfloat16* g_bf16;
  float* m;
  float* v;
  __nv_bfloat16* p_bf16;      // optional bf16 shadow of p
  const AdamwSeg* segs;       // device table, or nullptr to use seg0
  AdamwSeg seg0;              // the single segment when segs is nullptr
  const int* chunk_seg;       // first segment of every chunk of kAdamwChunk4 float4s
  long long begin4, end4;     // float4 range of the arena this launch steps
  const float2* bc_table;     // (1 - b1^t, 1 - b2^t) for t = 0 .. t_sat
  int t_sat;                  // t >= t_sat uses bc_table[t_sat] (both exactly 1)
  const long long* step_base; // device AdamW call counter before this step, or
  long long step_base_value;  // the counter by value when step_base is nullptr
  const int* skip;            // non-finite flag (nullptr = never skip)
  const float* grad_scale;    // device loss scale (nullptr = 1)
  float lr, b1, b2, eps, wd;
  float grad_divisor;         // GradAccumulator averaging divisor (1 = none)
  int fresh_state;            // m and v read as zero and not stored
};

constexpr long long kAdamwChunk4 = 2048;  // float4 per chunk-table entry

void launch_adamw(const AdamwArgs& a, int num_sms, cudaStream_t stream);

// One Muon matrix (rows x cols fp32, row-major) and where its NS input lives.
struct MuonMat {
  long long off;          // element offset of p / g / vel in the Muon arena
  int rows, cols;
  int transposed;         // rows > cols: X holds the transpose
  int xcls;               // shape-class index (selects x_base / x_bstride)
  int xbatch;             // index inside the class batch
  int tile0;              // first 64x64 tile index of this matrix (prefix sum)
  float lr_scale;         // lr * sqrt(rows / cols), computed in f32 on the host
  int norm_idx;           // slot of this matrix's norm in MuonArgs::norms
};

struct MuonClassPtr {
  void* x;            // class X buffer (items x n x ld): bf16, or fp32 when x_mode > 0
  long long bstride;  // elements between items (x_mode 2: two items, hi and lo, per matrix)
  int ld;
  int pad;
};

struct MuonArgs {
  float* p;
  const float* g;
  const __nv_bfloat16* g_bf16;
  float* vel;
  __nv_bfloat16* p_bf16;
  const MuonMat* mats;   // the matrices of this launch (a contiguous run of the table)
  int nmat;
  int tile_begin;        // mats[0].tile0: the launch covers tiles
  int total_tiles;       // [tile_begin, tile_begin + total_tiles)
  const MuonClassPtr* cls;
  float* partials;      // one fp32 sum of squares per tile (x_mode 1 and 2)
  float* norms;         // clamped Frobenius norms, slot mats[k].norm_idx
  const int* skip;
  const float* grad_scale;
  float momentum;
  int nesterov;
  float grad_divisor;
  int fresh_state;      // velocity read as zero
  int apply_divides_norm;  // zero Newton-Schulz steps: O = bf16(u) / norm (lib.rs:110)
  int vec_ok;              // p / g / vel bases are 16-byte aligned: matrices with
                           // cols % 4 == 0 and off % 4 == 0 take the 128-bit path
  int norm_scalar_rows;    // some matrix has oriented rows that are not a multiple of
                           // 8 elements (the norm launch adds its element-wise form)
  int x_mode;              // X storage: 0 bf16(u); 1 tf32(u) in fp32 words (TF32
                           // mode); 2 u as hi + lo tf32 planes (fp32 mode)
};

void launch_muon_momentum(const MuonArgs& a, int num_sms, cudaStream_t stream);
// Frobenius norms of the Newton-Schulz inputs of a.mats into a.norms: the
// reference's sequential fp32 sum reproduced bit for bit (x_mode 0, the
// reference and bf16 recipes; refnorm.cu), or the fixed-order sum of the
// momentum kernel's tile partials (x_mode 1 and 2, the TF32 and fp32 modes,
// which have no reference counterpart and aim at exact Newton-Schulz).
// `cluster` CTAs (1, 2, 4 or 8; see ref_norm_cluster) share each matrix's
// sequential sum.
void launch_muon_norms(const MuonArgs& a, cudaStream_t stream, int cluster = 1);
void launch_ref_norms(const MuonArgs& a, int cluster, cudaStream_t stream);
// Cluster size for a launch whose largest matrix has max_elems elements out
// of total_elems: large matrices are split until no CTA's share of the
// sequential sum is much longer than an even spread over the SMs.
int ref_norm_cluster(long long max_elems, long long total_elems, int nmat, int num_sms);
void launch_muon_apply(const MuonArgs& a, int num_sms, cudaStream_t stream);

// Non-finite scan of fp32 and bf16 grad arenas into *flag (flag must be zero).
void launch_nonfinite_scan(const float* g32, long long n32, const __nv_bfloat16* g16,
                           long long n16, int* flag, int num_sms, cudaStream_t stream);

// Data-parallel grad reduction over peer memory: dst[i] = src[0][i] + src[1][i]
// + ... + src[world-1][i] for i in [begin, end), accumulated in fp32 in rank
// order (bf16 grads: the fp32 sum rounded to bf16 once). src[rank] is this
// rank's own arena (== dst); the others are IPC mappings of the peers' arenas.
// With `scan`, any non-finite sum sets every rank's skip flag.
constexpr int kMaxRanks = 8;
struct GradReduceArgs {
  const void* src[kMaxRanks];
  void* dst;
  long long begin, end;   // elements; begin is a multiple of 8
  int world;
  int bf16;
  int scan;
  int* skip_flags[kMaxRanks];  // every rank's skip flag (this rank's own at [rank])
};
void launch_grad_reduce(const GradReduceArgs& a, int num_sms, cudaStream_t stream);

// Non-finite scan of one rank's part of the grad arenas whose verdict goes to
// every rank: any non-finite value sets flag[0..n) (this rank's flag and its
// peers', the latter through IPC mappings). Flags are only ever set here.
struct RankFlags {
  int* flag[kMaxRanks];
  int n;
};
void launch_nonfinite_scan_ranks(const float* g32, long long n32, const __nv_bfloat16* g16,
                                 long long n16, const RankFlags& f, int num_sms,
                                 cudaStream_t stream);

// End of step: advance the AdamW counter unless skipped; dynamic loss scale.
struct StepTail {
  long long* step_counter;
  long long adamw_calls;  // AdamW tensors per step
  int* skip;
  int reset_skip;         // clear *skip after use (grads reduced across ranks)
  float* grad_scale;      // nullptr when no loss scaling
  int* good_steps;
  int growth_interval;
  int* skipped_total;
};
void launch_step_tail(const StepTail& t, cudaStream_t stream);

}  // namespace mmn
