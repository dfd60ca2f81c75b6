// Host side of the batched Newton-Schulz iteration: one NsClass per matrix
// shape (n x m after orientation, n <= m), holding the working buffers of
// every matrix of that shape (bf16, or tf32-valued fp32 in the TF32 mode) and
// the TMA descriptors over them.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>
#include <vector>

namespace mmn {

enum NsMode : int {
  kNsReference = 0,  // reference recipe: fp32 B kept exact via two accumulators
  kNsBf16 = 1,       // B rounded to bf16, one accumulator (faster, looser)
  kNsTf32 = 2,       // the reference recipe with tf32 rounding points instead of
                     // bf16: fp32 storage, kind::tf32 MMAs, two accumulators
  kNsFp32 = 3,       // no rounding points: fp32 values held as hi + lo tf32
                     // planes, three-pass tf32 products, two accumulators
};

// Bytes per stored element of X, A and A2 in a mode, and planes per matrix.
inline int ns_elem_bytes(int mode) { return mode == kNsTf32 || mode == kNsFp32 ? 4 : 2; }
inline int ns_planes(int mode) { return mode == kNsFp32 ? 2 : 1; }

struct NsClass {
  int n = 0, m = 0;   // oriented shape, n <= m
  int batch = 0;      // matrices of this shape
  int esize = 2;      // bytes per element of X, A, A2: 2 (bf16) or 4 (tf32-valued fp32)
  int planes = 1;     // 2 in the fp32 mode: matrix b is stored as items 2b (hi), 2b + 1 (lo)
  int ld_x = 0;       // row stride of X (elements, multiple of 8)
  int ld_a = 0;       // row stride of A / A2 (elements, multiple of 8)
  void* x[2] = {nullptr, nullptr};  // ping-pong X (batch x n x ld_x)
  void* a = nullptr;                // round(X X^T)              (batch x n x ld_a)
  void* a2 = nullptr;               // round(A A) or bf16(B)     (batch x n x ld_a)
  float* norms = nullptr;                    // device, batch entries
  int2* sym_tiles = nullptr;                 // device (tm, tn) list, 128-row tiles
  int n_sym_tiles = 0;
  int2* sym_tiles2 = nullptr;                // device (tm, tn) list, 256-row tiles (CTA pairs)
  int n_sym_tiles2 = 0;
  CUtensorMap tm_x_a[2], tm_x_b[2], tm_x_mn[2];
  CUtensorMap tm_a_a, tm_a_b, tm_a2_a;
  CUtensorMap tm_a_n, tm_a2_n;  // A / A2 rows in 64-row boxes (B operands of the transposed Poly)
  CUtensorMap tm_a_out, tm_a2_out;  // 32 x 32 store boxes of the symmetric outputs
  bool owns_memory = false;

  size_t x_elems() const { return (size_t)batch * planes * n * ld_x; }
  size_t a_elems() const { return (size_t)batch * planes * n * ld_a; }
};

// Sizes the class, allocates its buffers (or uses the caller's when base is not
// null; base must then hold ns_class_bytes() bytes) and encodes the tensor maps.
// esize is ns_elem_bytes() of the mode the class runs in (2 unless TF32).
// Returns an empty string on success, else a message.
std::string ns_class_init(NsClass& c, int n, int m, int batch, void* base, int esize = 2,
                          int planes = 1);
size_t ns_class_bytes(int n, int m, int batch, int esize = 2, int planes = 1);
void ns_class_free(NsClass& c);

// Lays the class out over caller memory at `base` (ns_class_bytes() bytes) and
// encodes its tensor maps, touching no device memory: the caller clears the
// region and uploads `tiles_out` to c.sym_tiles on its own stream.
std::string ns_class_bind(NsClass& c, int n, int m, int batch, void* base,
                          std::vector<int2>* tiles_out, int esize = 2, int planes = 1);

// The Muon update fused into the last iteration: p -= lr*scale * O for every
// matrix of the class (apply[b] gives batch item b's parameter).
struct NsApply;
struct NsFused {
  float* p = nullptr;
  __nv_bfloat16* p_bf16 = nullptr;
  const NsApply* apply = nullptr;
};

// Runs `steps` iterations on every matrix of the class; X starts in x[0] with
// c.norms holding the first-iteration divisors. `mode` must match the class's
// element size and planes (ns_elem_bytes, ns_planes). Returns the index of the X
// buffer that holds the result, or -1 on a launch error (message in err). With
// `fused` (and steps >= 1) the last iteration updates the parameters instead
// of storing X.
int ns_class_run(NsClass& c, int steps, int mode, int* status, int num_sms,
                 cudaStream_t stream, std::string* err, const NsFused* fused = nullptr,
                 const int* skip = nullptr);

// Opt-in shared memory for every GEMM instantiation (once per device).
std::string ns_gemm_setup();

}  // namespace mmn
