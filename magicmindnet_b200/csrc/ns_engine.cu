#include "ns_engine.cuh"
#include "ns_gemm.cuh"

#include <cudaTypedefs.h>

#include <mutex>

namespace mmn {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

std::string get_encode() {
  static std::once_flag once;
  static std::string err;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      err = "cuTensorMapEncodeTiled is not available from the driver";
    else
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return err;
}

CUtensorMapDataType map_type(int esize) {
  return esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// 3-D map (inner, rows, batch) of bf16 (esize 2) or fp32 (esize 4) elements
// with 128-byte swizzle; box (128 bytes of inner elements, box_rows, 1).
// atom32: swizzle 32-byte chunks instead of 16-byte ones, the layout tcgen05
// needs for MN-major tf32 operands.
std::string encode_3d(CUtensorMap* map, const void* base, int inner, int rows, int batch,
                      int ld, int box_rows, int esize, bool atom32 = false) {
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * esize, (cuuint64_t)ld * esize * (cuuint64_t)rows};
  cuuint32_t box[3] = {(cuuint32_t)(128 / esize), (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, map_type(esize), 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
  return "";
}

// 3-D map for TMA stores of 32 x 32 blocks (unswizzled, row-major stage).
std::string encode_3d_store(CUtensorMap* map, const void* base, int inner, int rows, int batch,
                            int ld, int esize) {
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * esize, (cuuint64_t)ld * esize * (cuuint64_t)rows};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, map_type(esize), 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
  return "";
}

int round_up(int x, int a) { return (x + a - 1) / a * a; }

// Tiles of an n x n symmetric output that touch the upper triangle, for
// tile_m-row by 256-column tiles.
void sym_tile_list(int n, int tile_m, std::vector<int2>* out) {
  const int tm_n = (n + tile_m - 1) / tile_m, tn_n = (n + 255) / 256;
  for (int tm = 0; tm < tm_n; ++tm)
    for (int tn = 0; tn < tn_n; ++tn)
      if (tn * 256 + 255 >= tm * tile_m) out->push_back(make_int2(tm, tn));
}

size_t sym_tiles_total(int n) {
  const size_t a = (size_t)((n + 127) / 128) * ((n + 255) / 256);
  const size_t b = (size_t)((n + 255) / 256) * ((n + 255) / 256);
  return a + b;
}

// Lays out the buffers of a class over `p` and encodes its tensor maps.
std::string layout(NsClass& c, int n, int m, int batch, uint8_t* p,
                   std::vector<int2>* tiles, int esize, int planes) {
  c.n = n;
  c.m = m;
  c.batch = batch;
  c.esize = esize;
  c.planes = planes;
  c.ld_x = round_up(m, 8);
  c.ld_a = round_up(n, 8);
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  size_t off = 0;
  c.x[0] = p + off;
  off += al(c.x_elems() * esize);
  c.x[1] = p + off;
  off += al(c.x_elems() * esize);
  c.a = p + off;
  off += al(c.a_elems() * esize);
  c.a2 = p + off;
  off += al(c.a_elems() * esize);
  c.norms = reinterpret_cast<float*>(p + off);
  off += al((size_t)batch * 4);
  tiles->clear();
  sym_tile_list(n, kBM, tiles);
  c.n_sym_tiles = (int)tiles->size();
  sym_tile_list(n, 2 * kBM, tiles);
  c.n_sym_tiles2 = (int)tiles->size() - c.n_sym_tiles;
  c.sym_tiles = reinterpret_cast<int2*>(p + off);
  c.sym_tiles2 = c.sym_tiles + c.n_sym_tiles;
  std::string err;
  // MN-major X boxes: 128 bytes of columns by one stage of K rows (64 bf16 or
  // 32 tf32 rows); K-major boxes: one stage of K columns by the operand's rows.
  const int kb = 128 / esize;
  const int e = esize;
  const int nb = batch * planes;  // the maps index planes as batch items
  for (int i = 0; i < 2; ++i) {
    if (!(err = encode_3d(&c.tm_x_a[i], c.x[i], m, n, nb, c.ld_x, kBM, e)).empty()) return err;
    if (!(err = encode_3d(&c.tm_x_b[i], c.x[i], m, n, nb, c.ld_x, 256, e)).empty()) return err;
    // (in the TF32 and fp32 modes X is read MN-major only through this map)
    if (!(err = encode_3d(&c.tm_x_mn[i], c.x[i], m, n, nb, c.ld_x, kb, e, e == 4)).empty())
      return err;
  }
  if (!(err = encode_3d(&c.tm_a_a, c.a, n, n, nb, c.ld_a, kBM, e)).empty()) return err;
  if (!(err = encode_3d(&c.tm_a_b, c.a, n, n, nb, c.ld_a, 256, e)).empty()) return err;
  if (!(err = encode_3d(&c.tm_a2_a, c.a2, n, n, nb, c.ld_a, kBM, e)).empty()) return err;
  if (!(err = encode_3d(&c.tm_a_n, c.a, n, n, nb, c.ld_a, 64, e)).empty()) return err;
  if (!(err = encode_3d(&c.tm_a2_n, c.a2, n, n, nb, c.ld_a, 64, e)).empty()) return err;
  if (!(err = encode_3d_store(&c.tm_a_out, c.a, n, n, nb, c.ld_a, e)).empty()) return err;
  if (!(err = encode_3d_store(&c.tm_a2_out, c.a2, n, n, nb, c.ld_a, e)).empty()) return err;
  return "";
}

template <int BN, bool DUAL, bool B_MN, int EPI, bool PAIR, bool F32 = false, bool SPLIT = false>
cudaError_t set_smem() {
  using S = NsGemmShape<BN, DUAL, B_MN, PAIR, EPI, F32, SPLIT>;
  return cudaFuncSetAttribute(ns_gemm_kernel<BN, DUAL, B_MN, EPI, PAIR, F32, SPLIT>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
}

template <int BN, bool DUAL, bool B_MN, int EPI, bool PAIR, bool F32 = false, bool SPLIT = false>
cudaError_t launch(const CUtensorMap& a1, const CUtensorMap& a2, const CUtensorMap& b,
                   const NsGemmArgs& args, int num_sms, cudaStream_t stream) {
  using S = NsGemmShape<BN, DUAL, B_MN, PAIR, EPI, F32, SPLIT>;
  if (args.num_tiles <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(S::kThreads, 1, 1);
  cfg.dynamicSmemBytes = S::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int grid;
  if (!PAIR) {
    grid = args.num_tiles < num_sms ? args.num_tiles : num_sms;
  } else {
    // A persistent grid must not exceed the clusters that fit at once: a
    // cluster scheduled late would run its whole tile list after the others.
    static int max_pairs = 0;
    if (max_pairs == 0) {
      cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
      int n = 0;
      cudaError_t e = cudaOccupancyMaxActiveClusters(
          &n, ns_gemm_kernel<BN, DUAL, B_MN, EPI, PAIR, F32, SPLIT>, &cfg);
      if (e != cudaSuccess || n <= 0) return e != cudaSuccess ? e : cudaErrorLaunchOutOfResources;
      max_pairs = n < num_sms / 2 ? n : num_sms / 2;
    }
    grid = 2 * (args.num_tiles < max_pairs ? args.num_tiles : max_pairs);
  }
  cfg.gridDim = dim3(grid, 1, 1);
  // Programmatic dependent launch: this grid may be scheduled while the previous
  // kernel on the stream drains (its CTAs take SMs as the previous ones exit);
  // each CTA sets up its barriers and TMEM, then waits until that kernel has
  // completed before it touches global memory.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, ns_gemm_kernel<BN, DUAL, B_MN, EPI, PAIR, F32, SPLIT>, a1, a2,
                            b, args);
}

// CTA pairs pay off once a matrix fills 256-row tiles.
bool use_pairs(const NsClass& c) { return c.n >= 256; }

}  // namespace

std::string ns_gemm_setup() {
  cudaError_t e = cudaSuccess;
#define MMN_SET(BN, D, MN, E)                                  \
  if (e == cudaSuccess) e = set_smem<BN, D, MN, E, false>();   \
  if (e == cudaSuccess) e = set_smem<BN, D, MN, E, true>();
  MMN_SET(256, false, false, kEpiGram)
  MMN_SET(256, false, false, kEpiSquare)
  MMN_SET(256, false, false, kEpiSquareBf16)
  MMN_SET(128, true, true, kEpiPolyDual)
  MMN_SET(256, false, true, kEpiPolySingle)
#undef MMN_SET
  if (e == cudaSuccess) e = set_smem<128, true, false, kEpiPolyDualT, true>();
  // TF32 mode
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiGram, false, true>();
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiGram, true, true>();
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiSquare, false, true>();
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiSquare, true, true>();
  if (e == cudaSuccess) e = set_smem<128, true, true, kEpiPolyDual, false, true>();
  if (e == cudaSuccess) e = set_smem<128, true, false, kEpiPolyDualT, true, true>();
  // fp32 mode (split tf32 planes)
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiGram, false, true, true>();
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiGram, true, true, true>();
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiSquare, false, true, true>();
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiSquare, true, true, true>();
  if (e == cudaSuccess) e = set_smem<128, true, true, kEpiPolyDual, false, true, true>();
  if (e == cudaSuccess) e = set_smem<128, true, false, kEpiPolyDualT, true, true, true>();
  if (e != cudaSuccess) return std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
  return get_encode();
}

size_t ns_class_bytes(int n, int m, int batch, int esize, int planes) {
  const size_t ld_x = (size_t)round_up(m, 8), ld_a = (size_t)round_up(n, 8);
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t items = (size_t)batch * planes;
  return 2 * al(items * n * ld_x * esize) + 2 * al(items * n * ld_a * esize) +
         al((size_t)batch * 4) + al(sym_tiles_total(n) * sizeof(int2));
}

std::string ns_class_init(NsClass& c, int n, int m, int batch, void* base, int esize,
                          int planes) {
  if (n <= 0 || m <= 0 || n > m || batch <= 0) return "invalid Newton-Schulz class shape";
  if ((esize != 2 && esize != 4) || (planes != 1 && planes != 2) || (planes == 2 && esize != 4))
    return "invalid Newton-Schulz element size";
  std::string err = get_encode();
  if (!err.empty()) return err;
  const size_t bytes = ns_class_bytes(n, m, batch, esize, planes);
  uint8_t* p = static_cast<uint8_t*>(base);
  bool own = false;
  if (!p) {
    if (cudaMalloc(&p, bytes) != cudaSuccess) return "cudaMalloc failed for Newton-Schulz buffers";
    own = true;
  }
  std::vector<int2> tiles;
  err = layout(c, n, m, batch, p, &tiles, esize, planes);
  c.owns_memory = own;
  if (!err.empty()) return err;
  // Padding columns of X and A are never read (the tensor maps stop at n / m);
  // zero them once anyway.
  if (cudaMemset(p, 0, bytes) != cudaSuccess) return "cudaMemset failed";
  if (cudaMemcpy(c.sym_tiles, tiles.data(), tiles.size() * sizeof(int2), cudaMemcpyHostToDevice) !=
      cudaSuccess)
    return "cudaMemcpy of the tile list failed";
  return "";
}

std::string ns_class_bind(NsClass& c, int n, int m, int batch, void* base,
                          std::vector<int2>* tiles_out, int esize, int planes) {
  if (n <= 0 || m <= 0 || n > m || batch <= 0 || !base || !tiles_out ||
      (esize != 2 && esize != 4) || (planes != 1 && planes != 2) || (planes == 2 && esize != 4))
    return "invalid Newton-Schulz class shape or base";
  std::string err = get_encode();
  if (!err.empty()) return err;
  c = NsClass();
  return layout(c, n, m, batch, static_cast<uint8_t*>(base), tiles_out, esize, planes);
}

void ns_class_free(NsClass& c) {
  if (c.owns_memory && c.x[0]) cudaFree(c.x[0]);
  c = NsClass();
}

// Coefficients of the quintic iteration (crates/mmn-optim/src/lib.rs:84-86).
static constexpr float kNsA = 3.4445f, kNsB = -4.7750f, kNsC = 2.0315f;

namespace {

template <bool PAIR, bool F32, bool SPLIT>
cudaError_t run_iteration(NsClass& c, int cur, int nxt, const float* norms, int mode,
                          const NsGemmArgs& base, const NsFused* fused, int num_sms,
                          cudaStream_t stream) {
  const int tile_m = PAIR ? 2 * kBM : kBM;
  NsGemmArgs g = base;

  // A = round((X X^T) / s / s), round = bf16, tf32 in the TF32 mode, none
  // (hi + lo planes) in the fp32 mode
  g.out = c.a;
  g.out_bstride = (long long)c.n * c.ld_a;
  g.out_ld = c.ld_a;
  g.aux = nullptr;
  g.norms = norms;
  g.M = c.n;
  g.N = c.n;
  g.K = c.m;
  g.tile_list = PAIR ? c.sym_tiles2 : c.sym_tiles;
  g.tiles_per_matrix = PAIR ? c.n_sym_tiles2 : c.n_sym_tiles;
  g.tiles_n = 0;
  g.num_tiles = g.tiles_per_matrix * c.batch;
  // B is the same X rows: 128 rows per CTA of a pair, 256 for a single CTA.
  const CUtensorMap& xb = PAIR ? c.tm_x_a[cur] : c.tm_x_b[cur];
  cudaError_t e = launch<256, false, false, kEpiGram, PAIR, F32, SPLIT>(c.tm_x_a[cur], c.tm_a_out, xb, g,
                                                                 num_sms, stream);
  if (e != cudaSuccess) return e;

  // A2 = round(A A)   or   Bm = bf16(b*A + c*bf16(A A))
  g.out = c.a2;
  g.norms = nullptr;
  g.K = c.n;
  const CUtensorMap& ab = PAIR ? c.tm_a_a : c.tm_a_b;
  if constexpr (!F32) {
    if (mode == kNsBf16) {
      g.aux = c.a;
      g.aux_bstride = (long long)c.n * c.ld_a;
      g.aux_ld = c.ld_a;
      e = launch<256, false, false, kEpiSquareBf16, PAIR>(c.tm_a_a, c.tm_a2_out, ab, g, num_sms,
                                                         stream);
    } else {
      e = launch<256, false, false, kEpiSquare, PAIR>(c.tm_a_a, c.tm_a2_out, ab, g, num_sms,
                                                      stream);
    }
  } else {
    e = launch<256, false, false, kEpiSquare, PAIR, true, SPLIT>(c.tm_a_a, c.tm_a2_out, ab, g,
                                                                 num_sms, stream);
  }
  if (e != cudaSuccess) return e;

  // X' = round((X/s)*a + (b*(A X) + c*(A2 X))/s)   or   bf16((X/s)*a + (Bm X)/s)
  g.out = c.x[nxt];
  g.out_bstride = (long long)c.n * c.ld_x;
  g.out_ld = c.ld_x;
  g.aux = c.x[cur];
  g.aux_bstride = (long long)c.n * c.ld_x;
  g.aux_ld = c.ld_x;
  g.norms = norms;
  g.M = c.n;
  g.N = c.m;
  g.K = c.n;
  g.tile_list = nullptr;
  if (fused) {
    g.p = fused->p;
    g.p_bf16 = fused->p_bf16;
    g.apply = fused->apply;
  }
  if constexpr (!F32) {
    if (mode == kNsBf16) {
      g.tiles_n = (c.m + 255) / 256;
      g.tiles_per_matrix = ((c.n + tile_m - 1) / tile_m) * g.tiles_n;
      g.num_tiles = g.tiles_per_matrix * c.batch;
      return launch<256, false, true, kEpiPolySingle, PAIR>(c.tm_a2_a, c.tm_a2_a, c.tm_x_mn[cur],
                                                            g, num_sms, stream);
    }
  }
  // Two accumulators of 128 columns, double-buffered in TMEM. Measured against
  // 256-column dual tiles (single-buffered TMEM) and a stacked A|A2 pair that
  // swaps accumulator halves through shared memory, this shape was fastest.
  if (PAIR) {
    // transposed: 256 columns of X by 128 rows of A / A2 per tile
    g.tiles_n = (c.n + 127) / 128;
    g.tiles_per_matrix = ((c.m + 255) / 256) * g.tiles_n;
    g.num_tiles = g.tiles_per_matrix * c.batch;
    return launch<128, true, false, kEpiPolyDualT, true, F32, SPLIT>(
        c.tm_x_mn[cur], c.tm_a2_n, c.tm_a_n, g, num_sms, stream);
  }
  g.tiles_n = (c.m + 127) / 128;
  g.tiles_per_matrix = ((c.n + tile_m - 1) / tile_m) * g.tiles_n;
  g.num_tiles = g.tiles_per_matrix * c.batch;
  return launch<128, true, true, kEpiPolyDual, PAIR, F32, SPLIT>(c.tm_a_a, c.tm_a2_a,
                                                                 c.tm_x_mn[cur], g, num_sms, stream);
}

}  // namespace

int ns_class_run(NsClass& c, int steps, int mode, int* status, int num_sms,
                 cudaStream_t stream, std::string* err, const NsFused* fused, const int* skip) {
  int cur = 0;
  NsGemmArgs base{};
  base.status = status;
  base.skip = skip;
  base.coef_a = kNsA;
  base.coef_b = kNsB;
  base.coef_c = kNsC;
  const bool pair = use_pairs(c);
  const bool f32 = mode == kNsTf32 || mode == kNsFp32, split = mode == kNsFp32;
  if (c.esize != ns_elem_bytes(mode) || c.planes != ns_planes(mode)) {
    if (err) *err = "Newton-Schulz class buffers do not match the arithmetic mode";
    return -1;
  }
  for (int it = 0; it < steps; ++it) {
    const int nxt = cur ^ 1;
    const float* norms = it == 0 ? c.norms : nullptr;
    const NsFused* f = (fused && it == steps - 1) ? fused : nullptr;
    cudaError_t e;
    if (split)
      e = pair ? run_iteration<true, true, true>(c, cur, nxt, norms, mode, base, f, num_sms, stream)
               : run_iteration<false, true, true>(c, cur, nxt, norms, mode, base, f, num_sms,
                                                  stream);
    else if (f32)
      e = pair ? run_iteration<true, true, false>(c, cur, nxt, norms, mode, base, f, num_sms,
                                                  stream)
               : run_iteration<false, true, false>(c, cur, nxt, norms, mode, base, f, num_sms,
                                                   stream);
    else
      e = pair ? run_iteration<true, false, false>(c, cur, nxt, norms, mode, base, f, num_sms,
                                                   stream)
               : run_iteration<false, false, false>(c, cur, nxt, norms, mode, base, f, num_sms,
                                                    stream);
    if (e != cudaSuccess) {
      if (err) *err = std::string("Newton-Schulz GEMM launch: ") + cudaGetErrorString(e);
      return -1;
    }
    cur = nxt;
  }
  return cur;
}

}  // namespace mmn
