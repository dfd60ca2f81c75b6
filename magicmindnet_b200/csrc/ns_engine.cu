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

// 3-D bf16 map (inner, rows, batch) with 128-byte swizzle; box (64, box_rows, 1).
std::string encode_3d(CUtensorMap* map, const void* base, int inner, int rows, int batch,
                      int ld, int box_rows) {
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)ld * 2 * (cuuint64_t)rows};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
  return "";
}

int round_up(int x, int a) { return (x + a - 1) / a * a; }

template <int BN, bool DUAL, bool B_MN, int EPI>
cudaError_t set_smem() {
  using S = NsGemmShape<BN, DUAL, B_MN>;
  return cudaFuncSetAttribute(ns_gemm_kernel<BN, DUAL, B_MN, EPI>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
}

template <int BN, bool DUAL, bool B_MN, int EPI>
cudaError_t launch(const CUtensorMap& a1, const CUtensorMap& a2, const CUtensorMap& b,
                   const NsGemmArgs& args, int num_sms, cudaStream_t stream) {
  using S = NsGemmShape<BN, DUAL, B_MN>;
  if (args.num_tiles <= 0) return cudaSuccess;
  const int grid = args.num_tiles < num_sms ? args.num_tiles : num_sms;
  ns_gemm_kernel<BN, DUAL, B_MN, EPI><<<grid, 192, S::kSmemBytes, stream>>>(a1, a2, b, args);
  return cudaGetLastError();
}

}  // namespace

std::string ns_gemm_setup() {
  cudaError_t e = cudaSuccess;
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiGram>();
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiSquare>();
  if (e == cudaSuccess) e = set_smem<256, false, false, kEpiSquareBf16>();
  if (e == cudaSuccess) e = set_smem<128, true, true, kEpiPolyDual>();
  if (e == cudaSuccess) e = set_smem<256, false, true, kEpiPolySingle>();
  if (e != cudaSuccess) return std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
  return get_encode();
}

size_t ns_class_bytes(int n, int m, int batch) {
  const size_t ld_x = (size_t)round_up(m, 8), ld_a = (size_t)round_up(n, 8);
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  const int tm = (n + kBM - 1) / kBM, tn = (n + 255) / 256;
  return 2 * al((size_t)batch * n * ld_x * 2) + 2 * al((size_t)batch * n * ld_a * 2) +
         al((size_t)batch * 4) + al((size_t)tm * tn * sizeof(int2));
}

std::string ns_class_init(NsClass& c, int n, int m, int batch, void* base) {
  if (n <= 0 || m <= 0 || n > m || batch <= 0) return "invalid Newton-Schulz class shape";
  std::string err = get_encode();
  if (!err.empty()) return err;
  c.n = n;
  c.m = m;
  c.batch = batch;
  c.ld_x = round_up(m, 8);
  c.ld_a = round_up(n, 8);
  const size_t bytes = ns_class_bytes(n, m, batch);
  uint8_t* p = static_cast<uint8_t*>(base);
  if (!p) {
    if (cudaMalloc(&p, bytes) != cudaSuccess) return "cudaMalloc failed for Newton-Schulz buffers";
    c.owns_memory = true;
  }
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  size_t off = 0;
  c.x[0] = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += al(c.x_elems() * 2);
  c.x[1] = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += al(c.x_elems() * 2);
  c.a = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += al(c.a_elems() * 2);
  c.a2 = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += al(c.a_elems() * 2);
  c.norms = reinterpret_cast<float*>(p + off);
  off += al((size_t)batch * 4);
  c.sym_tiles = reinterpret_cast<int2*>(p + off);
  // Padding columns of X and A are never written by the kernels but are read
  // by nothing either (the tensor maps stop at n / m); zero them once anyway.
  if (cudaMemset(p, 0, bytes) != cudaSuccess) return "cudaMemset failed";

  // Tiles of an n x n symmetric output that touch the upper triangle.
  std::vector<int2> tiles;
  const int tm_n = (n + kBM - 1) / kBM, tn_n = (n + 255) / 256;
  for (int tm = 0; tm < tm_n; ++tm)
    for (int tn = 0; tn < tn_n; ++tn)
      if (tn * 256 + 255 >= tm * kBM) tiles.push_back(make_int2(tm, tn));
  c.n_sym_tiles = (int)tiles.size();
  if (cudaMemcpy(c.sym_tiles, tiles.data(), tiles.size() * sizeof(int2), cudaMemcpyHostToDevice) !=
      cudaSuccess)
    return "cudaMemcpy of the tile list failed";

  for (int i = 0; i < 2; ++i) {
    if (!(err = encode_3d(&c.tm_x_a[i], c.x[i], m, n, batch, c.ld_x, kBM)).empty()) return err;
    if (!(err = encode_3d(&c.tm_x_b[i], c.x[i], m, n, batch, c.ld_x, 256)).empty()) return err;
    if (!(err = encode_3d(&c.tm_x_mn[i], c.x[i], m, n, batch, c.ld_x, 64)).empty()) return err;
  }
  if (!(err = encode_3d(&c.tm_a_a, c.a, n, n, batch, c.ld_a, kBM)).empty()) return err;
  if (!(err = encode_3d(&c.tm_a_b, c.a, n, n, batch, c.ld_a, 256)).empty()) return err;
  if (!(err = encode_3d(&c.tm_a2_a, c.a2, n, n, batch, c.ld_a, kBM)).empty()) return err;
  return "";
}

std::string ns_class_bind(NsClass& c, int n, int m, int batch, void* base,
                          std::vector<int2>* tiles_out) {
  if (n <= 0 || m <= 0 || n > m || batch <= 0 || !base || !tiles_out)
    return "invalid Newton-Schulz class shape or base";
  std::string err = get_encode();
  if (!err.empty()) return err;
  c = NsClass();
  c.n = n;
  c.m = m;
  c.batch = batch;
  c.ld_x = round_up(m, 8);
  c.ld_a = round_up(n, 8);
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  c.x[0] = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += al(c.x_elems() * 2);
  c.x[1] = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += al(c.x_elems() * 2);
  c.a = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += al(c.a_elems() * 2);
  c.a2 = reinterpret_cast<__nv_bfloat16*>(p + off);
  off += al(c.a_elems() * 2);
  c.norms = reinterpret_cast<float*>(p + off);
  off += al((size_t)batch * 4);
  c.sym_tiles = reinterpret_cast<int2*>(p + off);
  tiles_out->clear();
  const int tm_n = (n + kBM - 1) / kBM, tn_n = (n + 255) / 256;
  for (int tm = 0; tm < tm_n; ++tm)
    for (int tn = 0; tn < tn_n; ++tn)
      if (tn * 256 + 255 >= tm * kBM) tiles_out->push_back(make_int2(tm, tn));
  c.n_sym_tiles = (int)tiles_out->size();
  for (int i = 0; i < 2; ++i) {
    if (!(err = encode_3d(&c.tm_x_a[i], c.x[i], m, n, batch, c.ld_x, kBM)).empty()) return err;
    if (!(err = encode_3d(&c.tm_x_b[i], c.x[i], m, n, batch, c.ld_x, 256)).empty()) return err;
    if (!(err = encode_3d(&c.tm_x_mn[i], c.x[i], m, n, batch, c.ld_x, 64)).empty()) return err;
  }
  if (!(err = encode_3d(&c.tm_a_a, c.a, n, n, batch, c.ld_a, kBM)).empty()) return err;
  if (!(err = encode_3d(&c.tm_a_b, c.a, n, n, batch, c.ld_a, 256)).empty()) return err;
  if (!(err = encode_3d(&c.tm_a2_a, c.a2, n, n, batch, c.ld_a, kBM)).empty()) return err;
  return "";
}

void ns_class_free(NsClass& c) {
  if (c.owns_memory && c.x[0]) cudaFree(c.x[0]);
  c = NsClass();
}

// Coefficients of the quintic iteration (crates/mmn-optim/src/lib.rs:84-86).
static constexpr float kNsA = 3.4445f, kNsB = -4.7750f, kNsC = 2.0315f;

int ns_class_run(NsClass& c, int steps, int mode, int* status, int num_sms,
                 cudaStream_t stream, std::string* err) {
  int cur = 0;
  for (int it = 0; it < steps; ++it) {
    const int nxt = cur ^ 1;
    const float* norms = it == 0 ? c.norms : nullptr;
    NsGemmArgs g{};
    g.status = status;
    g.coef_a = kNsA;
    g.coef_b = kNsB;
    g.coef_c = kNsC;

    // A = bf16((X X^T) / s / s)
    g.out = c.a;
    g.out_bstride = (long long)c.n * c.ld_a;
    g.out_ld = c.ld_a;
    g.aux = nullptr;
    g.norms = norms;
    g.M = c.n;
    g.N = c.n;
    g.K = c.m;
    g.tile_list = c.sym_tiles;
    g.tiles_per_matrix = c.n_sym_tiles;
    g.tiles_n = 0;
    g.num_tiles = c.n_sym_tiles * c.batch;
    cudaError_t e = launch<256, false, false, kEpiGram>(c.tm_x_a[cur], c.tm_x_a[cur],
                                                        c.tm_x_b[cur], g, num_sms, stream);

    // A2 = bf16(A A)   or   Bm = bf16(b*A + c*bf16(A A))
    g.out = c.a2;
    g.norms = nullptr;
    g.K = c.n;
    if (e == cudaSuccess) {
      if (mode == kNsBf16) {
        g.aux = c.a;
        g.aux_bstride = (long long)c.n * c.ld_a;
        g.aux_ld = c.ld_a;
        e = launch<256, false, false, kEpiSquareBf16>(c.tm_a_a, c.tm_a_a, c.tm_a_b, g, num_sms,
                                                      stream);
      } else {
        e = launch<256, false, false, kEpiSquare>(c.tm_a_a, c.tm_a_a, c.tm_a_b, g, num_sms,
                                                  stream);
      }
    }

    // X' = bf16((X/s)*a + (b*(A X) + c*(A2 X))/s)   or   bf16((X/s)*a + (Bm X)/s)
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
    if (e == cudaSuccess) {
      if (mode == kNsBf16) {
        g.tiles_n = (c.m + 255) / 256;
        g.tiles_per_matrix = ((c.n + kBM - 1) / kBM) * g.tiles_n;
        g.num_tiles = g.tiles_per_matrix * c.batch;
        e = launch<256, false, true, kEpiPolySingle>(c.tm_a2_a, c.tm_a2_a, c.tm_x_mn[cur], g,
                                                     num_sms, stream);
      } else {
        g.tiles_n = (c.m + 127) / 128;
        g.tiles_per_matrix = ((c.n + kBM - 1) / kBM) * g.tiles_n;
        g.num_tiles = g.tiles_per_matrix * c.batch;
        e = launch<128, true, true, kEpiPolyDual>(c.tm_a_a, c.tm_a2_a, c.tm_x_mn[cur], g,
                                                  num_sms, stream);
      }
    }
    if (e != cudaSuccess) {
      if (err) *err = std::string("Newton-Schulz GEMM launch: ") + cudaGetErrorString(e);
      return -1;
    }
    cur = nxt;
  }
  return cur;
}

}  // namespace mmn
