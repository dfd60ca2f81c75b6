// newton_schulz5 for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc: a process whose device memory is wholly
// owned by another framework's caching allocator or a fixed arena, a host that
// forbids allocation once it has started (real-time or certified runtimes), or
// code on a latency-critical path where cudaMalloc/cudaFree would implicitly
// synchronise the device. For them this entry point runs the same kernels as
// mmn_newton_schulz5 with every piece of scratch (the two bf16 X buffers, A,
// A2, the norm, the per-tile partial sums, the matrix descriptor and the
// status word) placed in one file-scope __device__ array of fixed size. Every
// GPU that loads the library holds that array until the process exits.
//
// The host only knows the array's name as a host-side stand-in; its device
// address is fetched once per device with cudaGetSymbolAddress (with that
// device current) on the first call, which is why the first call on a device
// should happen before any stream capture. All calls on a device share the one
// array, and each call clears the parts that must start at zero; calls that
// overlap on the GPU (other host threads, other streams) race on it.
#include <mutex>
#include <string>
#include <vector>

#include "capi_internal.cuh"
#include "elementwise.cuh"
#include "mmn_ptx.cuh"
#include "ns_engine.cuh"

namespace {

// Largest problem: min(rows, cols) <= 1024 and rows * cols <= 2^20.
constexpr int64_t kNoAllocMaxElems = int64_t(1) << 20;
constexpr int64_t kNoAllocMaxSide = 1024;
constexpr size_t kNoAllocScratchBytes = (size_t(8) << 20) + (size_t(256) << 10);  // 8.25 MiB

__device__ __align__(256) unsigned char g_ns_scratch[kNoAllocScratchBytes];

struct DeviceSlot {
  void* base = nullptr;  // device address of g_ns_scratch on this device
  int num_sms = 0;
  bool ready = false;
};

constexpr int kMaxDevices = 128;
std::mutex g_mutex;
DeviceSlot g_slots[kMaxDevices];

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Once per device, with the device current: resolve the array's device address.
int device_setup(int dev, DeviceSlot* out) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceSlot& s = g_slots[dev];
  if (!s.ready) {
    cudaDeviceProp prop;
    cudaError_t e = cudaGetDeviceProperties(&prop, dev);
    if (e != cudaSuccess) return mmn::cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
      return mmn::fail(MMN_E_NO_DEVICE, "this library is built for sm_100a (B200) devices only");
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ns_scratch);
    if (e != cudaSuccess) return mmn::cuda_fail(e, "cudaGetSymbolAddress(g_ns_scratch)");
    std::string err = mmn::ns_gemm_setup();
    if (!err.empty()) return mmn::fail(MMN_E_CUDA, err);
    s.base = p;
    s.num_sms = prop.multiProcessorCount;
    s.ready = true;
  }
  *out = s;
  return MMN_OK;
}

struct Meta {
  mmn::MuonMat mat;
  mmn::MuonClassPtr cls[2];
};

}  // namespace

extern "C" int mmn_newton_schulz5_noalloc(const float* g, int64_t rows, int64_t cols, int steps,
                                          int ns_mode, float* out, int device, void* stream) {
  using namespace mmn;
  if (!g || !out) return fail(MMN_E_INVALID, "null input or output");
  if (steps < 0) return fail(MMN_E_INVALID, "steps must be >= 0");
  if (ns_mode == MMN_NS_TF32 || ns_mode == MMN_NS_FP32)
    return fail(MMN_E_UNSUPPORTED,
                "the TF32 and fp32 modes need more than the fixed scratch of "
                "mmn_newton_schulz5_noalloc (use mmn_newton_schulz5)");
  if (ns_mode != MMN_NS_REFERENCE && ns_mode != MMN_NS_BF16)
    return fail(MMN_E_INVALID, "unknown ns_mode");
  if (rows < 1 || cols < 1) return fail(MMN_E_SHAPE, "empty matrix");
  const int64_t n = rows < cols ? rows : cols, m = rows < cols ? cols : rows;
  if (n > kNoAllocMaxSide || m > kNoAllocMaxElems / n)  // (rows * cols could overflow)
    return fail(MMN_E_UNSUPPORTED,
                "matrix exceeds the fixed scratch of mmn_newton_schulz5_noalloc: need "
                "min(rows, cols) <= 1024 and rows * cols <= 1048576 (use mmn_newton_schulz5)");
  if (device < 0 || device >= kMaxDevices) return fail(MMN_E_INVALID, "device out of range");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device >= count) {
    cudaGetLastError();
    return fail(MMN_E_NO_DEVICE, "GPU missing, but CUDA was requested.");
  }
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (cudaSetDevice(device) != cudaSuccess) return fail(MMN_E_CUDA, "cudaSetDevice failed");
  struct Restore {
    int d;
    ~Restore() {
      if (d >= 0) cudaSetDevice(d);
    }
  } restore{prev};

  DeviceSlot slot;
  int rc = device_setup(device, &slot);
  if (rc != MMN_OK) return rc;
  if ((rc = check_device_ptr(g, device, "g")) != MMN_OK) return rc;
  if ((rc = check_device_ptr(out, device, "out")) != MMN_OK) return rc;

  // Scratch layout: [Newton-Schulz class][status][partials][descriptor].
  const int ni = (int)n, mi = (int)m, ri = (int)rows, ci = (int)cols;
  const int tiles = ((ri + 63) / 64) * ((ci + 63) / 64);
  uint8_t* base = static_cast<uint8_t*>(slot.base);
  const size_t cls_bytes = align256(ns_class_bytes(ni, mi, 1));
  int* status = reinterpret_cast<int*>(base + cls_bytes);
  float* partials = reinterpret_cast<float*>(base + cls_bytes + 256);
  const size_t meta_off = cls_bytes + 256 + align256((size_t)tiles * 4);
  Meta* dmeta = reinterpret_cast<Meta*>(base + meta_off);
  const size_t used = meta_off + align256(sizeof(Meta));
  if (used > kNoAllocScratchBytes)
    return fail(MMN_E_UNSUPPORTED, "matrix exceeds the fixed scratch of mmn_newton_schulz5_noalloc");

  NsClass c;
  std::vector<int2> tile_list;
  std::string err = ns_class_bind(c, ni, mi, 1, base, &tile_list);
  if (!err.empty()) return fail(MMN_E_CUDA, err);

  Meta meta{};
  meta.mat.rows = ri;
  meta.mat.cols = ci;
  meta.mat.transposed = rows > cols;
  meta.mat.lr_scale = -1.0f;  // out = 0 - (-1 * O) = O
  meta.cls[0].x = c.x[0];
  meta.cls[0].bstride = (long long)c.n * c.ld_x;
  meta.cls[0].ld = c.ld_x;
  meta.cls[1] = meta.cls[0];
  meta.cls[1].x = c.x[steps % 2];

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The tile list and `meta` are pageable host objects of this call. The
  // runtime stages a pageable source before cudaMemcpyAsync returns, so an
  // early error return may drop them; on success the call also waits for its
  // stream before returning, so they outlive their copies either way.
  MMN_CUDA_TRY(cudaMemsetAsync(base, 0, used, s));
  MMN_CUDA_TRY(cudaMemcpyAsync(c.sym_tiles, tile_list.data(), tile_list.size() * sizeof(int2),
                               cudaMemcpyHostToDevice, s));
  MMN_CUDA_TRY(cudaMemcpyAsync(dmeta, &meta, sizeof(Meta), cudaMemcpyHostToDevice, s));

  // u = g (momentum 0, no Nesterov); the velocity slot is `out`, cleared again
  // below before the result is written into it.
  MuonArgs a{};
  a.p = out;
  a.g = g;
  a.vel = out;
  a.mats = &dmeta->mat;
  a.nmat = 1;
  a.total_tiles = tiles;
  a.cls = &dmeta->cls[0];
  a.partials = partials;
  a.norms = c.norms;
  a.momentum = 0.0f;
  a.nesterov = 0;
  a.grad_divisor = 1.0f;
  a.fresh_state = 1;
  a.apply_divides_norm = steps == 0;
  a.norm_scalar_rows = m % 8 != 0;
  launch_muon_momentum(a, slot.num_sms, s);
  launch_muon_norms(a, s, ref_norm_cluster(rows * cols, rows * cols, 1, slot.num_sms));
  MMN_CUDA_TRY(cudaGetLastError());
  if (ns_class_run(c, steps, ns_mode, status, slot.num_sms, s, &err) < 0)
    return fail(MMN_E_CUDA, err);
  MMN_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)rows * cols * 4, s));
  a.cls = &dmeta->cls[1];
  launch_muon_apply(a, slot.num_sms, s);
  MMN_CUDA_TRY(cudaGetLastError());
  // The status word comes back on the caller's stream, so the call waits for
  // that stream only (a plain cudaMemcpy would wait for the whole device).
  int st = 0;
  MMN_CUDA_TRY(cudaMemcpyAsync(&st, status, sizeof(int), cudaMemcpyDeviceToHost, s));
  MMN_CUDA_TRY(cudaStreamSynchronize(s));
  if (st != kDevOk)
    return fail(MMN_E_TIMEOUT, "a kernel gave up a bounded wait (device status " +
                                   std::to_string(st) + ")");
  return MMN_OK;
}
