// Shared pieces of the C ABI: error reporting, device contexts, the AdamW
// bias-correction table and the environment entry points.
#include <cmath>
#include <cstring>

#include "capi_internal.cuh"
#include "mmn_ptx.cuh"

namespace mmn {

namespace {
thread_local std::string t_last_error;
}

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? MMN_E_OOM : MMN_E_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

int Ctx::init(int dev, void* user_stream) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(MMN_E_NO_DEVICE, "GPU missing, but CUDA was requested.");
  }
  if (dev < 0 || dev >= count) return fail(MMN_E_INVALID, "device ordinal out of range");
  cudaDeviceProp prop;
  MMN_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
  if (prop.major != 10 || prop.minor != 0)
    return fail(MMN_E_NO_DEVICE, "this library is built for sm_100a (B200) devices only");
  device = dev;
  num_sms = prop.multiProcessorCount;
  MMN_CUDA_TRY(cudaSetDevice(dev));
  if (user_stream) {
    stream = static_cast<cudaStream_t>(user_stream);
    own_stream = false;
  } else {
    MMN_CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    own_stream = true;
  }
  MMN_CUDA_TRY(cudaMalloc(&status, sizeof(int)));
  MMN_CUDA_TRY(cudaMemset(status, 0, sizeof(int)));
  return MMN_OK;
}

void Ctx::release() {
  if (status) cudaFree(status);
  if (own_stream && stream) cudaStreamDestroy(stream);
  status = nullptr;
  stream = nullptr;
}

int Ctx::check_status() {
  MMN_CUDA_TRY(cudaStreamSynchronize(stream));
  int s = 0;
  MMN_CUDA_TRY(cudaMemcpy(&s, status, sizeof(int), cudaMemcpyDeviceToHost));
  if (s != kDevOk) {
    cudaMemset(status, 0, sizeof(int));
    return fail(MMN_E_TIMEOUT, "a kernel gave up a bounded wait (device status " +
                                   std::to_string(s) + ")");
  }
  return MMN_OK;
}

int Scratch::ensure(size_t need) {
  if (need <= bytes) return MMN_OK;
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
  size_t want = need < 4096 ? 4096 : need;
  MMN_CUDA_TRY(cudaMalloc(&ptr, want));
  bytes = want;
  return MMN_OK;
}

void Scratch::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
}

namespace {
// First t >= 1 from which 1 - beta^t is the same f32 for every later t, or -1.
int saturation_step(float beta, int cap) {
  if (beta == 1.0f || beta == 0.0f) return 1;  // beta^t constant for t >= 1
  if (!(beta > 0.0f && beta < 1.0f)) return -1;
  const float tiny = std::ldexp(1.0f, -26);  // 1 - x == 1.0f for every 0 <= x < 2^-25
  for (int t = 1; t <= cap; ++t)
    if (powf(beta, (float)t) < tiny) return t;
  return -1;
}
}  // namespace

int BiasTable::build(float b1, float b2) {
  const int cap = 1 << 22;
  const int s1 = saturation_step(b1, cap), s2 = saturation_step(b2, cap);
  if (s1 < 0 || s2 < 0)
    return fail(MMN_E_UNSUPPORTED,
                "AdamW betas must lie in [0, 1] and 1 - beta^t must reach 1.0f within 2^22 steps");
  t_sat = s1 > s2 ? s1 : s2;
  std::vector<float2> host((size_t)t_sat + 1);
  for (int t = 0; t <= t_sat; ++t) {
    host[t].x = 1.0f - powf(b1, (float)t);
    host[t].y = 1.0f - powf(b2, (float)t);
  }
  MMN_CUDA_TRY(cudaMalloc(&dev, host.size() * sizeof(float2)));
  MMN_CUDA_TRY(cudaMemcpy(dev, host.data(), host.size() * sizeof(float2), cudaMemcpyHostToDevice));
  return MMN_OK;
}

void BiasTable::release() {
  if (dev) cudaFree(dev);
  dev = nullptr;
}

int64_t shape_numel(const int64_t* shape, int ndim, int* err) {
  *err = MMN_OK;
  if (ndim < 0 || (ndim > 0 && !shape)) {
    *err = fail(MMN_E_INVALID, "shape pointer is null or ndim is negative");
    return 0;
  }
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] < 0) {
      *err = fail(MMN_E_INVALID, "negative dimension");
      return 0;
    }
    // elements stay below 2^62 so byte counts of 4-byte elements fit int64
    if (shape[i] > 0 && n > (int64_t(1) << 62) / shape[i]) {
      *err = fail(MMN_E_SHAPE, "tensor too large");
      return 0;
    }
    n *= shape[i];
  }
  return n;
}

int check_device_ptr(const void* p, int device, const char* what) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return fail(MMN_E_INVALID, std::string(what) + ": not a CUDA pointer");
  }
  if (at.type == cudaMemoryTypeManaged) return MMN_OK;
  if (at.type != cudaMemoryTypeDevice)
    return fail(MMN_E_INVALID, std::string(what) + ": host memory where device memory is needed");
  if (at.device != device)
    return fail(MMN_E_INVALID, std::string(what) + ": memory of device " +
                                   std::to_string(at.device) + ", handle on device " +
                                   std::to_string(device));
  return MMN_OK;
}

}  // namespace mmn

extern "C" {

int mmn_cuda_is_available(void) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  for (int d = 0; d < count; ++d) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, d) == cudaSuccess && prop.major == 10 && prop.minor == 0)
      return 1;
  }
  return 0;
}

int mmn_require_cuda(int cuda_requested) {
  if (cuda_requested && !mmn_cuda_is_available())
    return mmn::fail(MMN_E_NO_DEVICE,
                     "GPU missing, but CUDA was requested. Fix: install an NVIDIA GPU and CUDA "
                     "toolkit, or set cuda=False in TrainConfig.");
  return MMN_OK;
}

const char* mmn_last_error(void) { return mmn::t_last_error.c_str(); }

int mmn_abi_version(void) { return MMN_OPTIM_ABI_VERSION; }

namespace {
// Waits on an mbarrier phase that nothing completes, through the same bounded
// wait the GEMM kernels use, and records the time-out in *status.
__global__ void selftest_wait_kernel(uint64_t limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mmn::mbar_init(&bar, 1);
    abort_flag = 0;
    mmn::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mmn::mbar_wait(&bar, 0, &abort_flag, limit_ns))
    atomicExch(status, mmn::kDevWaitTimeout);
}
}  // namespace

int mmn_selftest_bounded_wait(int device, uint64_t limit_ns) {
  using namespace mmn;
  if (limit_ns == 0 || limit_ns > 2000000000ull) return fail(MMN_E_INVALID, "limit must be in (0, 2 s]");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return fail(MMN_E_NO_DEVICE, "no such CUDA device");
  }
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  int* d = nullptr;
  int st = -1;
  cudaError_t e = cudaMalloc(&d, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(d, 0, sizeof(int));
  if (e == cudaSuccess) {
    selftest_wait_kernel<<<1, 32>>>(limit_ns, d);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(&st, d, sizeof(int), cudaMemcpyDeviceToHost);
  if (d) cudaFree(d);
  if (prev >= 0) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "bounded-wait self-test");
  if (st == kDevWaitTimeout) return fail(MMN_E_TIMEOUT, "the wait gave up after its limit");
  return MMN_OK;
}

mmn_adamw_config mmn_adamw_config_default(void) {
  mmn_adamw_config c;
  c.lr = 3e-4f;
  c.beta1 = 0.9f;
  c.beta2 = 0.95f;
  c.eps = 1e-8f;
  c.weight_decay = 0.01f;
  return c;
}

mmn_muon_config mmn_muon_config_default(void) {
  mmn_muon_config c;
  c.lr = 0.02f;
  c.momentum = 0.95f;
  c.nesterov = 1;
  c.ns_steps = 5;
  return c;
}

int mmn_hybrid_classify_param(const int64_t* shape, int ndim) {
  if (ndim == 2 && shape && shape[0] > 1 && shape[1] > 1) return MMN_ROUTE_MUON;
  return MMN_ROUTE_ADAMW;
}

}  // extern "C"
