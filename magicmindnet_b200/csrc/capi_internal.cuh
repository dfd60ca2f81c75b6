// Internal helpers shared by the C ABI translation units.
#pragma once
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/mmn_optim.h"

namespace mmn {

// Thread-local message for mmn_last_error().
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define MMN_CUDA_TRY(expr)                          \
  do {                                              \
    cudaError_t _e = (expr);                        \
    if (_e != cudaSuccess) return cuda_fail(_e, #expr); \
  } while (0)

// Makes `dev` current for a scope and restores the previous device after it.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
};

// Device, stream and SM count of a handle.
struct Ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int* status = nullptr;  // device status word written by kernels on timeout

  int init(int dev, void* user_stream);
  void release();
  // Reads the device status word (synchronises the stream).
  int check_status();
};

// RAII-free device scratch that only grows.
struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
  int ensure(size_t need);
  void release();
};

// Host-side table of the AdamW bias-correction divisors (1 - b1^t, 1 - b2^t)
// computed with the C library's powf exactly as the reference's f32::powf
// (crates/mmn-optim/src/lib.rs:53-54), uploaded once; t_sat is the first step
// from which both divisors are exactly 1.0f for every later t.
struct BiasTable {
  float2* dev = nullptr;
  int t_sat = 0;
  int build(float b1, float b2);
  void release();
};

int64_t shape_numel(const int64_t* shape, int ndim, int* err);

// MMN_OK when `p` is device (or managed) memory of `device`, so that kernels
// launched there may read it; else MMN_E_INVALID naming `what`. Memory of
// another GPU is refused: kernels here never read a peer's memory.
int check_device_ptr(const void* p, int device, const char* what);

// fp32 -> tf32 value (10 leading mantissa bits), to nearest with ties to even
// on the 13 discarded bits; Inf and NaN pass through. The host form of the
// TF32 mode's rounding point.
inline float host_tf32_round(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

}  // namespace mmn
