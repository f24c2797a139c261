// Shared helpers of libxsake_hads: status/error plumbing, dtype helpers, bounded waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <string>

#include "xsake_hads.h"

namespace xsake {

// ----------------------------------------------------------------------------- host errors
int set_error(int code, const char* fmt, ...);   // records a message for this thread, returns code
void clear_error();

#define XSAKE_CUDA_TRY(expr)                                                              \
  do {                                                                                    \
    cudaError_t err__ = (expr);                                                           \
    if (err__ != cudaSuccess)                                                             \
      return ::xsake::set_error(XSAKE_ECUDA, "%s failed: %s (%s:%d)", #expr,              \
                                cudaGetErrorString(err__), __FILE__, __LINE__);           \
  } while (0)

#define XSAKE_REQUIRE(cond, code, ...)                                                    \
  do {                                                                                    \
    if (!(cond)) return ::xsake::set_error(code, __VA_ARGS__);                            \
  } while (0)

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(XSAKE_ECUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
  return XSAKE_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Per-device attributes, read once per device.
struct DeviceInfo {
  int sm_count = 0;
  int major = 0, minor = 0;
  size_t smem_optin = 0;
};
int device_info(DeviceInfo* out);

// ----------------------------------------------------------------------------- device errors
// Each translation unit owns one device error word (first error wins) and registers a
// reader; xsake_device_error() drains all of them.  Kinds (high byte of the word):
enum DeviceErrorKind : int32_t {
  DEV_ERR_TIMEOUT = 1,      // a bounded mbarrier / flag wait gave up
  DEV_ERR_PLAN = 2,         // the mask plan does not match the call
  DEV_ERR_BOUNDS = 3,       // an index check failed and the access was skipped
};

typedef int (*DeviceErrorReader)(cudaStream_t, int32_t*);
void register_device_error_reader(DeviceErrorReader fn);

#define XSAKE_DEFINE_DEVICE_ERROR(tag)                                                     \
  static __device__ int32_t g_dev_err_##tag = 0;                                           \
  static __device__ __forceinline__ void record_device_error(int32_t kind, int32_t detail) { \
    atomicCAS(&g_dev_err_##tag, 0, (kind << 24) | (detail & 0xFFFFFF));                    \
  }                                                                                        \
  static int read_clear_device_error_##tag(cudaStream_t s, int32_t* code) {                \
    int32_t v = 0, z = 0;                                                                  \
    if (cudaMemcpyFromSymbolAsync(&v, g_dev_err_##tag, sizeof(v), 0,                       \
                                  cudaMemcpyDeviceToHost, s) != cudaSuccess) return 1;     \
    if (cudaMemcpyToSymbolAsync(g_dev_err_##tag, &z, sizeof(z), 0,                         \
                                cudaMemcpyHostToDevice, s) != cudaSuccess) return 1;       \
    if (cudaStreamSynchronize(s) != cudaSuccess) return 1;                                 \
    *code = v;                                                                             \
    return 0;                                                                              \
  }                                                                                        \
  namespace {                                                                              \
  struct DevErrReg_##tag {                                                                 \
    DevErrReg_##tag() { ::xsake::register_device_error_reader(read_clear_device_error_##tag); } \
  } dev_err_reg_##tag;                                                                     \
  }

// ----------------------------------------------------------------------------- device helpers
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bound on any single device-side wait.  A healthy wait in these kernels lasts
// microseconds; after this long the waiting kernel records DEV_ERR_TIMEOUT and bails out.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

template <typename T> struct DT;
template <> struct DT<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct DT<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// float32 minimum, the fill value of masked scores in the reference.
constexpr float kMaskFill = -3.4028234663852886e38f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

}  // namespace xsake
