// Shared helpers of the omniwave_b200 kernels: element conversion, launch
// checks and the thread-local error message used by the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "omniwave_b200.h"

namespace ow {

// ---------------------------------------------------------------------------
// Error reporting.  Entry points catch nothing (no exceptions are thrown);
// helpers return a status and record the message here.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

#define OW_CHECK_ARG(cond, ...)                \
  do {                                         \
    if (!(cond)) {                             \
      ::ow::set_error(__VA_ARGS__);            \
      return OW_ERR_INVALID;                   \
    }                                          \
  } while (0)

void count_launches(int n);

// Records the caller's profiling event (ow_profile_events) for ``kernel``
// before (after == false) or after its launch on ``st``; no-op when unset.
void profile_mark(int kernel, bool after, cudaStream_t st);

#define OW_CHECK_LAUNCH(what)                                                   \
  do {                                                                          \
    cudaError_t e_ = cudaGetLastError();                                        \
    if (e_ != cudaSuccess) {                                                    \
      ::ow::set_error("%s: launch failed: %s", what, cudaGetErrorString(e_));   \
      return OW_ERR_CUDA;                                                       \
    }                                                                           \
  } while (0)

#define OW_RETURN_IF(status)      \
  do {                            \
    int s_ = (status);            \
    if (s_ != OW_OK) return s_;   \
  } while (0)

// Launch a kernel and count it (ow_launch_count()).
template <typename... KArgs, typename... Args>
inline void launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                   Args&&... args) {
  count_launches(1);
  kern<<<grid, block, smem, st>>>(static_cast<KArgs>(args)...);
}

inline size_t dtype_size(int dt) {
  switch (dt) {
    case OW_DTYPE_F32: return 4;
    case OW_DTYPE_F64: return 8;
    case OW_DTYPE_BF16: return 2;
    case OW_DTYPE_F16: return 2;
    default: return 0;
  }
}

inline const char* dtype_name(int dt) {
  switch (dt) {
    case OW_DTYPE_F32: return "float32";
    case OW_DTYPE_F64: return "float64";
    case OW_DTYPE_BF16: return "bfloat16";
    case OW_DTYPE_F16: return "float16";
    default: return "unknown";
  }
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// Element conversion between storage types and the compute type.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static double to_d(float v) { return v; }
  __device__ __forceinline__ static float from(float v) { return v; }
  __device__ __forceinline__ static float from(double v) { return (float)v; }
};
template <> struct Elem<double> {
  __device__ __forceinline__ static float to_f(double v) { return (float)v; }
  __device__ __forceinline__ static double to_d(double v) { return v; }
  __device__ __forceinline__ static double from(float v) { return v; }
  __device__ __forceinline__ static double from(double v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static double to_d(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
  __device__ __forceinline__ static __nv_bfloat16 from(double v) { return __double2bfloat16(v); }
};
template <> struct Elem<__half> {
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static double to_d(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from(float v) { return __float2half_rn(v); }
  __device__ __forceinline__ static __half from(double v) { return __double2half(v); }
};

// Load a storage element as compute type C.
template <typename C, typename S>
__device__ __forceinline__ C load_as(const S* p, int64_t i);
template <> __device__ __forceinline__ float load_as<float, float>(const float* p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ float load_as<float, double>(const double* p, int64_t i) { return (float)p[i]; }
template <> __device__ __forceinline__ float load_as<float, __nv_bfloat16>(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
template <> __device__ __forceinline__ float load_as<float, __half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <> __device__ __forceinline__ double load_as<double, double>(const double* p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ double load_as<double, float>(const float* p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ double load_as<double, __nv_bfloat16>(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
template <> __device__ __forceinline__ double load_as<double, __half>(const __half* p, int64_t i) { return __half2float(p[i]); }

// Round a compute value through a narrower type (identity for f32/f64).
__device__ __forceinline__ float round_through(float v, int dt) {
  if (dt == OW_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == OW_DTYPE_F16) return __half2float(__float2half_rn(v));
  return v;
}
__device__ __forceinline__ double round_through(double v, int dt) {
  if (dt == OW_DTYPE_BF16) return __bfloat162float(__double2bfloat16(v));
  if (dt == OW_DTYPE_F16) return __half2float(__double2half(v));
  if (dt == OW_DTYPE_F32) return (double)(float)v;
  return v;
}

__device__ __forceinline__ float ow_sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }
__device__ __forceinline__ double ow_sigmoid(double v) { return 1.0 / (1.0 + exp(-v)); }

}  // namespace ow
