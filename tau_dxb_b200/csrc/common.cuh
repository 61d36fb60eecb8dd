// Shared helpers for the tau-dxb B200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include "tau_dxb.h"

namespace taudxb {

// ---- error reporting (thread-local message, see capi.cu) -------------------
void set_last_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int check_launch(const char* what);

#define TDX_CHECK_ARG(cond, ...)                                                   \
  do {                                                                             \
    if (!(cond)) return ::taudxb::fail(TAU_DXB_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define TDX_CUDA(call)                                                             \
  do {                                                                             \
    cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess)                                                         \
      return ::taudxb::fail(TAU_DXB_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

int sm_count();  // SMs of the current device (cached per device)

// ---- element conversions ---------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

__device__ __forceinline__ float load_as_float(const void* p, int dtype, int64_t idx) {
  if (dtype == TAU_DXB_F32) return static_cast<const float*>(p)[idx];
  if (dtype == TAU_DXB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
  return __half2float(static_cast<const __half*>(p)[idx]);
}

// ---- tau-opus sigma functions (echo/stau_opus_operator.py:16-46) ----------
// Precise forms: CUDA's accurate math functions, fp32 throughout.
constexpr float kClampMin = 1e-8f;

__device__ __forceinline__ float sigma_precise(int sid, float x) {
  float v;
  switch (sid) {
    case TAU_DXB_SIGMA_SOFTPLUS: v = x > 20.f ? x : log1pf(expf(x)); break;
    case TAU_DXB_SIGMA_SIGMOID:  v = 1.f / (1.f + expf(-x)); break;
    case TAU_DXB_SIGMA_EXP:      v = expf(fminf(x, 20.f)); break;
    default:                     v = fmaxf(x, 0.f); break;  // relu
  }
  return fmaxf(v, kClampMin);
}

__device__ __forceinline__ float sigma_prime_precise(int sid, float x) {
  float v;
  switch (sid) {
    case TAU_DXB_SIGMA_SOFTPLUS: v = 1.f / (1.f + expf(-x)); break;
    case TAU_DXB_SIGMA_SIGMOID: { float s = 1.f / (1.f + expf(-x)); v = s * (1.f - s); } break;
    case TAU_DXB_SIGMA_EXP:      v = expf(fminf(x, 15.f)); break;
    default:                     v = x > 0.f ? 1.f : 0.f; break;
  }
  return fmaxf(v, kClampMin);
}

__device__ __forceinline__ float softplus_precise(float x) {
  return x > 20.f ? x : log1pf(expf(x));
}

constexpr float kMaskMin = -3.40282346638528859812e+38f;  // finfo(float32).min

}  // namespace taudxb
