// Shared device helpers for the Mamba-3 B200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mamba3_b200.h"

namespace m3 {

constexpr float kPi = 3.14159265358979323846f;
constexpr float kTwoPi = 6.28318530717958647692f;
constexpr float kLog2e = 1.44269504088896340736f;
constexpr float kAFloor = 1e-4f;  // mamba3/model.py:22
constexpr int kPhaseBlock = 64;   // mamba3/model.py:25

enum DeviceError : int {
  kErrNone = 0,
  kErrMbarTimeout = 1,
};

// ---------------------------------------------------------------------------
// dtype helpers
// ---------------------------------------------------------------------------

template <typename T> struct DType;
template <> struct DType<float> { static constexpr int id = M3_F32; };
template <> struct DType<__half> { static constexpr int id = M3_F16; };
template <> struct DType<__nv_bfloat16> { static constexpr int id = M3_BF16; };

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Round an fp32 value to the activation dtype and back: reproduces the rounding that the
// reference's activation-dtype tensor ops perform (identity for fp32).
template <typename T> __device__ __forceinline__ float rnd(float x) { return to_f(from_f<T>(x)); }

// Load element `idx` of a tensor whose dtype is only known at run time (scalars, params).
__device__ __forceinline__ float ld_any(const void* p, int dtype, int64_t idx) {
  if (dtype == M3_F32) return static_cast<const float*>(p)[idx];
  if (dtype == M3_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
  return __half2float(static_cast<const __half*>(p)[idx]);
}

__device__ __forceinline__ float ld_t(const m3_tensor& t, int64_t idx) { return ld_any(t.data, t.dtype, idx); }

// Store `v` (rounded to nearest) as element `idx` of a tensor whose dtype is known at run time.
__device__ __forceinline__ void st_t(const m3_tensor& t, int64_t idx, float v) {
  if (t.dtype == M3_F32) static_cast<float*>(t.data)[idx] = v;
  else if (t.dtype == M3_BF16) static_cast<__nv_bfloat16*>(t.data)[idx] = __float2bfloat16_rn(v);
  else static_cast<__half*>(t.data)[idx] = __float2half_rn(v);
}

// ---------------------------------------------------------------------------
// Scalar maps (mamba3/model.py:195-198, mamba3/ops.py:28-32)
// ---------------------------------------------------------------------------

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// torch.nn.functional.softplus with beta=1, threshold=20.
__device__ __forceinline__ float softplusf_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

__device__ __forceinline__ float heavy_tailf(float x) { return x >= 0.0f ? 1.0f + x : 1.0f / (1.0f - x); }

__device__ __forceinline__ float siluf_(float x) { return x * sigmoidf_(x); }

// Approximate 2^x (MUFU); used only for decay factors that are rounded to bf16/fp16.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_incl_scan(float v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    float n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

}  // namespace m3
