// common.cuh — device arithmetic shared by the GEMM epilogue and the
// elementwise/row kernels.
#pragma once
#include <cuda_runtime.h>

#include "../../include/oxf.h"

namespace oxf {

// apply_binary, src/cuda/device/elementwise.rs:5-13.
__device__ __forceinline__ float apply_binary(float lhs, float rhs, int op) {
  switch (op) {
    case OXF_ADD: return lhs + rhs;
    case OXF_SUB: return lhs - rhs;
    case OXF_MUL: return lhs * rhs;
    default: return lhs / rhs;
  }
}

// Activation::forward / derivative, src/net/linear.rs:21-70 (tanh GELU with
// GELU_SCALE = 0.7978846, GELU_CUBIC = 0.044715).
constexpr float kGeluScale = 0.7978846f;
constexpr float kGeluCubic = 0.044715f;

__device__ __forceinline__ float act_forward(int act, float x) {
  switch (act) {
    case OXF_ACT_GELU: {
      const float inner = kGeluScale * (x + kGeluCubic * x * x * x);
      return 0.5f * x * (1.0f + tanhf(inner));
    }
    case OXF_ACT_RELU: return x > 0.0f ? x : 0.0f;
    case OXF_ACT_SILU: return x / (1.0f + expf(-x));
    default: return x;
  }
}

__device__ __forceinline__ float act_derivative(int act, float x) {
  switch (act) {
    case OXF_ACT_GELU: {
      const float quad = kGeluScale * 3.0f * kGeluCubic;
      const float inner = kGeluScale * (x + kGeluCubic * x * x * x);
      const float th = tanhf(inner);
      const float dinner = kGeluScale + quad * x * x;
      return 0.5f * (1.0f + th) + 0.5f * x * (1.0f - th * th) * dinner;
    }
    case OXF_ACT_RELU: return x > 0.0f ? 1.0f : 0.0f;
    case OXF_ACT_SILU: {
      const float e = expf(-x);
      return 1.0f / (1.0f + e) + x * e / ((1.0f + e) * (1.0f + e));
    }
    default: return 1.0f;
  }
}

// Activation forms for GEMM epilogues, where each element costs issue slots
// of the few epilogue warps: tanh(u) = 1 - 2 / (exp(2u) + 1) from the
// hardware exp2-based __expf and the hardware reciprocal (rcp.approx, within
// 1 ulp). It saturates to +-1 for large |u| (1/inf = 0) without NaNs.
// Absolute error in tanh is ~2e-7, far inside the TF32 error of the
// product feeding it.
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float tanh_fast(float u) {
  const float e = __expf(2.0f * u);
  return 1.0f - 2.0f * rcp_approx(e + 1.0f);
}

__device__ __forceinline__ float act_forward_fast(int act, float x) {
  switch (act) {
    case OXF_ACT_GELU: {
      const float inner = kGeluScale * (x + kGeluCubic * x * x * x);
      return 0.5f * x * (1.0f + tanh_fast(inner));
    }
    case OXF_ACT_RELU: return x > 0.0f ? x : 0.0f;
    case OXF_ACT_SILU: return x * rcp_approx(1.0f + __expf(-x));
    default: return x;
  }
}

__device__ __forceinline__ float act_derivative_fast(int act, float x) {
  switch (act) {
    case OXF_ACT_GELU: {
      const float quad = kGeluScale * 3.0f * kGeluCubic;
      const float inner = kGeluScale * (x + kGeluCubic * x * x * x);
      const float th = tanh_fast(inner);
      const float dinner = kGeluScale + quad * x * x;
      return 0.5f * (1.0f + th) + 0.5f * x * (1.0f - th * th) * dinner;
    }
    case OXF_ACT_RELU: return x > 0.0f ? 1.0f : 0.0f;
    case OXF_ACT_SILU: {
      const float sg = rcp_approx(1.0f + __expf(-x));
      return sg + x * sg * (1.0f - sg);
    }
    default: return 1.0f;
  }
}

// Whole-chunk forms: the activation is a template constant inside the
// element loop, so the per-element switch folds away.
template <int ACT, int N>
__device__ __forceinline__ void act_forward_chunk(float (&v)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) v[j] = act_forward_fast(ACT, v[j]);
}

template <int N>
__device__ __forceinline__ void act_forward_chunk(int act, float (&v)[N]) {
  switch (act) {
    case OXF_ACT_GELU: act_forward_chunk<OXF_ACT_GELU>(v); break;
    case OXF_ACT_RELU: act_forward_chunk<OXF_ACT_RELU>(v); break;
    case OXF_ACT_SILU: act_forward_chunk<OXF_ACT_SILU>(v); break;
    default: break;
  }
}

// v[j] *= act'(x[j])
template <int ACT, int N>
__device__ __forceinline__ void act_grad_chunk(float (&v)[N], const float (&x)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) v[j] *= act_derivative_fast(ACT, x[j]);
}

template <int N>
__device__ __forceinline__ void act_grad_chunk(int act, float (&v)[N], const float (&x)[N]) {
  switch (act) {
    case OXF_ACT_GELU: act_grad_chunk<OXF_ACT_GELU>(v, x); break;
    case OXF_ACT_RELU: act_grad_chunk<OXF_ACT_RELU>(v, x); break;
    case OXF_ACT_SILU: act_grad_chunk<OXF_ACT_SILU>(v, x); break;
    default: break;
  }
}

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

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace oxf
