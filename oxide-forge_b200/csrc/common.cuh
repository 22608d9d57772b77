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
//
// The reference's 0.5·x·(1 + tanh(u)) is evaluated through the identity
// 1 + tanh(u) = 2·sigmoid(2u): GELU(x) = x / (1 + e^(-2u)), and with
// s = sigmoid(2u), 1 - tanh(u)^2 = 4·s·(1 - s) and 1 - s = e^(-2u)·s. This
// is the same function without the cancellation of 1 + tanh(u) for
// negative u, and one exponential replaces tanh. The exponent is capped at
// 80 (e^80 is finite in f32), where the sigmoid is already below 1e-34.
constexpr float kGeluScale = 0.7978846f;
constexpr float kGeluCubic = 0.044715f;

__device__ __forceinline__ float gelu_exp(float x) {
  const float inner = kGeluScale * (x + kGeluCubic * x * x * x);
  return fminf(-2.0f * inner, 80.0f);
}

__device__ __forceinline__ float act_forward(int act, float x) {
  switch (act) {
    case OXF_ACT_GELU: return x / (1.0f + expf(gelu_exp(x)));
    case OXF_ACT_RELU: return x > 0.0f ? x : 0.0f;
    case OXF_ACT_SILU: return x / (1.0f + expf(-x));
    default: return x;
  }
}

__device__ __forceinline__ float act_derivative(int act, float x) {
  switch (act) {
    case OXF_ACT_GELU: {
      const float quad = kGeluScale * 3.0f * kGeluCubic;
      const float e = expf(gelu_exp(x));
      const float sg = 1.0f / (1.0f + e);  // (1 + tanh(u)) / 2
      const float dinner = kGeluScale + quad * x * x;
      return sg * (1.0f + 2.0f * x * (e * sg) * dinner);
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
// of the few epilogue warps: the same sigmoid forms as above from the
// hardware exp2-based __expf and the hardware reciprocal (rcp.approx, within
// 1 ulp), relative error ~3e-7, far inside the TF32 error of the product
// feeding them.
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float act_forward_fast(int act, float x) {
  switch (act) {
    case OXF_ACT_GELU: return x * rcp_approx(1.0f + __expf(gelu_exp(x)));
    case OXF_ACT_RELU: return x > 0.0f ? x : 0.0f;
    case OXF_ACT_SILU: return x * rcp_approx(1.0f + __expf(-x));
    default: return x;
  }
}

__device__ __forceinline__ float act_derivative_fast(int act, float x) {
  switch (act) {
    case OXF_ACT_GELU: {
      const float quad = kGeluScale * 3.0f * kGeluCubic;
      const float e = __expf(gelu_exp(x));
      const float sg = rcp_approx(1.0f + e);
      const float dinner = kGeluScale + quad * x * x;
      return sg * (1.0f + 2.0f * x * (e * sg) * dinner);
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
