// Shared helpers for the Atlas scan kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "atlas_scan.h"

namespace atlas {

// Polar Express coefficients, atlas_jax/memory_layer.py:34-40.
#define ATLAS_PE_COEFFS                                        \
  {                                                            \
    {8.156554524902461, -22.48329292557795, 15.878769915207462},   \
    {4.042929935166739, -2.808917465908714, 0.5000178451051316},   \
    {3.8916678022926607, -2.772484153217685, 0.5060648178503393},  \
    {3.285753657755655, -2.3681294933425376, 0.46449024233003106}, \
    {2.3465413258596377, -1.7097828382687081, 0.42323551169305323} \
  }
__constant__ double kPE[5][3] = ATLAS_PE_COEFFS;
// host copy (launch-time epilogue coefficients)
constexpr double kPEHost[5][3] = ATLAS_PE_COEFFS;

// Kernels whose bounded waits expire record ATLAS_ERR_DEVICE_TIMEOUT in the
// library's device status word (passed to them as a pointer) and return
// instead of hanging.
__device__ __forceinline__ void set_status(int* st, int code) {
  if (st) atomicMax(st, code);
}

// ---- activation element access ------------------------------------------------
template <typename T> __device__ __forceinline__ float ld_act(const T* p, size_t i);
template <> __device__ __forceinline__ float ld_act<float>(const float* p, size_t i) { return p[i]; }
template <> __device__ __forceinline__ float ld_act<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) {
  return __bfloat162float(p[i]);
}
template <typename T> __device__ __forceinline__ void st_act(T* p, size_t i, float v);
template <> __device__ __forceinline__ void st_act<float>(float* p, size_t i, float v) { p[i] = v; }
template <> __device__ __forceinline__ void st_act<__nv_bfloat16>(__nv_bfloat16* p, size_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

// ---- GELU family (memory_layer.py:225-230, jax.nn.gelu approximate=True) ------
template <typename R> __device__ __forceinline__ R gelu_tanh(R x) {
  const R k0 = R(0.7978845608028654);  // sqrt(2/pi)
  R u = k0 * (x + R(0.044715) * x * x * x);
  return R(0.5) * x * (R(1) + tanh(u));
}
template <typename R> __device__ __forceinline__ R gelu_tanh_grad(R x) {
  const R k0 = R(0.7978845608028654);
  R u = k0 * (x + R(0.044715) * x * x * x);
  R t = tanh(u);
  R du = k0 * (R(1) + R(3 * 0.044715) * x * x);
  return R(0.5) * (R(1) + t) + R(0.5) * x * (R(1) - t * t) * du;
}
// exact d/dx [x Phi(x)] = Phi(x) + x phi(x)
template <typename R> __device__ __forceinline__ R gelu_erf_prime(R x) {
  R cdf = R(0.5) * (R(1) + erf(x * R(0.7071067811865476)));
  R pdf = exp(R(-0.5) * x * x) * R(0.3989422804014327);
  return cdf + x * pdf;
}
// d/dx of gelu_erf_prime = (2 - x^2) phi(x)
template <typename R> __device__ __forceinline__ R gelu_erf_second(R x) {
  R pdf = exp(R(-0.5) * x * x) * R(0.3989422804014327);
  return (R(2) - x * x) * pdf;
}

// Gate values at padded positions follow memory_layer.py:655-659.
struct Gates {
  float a, e, t, g;
};
__device__ __forceinline__ Gates load_gates(const float* alpha, const float* eta, const float* theta,
                                            const float* gamma, int T, int H, int b, int h, int tok) {
  Gates G;
  if (tok < T) {
    size_t i = ((size_t)b * T + tok) * H + h;
    G.a = alpha[i];
    G.e = eta[i];
    G.t = theta[i];
    G.g = gamma ? gamma[i] : 1.0f;
  } else {
    G.a = 1.f; G.e = 0.f; G.t = 0.f; G.g = 0.f;
  }
  return G;
}

}  // namespace atlas
