// act.cuh -- erf-GELU and its derivative, shared by the element-wise kernels
// (rowops.cu) and the linear layer's fused epilogues (gemm_tc.cu,
// gemm_simt.cu).
//
// gelu / gelu_bwd (Transformer_kernels/GeLU.cuh:7-29): y = x * Phi(x) and
// dx = dy * (Phi(x) + x * phi(x)), phi(x) = exp(-x^2 / 2) / sqrt(2 pi).
// Phi(x) = (1 + erf(x / sqrt 2)) / 2, the form torch's exact GELU uses; erff
// costs fewer instructions than normcdff, which keeps the element-wise kernels
// at the memory bound (normcdff's extra accuracy is in the far negative tail,
// where the products are below 1e-6 in absolute value).
#pragma once

namespace ct {

__device__ __forceinline__ float phi_cdf(float x) {
  return fmaf(0.5f, erff(x * 0.7071067811865476f), 0.5f);
}
__device__ __forceinline__ float gelu_f(float x) { return x * phi_cdf(x); }
// d gelu(x) / dx
__device__ __forceinline__ float gelu_d(float x) {
  const float inv_sqrt_2pi = 0.3989422804014327f;
  return phi_cdf(x) + x * inv_sqrt_2pi * expf(-0.5f * x * x);
}
__device__ __forceinline__ float gelu_g(float x, float dy) { return dy * gelu_d(x); }

}  // namespace ct
