// gemm_simt.cu -- FP32 CUDA-core GEMM with bias for layouts the tensor-core
// path cannot address with TMA (unaligned row pitch such as k = 65, or no
// unit-stride dimension) and for CT_PRECISION_FP32.  Same contract as
// fused_multiply_add (Transformer_kernels/fused_multiply_add.cuh:10-93):
// out[b] = x[b] @ W[b or 0] + bias with arbitrary input strides and a dense
// [batch, m, n] output.
//
// 64 x 64 output tile per CTA, 256 threads each owning a 4 x 4 block, K
// staged through shared memory 16 at a time.
#include "ct_internal.h"

namespace ct {
namespace {

constexpr int kTM = 64, kTN = 64, kTK = 16;

__global__ void __launch_bounds__(256)
    gemm_bias_simt_kernel(const float* __restrict__ x, int64_t xs0, int64_t xs1, int64_t xs2,
                          const float* __restrict__ w, int64_t ws0, int64_t ws1, int64_t ws2,
                          const float* __restrict__ bias, int64_t bs, float* __restrict__ out,
                          int64_t m, int64_t k, int64_t n) {
  __shared__ float As[kTK][kTM + 4];
  __shared__ float Bs[kTK][kTN + 4];
  const int64_t b = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * kTM, n0 = (int64_t)blockIdx.x * kTN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const float* xb = x + b * xs0;
  const float* wb = w + b * ws0;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < k; k0 += kTK) {
    for (int e = threadIdx.x; e < kTK * kTM; e += 256) {
      const int kk = e % kTK, mm = e / kTK;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < m && gk < k) ? __ldg(xb + gm * xs1 + gk * xs2) : 0.0f;
    }
    for (int e = threadIdx.x; e < kTK * kTN; e += 256) {
      const int nn = e % kTN, kk = e / kTN;
      const int64_t gn = n0 + nn, gk = k0 + kk;
      Bs[kk][nn] = (gn < n && gk < k) ? __ldg(wb + gk * ws1 + gn * ws2) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kTK; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bb[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * bb[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty * 4 + i;
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx * 4 + j;
      if (gn < n) out[(b * m + gm) * n + gn] = acc[i][j] + __ldg(bias + gn * bs);
    }
  }
}

}  // namespace

int launch_linear_simt(const GemmProblem& g, cudaStream_t st) {
  if (g.batch > 65535 || (g.m + kTM - 1) / kTM > 65535) return CT_ERR_INVALID_ARGUMENT;
  dim3 grid((unsigned)((g.n + kTN - 1) / kTN), (unsigned)((g.m + kTM - 1) / kTM),
            (unsigned)g.batch);
  gemm_bias_simt_kernel<<<grid, 256, 0, st>>>(g.x, g.xs[0], g.xs[1], g.xs[2], g.w, g.ws[0],
                                              g.ws[1], g.ws[2], g.bias, g.bias_s, g.out, g.m, g.k,
                                              g.n);
  return check_launch();
}

}  // namespace ct
