// gemm_simt.cu -- FP32 CUDA-core GEMM with bias for layouts the tensor-core
// path cannot address with TMA (unaligned row pitch such as k = 65, or no
// unit-stride dimension) and for CT_PRECISION_FP32.  Same contract as
// fused_multiply_add (Transformer_kernels/fused_multiply_add.cuh:10-93):
// out[b] = x[b] @ W[b or 0] + bias with arbitrary input strides and a dense
// [batch, m, n] output.
//
// 64 x 64 output tile per CTA, 256 threads each owning a 4 x 4 block, K
// staged through shared memory 16 at a time.  The fused options of
// ct_linear_fwd_ex (GELU epilogues, accumulate) apply in the store; the W
// column sums run as a separate kernel.
#include "act.cuh"
#include "ct_internal.h"

namespace ct {
namespace {

constexpr int kTM = 64, kTN = 64, kTK = 16;

__global__ void __launch_bounds__(256)
    gemm_bias_simt_kernel(const float* __restrict__ x, int64_t xs0, int64_t xs1, int64_t xs2,
                          const float* __restrict__ w, int64_t ws0, int64_t ws1, int64_t ws2,
                          const float* __restrict__ bias, int64_t bs, float* __restrict__ out,
                          int64_t m, int64_t k, int64_t n, int epi, float* __restrict__ out_act,
                          const float* __restrict__ act_in, int accumulate) {
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
      if (gn >= n) continue;
      const int64_t o = (b * m + gm) * n + gn;
      float v = acc[i][j] + __ldg(bias + gn * bs);
      if (epi == CT_EPILOGUE_GELU_GRAD) v *= gelu_d(__ldg(act_in + o));
      if (accumulate) v += out[o];
      out[o] = v;
      if (epi == CT_EPILOGUE_GELU) out_act[o] = gelu_f(v);
    }
  }
}

// cs[j] (+)= sum over (b, kk) of W[b | 0][kk][j]: 32 columns per CTA, eight
// row groups summed in parallel and combined in a fixed order.
__global__ void __launch_bounds__(256)
    w_colsum_simt_kernel(const float* __restrict__ w, int64_t ws0, int64_t ws1, int64_t ws2,
                         int64_t batch, int64_t k, int64_t n, float* __restrict__ cs,
                         int accumulate) {
  __shared__ float part[8][32];
  const int c = threadIdx.x % 32, g = threadIdx.x / 32;
  const int64_t j = (int64_t)blockIdx.x * 32 + c;
  float acc = 0.0f;
  if (j < n) {
    for (int64_t b = 0; b < batch; ++b)
      for (int64_t kk = g; kk < k; kk += 8) acc += __ldg(w + b * ws0 + kk * ws1 + j * ws2);
  }
  part[g][c] = acc;
  __syncthreads();
  if (g == 0 && j < n) {
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += part[i][c];
    cs[j] = accumulate ? cs[j] + t : t;
  }
}

}  // namespace

int launch_w_colsum_simt(const GemmProblem& g, cudaStream_t st) {
  if (!g.w_colsum || g.n <= 0) return CT_OK;
  w_colsum_simt_kernel<<<(unsigned)((g.n + 31) / 32), 256, 0, st>>>(
      g.w, g.ws[0], g.ws[1], g.ws[2], g.batch, g.k, g.n, g.w_colsum, g.accumulate ? 1 : 0);
  return check_launch();
}

int launch_linear_simt(const GemmProblem& g, cudaStream_t st) {
  if (g.batch > 65535 || (g.m + kTM - 1) / kTM > 65535) return CT_ERR_INVALID_ARGUMENT;
  dim3 grid((unsigned)((g.n + kTN - 1) / kTN), (unsigned)((g.m + kTM - 1) / kTM),
            (unsigned)g.batch);
  gemm_bias_simt_kernel<<<grid, 256, 0, st>>>(g.x, g.xs[0], g.xs[1], g.xs[2], g.w, g.ws[0],
                                              g.ws[1], g.ws[2], g.bias, g.bias_s, g.out, g.m, g.k,
                                              g.n, g.epilogue, g.out_act, g.act_in,
                                              g.accumulate ? 1 : 0);
  return check_launch();
}

}  // namespace ct
