// rowops.cu -- HBM-bound row-wise kernels: softmax fwd/bwd, erf-GELU
// fwd/bwd, LayerNorm fwd/bwd, the linear layer's bias gradient and the
// FlashAttention-2 backward delta.  Each keeps a row resident in registers so
// that it is read from HBM once and written once (128-bit accesses where the
// layout allows), and every reduction over rows is a fixed-order two-stage
// sum, so results are bit-reproducible run to run.
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "act.cuh"
#include "ct_internal.h"

namespace ct {
namespace {

constexpr int kWarp = 32;

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

// Block-wide reduction for THREADS threads; `red` holds THREADS/32 floats.
template <int THREADS, bool IS_MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  if constexpr (THREADS > kWarp) {
    const int w = threadIdx.x / kWarp, l = threadIdx.x % kWarp;
    __syncthreads();  // protect `red` against the previous reduction
    if (l == 0) red[w] = v;
    __syncthreads();
    v = (l < THREADS / kWarp) ? red[l] : (IS_MAX ? -INFINITY : 0.0f);
    v = IS_MAX ? warp_max(v) : warp_sum(v);
  }
  return v;
}

// A row slice owned by one thread: V slots of 4 floats.  In vector mode slot
// j covers elements 4*(j*THREADS+tid) .. +3 (one 128-bit access); in scalar
// mode slot j, lane q covers element (4*j+q)*THREADS+tid (coalesced scalars).
template <int THREADS, int V, bool VEC>
struct RowSlice {
  float v[V][4];
  __device__ __forceinline__ static int64_t idx(int j, int q) {
    return VEC ? (int64_t)4 * (j * THREADS + (int)threadIdx.x) + q
               : (int64_t)(4 * j + q) * THREADS + (int)threadIdx.x;
  }
  __device__ __forceinline__ void load(const float* __restrict__ p, int64_t n, float fill) {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (VEC) {
        const int64_t e = idx(j, 0);
        if (e < n) {
          const float4 x = __ldg(reinterpret_cast<const float4*>(p + e));
          v[j][0] = x.x; v[j][1] = x.y; v[j][2] = x.z; v[j][3] = x.w;
        } else {
          v[j][0] = v[j][1] = v[j][2] = v[j][3] = fill;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int64_t e = idx(j, q);
          v[j][q] = e < n ? __ldg(p + e) : fill;
        }
      }
    }
  }
  __device__ __forceinline__ void store(float* __restrict__ p, int64_t n) const {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (VEC) {
        const int64_t e = idx(j, 0);
        if (e < n) *reinterpret_cast<float4*>(p + e) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int64_t e = idx(j, q);
          if (e < n) p[e] = v[j][q];
        }
      }
    }
  }
};

// ------------------------------------------------------------------ softmax
// One row per CTA (THREADS threads, up to THREADS*V*4 elements).  Follows
// naive_softmax (Transformer_kernels/softmax.cuh:25-106): max, sum of exp,
// then exp(x - max) * (1/sum); here the row is read once instead of three times.
template <int THREADS, int V, bool VEC>
__global__ void __launch_bounds__(THREADS) softmax_fwd_kernel(const float* __restrict__ x,
                                                              float* __restrict__ y, int64_t n) {
  __shared__ float red[THREADS / kWarp > 0 ? THREADS / kWarp : 1];
  const int64_t row = blockIdx.x;
  RowSlice<THREADS, V, VEC> r;
  r.load(x + row * n, n, -INFINITY);
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) m = fmaxf(m, r.v[j][q]);
  m = block_reduce<THREADS, true>(m, red);
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float e = (r.v[j][q] == -INFINITY) ? 0.0f : expf(r.v[j][q] - m);
      r.v[j][q] = e;
      s += e;
    }
  s = block_reduce<THREADS, false>(s, red);
  const float inv = 1.0f / s;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) r.v[j][q] *= inv;
  r.store(y + row * n, n);
}

// dx = p * (dp - sum(p * dp)), naive_softmax_bwd (Transformer_kernels/softmax.cuh:108-159).
template <int THREADS, int V, bool VEC>
__global__ void __launch_bounds__(THREADS) softmax_bwd_kernel(const float* __restrict__ p,
                                                              const float* __restrict__ dp,
                                                              float* __restrict__ dx, int64_t n) {
  __shared__ float red[THREADS / kWarp > 0 ? THREADS / kWarp : 1];
  const int64_t row = blockIdx.x;
  RowSlice<THREADS, V, VEC> a, b;
  a.load(p + row * n, n, 0.0f);
  b.load(dp + row * n, n, 0.0f);
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) s += a.v[j][q] * b.v[j][q];
  s = block_reduce<THREADS, false>(s, red);
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) a.v[j][q] = a.v[j][q] * (b.v[j][q] - s);
  a.store(dx + row * n, n);
}

// Rows longer than the register-resident variants: online max/sum in one
// pass, then a second pass writes exp(x - m) / s.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_fwd_long_kernel(const float* __restrict__ x,
                                                                   float* __restrict__ y,
                                                                   int64_t n) {
  __shared__ float red[THREADS / kWarp];
  const int64_t row = blockIdx.x;
  const float* xr = x + row * n;
  float m = -INFINITY, s = 0.0f;
  for (int64_t i = threadIdx.x; i < n; i += THREADS) {
    const float v = __ldg(xr + i);
    if (v > m) {
      s = (m == -INFINITY) ? 0.0f : s * expf(m - v);
      m = v;
    }
    if (v != -INFINITY) s += expf(v - m);
  }
  const float gm = block_reduce<THREADS, true>(m, red);
  s = (m == -INFINITY) ? 0.0f : s * expf(m - gm);
  s = block_reduce<THREADS, false>(s, red);
  const float inv = 1.0f / s;
  float* yr = y + row * n;
  for (int64_t i = threadIdx.x; i < n; i += THREADS) {
    const float v = __ldg(xr + i);
    yr[i] = (v == -INFINITY) ? 0.0f : expf(v - gm) * inv;
  }
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_bwd_long_kernel(const float* __restrict__ p,
                                                                   const float* __restrict__ dp,
                                                                   float* __restrict__ dx,
                                                                   int64_t n) {
  __shared__ float red[THREADS / kWarp];
  const int64_t row = blockIdx.x;
  const float* pr = p + row * n;
  const float* dr = dp + row * n;
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < n; i += THREADS) s += __ldg(pr + i) * __ldg(dr + i);
  s = block_reduce<THREADS, false>(s, red);
  float* xr = dx + row * n;
  for (int64_t i = threadIdx.x; i < n; i += THREADS) xr[i] = __ldg(pr + i) * (__ldg(dr + i) - s);
}

// ------------------------------------------------------------------ GELU
// gelu / gelu_bwd (Transformer_kernels/GeLU.cuh:7-29), math in act.cuh.

__global__ void gelu_fwd_vec(const float4* __restrict__ x, float4* __restrict__ y, int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldg(x + i);
    y[i] = make_float4(gelu_f(a.x), gelu_f(a.y), gelu_f(a.z), gelu_f(a.w));
  }
}
__global__ void gelu_bwd_vec(const float4* __restrict__ x, const float4* __restrict__ dy,
                             float4* __restrict__ dx, int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldg(x + i), g = __ldg(dy + i);
    dx[i] = make_float4(gelu_g(a.x, g.x), gelu_g(a.y, g.y), gelu_g(a.z, g.z), gelu_g(a.w, g.w));
  }
}
__global__ void gelu_fwd_scalar(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                                int64_t start) {
  for (int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = gelu_f(__ldg(x + i));
}
__global__ void gelu_bwd_scalar(const float* __restrict__ x, const float* __restrict__ dy,
                                float* __restrict__ dx, int64_t n, int64_t start) {
  for (int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dx[i] = gelu_g(__ldg(x + i), __ldg(dy + i));
}

// ---------------------------------------------------------------- LayerNorm
// One warp per row; lane holds V slots of 4 columns (the same columns for
// every row, so per-column gradient partials stay in registers).  Math of the
// reference module gpt/gpt.py:55-58: biased variance, eps inside the sqrt.
template <int V, bool VEC>
struct WarpRow {
  float v[V][4];
  __device__ __forceinline__ static int col(int lane, int j, int q) {
    return VEC ? 4 * (j * kWarp + lane) + q : (4 * j + q) * kWarp + lane;
  }
  __device__ __forceinline__ void load(const float* __restrict__ p, int n, int lane) {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (VEC) {
        const int c = col(lane, j, 0);
        if (c < n) {
          const float4 x = __ldg(reinterpret_cast<const float4*>(p + c));
          v[j][0] = x.x; v[j][1] = x.y; v[j][2] = x.z; v[j][3] = x.w;
        } else {
          v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.0f;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = col(lane, j, q);
          v[j][q] = c < n ? __ldg(p + c) : 0.0f;
        }
      }
    }
  }
  __device__ __forceinline__ void store(float* __restrict__ p, int n, int lane) const {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (VEC) {
        const int c = col(lane, j, 0);
        if (c < n) *reinterpret_cast<float4*>(p + c) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = col(lane, j, q);
          if (c < n) p[c] = v[j][q];
        }
      }
    }
  }
};

constexpr int kLnWarps = 8;

template <int V, bool VEC>
__global__ void __launch_bounds__(kLnWarps* kWarp)
    layernorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                         const float* __restrict__ beta, float* __restrict__ y,
                         float* __restrict__ mean_out, float* __restrict__ rstd_out,
                         int64_t rows, int n, float eps) {
  const int lane = threadIdx.x % kWarp;
  WarpRow<V, VEC> g, b;
  g.load(gamma, n, lane);
  b.load(beta, n, lane);
  const int64_t stride = (int64_t)gridDim.x * kLnWarps;
  int64_t row = (int64_t)blockIdx.x * kLnWarps + threadIdx.x / kWarp;
  WarpRow<V, VEC> nx;  // the next row of this warp, loaded one row ahead
  if (row < rows) nx.load(x + row * n, n, lane);
  for (; row < rows; row += stride) {
  WarpRow<V, VEC> r = nx;
  if (row + stride < rows) nx.load(x + (row + stride) * n, n, lane);
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) s += r.v[j][q];
  const float mean = warp_sum(s) / (float)n;
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = WarpRow<V, VEC>::col(lane, j, q);
      const float d = (c < n) ? r.v[j][q] - mean : 0.0f;
      ss += d * d;
    }
  const float var = warp_sum(ss) / (float)n;
  const float rstd = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) r.v[j][q] = (r.v[j][q] - mean) * rstd * g.v[j][q] + b.v[j][q];
  r.store(y + row * n, n, lane);
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
  }
}

// dx = rstd * (g - mean(g) - xhat * mean(g * xhat)), g = dy * gamma.
// Per-CTA column partials of dy*xhat and dy go to ws[blockIdx.x][2][n].
template <int V, bool VEC>
__global__ void __launch_bounds__(kLnWarps* kWarp)
    layernorm_bwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                         const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                         const float* __restrict__ dy, float* __restrict__ dx,
                         float* __restrict__ ws, int64_t rows, int n) {
  extern __shared__ float lnsm[];  // [2][n]
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  WarpRow<V, VEC> gam;
  gam.load(gamma, n, lane);
  float pg[V][4], pb[V][4];
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) pg[j][q] = pb[j][q] = 0.0f;
  const int64_t stride = (int64_t)gridDim.x * kLnWarps;
  int64_t row0 = (int64_t)blockIdx.x * kLnWarps + warp;
  WarpRow<V, VEC> nx, ng;  // next row of this warp, loaded one row ahead
  float nmu = 0.0f, nrs = 0.0f;
  if (row0 < rows) {
    nx.load(x + row0 * n, n, lane);
    ng.load(dy + row0 * n, n, lane);
    nmu = __ldg(mean_in + row0);
    nrs = __ldg(rstd_in + row0);
  }
  constexpr bool kPrefetch = V <= 4;  // wider rows would not fit two in registers
  for (int64_t row = row0; row < rows; row += stride) {
    WarpRow<V, VEC> xr = nx, g = ng;
    const float mu = nmu, rs = nrs;
    const int64_t nrow = row + stride;
    if (nrow < rows) {
      if (kPrefetch) {
        nx.load(x + nrow * n, n, lane);
        ng.load(dy + nrow * n, n, lane);
      }
      nmu = __ldg(mean_in + nrow);
      nrs = __ldg(rstd_in + nrow);
    }
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float xh = (xr.v[j][q] - mu) * rs;
        const float gg = g.v[j][q] * gam.v[j][q];
        pg[j][q] += g.v[j][q] * xh;
        pb[j][q] += g.v[j][q];
        xr.v[j][q] = xh;
        g.v[j][q] = gg;
        s1 += gg;
        s2 += gg * xh;
      }
    s1 = warp_sum(s1) / (float)n;
    s2 = warp_sum(s2) / (float)n;
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) g.v[j][q] = rs * (g.v[j][q] - s1 - xr.v[j][q] * s2);
    g.store(dx + row * n, n, lane);
    if (!kPrefetch && nrow < rows) {
      nx.load(x + nrow * n, n, lane);
      ng.load(dy + nrow * n, n, lane);
    }
  }
  // CTA-level fixed-order reduction of the per-warp column partials: warps
  // add their partials into lnsm[2][n] one after another.
  for (int w = 0; w < kLnWarps; ++w) {
    if (warp == w) {
#pragma unroll
      for (int j = 0; j < V; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = WarpRow<V, VEC>::col(lane, j, q);
          if (c < n) {
            lnsm[c] = (w == 0 ? 0.0f : lnsm[c]) + pg[j][q];
            lnsm[n + c] = (w == 0 ? 0.0f : lnsm[n + c]) + pb[j][q];
          }
        }
    }
    __syncthreads();
  }
  float* out = ws + (size_t)blockIdx.x * 2 * n;
  for (int c = threadIdx.x; c < 2 * n; c += blockDim.x) out[c] = lnsm[c];
}

// ------------------------------------------------- LayerNorm, wide rows
// Rows of 1025..8192 columns: one 256-thread CTA per row (rows taken in turn
// by a persistent grid).  Thread t holds J slots of 4 columns: 4*(j*256 + t)
// .. +3 with float4 access (VEC), else (4j + q)*256 + t.  Same math and, in
// the backward, the same workspace layout ([CTA][2][n] column partials, each
// column owned by one thread) as the one-warp-per-row kernels above.
constexpr int kLnwThreads = 256, kLnwWarps = kLnwThreads / kWarp;

template <int J, bool VEC>
struct BlockRow {
  float v[J][4];
  __device__ __forceinline__ static int col(int t, int j, int q) {
    return VEC ? 4 * (j * kLnwThreads + t) + q : (4 * j + q) * kLnwThreads + t;
  }
  __device__ __forceinline__ void load(const float* __restrict__ p, int n, int t) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (VEC) {
        const int c = col(t, j, 0);
        if (c < n) {
          const float4 a = __ldg(reinterpret_cast<const float4*>(p + c));
          v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
        } else {
          v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.0f;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = col(t, j, q);
          v[j][q] = c < n ? __ldg(p + c) : 0.0f;
        }
      }
    }
  }
  __device__ __forceinline__ void store(float* __restrict__ p, int n, int t) const {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (VEC) {
        const int c = col(t, j, 0);
        if (c < n) *reinterpret_cast<float4*>(p + c) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = col(t, j, q);
          if (c < n) p[c] = v[j][q];
        }
      }
    }
  }
};

// Sums of NV values over the CTA, in a fixed order (warp butterflies, then
// the warps' totals in warp order); every thread gets the results.
template <int NV>
__device__ __forceinline__ void block_sums(float (&v)[NV], float (*red)[kLnwWarps]) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = warp_sum(v[i]);
    if (lane == 0) red[i][warp] = v[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kLnwWarps; ++w) s += red[i][w];
    v[i] = s;
  }
  __syncthreads();  // red is reused by the next call
}

template <int J, bool VEC>
__global__ void __launch_bounds__(kLnwThreads)
    layernorm_fwd_wide_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                              const float* __restrict__ beta, float* __restrict__ y,
                              float* __restrict__ mean_out, float* __restrict__ rstd_out,
                              int64_t rows, int n, float eps) {
  __shared__ float red[1][kLnwWarps];
  const int t = threadIdx.x;
  BlockRow<J, VEC> g, b;
  g.load(gamma, n, t);
  b.load(beta, n, t);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    BlockRow<J, VEC> r;
    r.load(x + row * n, n, t);
    float s[1] = {0.0f};
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) s[0] += r.v[j][q];
    block_sums<1>(s, red);
    const float mean = s[0] / (float)n;
    float ss[1] = {0.0f};
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float d = BlockRow<J, VEC>::col(t, j, q) < n ? r.v[j][q] - mean : 0.0f;
        ss[0] += d * d;
      }
    block_sums<1>(ss, red);
    const float rstd = 1.0f / sqrtf(ss[0] / (float)n + eps);
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) r.v[j][q] = (r.v[j][q] - mean) * rstd * g.v[j][q] + b.v[j][q];
    r.store(y + row * n, n, t);
    if (t == 0) {
      if (mean_out) mean_out[row] = mean;
      if (rstd_out) rstd_out[row] = rstd;
    }
  }
}

// dx = rstd * (g - mean(g) - xhat * mean(g * xhat)), g = dy * gamma; the
// column partials of dy*xhat and dy of this CTA's rows go to ws[blockIdx.x].
template <int J, bool VEC>
__global__ void __launch_bounds__(kLnwThreads)
    layernorm_bwd_wide_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                              const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                              const float* __restrict__ dy, float* __restrict__ dx,
                              float* __restrict__ ws, int64_t rows, int n) {
  __shared__ float red[2][kLnwWarps];
  const int t = threadIdx.x;
  BlockRow<J, VEC> gam;
  gam.load(gamma, n, t);
  float pg[J][4], pb[J][4];
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) pg[j][q] = pb[j][q] = 0.0f;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    BlockRow<J, VEC> xr, g;
    xr.load(x + row * n, n, t);
    g.load(dy + row * n, n, t);
    const float mu = __ldg(mean_in + row), rs = __ldg(rstd_in + row);
    float s[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float xh = (xr.v[j][q] - mu) * rs;
        const float gg = g.v[j][q] * gam.v[j][q];
        pg[j][q] += g.v[j][q] * xh;
        pb[j][q] += g.v[j][q];
        xr.v[j][q] = xh;
        g.v[j][q] = gg;
        s[0] += gg;
        s[1] += gg * xh;
      }
    block_sums<2>(s, red);
    const float s1 = s[0] / (float)n, s2 = s[1] / (float)n;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) g.v[j][q] = rs * (g.v[j][q] - s1 - xr.v[j][q] * s2);
    g.store(dx + row * n, n, t);
  }
  float* out = ws + (size_t)blockIdx.x * 2 * n;
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = BlockRow<J, VEC>::col(t, j, q);
      if (c < n) {
        out[c] = pg[j][q];
        out[n + c] = pb[j][q];
      }
    }
}

// Sums `parts` partial rows of length `len` (row stride `len`) column-wise;
// columns [0, split) go to out_a, the rest to out_b.  A 1024-thread block
// covers 32 columns: its 32 warps take every 32nd part (eight loads in flight
// per thread), then warp 0 adds the 32 partial sums.  The order of the
// additions depends only on (parts, len), so results are reproducible.
constexpr int kCsCols = 32, kCsGroups = 32;
__global__ void __launch_bounds__(kCsCols* kCsGroups)
    column_sum_parts(const float* __restrict__ ws, int parts, int64_t len,
                     float* __restrict__ out_a, float* __restrict__ out_b, int64_t split) {
  __shared__ float red[kCsGroups][kCsCols + 1];
  const int cx = threadIdx.x % kCsCols, gy = threadIdx.x / kCsCols;
  const int64_t c = (int64_t)blockIdx.x * kCsCols + cx;
  float acc = 0.0f;
  if (c < len) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int p = gy;
    for (; p + 7 * kCsGroups < parts; p += 8 * kCsGroups) {
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] += ws[(int64_t)(p + u * kCsGroups) * len + c];
    }
    for (; p < parts; p += kCsGroups) a[0] += ws[(int64_t)p * len + c];
    acc = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
  }
  red[gy][cx] = acc;
  __syncthreads();
  if (gy == 0 && c < len) {
    float s = 0.0f;
#pragma unroll
    for (int g = 0; g < kCsGroups; ++g) s += red[g][cx];
    if (c < split) out_a[c] = s;
    else out_b[c - split] = s;
  }
}

static unsigned column_sum_grid(int64_t len) { return (unsigned)((len + kCsCols - 1) / kCsCols); }

// ------------------------------------------------------------ bias gradient
// Stage 1: a CTA of up to kBgThreads threads owns 4 * blockDim consecutive
// columns (4 per thread, float4 loads; one CTA spans a whole row when
// n <= 1536) and sums a chunk of kBgRowsPerChunk rows, all of them in flight
// per thread; it writes one partial row per chunk.  Stage 2
// (column_sum_parts) adds the chunks in fixed order.  The shape was picked by
// measurement on B200: throughput grows with the CTAs in flight, not with
// deeper per-thread loops.  Replaces the one-block-per-column warp_sum_kernel
// (Transformer_kernels/warp_sum_kernel.cuh:13-51).
constexpr int kBgThreads = 384;
constexpr int kBgRowsPerChunk = 32;
constexpr int kBgUnroll = 8;

// FLAT: the batch stride is m row strides, so row r of the flattened
// (batch * m) rows starts at r * s1 (no division per row).
template <bool VEC, bool FLAT>
__global__ void __launch_bounds__(kBgThreads)
    bias_grad_partial(const float* __restrict__ dy, int64_t s0, int64_t s1, int64_t s2, int64_t m,
                      int64_t rows, int64_t n, float* __restrict__ ws) {
  // grid.x: row chunks (may exceed 65535), grid.y: column blocks
  const int64_t c0 = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (c0 >= n) return;
  const int64_t r0 = (int64_t)blockIdx.x * kBgRowsPerChunk;
  const int64_t r1 = min(rows, r0 + kBgRowsPerChunk);
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t r = r0; r < r1; r += kBgUnroll) {
    float4 v[kBgUnroll];
#pragma unroll
    for (int u = 0; u < kBgUnroll; ++u) {  // independent loads in flight
      v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int64_t rr = r + u;
      if (rr < r1) {
        const float* p = FLAT ? dy + rr * s1 : dy + (rr / m) * s0 + (rr % m) * s1;
        if (VEC && c0 + 3 < n) {
          v[u] = __ldg(reinterpret_cast<const float4*>(p + c0));
        } else {
          v[u].x = __ldg(p + c0 * s2);
          if (c0 + 1 < n) v[u].y = __ldg(p + (c0 + 1) * s2);
          if (c0 + 2 < n) v[u].z = __ldg(p + (c0 + 2) * s2);
          if (c0 + 3 < n) v[u].w = __ldg(p + (c0 + 3) * s2);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kBgUnroll; ++u) {
      a.x += v[u].x; a.y += v[u].y; a.z += v[u].z; a.w += v[u].w;
    }
  }
  float* out = ws + (int64_t)blockIdx.x * n;
  out[c0] = a.x;
  if (c0 + 1 < n) out[c0 + 1] = a.y;
  if (c0 + 2 < n) out[c0 + 2] = a.z;
  if (c0 + 3 < n) out[c0 + 3] = a.w;
}

// ---------------------------------------------------------- FA2 bwd delta
// delta[b,h,t] = sum_d O * dO (flash_attention_bwd_delta,
// Transformer_kernels/flash_attention.cuh:175-213).  D/4 lanes share a row,
// each lane reading 4 consecutive head-dim elements.
template <int D, bool VEC>
__global__ void __launch_bounds__(256)
    fa2_delta_kernel(const float* __restrict__ o, int64_t o0, int64_t o1, int64_t o2, int64_t o3,
                     const float* __restrict__ g, int64_t g0, int64_t g1, int64_t g2, int64_t g3,
                     float* __restrict__ delta, int64_t H, int64_t T, int64_t rows) {
  constexpr int LPR = D / 4;  // lanes per row
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = tid / LPR;
  const int sub = (int)(tid % LPR);
  float acc = 0.0f;
  if (row < rows) {
    const int64_t b = row / (H * T), rem = row % (H * T), h = rem / T, t = rem % T;
    const float* po = o + b * o0 + h * o1 + t * o2;
    const float* pg = g + b * g0 + h * g1 + t * g2;
    const int d = 4 * sub;
    if (VEC) {
      const float4 x = __ldg(reinterpret_cast<const float4*>(po + d));
      const float4 y = __ldg(reinterpret_cast<const float4*>(pg + d));
      acc = x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) acc += __ldg(po + (d + q) * o3) * __ldg(pg + (d + q) * g3);
    }
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off, LPR);
  if (row < rows && sub == 0) delta[row] = acc;
}

// The same sums for dense [B,H,T,D] O and dO (unit head-dim stride, rows D
// apart): the flat row index addresses both tensors, so no index division, and
// every lane has four float4 of each tensor in flight.  Lane l's u-th load is
// float4 u*32 + l of its warp's block of 128/(D/4) rows; each row is still
// summed as four products per lane and a butterfly over the row's D/4 lanes,
// the order fa2_delta_kernel uses (identical results).
template <int D>
__global__ void __launch_bounds__(256)
    fa2_delta_dense_kernel(const float4* __restrict__ o, const float4* __restrict__ g,
                           float* __restrict__ delta, int64_t rows) {
  constexpr int F = D / 4;        // float4 per row
  constexpr int RW = 128 / F;     // rows per warp
  const int lane = threadIdx.x & 31;
  const int64_t r0 = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * RW;
  const int64_t n4 = rows * F;
  float4 x[4], y[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t i = r0 * F + u * 32 + lane;
    x[u] = i < n4 ? __ldg(o + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    y[u] = i < n4 ? __ldg(g + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    float acc = x[u].x * y[u].x + x[u].y * y[u].y + x[u].z * y[u].z + x[u].w * y[u].w;
#pragma unroll
    for (int off = F / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off, F);
    const int64_t row = r0 + (u * 32 + lane) / F;
    if ((lane % F) == 0 && row < rows) delta[row] = acc;
  }
}

template <int THREADS, int V>
int softmax_dispatch_fwd(const float* x, float* y, int64_t rows, int64_t n, bool vec,
                         cudaStream_t st) {
  if (vec) softmax_fwd_kernel<THREADS, V, true><<<(unsigned)rows, THREADS, 0, st>>>(x, y, n);
  else softmax_fwd_kernel<THREADS, V, false><<<(unsigned)rows, THREADS, 0, st>>>(x, y, n);
  return check_launch();
}
template <int THREADS, int V>
int softmax_dispatch_bwd(const float* p, const float* dp, float* dx, int64_t rows, int64_t n,
                         bool vec, cudaStream_t st) {
  if (vec) softmax_bwd_kernel<THREADS, V, true><<<(unsigned)rows, THREADS, 0, st>>>(p, dp, dx, n);
  else softmax_bwd_kernel<THREADS, V, false><<<(unsigned)rows, THREADS, 0, st>>>(p, dp, dx, n);
  return check_launch();
}

template <int V, bool VEC>
void ln_fwd_launch(const float* x, const float* g, const float* b, float* y, float* mean,
                   float* rstd, int64_t rows, int n, float eps, cudaStream_t st) {
  // persistent: about four resident CTAs per SM, each warp taking rows in turn
  const int64_t want = (rows + kLnWarps - 1) / kLnWarps;
  const unsigned grid = (unsigned)(want < 148 * 4 ? want : 148 * 4);
  layernorm_fwd_kernel<V, VEC><<<grid, kLnWarps * kWarp, 0, st>>>(x, g, b, y, mean, rstd, rows, n,
                                                                  eps);
}

// Two CTAs per SM (each warp loops over rows); the per-CTA column partials
// are then few enough for one short reduction pass.
int ln_bwd_grid(int64_t rows) {
  const int64_t want = (rows + kLnWarps - 1) / kLnWarps;
  return (int)(want < 296 ? (want < 1 ? 1 : want) : 296);
}

template <int V, bool VEC>
int ln_bwd_launch(const float* x, const float* g, const float* mean, const float* rstd,
                  const float* dy, float* dx, float* ws, int64_t rows, int n, int grid,
                  cudaStream_t st) {
  const size_t smem = (size_t)2 * n * sizeof(float);
  auto kern = layernorm_bwd_kernel<V, VEC>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return CT_ERR_CUDA;
  }
  kern<<<grid, kLnWarps * kWarp, smem, st>>>(x, g, mean, rstd, dy, dx, ws, rows, n);
  return check_launch();
}

}  // namespace

// =============================================================== launchers
int launch_softmax_fwd(const float* x, float* y, int64_t rows, int64_t n, cudaStream_t st) {
  if (rows == 0 || n == 0) return CT_OK;
  const bool vec = (n % 4 == 0) && aligned16(x) && aligned16(y);
  if (n <= 128) return softmax_dispatch_fwd<32, 1>(x, y, rows, n, vec, st);
  if (n <= 512) return softmax_dispatch_fwd<128, 1>(x, y, rows, n, vec, st);
  if (n <= 1024) return softmax_dispatch_fwd<256, 1>(x, y, rows, n, vec, st);
  if (n <= 2048) return softmax_dispatch_fwd<256, 2>(x, y, rows, n, vec, st);
  if (n <= 4096) return softmax_dispatch_fwd<256, 4>(x, y, rows, n, vec, st);
  if (n <= 8192) return softmax_dispatch_fwd<512, 4>(x, y, rows, n, vec, st);
  if (n <= 16384) return softmax_dispatch_fwd<512, 8>(x, y, rows, n, vec, st);
  softmax_fwd_long_kernel<512><<<(unsigned)rows, 512, 0, st>>>(x, y, n);
  return check_launch();
}

int launch_softmax_bwd(const float* p, const float* dp, float* dx, int64_t rows, int64_t n,
                       cudaStream_t st) {
  if (rows == 0 || n == 0) return CT_OK;
  const bool vec = (n % 4 == 0) && aligned16(p) && aligned16(dp) && aligned16(dx);
  if (n <= 128) return softmax_dispatch_bwd<32, 1>(p, dp, dx, rows, n, vec, st);
  if (n <= 512) return softmax_dispatch_bwd<128, 1>(p, dp, dx, rows, n, vec, st);
  if (n <= 1024) return softmax_dispatch_bwd<256, 1>(p, dp, dx, rows, n, vec, st);
  if (n <= 2048) return softmax_dispatch_bwd<256, 2>(p, dp, dx, rows, n, vec, st);
  if (n <= 4096) return softmax_dispatch_bwd<256, 4>(p, dp, dx, rows, n, vec, st);
  if (n <= 8192) return softmax_dispatch_bwd<512, 4>(p, dp, dx, rows, n, vec, st);
  if (n <= 16384) return softmax_dispatch_bwd<512, 8>(p, dp, dx, rows, n, vec, st);
  softmax_bwd_long_kernel<512><<<(unsigned)rows, 512, 0, st>>>(p, dp, dx, n);
  return check_launch();
}

static unsigned elementwise_grid(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = 148 * 32;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

int launch_gelu_fwd(const float* x, float* y, int64_t numel, cudaStream_t st) {
  if (numel == 0) return CT_OK;
  int64_t done = 0;
  if (aligned16(x) && aligned16(y)) {
    const int64_t n4 = numel / 4;
    if (n4 > 0) {
      gelu_fwd_vec<<<elementwise_grid(n4, 256), 256, 0, st>>>(
          reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n4);
      done = n4 * 4;
    }
  }
  if (done < numel) gelu_fwd_scalar<<<elementwise_grid(numel - done, 256), 256, 0, st>>>(x, y, numel, done);
  return check_launch();
}

int launch_gelu_bwd(const float* x, const float* dy, float* dx, int64_t numel, cudaStream_t st) {
  if (numel == 0) return CT_OK;
  int64_t done = 0;
  if (aligned16(x) && aligned16(dy) && aligned16(dx)) {
    const int64_t n4 = numel / 4;
    if (n4 > 0) {
      gelu_bwd_vec<<<elementwise_grid(n4, 256), 256, 0, st>>>(
          reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(dy),
          reinterpret_cast<float4*>(dx), n4);
      done = n4 * 4;
    }
  }
  if (done < numel)
    gelu_bwd_scalar<<<elementwise_grid(numel - done, 256), 256, 0, st>>>(x, dy, dx, numel, done);
  return check_launch();
}

int launch_layernorm_fwd(const float* x, const float* g, const float* b, float* y, float* mean,
                         float* rstd, int64_t rows, int64_t n, float eps, cudaStream_t st) {
  if (rows == 0) return CT_OK;
  if (n <= 0 || n > kLayerNormMaxCols) return CT_ERR_INVALID_ARGUMENT;
  const bool vec = (n % 4 == 0) && aligned16(x) && aligned16(g) && aligned16(b) && aligned16(y);
  const int nn = (int)n;
  if (n > 1024) {  // one CTA per row
    const unsigned grid = (unsigned)(rows < 148 * 4 ? rows : 148 * 4);
#define CT_LNW_FWD(J)                                                                       \
  (vec ? layernorm_fwd_wide_kernel<J, true><<<grid, kLnwThreads, 0, st>>>(x, g, b, y, mean, \
                                                                          rstd, rows, nn, eps) \
       : layernorm_fwd_wide_kernel<J, false><<<grid, kLnwThreads, 0, st>>>(x, g, b, y, mean, \
                                                                           rstd, rows, nn, eps))
    if (n <= 2048) CT_LNW_FWD(2);
    else if (n <= 4096) CT_LNW_FWD(4);
    else CT_LNW_FWD(8);
#undef CT_LNW_FWD
    return check_launch();
  }
#define CT_LN_FWD(V) \
  (vec ? ln_fwd_launch<V, true>(x, g, b, y, mean, rstd, rows, nn, eps, st) \
       : ln_fwd_launch<V, false>(x, g, b, y, mean, rstd, rows, nn, eps, st))
  if (n <= 128) CT_LN_FWD(1);
  else if (n <= 256) CT_LN_FWD(2);
  else if (n <= 384) CT_LN_FWD(3);
  else if (n <= 512) CT_LN_FWD(4);
  else CT_LN_FWD(8);
#undef CT_LN_FWD
  return check_launch();
}

size_t layernorm_bwd_workspace(int64_t rows, int64_t n) {
  return (size_t)ln_bwd_grid(rows) * 2 * (size_t)n * sizeof(float);
}

int launch_layernorm_bwd(const float* x, const float* g, const float* mean, const float* rstd,
                         const float* dy, float* dx, float* dg, float* db, int64_t rows,
                         int64_t n, float* ws, cudaStream_t st) {
  if (n <= 0 || n > kLayerNormMaxCols) return CT_ERR_INVALID_ARGUMENT;
  if (rows == 0) {
    if (cudaMemsetAsync(dg, 0, n * sizeof(float), st) != cudaSuccess) return CT_ERR_CUDA;
    if (cudaMemsetAsync(db, 0, n * sizeof(float), st) != cudaSuccess) return CT_ERR_CUDA;
    return CT_OK;
  }
  const bool vec = (n % 4 == 0) && aligned16(x) && aligned16(g) && aligned16(dy) && aligned16(dx);
  const int nn = (int)n, grid = ln_bwd_grid(rows);
  int rc;
  if (n > 1024) {  // one CTA per row, the same [grid][2][n] partials
#define CT_LNW_BWD(J)                                                                          \
  (vec ? layernorm_bwd_wide_kernel<J, true><<<grid, kLnwThreads, 0, st>>>(x, g, mean, rstd, dy, \
                                                                          dx, ws, rows, nn)   \
       : layernorm_bwd_wide_kernel<J, false><<<grid, kLnwThreads, 0, st>>>(x, g, mean, rstd, dy, \
                                                                           dx, ws, rows, nn))
    if (n <= 2048) CT_LNW_BWD(2);
    else if (n <= 4096) CT_LNW_BWD(4);
    else CT_LNW_BWD(8);
#undef CT_LNW_BWD
    rc = check_launch();
    if (rc != CT_OK) return rc;
    column_sum_parts<<<column_sum_grid(2 * n), kCsCols * kCsGroups, 0, st>>>(ws, grid, 2 * n, dg, db, n);
    return check_launch();
  }
#define CT_LN_BWD(V) \
  rc = vec ? ln_bwd_launch<V, true>(x, g, mean, rstd, dy, dx, ws, rows, nn, grid, st) \
           : ln_bwd_launch<V, false>(x, g, mean, rstd, dy, dx, ws, rows, nn, grid, st)
  if (n <= 128) CT_LN_BWD(1);
  else if (n <= 256) CT_LN_BWD(2);
  else if (n <= 384) CT_LN_BWD(3);
  else if (n <= 512) CT_LN_BWD(4);
  else CT_LN_BWD(8);
#undef CT_LN_BWD
  if (rc != CT_OK) return rc;
  column_sum_parts<<<column_sum_grid(2 * n), kCsCols * kCsGroups, 0, st>>>(ws, grid, 2 * n, dg, db, n);
  return check_launch();
}

size_t bias_grad_workspace(int64_t rows, int64_t n) {
  const int64_t chunks = (rows + kBgRowsPerChunk - 1) / kBgRowsPerChunk;
  return (size_t)(chunks < 1 ? 1 : chunks) * (size_t)n * sizeof(float);
}

int launch_bias_grad(const float* dy, const int64_t s[3], float* db, int64_t batch, int64_t m,
                     int64_t n, float* ws, cudaStream_t st) {
  if (n == 0) return CT_OK;
  const int64_t rows = batch * m;
  if (rows == 0) return cudaMemsetAsync(db, 0, n * sizeof(float), st) == cudaSuccess ? CT_OK : CT_ERR_CUDA;
  const int64_t chunks = (rows + kBgRowsPerChunk - 1) / kBgRowsPerChunk;
  if (chunks >= (1ll << 31)) return CT_ERR_INVALID_ARGUMENT;
  const bool vec = s[2] == 1 && s[1] % 4 == 0 && s[0] % 4 == 0 && aligned16(dy);
  const int64_t quads = (n + 3) / 4;
  const unsigned th = (unsigned)std::min<int64_t>((quads + 31) / 32 * 32, kBgThreads);
  if ((quads + th - 1) / th > 65535) return CT_ERR_INVALID_ARGUMENT;
  dim3 grid((unsigned)chunks, (unsigned)((quads + th - 1) / th));
  const bool flat = batch == 1 || s[0] == m * s[1];
  if (vec && flat) bias_grad_partial<true, true><<<grid, th, 0, st>>>(dy, s[0], s[1], s[2], m, rows, n, ws);
  else if (vec) bias_grad_partial<true, false><<<grid, th, 0, st>>>(dy, s[0], s[1], s[2], m, rows, n, ws);
  else if (flat) bias_grad_partial<false, true><<<grid, th, 0, st>>>(dy, s[0], s[1], s[2], m, rows, n, ws);
  else bias_grad_partial<false, false><<<grid, th, 0, st>>>(dy, s[0], s[1], s[2], m, rows, n, ws);
  int rc = check_launch();
  if (rc != CT_OK) return rc;
  column_sum_parts<<<column_sum_grid(n), kCsCols * kCsGroups, 0, st>>>(ws, (int)chunks, n, db, db, n);
  return check_launch();
}

int launch_fa2_delta(const Fa2Problem& p, Strided4 o, Strided4 dO, float* delta, cudaStream_t st) {
  const int64_t rows = p.B * p.H * p.T;
  if (rows == 0) return CT_OK;
  const bool vec = o.s[3] == 1 && dO.s[3] == 1 && aligned16(o.ptr) && aligned16(dO.ptr) &&
                   o.s[0] % 4 == 0 && o.s[1] % 4 == 0 && o.s[2] % 4 == 0 && dO.s[0] % 4 == 0 &&
                   dO.s[1] % 4 == 0 && dO.s[2] % 4 == 0;
  const auto dense = [&](const Strided4& t) {
    return t.s[3] == 1 && t.s[2] == p.D && t.s[1] == p.T * p.D && t.s[0] == p.H * p.T * p.D &&
           aligned16(t.ptr);
  };
  if (dense(o) && dense(dO)) {
    const int64_t rows_per_cta = 8 * (128 / (p.D / 4));
    const unsigned g = (unsigned)((rows + rows_per_cta - 1) / rows_per_cta);
    const float4* o4 = reinterpret_cast<const float4*>(o.ptr);
    const float4* g4 = reinterpret_cast<const float4*>(dO.ptr);
    switch (p.D) {
      case 32: fa2_delta_dense_kernel<32><<<g, 256, 0, st>>>(o4, g4, delta, rows); break;
      case 64: fa2_delta_dense_kernel<64><<<g, 256, 0, st>>>(o4, g4, delta, rows); break;
      case 128: fa2_delta_dense_kernel<128><<<g, 256, 0, st>>>(o4, g4, delta, rows); break;
      default: return CT_ERR_UNSUPPORTED_HEAD_DIM;
    }
    return check_launch();
  }
  const int64_t threads = rows * (p.D / 4);
  const unsigned grid = (unsigned)((threads + 255) / 256);
#define CT_DELTA(DD)                                                                          \
  if (vec)                                                                                    \
    fa2_delta_kernel<DD, true><<<grid, 256, 0, st>>>(o.ptr, o.s[0], o.s[1], o.s[2], o.s[3],   \
                                                     dO.ptr, dO.s[0], dO.s[1], dO.s[2],       \
                                                     dO.s[3], delta, p.H, p.T, rows);         \
  else                                                                                        \
    fa2_delta_kernel<DD, false><<<grid, 256, 0, st>>>(o.ptr, o.s[0], o.s[1], o.s[2], o.s[3],  \
                                                      dO.ptr, dO.s[0], dO.s[1], dO.s[2],      \
                                                      dO.s[3], delta, p.H, p.T, rows);
  switch (p.D) {
    case 32: CT_DELTA(32) break;
    case 64: CT_DELTA(64) break;
    case 128: CT_DELTA(128) break;
    default: return CT_ERR_UNSUPPORTED_HEAD_DIM;
  }
#undef CT_DELTA
  return check_launch();
}


// ----------------------------------------------------------- cross entropy
// F.cross_entropy over the lm_head logits (gpt/gpt.py:170-175; the reference
// calls torch for it), forward and backward of one row together:
//   loss_row = logsumexp(x) - x[t],   dx = softmax(x) - onehot(t)
// written over x in place (the caller scales by 1 / rows afterwards).  A
// target equal to `ignore` gives loss 0 and a zero gradient row; a target
// outside [0, vocab) gives NaN (the row is poisoned, not silently wrong).
// TPR threads per row: a warp (8 rows per CTA) for short rows, the CTA for
// long ones.  Pass 1 keeps a running (max, sum of exp) per thread, combined
// across threads in a fixed order; pass 2 writes the gradient.
__device__ __forceinline__ void online_combine(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;  // both empty
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

template <int TPR, bool VEC>
__global__ void __launch_bounds__(256)
    ce_fwd_bwd_kernel(float* __restrict__ x, int64_t ld, int64_t rows, int64_t vocab,
                      const int64_t* __restrict__ targets, int64_t ignore,
                      float* __restrict__ loss_rows) {
  constexpr int RPB = 256 / TPR;  // rows per CTA
  __shared__ float red_m[256 / 32], red_s[256 / 32];
  __shared__ float sh_lse[RPB];
  const int sub = threadIdx.x / TPR, t_in = threadIdx.x % TPR;
  const int64_t row = (int64_t)blockIdx.x * RPB + sub;
  const bool live = row < rows;
  float* xr = x + (live ? row : 0) * ld;
  const int64_t tgt = live ? targets[row] : ignore;
  // pass 1: running max and sum of exp
  float m = -INFINITY, sum = 0.0f;
  if (live) {
    if constexpr (VEC) {
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      for (int64_t i = t_in; i < vocab / 4; i += TPR) {
        const float4 v = x4[i];
        const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
        if (mx > m) {
          sum *= expf(m - mx);
          m = mx;
        }
        sum += expf(v.x - m) + expf(v.y - m) + expf(v.z - m) + expf(v.w - m);
      }
    } else {
      for (int64_t i = t_in; i < vocab; i += TPR) {
        const float v = xr[i];
        if (v > m) {
          sum *= expf(m - v);
          m = v;
        }
        sum += expf(v - m);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float s2 = __shfl_xor_sync(0xffffffffu, sum, off);
    online_combine(m, sum, m2, s2);
  }
  if constexpr (TPR > 32) {
    const int w = threadIdx.x / 32;
    if ((threadIdx.x & 31) == 0) {
      red_m[w] = m;
      red_s[w] = sum;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float mm = red_m[0], ss = red_s[0];
      for (int i = 1; i < TPR / 32; ++i) online_combine(mm, ss, red_m[i], red_s[i]);
      sh_lse[0] = mm + logf(ss);
    }
  } else if (t_in == 0) {
    sh_lse[sub] = m + logf(sum);
  }
  __syncthreads();
  const float lse = sh_lse[sub];
  const bool ignored = tgt == ignore;
  const bool bad = !ignored && (tgt < 0 || tgt >= vocab);
  if (live && t_in == 0)
    loss_rows[row] = ignored ? 0.0f : (bad ? NAN : lse - xr[tgt]);
  if constexpr (TPR > 32) __syncthreads();  // x[t] read before the row is overwritten
  else __syncwarp();
  if (!live) return;
  // pass 2: dx = softmax - onehot, in place
  if constexpr (VEC) {
    float4* x4 = reinterpret_cast<float4*>(xr);
    for (int64_t i = t_in; i < vocab / 4; i += TPR) {
      float4 v = x4[i];
      if (ignored) {
        v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      } else {
        v = make_float4(expf(v.x - lse), expf(v.y - lse), expf(v.z - lse), expf(v.w - lse));
        if (bad) v = make_float4(NAN, NAN, NAN, NAN);
        if (tgt / 4 == i) {
          const int c = (int)(tgt % 4);
          if (c == 0) v.x -= 1.0f; else if (c == 1) v.y -= 1.0f; else if (c == 2) v.z -= 1.0f; else v.w -= 1.0f;
        }
      }
      x4[i] = v;
    }
  } else {
    for (int64_t i = t_in; i < vocab; i += TPR) {
      float v = ignored ? 0.0f : (bad ? NAN : expf(xr[i] - lse) - (i == tgt ? 1.0f : 0.0f));
      xr[i] = v;
    }
  }
}

int launch_cross_entropy(float* x, int64_t ld, int64_t rows, int64_t vocab, const int64_t* targets,
                         int64_t ignore, float* loss_rows, cudaStream_t st) {
  if (rows == 0) return CT_OK;
  const bool vec = (vocab % 4) == 0 && (ld % 4) == 0 && aligned16(x);
  if (vocab <= 2048) {
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (vec) ce_fwd_bwd_kernel<32, true><<<grid, 256, 0, st>>>(x, ld, rows, vocab, targets, ignore, loss_rows);
    else ce_fwd_bwd_kernel<32, false><<<grid, 256, 0, st>>>(x, ld, rows, vocab, targets, ignore, loss_rows);
  } else {
    if (rows > 0x7fffffffll) return CT_ERR_INVALID_ARGUMENT;
    const unsigned grid = (unsigned)rows;
    if (vec) ce_fwd_bwd_kernel<256, true><<<grid, 256, 0, st>>>(x, ld, rows, vocab, targets, ignore, loss_rows);
    else ce_fwd_bwd_kernel<256, false><<<grid, 256, 0, st>>>(x, ld, rows, vocab, targets, ignore, loss_rows);
  }
  return check_launch();
}

}  // namespace ct
