// fa2_simt.cu -- FlashAttention-2 forward and backward on the CUDA cores in
// FP32 (FFMA).  Serves head dims the tensor-core backward does not cover yet
// (D = 128) and the CT_PRECISION_FP32 mode.  Same math as
// Transformer_kernels/flash_attention.cuh (fwd :27-170, dq :216-354,
// dk_dv :357-504) including the causal tile skip in all three passes.
//
// Layout: a CTA owns ROWS stationary rows, one warp per row at a time; the
// streamed K/V (or Q/dO) tile of 32 rows sits in shared memory with a padded
// row pitch (D + 1) so lane j reading row j hits distinct banks.  Lane j owns
// column j of the 32-wide score tile; head-dim outputs are spread over lanes
// (d = lane + 32 * i).
#include <cmath>

#include "ct_internal.h"

namespace ct {
namespace {

constexpr int kSRows = 16;     // stationary rows per CTA (forward)
constexpr int kBRows = 8;      // stationary rows per CTA (backward: two stationary tiles)
constexpr int kSWarps = 4;
constexpr int kSTile = 32;     // streamed rows per tile

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

struct P4 {
  const float* p;
  int64_t s0, s1, s2, s3;
  __device__ __forceinline__ float at(int64_t b, int64_t h, int64_t t, int d) const {
    return __ldg(p + b * s0 + h * s1 + t * s2 + d * s3);
  }
};

// Loads rows [t0, t0 + n) of a [B,H,T,D] tensor into smem[n][D + 1].
template <int D>
__device__ __forceinline__ void stage_rows(float* sm, const P4& t, int64_t b, int64_t h, int t0,
                                           int n, int T) {
  for (int e = threadIdx.x; e < n * D; e += blockDim.x) {
    const int r = e / D, d = e % D;
    sm[r * (D + 1) + d] = (t0 + r < T) ? t.at(b, h, t0 + r, d) : 0.0f;
  }
}

template <int D>
__global__ void __launch_bounds__(kSWarps * 32)
    fa2_fwd_simt_kernel(P4 q, P4 k, P4 v, float* __restrict__ o, float* __restrict__ lse, int H,
                        int T, int causal, float scale) {
  constexpr int DL = D / 32;
  __shared__ float qs[kSRows * (D + 1)];
  __shared__ float ks[kSTile * (D + 1)];
  __shared__ float vs[kSTile * (D + 1)];
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * kSRows;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  stage_rows<D>(qs, q, b, h, q0, kSRows, T);
  float acc[kSRows / kSWarps][DL];
  float m[kSRows / kSWarps], l[kSRows / kSWarps];
#pragma unroll
  for (int i = 0; i < kSRows / kSWarps; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int c = 0; c < DL; ++c) acc[i][c] = 0.0f;
  }
  const int last = min(q0 + kSRows - 1, T - 1);
  const int kv_end = causal ? last + 1 : T;
  for (int kv0 = 0; kv0 < kv_end; kv0 += kSTile) {
    __syncthreads();
    stage_rows<D>(ks, k, b, h, kv0, kSTile, T);
    stage_rows<D>(vs, v, b, h, kv0, kSTile, T);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kSRows / kSWarps; ++i) {
      const int r = warp + kSWarps * i, row = q0 + r;
      const int kv = kv0 + lane;
      float s = 0.0f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) s += qs[r * (D + 1) + d] * ks[lane * (D + 1) + d];
      s *= scale;
      if (!(kv < T && (!causal || kv <= row))) s = -INFINITY;
      const float mn = fmaxf(m[i], wmax(s));
      const float p = (mn == -INFINITY) ? 0.0f : expf(s - mn);
      const float alpha = (m[i] == -INFINITY) ? 0.0f : expf(m[i] - mn);
      l[i] = l[i] * alpha + wsum(p);
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < DL; ++c) acc[i][c] *= alpha;
      for (int j = 0; j < kSTile; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
        for (int c = 0; c < DL; ++c) acc[i][c] += pj * vs[j * (D + 1) + lane + 32 * c];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kSRows / kSWarps; ++i) {
    const int row = q0 + warp + kSWarps * i;
    if (row < T) {
      float* orow = o + ((int64_t)bh * T + row) * D;
#pragma unroll
      for (int c = 0; c < DL; ++c) orow[lane + 32 * c] = acc[i][c] / l[i];
      if (lane == 0) lse[(int64_t)bh * T + row] = m[i] + logf(l[i]);
    }
  }
}

template <int D>
__global__ void __launch_bounds__(kSWarps * 32)
    fa2_dq_simt_kernel(P4 q, P4 k, P4 v, P4 dO, const float* __restrict__ lse, int64_t l0,
                       int64_t l1, int64_t l2, const float* __restrict__ delta,
                       float* __restrict__ dq, int H, int T, int causal, float scale) {
  constexpr int DL = D / 32;
  __shared__ float qs[kBRows * (D + 1)];
  __shared__ float gs[kBRows * (D + 1)];
  __shared__ float ks[kSTile * (D + 1)];
  __shared__ float vs[kSTile * (D + 1)];
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * kBRows;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  stage_rows<D>(qs, q, b, h, q0, kBRows, T);
  stage_rows<D>(gs, dO, b, h, q0, kBRows, T);
  float acc[kBRows / kSWarps][DL];
  float lr[kBRows / kSWarps], dr[kBRows / kSWarps];
#pragma unroll
  for (int i = 0; i < kBRows / kSWarps; ++i) {
    const int row = q0 + warp + kSWarps * i;
    lr[i] = row < T ? __ldg(lse + b * l0 + h * l1 + (int64_t)row * l2) : 0.0f;
    dr[i] = row < T ? __ldg(delta + (int64_t)bh * T + row) : 0.0f;
#pragma unroll
    for (int c = 0; c < DL; ++c) acc[i][c] = 0.0f;
  }
  const int last = min(q0 + kBRows - 1, T - 1);
  const int kv_end = causal ? last + 1 : T;
  for (int kv0 = 0; kv0 < kv_end; kv0 += kSTile) {
    __syncthreads();
    stage_rows<D>(ks, k, b, h, kv0, kSTile, T);
    stage_rows<D>(vs, v, b, h, kv0, kSTile, T);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kBRows / kSWarps; ++i) {
      const int r = warp + kSWarps * i, row = q0 + r;
      const int kv = kv0 + lane;
      float s = 0.0f, dp = 0.0f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) {
        s += qs[r * (D + 1) + d] * ks[lane * (D + 1) + d];
        dp += gs[r * (D + 1) + d] * vs[lane * (D + 1) + d];
      }
      const bool keep = kv < T && row < T && (!causal || kv <= row);
      const float p = keep ? expf(s * scale - lr[i]) : 0.0f;
      const float ds = p * (dp - dr[i]);
      for (int j = 0; j < kSTile; ++j) {
        const float dj = __shfl_sync(0xffffffffu, ds, j);
#pragma unroll
        for (int c = 0; c < DL; ++c) acc[i][c] += dj * ks[j * (D + 1) + lane + 32 * c];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kBRows / kSWarps; ++i) {
    const int row = q0 + warp + kSWarps * i;
    if (row < T) {
      float* out = dq + ((int64_t)bh * T + row) * D;
#pragma unroll
      for (int c = 0; c < DL; ++c) out[lane + 32 * c] = acc[i][c] * scale;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(kSWarps * 32)
    fa2_dkdv_simt_kernel(P4 q, P4 k, P4 v, P4 dO, const float* __restrict__ lse, int64_t l0,
                         int64_t l1, int64_t l2, const float* __restrict__ delta,
                         float* __restrict__ dk, float* __restrict__ dv, int H, int T, int causal,
                         float scale) {
  constexpr int DL = D / 32;
  __shared__ float ksm[kBRows * (D + 1)];
  __shared__ float vsm[kBRows * (D + 1)];
  __shared__ float qs[kSTile * (D + 1)];
  __shared__ float gs[kSTile * (D + 1)];
  __shared__ float ls[kSTile], ds_[kSTile];
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int k0 = blockIdx.x * kBRows;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  stage_rows<D>(ksm, k, b, h, k0, kBRows, T);
  stage_rows<D>(vsm, v, b, h, k0, kBRows, T);
  float ak[kBRows / kSWarps][DL], av[kBRows / kSWarps][DL];
#pragma unroll
  for (int i = 0; i < kBRows / kSWarps; ++i)
#pragma unroll
    for (int c = 0; c < DL; ++c) ak[i][c] = av[i][c] = 0.0f;
  const int q_begin = causal ? (k0 / kSTile) * kSTile : 0;
  for (int qs0 = q_begin; qs0 < T; qs0 += kSTile) {
    __syncthreads();
    stage_rows<D>(qs, q, b, h, qs0, kSTile, T);
    stage_rows<D>(gs, dO, b, h, qs0, kSTile, T);
    for (int e = threadIdx.x; e < kSTile; e += blockDim.x) {
      const int t = qs0 + e;
      ls[e] = t < T ? __ldg(lse + b * l0 + h * l1 + (int64_t)t * l2) : 0.0f;
      ds_[e] = t < T ? __ldg(delta + (int64_t)bh * T + t) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kBRows / kSWarps; ++i) {
      const int r = warp + kSWarps * i, kvrow = k0 + r;
      const int qi = qs0 + lane;
      float s = 0.0f, dp = 0.0f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) {
        s += qs[lane * (D + 1) + d] * ksm[r * (D + 1) + d];
        dp += gs[lane * (D + 1) + d] * vsm[r * (D + 1) + d];
      }
      const bool keep = qi < T && kvrow < T && (!causal || qi >= kvrow);
      const float p = keep ? expf(s * scale - ls[lane]) : 0.0f;
      const float dsv = p * (dp - ds_[lane]);
      for (int j = 0; j < kSTile; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const float dj = __shfl_sync(0xffffffffu, dsv, j);
#pragma unroll
        for (int c = 0; c < DL; ++c) {
          av[i][c] += pj * gs[j * (D + 1) + lane + 32 * c];
          ak[i][c] += dj * qs[j * (D + 1) + lane + 32 * c];
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kBRows / kSWarps; ++i) {
    const int row = k0 + warp + kSWarps * i;
    if (row < T) {
      float* pk = dk + ((int64_t)bh * T + row) * D;
      float* pv = dv + ((int64_t)bh * T + row) * D;
#pragma unroll
      for (int c = 0; c < DL; ++c) {
        pk[lane + 32 * c] = ak[i][c] * scale;
        pv[lane + 32 * c] = av[i][c];
      }
    }
  }
}

P4 to_p4(const Strided4& t) { return P4{t.ptr, t.s[0], t.s[1], t.s[2], t.s[3]}; }

dim3 simt_grid(const Fa2Problem& p, int rows) {
  return dim3((unsigned)((p.T + rows - 1) / rows), (unsigned)(p.B * p.H));
}

}  // namespace

int launch_fa2_fwd_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, float* o,
                        float* lse, cudaStream_t st) {
  if (p.B * p.H > 65535) return CT_ERR_INVALID_ARGUMENT;
  const float scale = (float)(1.0 / std::sqrt((double)p.D));
  const dim3 g = simt_grid(p, kSRows);
  const int c = p.causal ? 1 : 0;
  switch (p.D) {
    case 32: fa2_fwd_simt_kernel<32><<<g, kSWarps * 32, 0, st>>>(to_p4(q), to_p4(k), to_p4(v), o, lse, (int)p.H, (int)p.T, c, scale); break;
    case 64: fa2_fwd_simt_kernel<64><<<g, kSWarps * 32, 0, st>>>(to_p4(q), to_p4(k), to_p4(v), o, lse, (int)p.H, (int)p.T, c, scale); break;
    case 128: fa2_fwd_simt_kernel<128><<<g, kSWarps * 32, 0, st>>>(to_p4(q), to_p4(k), to_p4(v), o, lse, (int)p.H, (int)p.T, c, scale); break;
    default: return CT_ERR_UNSUPPORTED_HEAD_DIM;
  }
  return check_launch();
}

int launch_fa2_bwd_dq_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 dO,
                           const float* lse, const int64_t ls[3], const float* delta, float* dq,
                           cudaStream_t st) {
  if (p.B * p.H > 65535) return CT_ERR_INVALID_ARGUMENT;
  const float scale = (float)(1.0 / std::sqrt((double)p.D));
  const dim3 g = simt_grid(p, kBRows);
  const int c = p.causal ? 1 : 0;
#define CT_DQ(DD)                                                                          \
  fa2_dq_simt_kernel<DD><<<g, kSWarps * 32, 0, st>>>(to_p4(q), to_p4(k), to_p4(v),         \
                                                     to_p4(dO), lse, ls[0], ls[1], ls[2],  \
                                                     delta, dq, (int)p.H, (int)p.T, c, scale)
  switch (p.D) {
    case 32: CT_DQ(32); break;
    case 64: CT_DQ(64); break;
    case 128: CT_DQ(128); break;
    default: return CT_ERR_UNSUPPORTED_HEAD_DIM;
  }
#undef CT_DQ
  return check_launch();
}

int launch_fa2_bwd_dkdv_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v,
                             Strided4 dO, const float* lse, const int64_t ls[3],
                             const float* delta, float* dk, float* dv, cudaStream_t st) {
  if (p.B * p.H > 65535) return CT_ERR_INVALID_ARGUMENT;
  const float scale = (float)(1.0 / std::sqrt((double)p.D));
  const dim3 g = simt_grid(p, kBRows);
  const int c = p.causal ? 1 : 0;
#define CT_DKDV(DD)                                                                           \
  fa2_dkdv_simt_kernel<DD><<<g, kSWarps * 32, 0, st>>>(to_p4(q), to_p4(k), to_p4(v),          \
                                                       to_p4(dO), lse, ls[0], ls[1], ls[2],   \
                                                       delta, dk, dv, (int)p.H, (int)p.T, c,  \
                                                       scale)
  switch (p.D) {
    case 32: CT_DKDV(32); break;
    case 64: CT_DKDV(64); break;
    case 128: CT_DKDV(128); break;
    default: return CT_ERR_UNSUPPORTED_HEAD_DIM;
  }
#undef CT_DKDV
  return check_launch();
}

}  // namespace ct
