// fa2_simt.cu -- FlashAttention-2 forward and backward on the CUDA cores in
// FP32 (FFMA).  Serves the CT_PRECISION_FP32 mode and the head-dim-128
// backward in 3xTF32 mode (which the tensor-core kernels do not cover).  Same
// math as Transformer_kernels/flash_attention.cuh (fwd :27-170, dq :216-354,
// dk_dv :357-504) including the causal tile skip in all three passes.
//
// Layout: a CTA owns 32 stationary rows, eight per warp taken together; the
// streamed K/V (or Q/dO) tile of 32 rows sits in shared memory with a padded
// row pitch (D + 1) so lane j reading row j hits distinct banks.  Lane j owns
// column j of the 32-wide score tile; head-dim outputs are spread over lanes
// (d = lane + 32 * i).
#include <cmath>

#include "ct_internal.h"

namespace ct {
namespace {

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

P4 to_p4_(const Strided4& t) { return P4{t.ptr, t.s[0], t.s[1], t.s[2], t.s[3]}; }

// ---------------------------------------------------------- shared layout
// 32 stationary rows per CTA, 8 per warp computed together: per head-dim step
// a lane reads its streamed row once (padded pitch, conflict-free) and the
// warp's 8 stationary rows as float4 broadcasts, so a shared-memory load feeds
// about three FMAs instead of one half, and every streamed tile staged in
// shared memory serves 32 rows.  The elementwise dS (dQ pass) or P^T, dS^T
// (dK/dV pass) of the warp's rows go through a warp-private shared buffer and
// are read back as float4 broadcasts for the head-dim accumulation.
constexpr int kBRows = 32;                  // stationary rows per CTA
constexpr int kBWarpRows = kBRows / kSWarps;  // rows per warp

template <int D>
struct SimtBwdSmem {
  // stationary rows [kBRows][D] x 2 (pitch D: float4 broadcast reads), streamed
  // rows [kSTile][D + 1] x 2, then per-warp [kBWarpRows][kSTile] buffers
  static constexpr int ST = kBRows * D, SM = kSTile * (D + 1), WB = kBWarpRows * kSTile;
  static constexpr size_t bytes(int nbuf) {
    return (size_t)(2 * ST + 2 * SM + nbuf * kSWarps * WB + 2 * kSTile) * sizeof(float);
  }
};

// Rows [t0, t0 + n) of a [B,H,T,D] tensor into sm[n][PITCH] (zeros past T).
template <int D, int PITCH>
__device__ __forceinline__ void stage_rows_p(float* sm, const P4& t, int64_t b, int64_t h, int t0,
                                             int n, int T) {
  for (int e = threadIdx.x; e < n * D; e += blockDim.x) {
    const int r = e / D, d = e % D;
    sm[r * PITCH + d] = (t0 + r < T) ? t.at(b, h, t0 + r, d) : 0.0f;
  }
}

// s[i] += A[i] . x and t[i] += C[i] . y over the head dim, for the warp's 8
// stationary rows A, C (pitch D, broadcast) and this lane's streamed rows x, y
// (pitch D + 1).
template <int D>
__device__ __forceinline__ void dot8x2(const float* __restrict__ A, const float* __restrict__ C,
                                       const float* __restrict__ x, const float* __restrict__ y,
                                       float (&s)[kBWarpRows], float (&u)[kBWarpRows]) {
#pragma unroll 2
  for (int d = 0; d < D; d += 4) {
    const float x0 = x[d], x1 = x[d + 1], x2 = x[d + 2], x3 = x[d + 3];
    const float y0 = y[d], y1 = y[d + 1], y2 = y[d + 2], y3 = y[d + 3];
#pragma unroll
    for (int i = 0; i < kBWarpRows; ++i) {
      const float4 a = *reinterpret_cast<const float4*>(A + i * D + d);
      const float4 c = *reinterpret_cast<const float4*>(C + i * D + d);
      s[i] = fmaf(a.x, x0, s[i]); s[i] = fmaf(a.y, x1, s[i]);
      s[i] = fmaf(a.z, x2, s[i]); s[i] = fmaf(a.w, x3, s[i]);
      u[i] = fmaf(c.x, y0, u[i]); u[i] = fmaf(c.y, y1, u[i]);
      u[i] = fmaf(c.z, y2, u[i]); u[i] = fmaf(c.w, y3, u[i]);
    }
  }
}

// acc[i][c] += sum_j w[i][j] * M[j][lane + 32 c] over the tile's kSTile rows
// (w: this warp's [kBWarpRows][kSTile] buffer, broadcast; M pitch D + 1).
template <int D>
__device__ __forceinline__ void accum8(const float* __restrict__ w, const float* __restrict__ M,
                                       float (&acc)[kBWarpRows][D / 32], int lane) {
  constexpr int DL = D / 32;
#pragma unroll 1
  for (int j = 0; j < kSTile; j += 4) {
    float m[4][DL];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int c = 0; c < DL; ++c) m[u][c] = M[(j + u) * (D + 1) + lane + 32 * c];
#pragma unroll
    for (int i = 0; i < kBWarpRows; ++i) {
      const float4 q = *reinterpret_cast<const float4*>(w + i * kSTile + j);
#pragma unroll
      for (int c = 0; c < DL; ++c) {
        acc[i][c] = fmaf(q.x, m[0][c], acc[i][c]);
        acc[i][c] = fmaf(q.y, m[1][c], acc[i][c]);
        acc[i][c] = fmaf(q.z, m[2][c], acc[i][c]);
        acc[i][c] = fmaf(q.w, m[3][c], acc[i][c]);
      }
    }
  }
}

// s[i] += A[i] . x over the head dim (8 stationary rows A, pitch D, broadcast;
// this lane's streamed row x, pitch D + 1).
template <int D>
__device__ __forceinline__ void dot8(const float* __restrict__ A, const float* __restrict__ x,
                                     float (&s)[kBWarpRows]) {
#pragma unroll 4
  for (int d = 0; d < D; d += 4) {
    const float x0 = x[d], x1 = x[d + 1], x2 = x[d + 2], x3 = x[d + 3];
#pragma unroll
    for (int i = 0; i < kBWarpRows; ++i) {
      const float4 a = *reinterpret_cast<const float4*>(A + i * D + d);
      s[i] = fmaf(a.x, x0, s[i]); s[i] = fmaf(a.y, x1, s[i]);
      s[i] = fmaf(a.z, x2, s[i]); s[i] = fmaf(a.w, x3, s[i]);
    }
  }
}

// O, LSE per 32 query rows with the online softmax (reference
// flash_attention_fwd_kernel, :27-170): the warp's 8 rows take each K/V tile
// together; P goes through the warp's buffer into the O accumulation.
template <int D>
__global__ void __launch_bounds__(kSWarps * 32)
    fa2_fwd_simt_kernel(P4 q, P4 k, P4 v, float* __restrict__ o, float* __restrict__ lse, int H,
                        int T, int causal, float scale) {
  using L = SimtBwdSmem<D>;
  constexpr int DL = D / 32, R = kBWarpRows;
  extern __shared__ __align__(16) float sm_simt[];
  float* qs = sm_simt;
  float* ks = qs + L::ST;
  float* vs = ks + L::SM;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* pw = vs + L::SM + warp * L::WB;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * kBRows;
  stage_rows_p<D, D>(qs, q, b, h, q0, kBRows, T);
  const float* qw = qs + warp * R * D;
  float acc[R][DL], m[R], l[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int c = 0; c < DL; ++c) acc[i][c] = 0.0f;
  }
  const int last = min(q0 + kBRows - 1, T - 1);
  const int kv_end = causal ? last + 1 : T;
  for (int kv0 = 0; kv0 < kv_end; kv0 += kSTile) {
    __syncthreads();
    stage_rows_p<D, D + 1>(ks, k, b, h, kv0, kSTile, T);
    stage_rows_p<D, D + 1>(vs, v, b, h, kv0, kSTile, T);
    __syncthreads();
    float s[R];
#pragma unroll
    for (int i = 0; i < R; ++i) s[i] = 0.0f;
    dot8<D>(qw, ks + lane * (D + 1), s);
    const int kv = kv0 + lane;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int row = q0 + warp * R + i;
      float si = s[i] * scale;
      if (!(kv < T && (!causal || kv <= row))) si = -INFINITY;
      const float mn = fmaxf(m[i], wmax(si));
      const float p = (mn == -INFINITY) ? 0.0f : expf(si - mn);
      const float alpha = (m[i] == -INFINITY) ? 0.0f : expf(m[i] - mn);
      l[i] = l[i] * alpha + wsum(p);
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < DL; ++c) acc[i][c] *= alpha;
      pw[i * kSTile + lane] = p;
    }
    __syncwarp();
    accum8<D>(pw, vs, acc, lane);
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int row = q0 + warp * R + i;
    if (row < T) {
      float* orow = o + ((int64_t)bh * T + row) * D;
#pragma unroll
      for (int c = 0; c < DL; ++c) orow[lane + 32 * c] = acc[i][c] / l[i];
      if (lane == 0) lse[(int64_t)bh * T + row] = m[i] + logf(l[i]);
    }
  }
}

// dQ_i = scale * sum_j dS_ij K_j, dS = P (dP - delta), P = exp(S scale - L),
// per 32 query rows (reference flash_attention_bwd_dq, :216-354).
template <int D>
__global__ void __launch_bounds__(kSWarps * 32)
    fa2_dq_simt_kernel(P4 q, P4 k, P4 v, P4 dO, const float* __restrict__ lse, int64_t l0,
                       int64_t l1, int64_t l2, const float* __restrict__ delta,
                       float* __restrict__ dq, int H, int T, int causal, float scale) {
  using L = SimtBwdSmem<D>;
  constexpr int DL = D / 32, R = kBWarpRows;
  extern __shared__ __align__(16) float sm_simt[];
  float* qs = sm_simt;
  float* gs = qs + L::ST;
  float* ks = gs + L::ST;
  float* vs = ks + L::SM;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* dsw = vs + L::SM + warp * L::WB;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int q0 = blockIdx.x * kBRows;
  stage_rows_p<D, D>(qs, q, b, h, q0, kBRows, T);
  stage_rows_p<D, D>(gs, dO, b, h, q0, kBRows, T);
  const float* qw = qs + warp * R * D;
  const float* gw = gs + warp * R * D;
  float acc[R][DL], lr[R], dr[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int row = q0 + warp * R + i;
    lr[i] = row < T ? __ldg(lse + b * l0 + h * l1 + (int64_t)row * l2) : 0.0f;
    dr[i] = row < T ? __ldg(delta + (int64_t)bh * T + row) : 0.0f;
#pragma unroll
    for (int c = 0; c < DL; ++c) acc[i][c] = 0.0f;
  }
  const int last = min(q0 + kBRows - 1, T - 1);
  const int kv_end = causal ? last + 1 : T;
  for (int kv0 = 0; kv0 < kv_end; kv0 += kSTile) {
    __syncthreads();
    stage_rows_p<D, D + 1>(ks, k, b, h, kv0, kSTile, T);
    stage_rows_p<D, D + 1>(vs, v, b, h, kv0, kSTile, T);
    __syncthreads();
    float s[R], dp[R];
#pragma unroll
    for (int i = 0; i < R; ++i) s[i] = dp[i] = 0.0f;
    dot8x2<D>(qw, gw, ks + lane * (D + 1), vs + lane * (D + 1), s, dp);
    const int kv = kv0 + lane;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int row = q0 + warp * R + i;
      const bool keep = kv < T && row < T && (!causal || kv <= row);
      const float p = keep ? expf(s[i] * scale - lr[i]) : 0.0f;
      dsw[i * kSTile + lane] = p * (dp[i] - dr[i]);
    }
    __syncwarp();
    accum8<D>(dsw, ks, acc, lane);
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int row = q0 + warp * R + i;
    if (row < T) {
      float* out = dq + ((int64_t)bh * T + row) * D;
#pragma unroll
      for (int c = 0; c < DL; ++c) out[lane + 32 * c] = acc[i][c] * scale;
    }
  }
}

// dV_j = sum_i P_ij dO_i and dK_j = scale * sum_i dS_ij Q_i per 32 key rows,
// from the causal diagonal on (reference flash_attention_bwd_dk_dv, :357-504).
template <int D>
__global__ void __launch_bounds__(kSWarps * 32)
    fa2_dkdv_simt_kernel(P4 q, P4 k, P4 v, P4 dO, const float* __restrict__ lse, int64_t l0,
                         int64_t l1, int64_t l2, const float* __restrict__ delta,
                         float* __restrict__ dk, float* __restrict__ dv, int H, int T, int causal,
                         float scale) {
  using L = SimtBwdSmem<D>;
  constexpr int DL = D / 32, R = kBWarpRows;
  extern __shared__ __align__(16) float sm_simt[];
  float* ksm = sm_simt;
  float* vsm = ksm + L::ST;
  float* qs = vsm + L::ST;
  float* gs = qs + L::SM;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* pw = gs + L::SM + warp * L::WB;         // P^T of the warp's key rows
  float* dsw = pw + kSWarps * L::WB;             // dS^T
  float* ls = gs + L::SM + 2 * kSWarps * L::WB;  // the tile's LSE and delta
  float* dls = ls + kSTile;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int k0 = blockIdx.x * kBRows;
  stage_rows_p<D, D>(ksm, k, b, h, k0, kBRows, T);
  stage_rows_p<D, D>(vsm, v, b, h, k0, kBRows, T);
  const float* kw = ksm + warp * R * D;
  const float* vw = vsm + warp * R * D;
  float ak[R][DL], av[R][DL];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int c = 0; c < DL; ++c) ak[i][c] = av[i][c] = 0.0f;
  const int q_begin = causal ? (k0 / kSTile) * kSTile : 0;
  for (int qs0 = q_begin; qs0 < T; qs0 += kSTile) {
    __syncthreads();
    stage_rows_p<D, D + 1>(qs, q, b, h, qs0, kSTile, T);
    stage_rows_p<D, D + 1>(gs, dO, b, h, qs0, kSTile, T);
    for (int e = threadIdx.x; e < kSTile; e += blockDim.x) {
      const int t = qs0 + e;
      ls[e] = t < T ? __ldg(lse + b * l0 + h * l1 + (int64_t)t * l2) : 0.0f;
      dls[e] = t < T ? __ldg(delta + (int64_t)bh * T + t) : 0.0f;
    }
    __syncthreads();
    float s[R], dp[R];
#pragma unroll
    for (int i = 0; i < R; ++i) s[i] = dp[i] = 0.0f;
    dot8x2<D>(kw, vw, qs + lane * (D + 1), gs + lane * (D + 1), s, dp);
    const int qi = qs0 + lane;
    const float lq = ls[lane], dq_ = dls[lane];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int krow = k0 + warp * R + i;
      const bool keep = qi < T && krow < T && (!causal || qi >= krow);
      const float p = keep ? expf(s[i] * scale - lq) : 0.0f;
      pw[i * kSTile + lane] = p;
      dsw[i * kSTile + lane] = p * (dp[i] - dq_);
    }
    __syncwarp();
    accum8<D>(pw, gs, av, lane);
    accum8<D>(dsw, qs, ak, lane);
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int row = k0 + warp * R + i;
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

// Dynamic shared memory above 48 KB needs the per-kernel opt-in, once per
// device (bit d of *done).
template <class K>
int simt_smem_attr(K kernel, size_t bytes, unsigned long long* done) {
  if (bytes <= 48 * 1024) return CT_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CT_ERR_CUDA;
  const unsigned long long bit = 1ull << (dev & 63);
  if (__atomic_load_n(done, __ATOMIC_ACQUIRE) & bit) return CT_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
      cudaSuccess)
    return CT_ERR_CUDA;
  __atomic_fetch_or(done, bit, __ATOMIC_RELEASE);
  return CT_OK;
}

template <int D>
int run_fwd_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, float* o, float* lse,
                 int c, float scale, dim3 g, cudaStream_t st) {
  static unsigned long long done = 0;
  using L = SimtBwdSmem<D>;
  const size_t smem = (size_t)(L::ST + 2 * L::SM + kSWarps * L::WB) * sizeof(float);
  const int rc = simt_smem_attr(fa2_fwd_simt_kernel<D>, smem, &done);
  if (rc != CT_OK) return rc;
  fa2_fwd_simt_kernel<D><<<g, kSWarps * 32, smem, st>>>(to_p4_(q), to_p4_(k), to_p4_(v), o, lse,
                                                       (int)p.H, (int)p.T, c, scale);
  return check_launch();
}

template <int D>
int run_dq_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 dO,
                const float* lse, const int64_t ls[3], const float* delta, float* dq, int c,
                float scale, dim3 g, cudaStream_t st) {
  static unsigned long long done = 0;
  const size_t smem = SimtBwdSmem<D>::bytes(1);
  const int rc = simt_smem_attr(fa2_dq_simt_kernel<D>, smem, &done);
  if (rc != CT_OK) return rc;
  fa2_dq_simt_kernel<D><<<g, kSWarps * 32, smem, st>>>(to_p4_(q), to_p4_(k), to_p4_(v),
                                                      to_p4_(dO), lse, ls[0], ls[1], ls[2], delta,
                                                      dq, (int)p.H, (int)p.T, c, scale);
  return check_launch();
}

template <int D>
int run_dkdv_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 dO,
                  const float* lse, const int64_t ls[3], const float* delta, float* dk, float* dv,
                  int c, float scale, dim3 g, cudaStream_t st) {
  static unsigned long long done = 0;
  const size_t smem = SimtBwdSmem<D>::bytes(2);
  const int rc = simt_smem_attr(fa2_dkdv_simt_kernel<D>, smem, &done);
  if (rc != CT_OK) return rc;
  fa2_dkdv_simt_kernel<D><<<g, kSWarps * 32, smem, st>>>(to_p4_(q), to_p4_(k), to_p4_(v),
                                                        to_p4_(dO), lse, ls[0], ls[1], ls[2],
                                                        delta, dk, dv, (int)p.H, (int)p.T, c,
                                                        scale);
  return check_launch();
}

P4 to_p4(const Strided4& t) { return to_p4_(t); }

dim3 simt_grid(const Fa2Problem& p, int rows) {
  return dim3((unsigned)((p.T + rows - 1) / rows), (unsigned)(p.B * p.H));
}

}  // namespace

int launch_fa2_fwd_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, float* o,
                        float* lse, cudaStream_t st) {
  if (p.B * p.H > 65535) return CT_ERR_INVALID_ARGUMENT;
  const float scale = (float)(1.0 / std::sqrt((double)p.D));
  const dim3 g = simt_grid(p, kBRows);
  const int c = p.causal ? 1 : 0;
  switch (p.D) {
    case 32: return run_fwd_simt<32>(p, q, k, v, o, lse, c, scale, g, st);
    case 64: return run_fwd_simt<64>(p, q, k, v, o, lse, c, scale, g, st);
    case 128: return run_fwd_simt<128>(p, q, k, v, o, lse, c, scale, g, st);
    default: return CT_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

int launch_fa2_bwd_dq_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 dO,
                           const float* lse, const int64_t ls[3], const float* delta, float* dq,
                           cudaStream_t st) {
  if (p.B * p.H > 65535) return CT_ERR_INVALID_ARGUMENT;
  const float scale = (float)(1.0 / std::sqrt((double)p.D));
  const dim3 g = simt_grid(p, kBRows);
  const int c = p.causal ? 1 : 0;
  switch (p.D) {
    case 32: return run_dq_simt<32>(p, q, k, v, dO, lse, ls, delta, dq, c, scale, g, st);
    case 64: return run_dq_simt<64>(p, q, k, v, dO, lse, ls, delta, dq, c, scale, g, st);
    case 128: return run_dq_simt<128>(p, q, k, v, dO, lse, ls, delta, dq, c, scale, g, st);
    default: return CT_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

int launch_fa2_bwd_dkdv_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v,
                             Strided4 dO, const float* lse, const int64_t ls[3],
                             const float* delta, float* dk, float* dv, cudaStream_t st) {
  if (p.B * p.H > 65535) return CT_ERR_INVALID_ARGUMENT;
  const float scale = (float)(1.0 / std::sqrt((double)p.D));
  const dim3 g = simt_grid(p, kBRows);
  const int c = p.causal ? 1 : 0;
  switch (p.D) {
    case 32: return run_dkdv_simt<32>(p, q, k, v, dO, lse, ls, delta, dk, dv, c, scale, g, st);
    case 64: return run_dkdv_simt<64>(p, q, k, v, dO, lse, ls, delta, dk, dv, c, scale, g, st);
    case 128: return run_dkdv_simt<128>(p, q, k, v, dO, lse, ls, delta, dk, dv, c, scale, g, st);
    default: return CT_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

}  // namespace ct
