// ct_internal.h -- host-side declarations shared by the kernel translation
// units and the C-ABI layer (capi.cu).  No torch types anywhere.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/ct_b200.h"

namespace ct {

// Per-device state, created on first use with the device current.
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  uint32_t* status = nullptr;  // device address of the watchdog word
};

// Returns the state of the current device (initialising it on first use), or
// nullptr with *err set on failure.
const DeviceInfo* current_device(int* err);

// Encodes a TMA descriptor for an FP32 tensor of rank 3 or 4 with a 32-float
// (128-byte) inner box.  `mn_major` selects CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
// (tiles the tensor core reads MN-major) instead of CU_TENSOR_MAP_SWIZZLE_128B
// (tiles read K-major).  dims[0] is the contiguous dimension; strides_bytes[i]
// is the stride of dims[i + 1].  Returns CT_OK or CT_ERR_UNSUPPORTED_LAYOUT
// when TMA cannot address the tensor.
int make_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, bool mn_major = false);

// True when a float tensor with these element strides (innermost first
// omitted) can be described by a TMA map: unit inner stride, 16-byte aligned
// base and outer strides.
bool tma_compatible(const void* base, int64_t inner_stride, const int64_t* outer, int n_outer);

inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CT_OK : CT_ERR_LAUNCH_FAILED;
}

// ---------------------------------------------------------------- FA2 args
struct Fa2Problem {
  int64_t B, H, T, D;
  bool causal;
  int precision;
};
struct Strided4 {
  const float* ptr;
  int64_t s[4];  // batch, head, seq, dim (elements)
};

// ------------------------------------------ FA2 entry-point validation / dispatch
// Shared by every FA2 entry point of the C ABI (capi.cu, fa2_bwd_noalloc.cu).
// Shape check without any CUDA call: sizes non-negative, head_dim positive,
// T < 2^31 and B*H < 2^31 (each factor bounded before the product is formed,
// so the product cannot overflow).  After it, B*H*T < 2^62.
bool fa2_shape_ok(int64_t B, int64_t H, int64_t T, int64_t D);
bool valid_precision(int p);
// fa2_shape_ok + precision + head dim in {32, 64, 128} (status, no CUDA call).
int fa2_validate(int64_t B, int64_t H, int64_t T, int64_t D, int precision);
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline Strided4 s4(const float* p, const int64_t* s) {
  Strided4 t;
  t.ptr = p;
  for (int i = 0; i < 4; ++i) t.s[i] = s[i];
  return t;
}
// dQ / dK-dV launch on the tensor cores when they cover the problem, else on
// the FP32 CUDA-core kernels.
int fa2_dq_dispatch(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
                    const float* lse, const int64_t* ls, const float* delta, float* dq,
                    const DeviceInfo& dev, cudaStream_t st);
int fa2_dkdv_dispatch(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
                      const float* lse, const int64_t* ls, const float* delta, float* dk,
                      float* dv, const DeviceInfo& dev, cudaStream_t st);

// Kernel launchers (one translation unit each).  All return a ct status.
int launch_fa2_fwd_tc(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, float* o,
                      float* lse, const DeviceInfo& dev, cudaStream_t st);
int launch_fa2_bwd_dq_tc(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 dO,
                         const float* lse, const int64_t lse_s[3], const float* delta, float* dq,
                         const DeviceInfo& dev, cudaStream_t st);
int launch_fa2_bwd_dkdv_tc(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 dO,
                           const float* lse, const int64_t lse_s[3], const float* delta,
                           float* dk, float* dv, const DeviceInfo& dev, cudaStream_t st);
// The one-kernel backward (TF32, head dim 64): dQ, dK and dV from one
// key/value-stationary pass, dQ added in a fixed key-tile order.  sync_words:
// fa2_bwd_fused_sync_words(B, H, T) 32-bit words of device scratch (ordering
// counters and per-launch tickets), zeroed by the launcher on `st`.
int launch_fa2_bwd_fused_tc(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 dO,
                            const float* lse, const int64_t lse_s[3], const float* delta,
                            float* dq, float* dk, float* dv, uint32_t* sync_words,
                            const DeviceInfo& dev, cudaStream_t st);
size_t fa2_bwd_fused_sync_words(int64_t B, int64_t H, int64_t T);
// dK/dV on CTA pairs (TF32, head dim 64; fa2_bwd_pair.cu): the default for
// that case unless CT_FA2_PAIR_DKDV=0.
int launch_fa2_bwd_dkdv_pair(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v,
                             Strided4 dO, const float* lse, const int64_t lse_s[3],
                             const float* delta, float* dk, float* dv, const DeviceInfo& dev,
                             cudaStream_t st);
bool fa2_bwd_pair_supported(const Fa2Problem& p);
// Persistent dQ (TF32, head dim 64; fa2_bwd_dq_persist.cu): the default for
// that case unless CT_FA2_PERSIST_DQ=0.
int launch_fa2_bwd_dq_persist(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v,
                              Strided4 dO, const float* lse, const int64_t lse_s[3],
                              const float* delta, float* dq, const DeviceInfo& dev,
                              cudaStream_t st);
bool fa2_bwd_dq_persist_supported(const Fa2Problem& p);
// Whether the tensor-core kernels cover this problem (head dim / precision).
bool fa2_fwd_tc_supported(const Fa2Problem& p);
bool fa2_bwd_tc_supported(const Fa2Problem& p);
bool fa2_bwd_fused_supported(const Fa2Problem& p);

// CUDA-core FP32 kernels: any strides, head_dim in {32, 64, 128}.
int launch_fa2_fwd_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, float* o,
                        float* lse, cudaStream_t st);
int launch_fa2_bwd_dq_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 dO,
                           const float* lse, const int64_t lse_s[3], const float* delta,
                           float* dq, cudaStream_t st);
int launch_fa2_bwd_dkdv_simt(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v,
                             Strided4 dO, const float* lse, const int64_t lse_s[3],
                             const float* delta, float* dk, float* dv, cudaStream_t st);
int launch_fa2_delta(const Fa2Problem& p, Strided4 o, Strided4 dO, float* delta, cudaStream_t st);

// ------------------------------------------------------------- GEMM args
struct GemmProblem {
  int64_t batch, m, k, n;
  const float* x;
  int64_t xs[3];  // batch, row (m), col (k)
  const float* w;
  int64_t ws[3];  // batch (0 = shared), row (k), col (n)
  const float* bias;
  int64_t bias_s;
  float* out;     // contiguous [batch, m, n]
  int precision;
  // Fused epilogues (CT_EPILOGUE_*): GELU writes gelu(out) to out_act as well;
  // GELU_GRAD multiplies out by gelu'(act_in) (act_in dense [batch, m, n]).
  int epilogue = CT_EPILOGUE_NONE;
  float* out_act = nullptr;
  const float* act_in = nullptr;
  // Column sums of the W operand over the batch and reduction indices, [n]
  // (the bias gradient when W is dY); batch == 1.
  float* w_colsum = nullptr;
  bool accumulate = false;  // out (and w_colsum) += instead of =
};
// ws / ws_bytes: optional per-tile counters that enable the split-K schedule.
int launch_linear_tc(const GemmProblem& g, void* ws, size_t ws_bytes, const DeviceInfo& dev,
                     cudaStream_t st);
size_t linear_workspace_bytes(int64_t batch, int64_t m, int64_t n);
bool linear_tc_supported(const GemmProblem& g);
int launch_linear_simt(const GemmProblem& g, cudaStream_t st);
// w_colsum of a GemmProblem on the CUDA cores (fallback path).
int launch_w_colsum_simt(const GemmProblem& g, cudaStream_t st);

// -------------------------------------------------------- row-wise kernels
size_t bias_grad_workspace(int64_t rows, int64_t n);
int launch_bias_grad(const float* dy, const int64_t s[3], float* db, int64_t batch, int64_t m,
                     int64_t n, float* ws, cudaStream_t st);
int launch_softmax_fwd(const float* x, float* y, int64_t rows, int64_t n, cudaStream_t st);
int launch_softmax_bwd(const float* p, const float* dp, float* dx, int64_t rows, int64_t n,
                       cudaStream_t st);
int launch_gelu_fwd(const float* x, float* y, int64_t numel, cudaStream_t st);
int launch_gelu_bwd(const float* x, const float* dy, float* dx, int64_t numel, cudaStream_t st);
// Widest LayerNorm row: one warp per row up to 1024 columns, one CTA per row above.
constexpr int64_t kLayerNormMaxCols = 8192;
int launch_layernorm_fwd(const float* x, const float* g, const float* b, float* y, float* mean,
                         float* rstd, int64_t rows, int64_t n, float eps, cudaStream_t st);
size_t layernorm_bwd_workspace(int64_t rows, int64_t n);
int launch_layernorm_bwd(const float* x, const float* g, const float* mean, const float* rstd,
                         const float* dy, float* dx, float* dg, float* db, int64_t rows,
                         int64_t n, float* ws, cudaStream_t st);

// Cross entropy of logit rows (loss per row; gradient written over the logits).
int launch_cross_entropy(float* x, int64_t ld, int64_t rows, int64_t vocab, const int64_t* targets,
                         int64_t ignore, float* loss_rows, cudaStream_t st);

// ------------------------------------------------------------ watchdog
// One CTA whose waits on a barrier phase that nothing completes run out after
// the device's wait limit, followed by the kernels' abort teardown.
int launch_watchdog_selftest(const DeviceInfo& dev, cudaStream_t st);

}  // namespace ct
