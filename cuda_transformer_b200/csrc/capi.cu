// capi.cu -- the extern "C" entry points declared in include/ct_b200.h:
// argument validation, per-device state (SM count, watchdog word), TMA
// descriptor encoding and dispatch to the kernel launchers.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "ct_internal.h"
#include "tc_ptx.cuh"

namespace {
// Watchdog block: bounded device-side waits OR CT_DEVSTAT_* bits into its
// status word and give up after its limit_ns.
__device__ ct::WatchBlock g_ct_watch = {0u, 0u, CT_WAIT_TIMEOUT_NS};
}  // namespace

namespace ct {
namespace {

constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
bool g_dev_ready[kMaxDevices];
std::mutex g_dev_mu;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

}  // namespace

const DeviceInfo* current_device(int* err) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = CT_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_dev_ready[dev]) {
    DeviceInfo d;
    d.device = dev;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
      *err = CT_ERR_CUDA;
      return nullptr;
    }
    if (d.cc_major != 10 || d.cc_minor != 0) {
      *err = CT_ERR_UNSUPPORTED_DEVICE;
      return nullptr;
    }
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_ct_watch) != cudaSuccess) {
      *err = CT_ERR_CUDA;
      return nullptr;
    }
    d.status = static_cast<uint32_t*>(addr);
    g_dev[dev] = d;
    g_dev_ready[dev] = true;
  }
  *err = CT_OK;
  return &g_dev[dev];
}

bool tma_compatible(const void* base, int64_t inner_stride, const int64_t* outer, int n_outer) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || inner_stride != 1) return false;
  for (int i = 0; i < n_outer; ++i) {
    if (outer[i] < 0 || (outer[i] * 4) % 16 != 0 || outer[i] * 4 >= (1ll << 40)) return false;
  }
  return true;
}

int make_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, bool mn_major) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return CT_ERR_CUDA;
  cuuint64_t gd[5];
  cuuint64_t gs[4];
  cuuint32_t bd[5], es[5];
  for (int i = 0; i < rank; ++i) {
    if (dims[i] == 0 || dims[i] > (1ull << 32)) return CT_ERR_UNSUPPORTED_LAYOUT;
    gd[i] = dims[i];
    bd[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    // A broadcast (zero) stride is legal for the math but not for TMA.
    if (strides_bytes[i] % 16 != 0 || strides_bytes[i] == 0) return CT_ERR_UNSUPPORTED_LAYOUT;
    gs[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank,
                        const_cast<void*>(base), gd, gs, bd, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CT_OK : CT_ERR_UNSUPPORTED_LAYOUT;
}

bool fa2_shape_ok(int64_t B, int64_t H, int64_t T, int64_t D) {
  constexpr int64_t kLim = 1ll << 31;
  return B >= 0 && H >= 0 && T >= 0 && D > 0 && T < kLim && B < kLim && H < kLim &&
         B * H < kLim;
}

bool valid_precision(int p) {
  return p == CT_PRECISION_3XTF32 || p == CT_PRECISION_TF32 || p == CT_PRECISION_FP32;
}

int fa2_validate(int64_t B, int64_t H, int64_t T, int64_t D, int precision) {
  if (!fa2_shape_ok(B, H, T, D) || !valid_precision(precision)) return CT_ERR_INVALID_ARGUMENT;
  if (!(D == 32 || D == 64 || D == 128)) return CT_ERR_UNSUPPORTED_HEAD_DIM;
  return CT_OK;
}

namespace {

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Common preamble of every FA2 entry point.
int fa2_prelude(int64_t B, int64_t H, int64_t T, int64_t D, int precision, const DeviceInfo** dev) {
  const int rc = fa2_validate(B, H, T, D, precision);
  if (rc != CT_OK) return rc;
  int err = CT_OK;
  *dev = current_device(&err);
  return err;
}

}  // namespace

int fa2_dq_dispatch(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
                    const float* lse, const int64_t* ls, const float* delta, float* dq,
                    const DeviceInfo& dev, cudaStream_t st) {
  if (p.precision != CT_PRECISION_FP32 && fa2_bwd_tc_supported(p))
    return launch_fa2_bwd_dq_tc(p, q, k, v, g, lse, ls, delta, dq, dev, st);
  return launch_fa2_bwd_dq_simt(p, q, k, v, g, lse, ls, delta, dq, st);
}

int fa2_dkdv_dispatch(const Fa2Problem& p, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
                      const float* lse, const int64_t* ls, const float* delta, float* dk,
                      float* dv, const DeviceInfo& dev, cudaStream_t st) {
  if (p.precision != CT_PRECISION_FP32 && fa2_bwd_tc_supported(p))
    return launch_fa2_bwd_dkdv_tc(p, q, k, v, g, lse, ls, delta, dk, dv, dev, st);
  return launch_fa2_bwd_dkdv_simt(p, q, k, v, g, lse, ls, delta, dk, dv, st);
}

}  // namespace ct

using namespace ct;

extern "C" {

const char* ct_status_string(int status) {
  switch (status) {
    case CT_OK: return "ok";
    case CT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CT_ERR_UNSUPPORTED_HEAD_DIM:
      return "Unsupported head dimension! Only hs=32, hs=64, and hs=128 are supported.";
    case CT_ERR_UNSUPPORTED_LAYOUT: return "tensor layout not addressable by TMA (strides/alignment)";
    case CT_ERR_LAUNCH_FAILED: return "kernel launch failed";
    case CT_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case CT_ERR_CUDA: return "CUDA runtime error";
    case CT_ERR_UNSUPPORTED_DEVICE: return "device is not sm_100 (B200)";
    case CT_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    default: return "unknown status";
  }
}

int ct_version(void) { return 10000; }

int ct_device_status(int device, int clear, unsigned int* flag_out) {
  if (!flag_out) return CT_ERR_INVALID_ARGUMENT;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return CT_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return CT_ERR_CUDA;
  int err = CT_OK;
  const DeviceInfo* dev = current_device(&err);
  unsigned int v = 0;
  if (err == CT_OK) {
    if (cudaMemcpy(&v, dev->status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
      err = CT_ERR_CUDA;
    else if (clear && v != 0 && cudaMemset(dev->status, 0, sizeof(v)) != cudaSuccess)
      err = CT_ERR_CUDA;
  }
  cudaSetDevice(prev);
  *flag_out = v;
  return err;
}

int ct_set_wait_limit_ns(int device, unsigned long long limit_ns) {
  if (limit_ns < CT_WAIT_LIMIT_MIN_NS || limit_ns > CT_WAIT_LIMIT_MAX_NS)
    return CT_ERR_INVALID_ARGUMENT;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return CT_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return CT_ERR_CUDA;
  int err = CT_OK;
  const DeviceInfo* dev = current_device(&err);
  if (err == CT_OK) {
    auto* blk = reinterpret_cast<WatchBlock*>(dev->status);
    if (cudaMemcpy(&blk->limit_ns, &limit_ns, sizeof(limit_ns), cudaMemcpyHostToDevice) !=
        cudaSuccess)
      err = CT_ERR_CUDA;
  }
  cudaSetDevice(prev);
  return err;
}

int ct_get_wait_limit_ns(int device, unsigned long long* limit_ns) {
  if (!limit_ns) return CT_ERR_INVALID_ARGUMENT;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return CT_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return CT_ERR_CUDA;
  int err = CT_OK;
  const DeviceInfo* dev = current_device(&err);
  if (err == CT_OK) {
    const auto* blk = reinterpret_cast<const WatchBlock*>(dev->status);
    if (cudaMemcpy(limit_ns, &blk->limit_ns, sizeof(*limit_ns), cudaMemcpyDeviceToHost) !=
        cudaSuccess)
      err = CT_ERR_CUDA;
  }
  cudaSetDevice(prev);
  return err;
}

int ct_watchdog_selftest(void* stream) {
  int err = CT_OK;
  const DeviceInfo* dev = current_device(&err);
  if (err != CT_OK) return err;
  return launch_watchdog_selftest(*dev, as_stream(stream));
}

int ct_fa2_fwd(const float* q, const int64_t q_stride[4], const float* k, const int64_t k_stride[4],
               const float* v, const int64_t v_stride[4], float* o, float* lse, int64_t batch,
               int64_t heads, int64_t seq_len, int64_t head_dim, int causal, int precision,
               void* stream) {
  const DeviceInfo* dev = nullptr;
  int rc = fa2_prelude(batch, heads, seq_len, head_dim, precision, &dev);
  if (rc != CT_OK) return rc;
  if (batch * heads * seq_len == 0) return CT_OK;
  if (!q || !k || !v || !o || !lse || !q_stride || !k_stride || !v_stride || !aligned16(o))
    return CT_ERR_INVALID_ARGUMENT;
  Fa2Problem p{batch, heads, seq_len, head_dim, causal != 0, precision};
  if (precision != CT_PRECISION_FP32 && fa2_fwd_tc_supported(p))
    return launch_fa2_fwd_tc(p, s4(q, q_stride), s4(k, k_stride), s4(v, v_stride), o, lse, *dev,
                             as_stream(stream));
  return launch_fa2_fwd_simt(p, s4(q, q_stride), s4(k, k_stride), s4(v, v_stride), o, lse,
                             as_stream(stream));
}

int ct_fa2_bwd_delta(const float* o, const int64_t o_stride[4], const float* d_o,
                     const int64_t do_stride[4], float* delta, int64_t batch, int64_t heads,
                     int64_t seq_len, int64_t head_dim, void* stream) {
  const DeviceInfo* dev = nullptr;
  int rc = fa2_prelude(batch, heads, seq_len, head_dim, CT_PRECISION_FP32, &dev);
  if (rc != CT_OK) return rc;
  if (batch * heads * seq_len == 0) return CT_OK;
  if (!o || !d_o || !delta || !o_stride || !do_stride) return CT_ERR_INVALID_ARGUMENT;
  Fa2Problem p{batch, heads, seq_len, head_dim, false, CT_PRECISION_FP32};
  return launch_fa2_delta(p, s4(o, o_stride), s4(d_o, do_stride), delta, as_stream(stream));
}

int ct_fa2_bwd_dq(const float* q, const int64_t q_stride[4], const float* k,
                  const int64_t k_stride[4], const float* v, const int64_t v_stride[4],
                  const float* d_o, const int64_t do_stride[4], const float* lse,
                  const int64_t lse_stride[3], const float* delta, float* dq, int64_t batch,
                  int64_t heads, int64_t seq_len, int64_t head_dim, int causal, int precision,
                  void* stream) {
  const DeviceInfo* dev = nullptr;
  int rc = fa2_prelude(batch, heads, seq_len, head_dim, precision, &dev);
  if (rc != CT_OK) return rc;
  if (batch * heads * seq_len == 0) return CT_OK;
  if (!q || !k || !v || !d_o || !lse || !delta || !dq || !lse_stride || !aligned16(dq))
    return CT_ERR_INVALID_ARGUMENT;
  Fa2Problem p{batch, heads, seq_len, head_dim, causal != 0, precision};
  return fa2_dq_dispatch(p, s4(q, q_stride), s4(k, k_stride), s4(v, v_stride),
                         s4(d_o, do_stride), lse, lse_stride, delta, dq, *dev, as_stream(stream));
}

int ct_fa2_bwd_dkdv(const float* q, const int64_t q_stride[4], const float* k,
                    const int64_t k_stride[4], const float* v, const int64_t v_stride[4],
                    const float* d_o, const int64_t do_stride[4], const float* lse,
                    const int64_t lse_stride[3], const float* delta, float* dk, float* dv,
                    int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int causal,
                    int precision, void* stream) {
  const DeviceInfo* dev = nullptr;
  int rc = fa2_prelude(batch, heads, seq_len, head_dim, precision, &dev);
  if (rc != CT_OK) return rc;
  if (batch * heads * seq_len == 0) return CT_OK;
  if (!q || !k || !v || !d_o || !lse || !delta || !dk || !dv || !lse_stride || !aligned16(dk) ||
      !aligned16(dv))
    return CT_ERR_INVALID_ARGUMENT;
  Fa2Problem p{batch, heads, seq_len, head_dim, causal != 0, precision};
  return fa2_dkdv_dispatch(p, s4(q, q_stride), s4(k, k_stride), s4(v, v_stride),
                           s4(d_o, do_stride), lse, lse_stride, delta, dk, dv, *dev,
                           as_stream(stream));
}

namespace {
// ct_fa2_bwd's workspace: delta (B*H*T floats), then at a 256-byte boundary
// the one-kernel backward's ordering counters and tickets.
size_t fa2_bwd_delta_bytes(int64_t B, int64_t H, int64_t T) {
  return ((size_t)(B * H * T) * sizeof(float) + 255u) & ~(size_t)255u;
}
}  // namespace

size_t ct_fa2_bwd_workspace_size(int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim) {
  (void)head_dim;
  if (!fa2_shape_ok(batch, heads, seq_len, 1)) return 0;
  return fa2_bwd_delta_bytes(batch, heads, seq_len) +
         fa2_bwd_fused_sync_words(batch, heads, seq_len) * sizeof(uint32_t);
}

int ct_fa2_bwd(const float* q, const int64_t q_stride[4], const float* k, const int64_t k_stride[4],
               const float* v, const int64_t v_stride[4], const float* o,
               const int64_t o_stride[4], const float* d_o, const int64_t do_stride[4],
               const float* lse, const int64_t lse_stride[3], float* dq, float* dk, float* dv,
               void* workspace, size_t workspace_bytes, int64_t batch, int64_t heads,
               int64_t seq_len, int64_t head_dim, int causal, int precision, void* stream) {
  const DeviceInfo* dev = nullptr;
  int rc = fa2_prelude(batch, heads, seq_len, head_dim, precision, &dev);
  if (rc != CT_OK) return rc;
  if (batch * heads * seq_len == 0) return CT_OK;
  if (!q || !k || !v || !o || !d_o || !lse || !dq || !dk || !dv || !lse_stride ||
      !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    return CT_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < ct_fa2_bwd_workspace_size(batch, heads, seq_len, head_dim))
    return CT_ERR_WORKSPACE_TOO_SMALL;
  Fa2Problem p{batch, heads, seq_len, head_dim, causal != 0, precision};
  cudaStream_t st = as_stream(stream);
  float* delta = static_cast<float*>(workspace);
  rc = launch_fa2_delta(p, s4(o, o_stride), s4(d_o, do_stride), delta, st);
  if (rc != CT_OK) return rc;
  rc = fa2_dq_dispatch(p, s4(q, q_stride), s4(k, k_stride), s4(v, v_stride), s4(d_o, do_stride),
                       lse, lse_stride, delta, dq, *dev, st);
  if (rc != CT_OK) return rc;
  return fa2_dkdv_dispatch(p, s4(q, q_stride), s4(k, k_stride), s4(v, v_stride),
                           s4(d_o, do_stride), lse, lse_stride, delta, dk, dv, *dev, st);
}

int ct_fa2_bwd_fused(const float* q, const int64_t q_stride[4], const float* k,
                     const int64_t k_stride[4], const float* v, const int64_t v_stride[4],
                     const float* o, const int64_t o_stride[4], const float* d_o,
                     const int64_t do_stride[4], const float* lse, const int64_t lse_stride[3],
                     float* dq, float* dk, float* dv, void* workspace, size_t workspace_bytes,
                     int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int causal,
                     int precision, void* stream) {
  const DeviceInfo* dev = nullptr;
  int rc = fa2_validate(batch, heads, seq_len, head_dim, precision);
  if (rc != CT_OK) return rc;
  if (head_dim != 64) return CT_ERR_UNSUPPORTED_HEAD_DIM;
  if (precision != CT_PRECISION_TF32) return CT_ERR_INVALID_ARGUMENT;
  if (batch * heads * seq_len == 0) return CT_OK;
  if (!q || !k || !v || !o || !d_o || !lse || !dq || !dk || !dv || !lse_stride ||
      !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    return CT_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < ct_fa2_bwd_workspace_size(batch, heads, seq_len, head_dim))
    return CT_ERR_WORKSPACE_TOO_SMALL;
  rc = fa2_prelude(batch, heads, seq_len, head_dim, precision, &dev);
  if (rc != CT_OK) return rc;
  Fa2Problem p{batch, heads, seq_len, head_dim, causal != 0, precision};
  if (!fa2_bwd_fused_supported(p)) return CT_ERR_INVALID_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  float* delta = static_cast<float*>(workspace);
  rc = launch_fa2_delta(p, s4(o, o_stride), s4(d_o, do_stride), delta, st);
  if (rc != CT_OK) return rc;
  uint32_t* sync_words = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) +
                                                     fa2_bwd_delta_bytes(batch, heads, seq_len));
  return launch_fa2_bwd_fused_tc(p, s4(q, q_stride), s4(k, k_stride), s4(v, v_stride),
                                 s4(d_o, do_stride), lse, lse_stride, delta, dq, dk, dv,
                                 sync_words, *dev, st);
}

size_t ct_linear_workspace_size(int64_t batch, int64_t m, int64_t k, int64_t n) {
  if (batch < 0 || m < 0 || k < 0 || n < 0) return 0;
  return linear_workspace_bytes(batch, m, n);
}

int ct_linear_fwd_ws(const float* x, const int64_t x_stride[3], const float* w,
                     const int64_t w_stride[3], const float* bias, int64_t bias_stride, float* out,
                     int64_t batch, int64_t m, int64_t k, int64_t n, int64_t w_batch,
                     int precision, void* workspace, size_t workspace_bytes, void* stream) {
  if (batch < 0 || m < 0 || k < 0 || n < 0 || !valid_precision(precision) ||
      !(w_batch == 1 || w_batch == batch))
    return CT_ERR_INVALID_ARGUMENT;
  if (batch * m * n == 0) return CT_OK;
  if (!x || !w || !bias || !out || !x_stride || !w_stride) return CT_ERR_INVALID_ARGUMENT;
  if (workspace_bytes > 0 && !workspace) return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  const DeviceInfo* dev = current_device(&err);
  if (err != CT_OK) return err;
  GemmProblem g;
  g.batch = batch; g.m = m; g.k = k; g.n = n;
  g.x = x; g.w = w; g.bias = bias; g.bias_s = bias_stride; g.out = out;
  for (int i = 0; i < 3; ++i) { g.xs[i] = x_stride[i]; g.ws[i] = w_stride[i]; }
  if (w_batch == 1) g.ws[0] = 0;
  g.precision = precision;
  if (precision != CT_PRECISION_FP32 && linear_tc_supported(g)) {
    const int rc = launch_linear_tc(g, workspace, workspace_bytes, *dev, as_stream(stream));
    if (rc != CT_ERR_UNSUPPORTED_LAYOUT) return rc;  // else: TMA cannot address it
  }
  return launch_linear_simt(g, as_stream(stream));
}

int ct_linear_fwd_ex(const float* x, const int64_t x_stride[3], const float* w,
                     const int64_t w_stride[3], const float* bias, int64_t bias_stride, float* out,
                     int64_t batch, int64_t m, int64_t k, int64_t n, int64_t w_batch,
                     int precision, int epilogue, float* act_out, const float* act_in,
                     float* w_colsum, int accumulate, void* workspace, size_t workspace_bytes,
                     void* stream) {
  if (batch < 0 || m < 0 || k < 0 || n < 0 || !valid_precision(precision) ||
      !(w_batch == 1 || w_batch == batch) ||
      !(epilogue == CT_EPILOGUE_NONE || epilogue == CT_EPILOGUE_GELU ||
        epilogue == CT_EPILOGUE_GELU_GRAD) ||
      (epilogue == CT_EPILOGUE_GELU && !act_out) ||
      (epilogue == CT_EPILOGUE_GELU_GRAD && !act_in) ||
      (accumulate && epilogue != CT_EPILOGUE_NONE) || (w_colsum && batch != 1))
    return CT_ERR_INVALID_ARGUMENT;
  if (batch * n == 0) return CT_OK;
  if (!x_stride || !w_stride || (m > 0 && (!x || !bias || !out)) || (k > 0 && !w))
    return CT_ERR_INVALID_ARGUMENT;
  if (workspace_bytes > 0 && !workspace) return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  const DeviceInfo* dev = current_device(&err);
  if (err != CT_OK) return err;
  GemmProblem g;
  g.batch = batch; g.m = m; g.k = k; g.n = n;
  g.x = x; g.w = w; g.bias = bias; g.bias_s = bias_stride; g.out = out;
  for (int i = 0; i < 3; ++i) { g.xs[i] = x_stride[i]; g.ws[i] = w_stride[i]; }
  if (w_batch == 1) g.ws[0] = 0;
  g.precision = precision;
  g.epilogue = epilogue;
  g.out_act = act_out;
  g.act_in = act_in;
  g.w_colsum = w_colsum;
  g.accumulate = accumulate != 0;
  if (m > 0 && precision != CT_PRECISION_FP32 && linear_tc_supported(g)) {
    const int rc = launch_linear_tc(g, workspace, workspace_bytes, *dev, as_stream(stream));
    if (rc != CT_ERR_UNSUPPORTED_LAYOUT) return rc;  // else: TMA cannot address it
  }
  if (m > 0) {
    const int rc = launch_linear_simt(g, as_stream(stream));
    if (rc != CT_OK) return rc;
  }
  return launch_w_colsum_simt(g, as_stream(stream));
}

int ct_linear_fwd(const float* x, const int64_t x_stride[3], const float* w,
                  const int64_t w_stride[3], const float* bias, int64_t bias_stride, float* out,
                  int64_t batch, int64_t m, int64_t k, int64_t n, int64_t w_batch, int precision,
                  void* stream) {
  return ct_linear_fwd_ws(x, x_stride, w, w_stride, bias, bias_stride, out, batch, m, k, n,
                          w_batch, precision, nullptr, 0, stream);
}

size_t ct_bias_grad_workspace_size(int64_t batch, int64_t m, int64_t n) {
  if (batch < 0 || m < 0 || n < 0) return 0;
  return bias_grad_workspace(batch * m, n);
}

int ct_bias_grad(const float* dy, const int64_t dy_stride[3], float* db, int64_t batch, int64_t m,
                 int64_t n, void* workspace, size_t workspace_bytes, void* stream) {
  if (batch < 0 || m < 0 || n < 0 || !dy || !db || !dy_stride) return CT_ERR_INVALID_ARGUMENT;
  if (n == 0) return CT_OK;
  int err = CT_OK;
  current_device(&err);
  if (err != CT_OK) return err;
  if (!workspace || workspace_bytes < ct_bias_grad_workspace_size(batch, m, n))
    return CT_ERR_WORKSPACE_TOO_SMALL;
  return launch_bias_grad(dy, dy_stride, db, batch, m, n, static_cast<float*>(workspace),
                          as_stream(stream));
}

int ct_softmax_fwd(const float* x, float* y, int64_t rows, int64_t n, void* stream) {
  if (rows < 0 || n < 0 || ((!x || !y) && rows * n > 0) || rows > 0x7fffffffll)
    return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  current_device(&err);
  if (err != CT_OK) return err;
  return launch_softmax_fwd(x, y, rows, n, as_stream(stream));
}

int ct_softmax_bwd(const float* p, const float* dp, float* dx, int64_t rows, int64_t n,
                   void* stream) {
  if (rows < 0 || n < 0 || ((!p || !dp || !dx) && rows * n > 0) || rows > 0x7fffffffll)
    return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  current_device(&err);
  if (err != CT_OK) return err;
  return launch_softmax_bwd(p, dp, dx, rows, n, as_stream(stream));
}

int ct_gelu_fwd(const float* x, float* y, int64_t numel, void* stream) {
  if (numel < 0 || ((!x || !y) && numel > 0)) return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  current_device(&err);
  if (err != CT_OK) return err;
  return launch_gelu_fwd(x, y, numel, as_stream(stream));
}

int ct_gelu_bwd(const float* x, const float* dy, float* dx, int64_t numel, void* stream) {
  if (numel < 0 || ((!x || !dy || !dx) && numel > 0)) return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  current_device(&err);
  if (err != CT_OK) return err;
  return launch_gelu_bwd(x, dy, dx, numel, as_stream(stream));
}

int ct_layernorm_fwd(const float* x, const float* gamma, const float* beta, float* y, float* mean,
                     float* rstd, int64_t rows, int64_t n, float eps, void* stream) {
  if (rows < 0 || n <= 0 || n > kLayerNormMaxCols || ((!x || !gamma || !beta || !y) && rows > 0))
    return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  current_device(&err);
  if (err != CT_OK) return err;
  return launch_layernorm_fwd(x, gamma, beta, y, mean, rstd, rows, n, eps, as_stream(stream));
}

size_t ct_layernorm_bwd_workspace_size(int64_t rows, int64_t n) {
  if (rows < 0 || n <= 0) return 0;
  return layernorm_bwd_workspace(rows, n);
}

int ct_layernorm_bwd(const float* x, const float* gamma, const float* mean, const float* rstd,
                     const float* dy, float* dx, float* dgamma, float* dbeta, int64_t rows,
                     int64_t n, void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || n <= 0 || n > kLayerNormMaxCols || !gamma || !dgamma || !dbeta ||
      ((!x || !mean || !rstd || !dy || !dx) && rows > 0))
    return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  current_device(&err);
  if (err != CT_OK) return err;
  if (rows > 0 && (!workspace || workspace_bytes < ct_layernorm_bwd_workspace_size(rows, n)))
    return CT_ERR_WORKSPACE_TOO_SMALL;
  return launch_layernorm_bwd(x, gamma, mean, rstd, dy, dx, dgamma, dbeta, rows, n,
                              static_cast<float*>(workspace), as_stream(stream));
}

int ct_cross_entropy_fwd_bwd(float* logits, int64_t ld, int64_t rows, int64_t vocab,
                             const int64_t* targets, int64_t ignore_index, float* loss_rows,
                             void* stream) {
  if (rows < 0 || vocab <= 0 || ld < vocab || ((!logits || !targets || !loss_rows) && rows > 0))
    return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  current_device(&err);
  if (err != CT_OK) return err;
  return launch_cross_entropy(logits, ld, rows, vocab, targets, ignore_index, loss_rows,
                              as_stream(stream));
}

}  // extern "C"
