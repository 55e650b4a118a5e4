// fa2_bwd_noalloc.cu -- FlashAttention-2 backward that allocates nothing.
//
// ct_fa2_bwd needs a caller-provided workspace for the per-row delta vector
// (delta = rowsum(O * dO)).  Some callers cannot provide one: a plugin that is
// handed only tensor pointers by a host runtime whose allocator it cannot
// reach, or a service that forbids device allocation once it has started (a
// fixed memory budget, no cudaMalloc on the request path).  For them,
// ct_fa2_bwd_noalloc keeps delta in a fixed device array compiled into this
// library instead.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds CT_FA2_BWD_NOALLOC_MAX_ROWS floats (8 MiB) for it until the
// process exits.  Host code cannot use the array's name as a device address,
// so the first call on each device looks the address up with
// cudaGetSymbolAddress (with that device current) and caches it; make that
// first call before any stream capture.  All calls share the one array and it
// keeps the previous call's contents; every element a call reads is written by
// the same call first (the delta kernel fills rows [0, B*H*T) before the
// gradient kernels read them), so nothing needs clearing.  Two calls whose
// work overlaps on the GPU (different streams, no ordering between them) race
// on the array: order such calls on one stream or with events.
#include <mutex>

#include "ct_internal.h"

namespace {

__device__ __align__(256) float g_fa2_bwd_delta_scratch[CT_FA2_BWD_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_addr[kMaxDevices];

// Device address of the scratch array on the current device (looked up once
// per device and cached).
int scratch_address(int device, float** out) {
  if (device < 0 || device >= kMaxDevices) return CT_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_addr[device] == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_fa2_bwd_delta_scratch) != cudaSuccess || addr == nullptr)
      return CT_ERR_CUDA;
    g_scratch_addr[device] = static_cast<float*>(addr);
  }
  *out = g_scratch_addr[device];
  return CT_OK;
}

ct::Strided4 view4(const float* p, const int64_t* s) {
  ct::Strided4 t;
  t.ptr = p;
  for (int i = 0; i < 4; ++i) t.s[i] = s[i];
  return t;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int ct_fa2_bwd_noalloc(const float* q, const int64_t q_stride[4], const float* k,
                                  const int64_t k_stride[4], const float* v,
                                  const int64_t v_stride[4], const float* o,
                                  const int64_t o_stride[4], const float* d_o,
                                  const int64_t do_stride[4], const float* lse,
                                  const int64_t lse_stride[3], float* dq, float* dk, float* dv,
                                  int64_t batch, int64_t heads, int64_t seq_len,
                                  int64_t head_dim, int causal, int precision, void* stream) {
  using namespace ct;
  if (batch < 0 || heads < 0 || seq_len < 0 || seq_len >= (1ll << 31) ||
      !(precision == CT_PRECISION_3XTF32 || precision == CT_PRECISION_TF32 ||
        precision == CT_PRECISION_FP32))
    return CT_ERR_INVALID_ARGUMENT;
  if (!(head_dim == 32 || head_dim == 64 || head_dim == 128)) return CT_ERR_UNSUPPORTED_HEAD_DIM;
  const int64_t rows = batch * heads * seq_len;
  if (rows == 0) return CT_OK;
  if (rows > CT_FA2_BWD_NOALLOC_MAX_ROWS) return CT_ERR_WORKSPACE_TOO_SMALL;
  if (!q || !k || !v || !o || !d_o || !lse || !dq || !dk || !dv || !q_stride || !k_stride ||
      !v_stride || !o_stride || !do_stride || !lse_stride || !aligned16(dq) || !aligned16(dk) ||
      !aligned16(dv))
    return CT_ERR_INVALID_ARGUMENT;
  int err = CT_OK;
  const DeviceInfo* dev = current_device(&err);
  if (err != CT_OK) return err;
  float* delta = nullptr;
  err = scratch_address(dev->device, &delta);
  if (err != CT_OK) return err;

  const Fa2Problem p{batch, heads, seq_len, head_dim, causal != 0, precision};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const Strided4 tq = view4(q, q_stride), tk = view4(k, k_stride), tv = view4(v, v_stride);
  const Strided4 tg = view4(d_o, do_stride);
  int rc = launch_fa2_delta(p, view4(o, o_stride), tg, delta, st);
  if (rc != CT_OK) return rc;
  const bool tc = precision != CT_PRECISION_FP32 && fa2_bwd_tc_supported(p);
  rc = tc ? launch_fa2_bwd_dq_tc(p, tq, tk, tv, tg, lse, lse_stride, delta, dq, *dev, st)
          : launch_fa2_bwd_dq_simt(p, tq, tk, tv, tg, lse, lse_stride, delta, dq, st);
  if (rc != CT_OK) return rc;
  return tc ? launch_fa2_bwd_dkdv_tc(p, tq, tk, tv, tg, lse, lse_stride, delta, dk, dv, *dev, st)
            : launch_fa2_bwd_dkdv_simt(p, tq, tk, tv, tg, lse, lse_stride, delta, dk, dv, st);
}
