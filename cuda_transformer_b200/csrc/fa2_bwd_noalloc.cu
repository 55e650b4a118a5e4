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
// so the first call on each device (in each CUDA context) looks the address up
// with cudaGetSymbolAddress, with that device current, and caches it per
// context; make that first call before any stream capture.  A call from a
// different context on the same device (a non-primary driver context, or the
// primary context re-created after cudaDeviceReset) looks the address up again,
// because the module is loaded anew there.  All calls share the one array and
// it keeps the previous call's contents; every element a call reads is written
// by the same call first (the delta kernel fills rows [0, B*H*T) before the
// gradient kernels read them), so nothing needs clearing.  Two calls whose
// work overlaps on the GPU (different streams, no ordering between them) race
// on the array: order such calls on one stream or with events.
#include <cudaTypedefs.h>

#include <mutex>

#include "ct_internal.h"

namespace {

__device__ __align__(256) float g_fa2_bwd_delta_scratch[CT_FA2_BWD_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 64;
struct ScratchSlot {
  CUcontext ctx = nullptr;  // context the cached address belongs to
  float* addr = nullptr;
};
std::mutex g_scratch_mu;
ScratchSlot g_scratch[kMaxDevices];

PFN_cuCtxGetCurrent_v4000 g_ctx_get = nullptr;
std::once_flag g_ctx_get_once;

void load_ctx_get() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_get = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
}

// Device address of the scratch array in the current device's current context
// (looked up once per context and cached).
int scratch_address(int device, float** out) {
  if (device < 0 || device >= kMaxDevices) return CT_ERR_CUDA;
  std::call_once(g_ctx_get_once, load_ctx_get);
  CUcontext ctx = nullptr;
  if (!g_ctx_get || g_ctx_get(&ctx) != CUDA_SUCCESS || ctx == nullptr) return CT_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  ScratchSlot& slot = g_scratch[device];
  if (slot.addr == nullptr || slot.ctx != ctx) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_fa2_bwd_delta_scratch) != cudaSuccess || addr == nullptr)
      return CT_ERR_CUDA;
    slot.ctx = ctx;
    slot.addr = static_cast<float*>(addr);
  }
  *out = slot.addr;
  return CT_OK;
}

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
  // The same validation as ct_fa2_bwd, before any CUDA call: it bounds B*H and
  // T, so the row count below cannot overflow.
  int rc = fa2_validate(batch, heads, seq_len, head_dim, precision);
  if (rc != CT_OK) return rc;
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
  const Strided4 tq = s4(q, q_stride), tk = s4(k, k_stride), tv = s4(v, v_stride);
  const Strided4 tg = s4(d_o, do_stride);
  rc = launch_fa2_delta(p, s4(o, o_stride), tg, delta, st);
  if (rc != CT_OK) return rc;
  rc = fa2_dq_dispatch(p, tq, tk, tv, tg, lse, lse_stride, delta, dq, *dev, st);
  if (rc != CT_OK) return rc;
  return fa2_dkdv_dispatch(p, tq, tk, tv, tg, lse, lse_stride, delta, dk, dv, *dev, st);
}
