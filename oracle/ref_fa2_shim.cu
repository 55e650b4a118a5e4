// ref_fa2_shim.cu -- TEST INFRASTRUCTURE: a C entry point around the
// reference's own FlashAttention-2 kernels (Transformer_kernels/flash_attention.cuh,
// included from the reference checkout at build time, never copied), compiled
// for sm_100a by oracle/build_ref.py into oracle/_ref/libref_fa2.so.
//
// The launch configuration restates the reference launcher
// (Transformer_launchers/flash_attn_launcher.cu:41-56 forward, :95-133
// backward): br = bc = 16, 256 threads, grid (1, ceil(T/16), B*nh); delta with
// grid (1, T, B*nh) x 1024 threads; hs = 128 dK/dV with 8 x 8 tiles; the
// kernels receive sm_scale = sqrt(hs) and int strides.  Used by the GPU tests
// as a second parity reference and as the "reference kernels on the same
// B200" timing baseline.  Inputs are contiguous [B,nh,T,hs] FP32.
#include <cmath>
#include <cuda_runtime.h>

#include "Transformer_kernels/flash_attention.cuh"

namespace {

template <int HS>
void fwd_launch(const float* q, const float* k, const float* v, float* o, float* l, int B, int nh,
                int T, bool causal, cudaStream_t st) {
  const float sm_scale = std::sqrt(static_cast<float>(HS));
  const int s_t = HS, s_h = T * HS, s_b = nh * T * HS;
  dim3 grid(1, (T + 15) / 16, B * nh), block(256);
  flash_attention_fwd_kernel<16, 16, HS><<<grid, block, 0, st>>>(
      q, k, v, o, l, B, nh, T, sm_scale, causal, s_b, s_h, s_t, 1, s_b, s_h, s_t, 1, s_b, s_h, s_t, 1);
}

template <int HS>
void bwd_launch(const float* q, const float* k, const float* v, const float* o, const float* dO,
                const float* l, float* dq, float* dk, float* dv, float* delta, int B, int nh, int T,
                bool causal, cudaStream_t st) {
  const float sm_scale = std::sqrt(static_cast<float>(HS));
  const int s_t = HS, s_h = T * HS, s_b = nh * T * HS;
  flash_attention_bwd_delta<<<dim3(1, T, B * nh), dim3(1024), 0, st>>>(o, dO, delta, B, nh, T, HS,
                                                                      s_b, s_h, s_t, 1, s_b, s_h, s_t, 1);
  dim3 grid(1, (T + 15) / 16, B * nh), block(256);
  flash_attention_bwd_dq<16, 16, HS><<<grid, block, 0, st>>>(
      q, k, v, delta, l, dO, dq, B, nh, T, sm_scale, causal, s_b, s_h, s_t, 1, s_b, s_h, s_t, 1,
      s_b, s_h, s_t, 1, nh * T, T, 1, s_b, s_h, s_t, 1);
  if constexpr (HS == 128) {
    flash_attention_bwd_dk_dv<8, 8, HS><<<dim3(1, (T + 7) / 8, B * nh), block, 0, st>>>(
        q, k, v, delta, l, dO, dk, dv, B, nh, T, sm_scale, causal, s_b, s_h, s_t, 1, s_b, s_h, s_t,
        1, s_b, s_h, s_t, 1, nh * T, T, 1, s_b, s_h, s_t, 1);
  } else {
    flash_attention_bwd_dk_dv<16, 16, HS><<<grid, block, 0, st>>>(
        q, k, v, delta, l, dO, dk, dv, B, nh, T, sm_scale, causal, s_b, s_h, s_t, 1, s_b, s_h, s_t,
        1, s_b, s_h, s_t, 1, nh * T, T, 1, s_b, s_h, s_t, 1);
  }
}

}  // namespace

extern "C" int ref_fa2_fwd(const float* q, const float* k, const float* v, float* o, float* l,
                           int B, int nh, int T, int hs, int causal, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (hs) {
    case 32: fwd_launch<32>(q, k, v, o, l, B, nh, T, causal != 0, st); break;
    case 64: fwd_launch<64>(q, k, v, o, l, B, nh, T, causal != 0, st); break;
    case 128: fwd_launch<128>(q, k, v, o, l, B, nh, T, causal != 0, st); break;
    default: return 2;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int ref_fa2_bwd(const float* q, const float* k, const float* v, const float* o,
                           const float* dO, const float* l, float* dq, float* dk, float* dv,
                           float* delta, int B, int nh, int T, int hs, int causal, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (hs) {
    case 32: bwd_launch<32>(q, k, v, o, dO, l, dq, dk, dv, delta, B, nh, T, causal != 0, st); break;
    case 64: bwd_launch<64>(q, k, v, o, dO, l, dq, dk, dv, delta, B, nh, T, causal != 0, st); break;
    case 128: bwd_launch<128>(q, k, v, o, dO, l, dq, dk, dv, delta, B, nh, T, causal != 0, st); break;
    default: return 2;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
