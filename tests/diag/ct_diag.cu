// ct_diag.cu -- TEST-ONLY diagnostics library (tests/diag/libct_diag.so), not
// part of the product library.
//
// * ct_diag_umma_tf32: a single-CTA 128 x n x 32 TF32 tensor-core product used
//   by the test-suite to check, on the device, the operand layouts that the
//   FlashAttention and GEMM kernels rely on: K-major and MN-major shared-memory
//   operands in the 128-byte swizzle, A read from Tensor Memory, and how the
//   tensor core treats the 13 low mantissa bits of an FP32 operand.
// * ct_diag_umma_pair: the same check for a CTA pair (cta_group::2, M = 256):
//   which rows of A, B and D each CTA of the pair holds.
// * ct_diag_mma_rate: a throughput probe -- back-to-back kind::tf32 MMAs of one
//   shape, timed in SM cycles on every SM (the tensor-pipe ceiling the tile
//   shapes of the product kernels are chosen against).
//
// Built from the product's PTX layer (cuda_transformer_b200/csrc/tc_ptx.cuh)
// with its own watchdog block; declared in tests/diag/ct_diag.h.
#include <cuda_runtime.h>

#include "ct_diag.h"
#include "tc_ptx.cuh"

namespace {
__device__ ct::WatchBlock g_diag_watch = {0u, 0u, CT_WAIT_TIMEOUT_NS};
}  // namespace

namespace ct {
namespace {

int launch_ok() { return cudaGetLastError() == cudaSuccess ? 0 : 4; }

uint32_t* diag_status() {
  void* addr = nullptr;
  return cudaGetSymbolAddress(&addr, g_diag_watch) == cudaSuccess ? static_cast<uint32_t*>(addr)
                                                                   : nullptr;
}

struct DiagSmem {
  uint64_t bar, bar2;
  CtaCtl ctl;
};

// 128 threads.  smem: [header][pad to 1024][A 16 KB][B n*128 bytes].
__global__ void __launch_bounds__(128, 1)
    umma_diag_kernel(int mode, const float* __restrict__ a, const float* __restrict__ b,
                     float* __restrict__ d, int n, uint32_t* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  DiagSmem* hs = reinterpret_cast<DiagSmem*>(smem_raw);
  const uint32_t base = (smem_u32(smem_raw) + sizeof(DiagSmem) + 1023u) & ~1023u;
  const uint32_t sa = base, sb = base + 128u * 128u;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const bool a_tmem = (mode == 2 || mode == 3);
  const bool a_mn = (mode == 4);
  const bool b_mn = (mode == 1 || mode == 3 || mode == 4);

  if (tid == 0) {
    mbar_init(smem_u32(&hs->bar), 1);
    hs->ctl.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&hs->ctl.tmem_base), 256);
    tmem_relinquish();
  }
  // Operands into swizzled smem exactly as TMA would lay them out (K-major:
  // SWIZZLE_128B; MN-major: SWIZZLE_128B_ATOM_32B).
  for (int e = tid; e < 128 * 32; e += 128) {
    if (!a_tmem) {
      if (a_mn) {  // a is [32 (k)][128 (m)], m contiguous
        const int kk = e / 128, mm = e % 128;
        *reinterpret_cast<float*>(smem_raw + (sa - smem_u32(smem_raw)) + sw128_32b_offset(kk, mm, 32)) = a[e];
      } else {  // a is [128 (m)][32 (k)]
        const int mm = e / 32, kk = e % 32;
        *reinterpret_cast<float*>(smem_raw + (sa - smem_u32(smem_raw)) + sw128_offset(mm, kk, 128)) = a[e];
      }
    }
  }
  for (int e = tid; e < n * 32; e += 128) {
    if (b_mn) {  // b is [32 (k)][n], n contiguous
      const int kk = e / n, nn = e % n;
      *reinterpret_cast<float*>(smem_raw + (sb - smem_u32(smem_raw)) + sw128_32b_offset(kk, nn, 32)) = b[e];
    } else {  // b is [n][32 (k)]
      const int nn = e / 32, kk = e % 32;
      *reinterpret_cast<float*>(smem_raw + (sb - smem_u32(smem_raw)) + sw128_offset(nn, kk, n)) = b[e];
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = hs->ctl.tmem_base;
  const uint32_t lane_base = tmem_addr(tmem, 32u * warp, 0);
  if (a_tmem) {  // row tid of A into columns 128..159 of lane tid
    float row[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) row[i] = a[tid * 32 + i];
    tmem_st32(lane_base + 128u, row);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    tc_fence_after();
    const uint32_t idesc = idesc_tf32(128, n, a_mn, b_mn);
    for (int k = 0; k < 4; ++k) {
      const uint64_t bd = b_mn ? sdesc_mnmajor(sb + k * 1024u, 32u * 128u)
                               : sdesc_kmajor(sb + k * 32u);
      if (a_tmem) {
        umma_tf32_ts(tmem, tmem + 128u + 8u * k, bd, idesc, k > 0);
      } else {
        const uint64_t ad = a_mn ? sdesc_mnmajor(sa + k * 1024u, 32u * 128u)
                                 : sdesc_kmajor(sa + k * 32u);
        umma_tf32_ss(tmem, ad, bd, idesc, k > 0);
      }
    }
    umma_commit(smem_u32(&hs->bar));
  }
  __syncwarp();
  const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&hs->bar), 0, &hs->ctl, status));
  if (ok) {
    tc_fence_after();
    for (int c = 0; c < n; c += 32) {
      float v[32];
      tmem_ld32(lane_base + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) d[tid * n + c + i] = v[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// A CTA pair (cluster of two, cta_group::2): D[256 x n] = A[256 x 64] B^T over
// K = 64 in eight MMAs of M = 256 issued by the even CTA.  A from Tensor
// Memory: CTA r holds rows 128r..128r+127 in its lanes (columns 128..191).  B
// split along N: CTA r holds B's rows [r n/2, (r+1) n/2) in its shared memory
// at the same address, K-major (mode 0: b is [n][64]) or MN-major (mode 1: b is
// [64][n]).  The odd CTA reports its operands ready with a remote arrival on
// the even CTA's barrier; the commit arrives on both CTAs' barriers.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1)
    umma_pair_diag_kernel(int mode, const float* __restrict__ a, const float* __restrict__ b,
                          float* __restrict__ d, int n, uint32_t* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  DiagSmem* hs = reinterpret_cast<DiagSmem*>(smem_raw);
  const uint32_t base = (smem_u32(smem_raw) + sizeof(DiagSmem) + 1023u) & ~1023u;
  uint8_t* sbp = smem_raw + (base - smem_u32(smem_raw));
  const int tid = threadIdx.x, warp = tid / 32;
  const uint32_t rank = cluster_ctarank();
  const bool b_mn = mode == 1;
  const int nh = n / 2;

  if (tid == 0) {
    mbar_init(smem_u32(&hs->bar), 1);   // the pair's commit
    mbar_init(smem_u32(&hs->bar2), 2);  // operands ready: one arrival per CTA
    hs->ctl.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(smem_u32(&hs->ctl.tmem_base), 256);
    tmem_relinquish_pair();
  }
  for (int e = tid; e < nh * 64; e += 128) {
    if (b_mn) {  // rows k, 128-byte rows of 32 n values, n chunks of 64 rows
      const int kk = e / nh, nl = e % nh;
      *reinterpret_cast<float*>(sbp + sw128_32b_offset(kk, nl, 64)) = b[kk * n + rank * nh + nl];
    } else {  // rows n, 128-byte rows of 32 k values, k chunks of nh rows
      const int nl = e / 64, kk = e % 64;
      *reinterpret_cast<float*>(sbp + sw128_offset(nl, kk, nh)) = b[(rank * nh + nl) * 64 + kk];
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = hs->ctl.tmem_base;
  const uint32_t lane_base = tmem_addr(tmem, 32u * warp, 0);
  for (int h = 0; h < 2; ++h) {
    float row[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) row[i] = a[(128 * rank + tid) * 64 + 32 * h + i];
    tmem_st32(lane_base + 128u + 32u * h, row);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncthreads();
  if (tid == 0) mbar_arrive_remote(mapa_shared(smem_u32(&hs->bar2), 0));
  if (rank == 0 && tid == 0) {
    if (mbar_wait(smem_u32(&hs->bar2), 0, &hs->ctl, status)) {
      tc_fence_after();
      const uint32_t idesc = idesc_tf32(256, n, false, b_mn);
      for (int k = 0; k < 8; ++k) {
        const uint64_t bd =
            b_mn ? sdesc_mnmajor(base + k * 1024u, 64u * 128u)
                 : sdesc_kmajor(base + (uint32_t)(k / 4) * nh * 128u + (uint32_t)(k % 4) * 32u);
        umma_tf32_ts_pair(tmem, tmem + 128u + 8u * k, bd, idesc, k > 0);
      }
      umma_commit_pair(smem_u32(&hs->bar));
    }
  }
  __syncwarp();
  const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&hs->bar), 0, &hs->ctl, status));
  if (ok) {
    tc_fence_after();
    for (int c = 0; c < n; c += 32) {
      float v[32];
      tmem_ld32(lane_base + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) d[(128 * rank + tid) * n + c + i] = v[i];
    }
  }
  tc_fence_before();
  cluster_sync_all();  // no MMA, load or remote arrival of either CTA still pending
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 256);
  }
}

// One CTA per SM (the shared-memory request keeps a second CTA off the SM):
// thread 0 issues `reps` x 4 MMAs D[128 x N] += A[128 x 8] B[8 x N] on zeroed
// operands (A in TMEM when TS, else shared memory; B K-major in shared
// memory) and records the clock64 span from the first issue to the commit's
// completion in cycles[blockIdx.x].
// tcgen05.ld of 16 lanes x 32-bit, two halves: threads 0-15 read lanes
// base..base+15 at columns [col, col + N), threads 16-31 the same lanes at
// columns [col + N, col + 2N) (immediate half-split offset N).
__device__ __forceinline__ void tmem_ld_16x32bx2_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16], 16;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// M = 64 product D[64 x n] = A[64 x 32] B[n x 32]^T, B K-major in shared
// memory, checking the M = 64 data-path layout of TMEM: row r of D (and of a
// TMEM A operand) sits in lane 32 * (r / 16) + r % 16 + L.  mode bit 0: A from
// TMEM (columns 128..159), else shared memory K-major; bit 1: L = 16 (the
// upper half of each warp's lane quadrant), else 0; bit 2: D read with the
// 16-lane 16x32bx2 shape (n = 32: threads 0-15 columns 0-15, threads 16-31
// columns 16-31 of the same rows), else with 32x32b; bit 3: A and B both from
// shared memory MN-major (a is [32 (k)][64 (m)], b is [32 (k)][n]).
__global__ void __launch_bounds__(128, 1)
    umma_m64_kernel(int mode, const float* __restrict__ a, const float* __restrict__ b,
                    float* __restrict__ d, int n, uint32_t* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  DiagSmem* hs = reinterpret_cast<DiagSmem*>(smem_raw);
  const uint32_t base = (smem_u32(smem_raw) + sizeof(DiagSmem) + 1023u) & ~1023u;
  uint8_t* gen = smem_raw + (base - smem_u32(smem_raw));
  const uint32_t sa = base, sb = base + 64u * 128u;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const bool a_tmem = (mode & 1) != 0, x2 = (mode & 4) != 0, mn = (mode & 8) != 0;
  const uint32_t L = (mode & 2) ? 16u : 0u;
  if (tid == 0) {
    mbar_init(smem_u32(&hs->bar), 1);
    hs->ctl.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&hs->ctl.tmem_base), 256);
    tmem_relinquish();
  }
  for (int e = tid; e < 64 * 32; e += 128)
    *reinterpret_cast<float*>(gen + (mn ? sw128_32b_offset(e / 64, e % 64, 32)
                                        : sw128_offset(e / 32, e % 32, 64))) = a[e];
  for (int e = tid; e < n * 32; e += 128)
    *reinterpret_cast<float*>(gen + (sb - sa) + (mn ? sw128_32b_offset(e / n, e % n, 32)
                                                    : sw128_offset(e / 32, e % 32, n))) = b[e];
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = hs->ctl.tmem_base;
  const bool mine = (uint32_t)lane >= L && (uint32_t)lane < L + 16u;  // this lane holds a row
  const int r = 16 * warp + lane - (int)L;
  if (a_tmem) {
    float row[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) row[i] = mine ? a[r * 32 + i] : 0.0f;
    tmem_st32(tmem_addr(tmem, 32u * warp, 128), row);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    tc_fence_after();
    const uint32_t idesc = idesc_tf32(64, n, mn, mn);
    const uint32_t dt = tmem + (L << 16);
    for (int k = 0; k < 4; ++k) {
      const uint64_t bd = mn ? sdesc_mnmajor(sb + k * 1024u, 32u * 128u) : sdesc_kmajor(sb + k * 32u);
      if (a_tmem) umma_tf32_ts(dt, tmem + (L << 16) + 128u + 8u * k, bd, idesc, k > 0);
      else if (mn) umma_tf32_ss(dt, sdesc_mnmajor(sa + k * 1024u, 32u * 128u), bd, idesc, k > 0);
      else umma_tf32_ss(dt, sdesc_kmajor(sa + k * 32u), bd, idesc, k > 0);
    }
    umma_commit(smem_u32(&hs->bar));
  }
  __syncwarp();
  const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&hs->bar), 0, &hs->ctl, status));
  if (ok) {
    tc_fence_after();
    if (x2) {  // n == 32
      float v[16];
      tmem_ld_16x32bx2_x16(tmem + ((32u * warp + L) << 16), v);
      const int rr = 16 * warp + (lane & 15), c0 = (lane >> 4) * 16;
#pragma unroll
      for (int i = 0; i < 16; ++i) d[rr * n + c0 + i] = v[i];
    } else {
      for (int c = 0; c < n; c += 32) {
        float v[32];
        tmem_ld32(tmem_addr(tmem, 32u * warp, c), v);
        if (mine) {
#pragma unroll
          for (int i = 0; i < 32; ++i) d[r * n + c + i] = v[i];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <int N, bool TS, bool BMN, bool TWO>
__global__ void __launch_bounds__(128, 1)
    mma_rate_kernel(int reps, long long* __restrict__ cycles, uint32_t* status) {
  // One or two issuing threads (thread 0, and thread 32 of the next warp with
  // TWO), each driving its own accumulator (columns 0 and N); B K-major or
  // MN-major (BMN); A from shared memory or TMEM columns 256..287.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  DiagSmem* hs = reinterpret_cast<DiagSmem*>(smem_raw);
  const uint32_t base = (smem_u32(smem_raw) + sizeof(DiagSmem) + 1023u) & ~1023u;
  const uint32_t sa = base, sb = base + 16384u;
  float* f = reinterpret_cast<float*>(smem_raw + (base - smem_u32(smem_raw)));
  for (int i = threadIdx.x; i < (16384 + N * 128) / 4; i += 128) f[i] = 0.0f;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&hs->bar), 1);
    mbar_init(smem_u32(&hs->bar2), 1);
    hs->ctl.abort = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(smem_u32(&hs->ctl.tmem_base), 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = hs->ctl.tmem_base;
  if (threadIdx.x < 128 && TS) {  // A operand columns 256..287: zeros
    float z[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) z[i] = 0.0f;
    tmem_st32(tmem_addr(tmem, 32u * (threadIdx.x / 32), 256), z);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool issuer = threadIdx.x == 0 || (TWO && threadIdx.x == 32);
  if (issuer) {
    const uint32_t d = tmem + (threadIdx.x == 0 ? 0u : (uint32_t)N);
    const uint32_t bar = smem_u32(threadIdx.x == 0 ? &hs->bar : &hs->bar2);
    const uint32_t id = idesc_tf32(128, N, false, BMN);
    // MN-major B: K = 32 rows of 128-byte N chunks (chunk stride 32 * 128),
    // k-step +1024 bytes; K-major: k-step +32 bytes
    const uint64_t ad = sdesc_kmajor(sa);
    const uint64_t bd = BMN ? sdesc_mnmajor(sb, 32u * 128u) : sdesc_kmajor(sb);
    const uint32_t kstep = BMN ? 1024u : 32u;
    const long long t0 = clock64();
    for (int r = 0; r < reps; ++r) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (TS) umma_tf32_ts(d, tmem + 256 + 8 * k, bd + (kstep * k >> 4), id, (r | k) ? 1u : 0u);
        else umma_tf32_ss(d, ad + (32u * k >> 4), bd + (kstep * k >> 4), id, (r | k) ? 1u : 0u);
      }
    }
    umma_commit(bar);
    const bool ok = mbar_wait(bar, 0, &hs->ctl, status);
    if (threadIdx.x == 0) cycles[blockIdx.x] = ok ? clock64() - t0 : -1;
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int N, bool TS, bool BMN, bool TWO>
int run_mma_rate(int reps, int blocks, long long* cycles, uint32_t* status, cudaStream_t st) {
  const size_t smem = 120 * 1024;  // one CTA per SM: each allocates all 512 TMEM columns
  if (cudaFuncSetAttribute(mma_rate_kernel<N, TS, BMN, TWO>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return 6;
  mma_rate_kernel<N, TS, BMN, TWO><<<blocks, 128, smem, st>>>(reps, cycles, status);
  return launch_ok();
}

template <int N>
int run_mma_rate_n(int flags, int reps, int blocks, long long* cycles, uint32_t* status,
                   cudaStream_t st) {
  const bool ts = flags & 1, bmn = flags & 2, two = flags & 4;
  if (two && N > 128) return 1;  // two accumulators must fit below A
  if (two) {
    if (ts) return bmn ? run_mma_rate<N, true, true, true>(reps, blocks, cycles, status, st)
                       : run_mma_rate<N, true, false, true>(reps, blocks, cycles, status, st);
    return bmn ? run_mma_rate<N, false, true, true>(reps, blocks, cycles, status, st)
               : run_mma_rate<N, false, false, true>(reps, blocks, cycles, status, st);
  }
  if (ts) return bmn ? run_mma_rate<N, true, true, false>(reps, blocks, cycles, status, st)
                     : run_mma_rate<N, true, false, false>(reps, blocks, cycles, status, st);
  return bmn ? run_mma_rate<N, false, true, false>(reps, blocks, cycles, status, st)
             : run_mma_rate<N, false, false, false>(reps, blocks, cycles, status, st);
}

}  // namespace
}  // namespace ct

extern "C" {

// flags: bit 0 A from TMEM, bit 1 B MN-major, bit 2 two issuing threads.
int ct_diag_mma_rate(int n, int flags, int reps, int blocks, long long* cycles, void* stream) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 6;
  if (reps <= 0 || reps > (1 << 20) || blocks <= 0 || blocks > sms || !cycles || flags < 0 ||
      flags > 7)
    return 1;
  uint32_t* status = ct::diag_status();
  if (!status) return 6;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (n) {
    case 32: return ct::run_mma_rate_n<32>(flags, reps, blocks, cycles, status, st);
    case 64: return ct::run_mma_rate_n<64>(flags, reps, blocks, cycles, status, st);
    case 128: return ct::run_mma_rate_n<128>(flags, reps, blocks, cycles, status, st);
    case 256: return ct::run_mma_rate_n<256>(flags, reps, blocks, cycles, status, st);
    default: return 1;
  }
}

int ct_diag_umma_tf32(int mode, const float* a, const float* b, float* d, int n, void* stream) {
  if (!a || !b || !d || mode < 0 || mode > 4 || !(n == 32 || n == 64 || n == 128)) return 1;
  uint32_t* status = ct::diag_status();
  if (!status) return 6;
  const size_t smem = 1024 + 1024 + 128 * 128 + (size_t)n * 128;
  if (cudaFuncSetAttribute(ct::umma_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return 6;
  ct::umma_diag_kernel<<<1, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(mode, a, b, d,
                                                                                 n, status);
  return ct::launch_ok();
}

int ct_diag_umma_m64(int mode, const float* a, const float* b, float* d, int n, void* stream) {
  if (!a || !b || !d || mode < 0 || mode > 15 || !(n == 32 || n == 64) || ((mode & 4) && n != 32) ||
      ((mode & 8) && (mode & 1)))
    return 1;
  uint32_t* status = ct::diag_status();
  if (!status) return 6;
  const size_t smem = 1024 + 1024 + 64 * 128 + (size_t)n * 128;
  if (cudaFuncSetAttribute(ct::umma_m64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return 6;
  ct::umma_m64_kernel<<<1, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(mode, a, b, d, n,
                                                                                status);
  return ct::launch_ok();
}

int ct_diag_umma_pair(int mode, const float* a, const float* b, float* d, int n, void* stream) {
  if (!a || !b || !d || mode < 0 || mode > 1 || !(n == 64 || n == 128)) return 1;
  uint32_t* status = ct::diag_status();
  if (!status) return 6;
  const size_t smem = 1024 + 1024 + (size_t)(n / 2) * 64 * 4;
  if (cudaFuncSetAttribute(ct::umma_pair_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return 6;
  ct::umma_pair_diag_kernel<<<2, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(mode, a, b,
                                                                                      d, n, status);
  return ct::launch_ok();
}

int ct_diag_status(unsigned int* flag_out) {
  if (!flag_out) return 1;
  uint32_t* status = ct::diag_status();
  if (!status) return 6;
  return cudaMemcpy(flag_out, status, sizeof(*flag_out), cudaMemcpyDeviceToHost) == cudaSuccess
             ? 0
             : 6;
}

}  // extern "C"
