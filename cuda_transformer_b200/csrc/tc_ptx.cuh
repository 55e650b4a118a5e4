// tc_ptx.cuh -- thin inline-PTX layer for sm_100a: mbarriers with bounded
// waits, TMA tile loads, Tensor Memory (TMEM) allocation / load / store, and
// tcgen05.mma (kind::tf32) with shared-memory matrix descriptors.
//
// Every wait in this file is bounded: after the device's wait limit (the
// watchdog block's limit_ns, 2 s unless set through ct_set_wait_limit_ns) it
// records CT_DEVSTAT_TIMEOUT in the device status word, raises the CTA's abort
// flag and returns false.  Callers then skip the rest of their work and fall
// through to the kernel teardown (drain in-flight copies, release TMEM).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

// Default wait limit, and the bound of teardown drains (waits for copies and
// MMAs already in flight, which complete on their own).
#ifndef CT_WAIT_TIMEOUT_NS
#define CT_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: legitimate waits are microseconds
#endif

namespace ct {

// Device status word bits (see ct_device_status in the C ABI).
constexpr uint32_t CT_DEVSTAT_TIMEOUT = 1u;

// Per-device watchdog block (one __device__ instance in capi.cu).  Kernels get
// the address of its first member as `uint32_t* status`: the status word that
// expired waits OR CT_DEVSTAT_* bits into, followed by the limit of every
// bounded wait in nanoseconds (set by ct_set_wait_limit_ns).
struct WatchBlock {
  uint32_t status;
  uint32_t reserved;
  unsigned long long limit_ns;
};
__host__ __device__ __forceinline__ unsigned long long wait_limit_ns(const uint32_t* status) {
  return reinterpret_cast<const volatile WatchBlock*>(status)->limit_ns;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Per-CTA control block placed in shared memory by every tcgen05 kernel.
struct CtaCtl {
  volatile uint32_t abort;   // set when any wait in this CTA expired
  uint32_t tmem_base;        // written by tcgen05.alloc
};

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy accesses (TMA writes, tensor-core operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of a phase (test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase has not completed is
// suspended by the hardware (woken when the phase completes or after at most
// `hint_ns`) instead of spinning, so waiting warps leave their scheduler's
// issue slots to the warps doing work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Slow path of mbar_wait: suspend-hinted polls bounded by the device's wait
// limit.  Kept out of line so the fast path is one try_wait and a branch.
static __device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, CtaCtl* ctl,
                                                   uint32_t* status) {
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(status);
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
    if ((i & 15u) == 0u) {
      if (ctl->abort) return false;
      if (*reinterpret_cast<volatile uint32_t*>(status) != 0u) {  // another CTA gave up
        ctl->abort = 1u;
        return false;
      }
      if (globaltimer_ns() - t0 > limit) {
        ctl->abort = 1u;
        atomicOr(status, CT_DEVSTAT_TIMEOUT);
        return false;
      }
    }
  }
}

// Waits until the phase with the given parity of barrier `bar` has completed.
// Returns false (and raises ctl->abort and the device status word) if the
// wait exceeds the device's wait limit or another wait of this CTA already
// failed.
// The common case -- the phase has completed -- costs one try_wait: the MMA
// issuing thread pays for every instruction between two MMA groups, because
// the tensor pipe idles while that thread is away (measured on B200).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, CtaCtl* ctl,
                                          uint32_t* status) {
  if (__builtin_expect(mbar_try_wait(bar, parity), 1)) return true;
  return mbar_wait_slow(bar, parity, ctl, status);
}

// ------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(bar)
      : "memory");
}

// TMA stores from shared memory (bulk-group completion).  Coordinates must be
// non-negative; the innermost one times the element size a multiple of 16.
// Box elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(src)
      : "memory");
}
// Element-wise global += shared (the add happens in L2, per element).
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, uint32_t src, int c0,
                                                  int c1, int c2) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%1, %2, %3}], [%4];" ::
          "l"(reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(src)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until at most N committed bulk groups are incomplete (writes done).
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Orders async-proxy (TMA) global accesses with this thread's generic ones.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ------------------------------------------------------------ tcgen05 sync
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------- TMEM allocation
// Executed by one full warp.  The allocated base address is written to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// TMEM address of (lane, column): lane in bits 31..16, column in 15..0.
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// ------------------------------------------------------- TMEM load/store
// 32 lanes x 32 columns of 32-bit: thread t of the warp gets lane (quadrant
// base + t), columns col..col+31.  The wait is inside the same asm statement
// so the registers are valid when the statement retires.
#define CT_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), \
                 "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define CT_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), \
                 "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : CT_R8(0), CT_R8(8), CT_R8(16), CT_R8(24)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : CT_R8(0), CT_R8(8)
      : "r"(taddr)
      : "memory");
}
// Stores do not wait; call tmem_wait_st() before publishing them.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      CT_W8(0), CT_W8(8), CT_W8(16), CT_W8(24)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      CT_W8(0), CT_W8(8)
      : "memory");
}
// 16 lanes x 32-bit, two halves (M = 64 accumulators, whose rows occupy 16
// lanes of each warp's quadrant): threads 0-15 access lanes base .. base + 15
// at columns [col, col + N), threads 16-31 the same lanes at [col + N,
// col + 2N) (half-split offset N).  The address's lane field selects the
// quadrant's lower (+0) or upper (+16) half.  N in {8, 16, 32}.
template <int N>
__device__ __forceinline__ void tmem_ld_16x32bx2(uint32_t taddr, float (&v)[N]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  static_assert(N == 8 || N == 16 || N == 32, "16x32bx2 width");
  if constexpr (N == 8) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x32bx2.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], 8;\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : CT_R8(0)
        : "r"(taddr)
        : "memory");
  } else if constexpr (N == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x32bx2.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15}, [%16], 16;\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : CT_R8(0), CT_R8(8)
        : "r"(taddr)
        : "memory");
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], "
        "32;\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : CT_R8(0), CT_R8(8), CT_R8(16), CT_R8(24)
        : "r"(taddr)
        : "memory");
  }
}
// Store counterpart of tmem_ld_16x32bx2 (does not wait; tmem_wait_st before
// publishing).
template <int N>
__device__ __forceinline__ void tmem_st_16x32bx2(uint32_t taddr, const float (&v)[N]) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  static_assert(N == 8 || N == 16, "16x32bx2 width");
  if constexpr (N == 8) {
    asm volatile("tcgen05.st.sync.aligned.16x32bx2.x8.b32 [%0], 8, {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
                     taddr),
                 CT_W8(0)
                 : "memory");
  } else {
    asm volatile(
        "tcgen05.st.sync.aligned.16x32bx2.x16.b32 [%0], 16, {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,"
        "%12,%13,%14,%15,%16};" ::"r"(taddr),
        CT_W8(0), CT_W8(8)
        : "memory");
  }
}
#undef CT_R8
#undef CT_W8

// --------------------------------------------------- UMMA descriptors
// Shared-memory matrix descriptor (64-bit):
//   bits  0-13 start address >> 4      bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4 bits 46-47 version (1 on sm_100)
//   bits 49-51 base offset (0)         bits 61-63 layout (2 = SWIZZLE_128B,
//                                                  1 = SWIZZLE_128B_BASE32B)
// K-major operand (layout 2, the pattern TMA writes with
//   CU_TENSOR_MAP_SWIZZLE_128B): rows of 128 bytes hold 32 fp32 along K; 16-byte
//   units are XOR-swizzled with row % 8; SBO = distance between 8-row groups
//   (1024 when dense), LBO unused (16).  Stepping K by 8 fp32 inside the
//   128-byte row advances the start address by 32 bytes.
// MN-major operand (layout 1, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B; the only
//   MN-major layout the tensor core accepts for TF32): 128-byte rows hold 32
//   consecutive M (or N) elements, one row per K index; 32-byte units are
//   XOR-swizzled with row % 4; LBO = distance between consecutive 32-element
//   M/N chunks, SBO = distance between 4-row K groups (512 when dense).
//   Stepping K by 8 advances the start address by 1024 bytes.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                          uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)layout << 61;
  return d;
}
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t saddr) {
  return sdesc(saddr, 16u, 1024u, 2u);
}
__device__ __forceinline__ uint64_t sdesc_mnmajor(uint32_t saddr, uint32_t chunk_stride_bytes) {
  return sdesc(saddr, chunk_stride_bytes, 512u, 1u);
}

// Instruction descriptor for kind::tf32 with an FP32 accumulator:
//   bits 4-5 D format (1 = F32), 7-9 A format (2 = TF32), 10-12 B format,
//   15 A major (1 = MN), 16 B major, 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ------------------------------------------------------------- MMA issue
// D[tmem] (+)= A * B, A and B from shared memory.
__device__ __forceinline__ void umma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A * B, A from TMEM (rows = lanes, K = columns), B from smem.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on `bar` when all previously issued tcgen05 async ops of this
// thread have completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// ------------------------------------------------- CTA pairs (cta_group::2)
// A cluster of two CTAs on two SMs runs one tensor-core product of M = 256:
// rows 0-127 of A and D live in the even CTA's Tensor Memory and rows 128-255
// in the odd CTA's (same TMEM address in both); B's N rows are split, rows
// [0, N/2) in the even CTA's shared memory and [N/2, N) in the odd CTA's, both
// at the address the descriptor names.  The even CTA's thread issues, and its
// commits arrive on the barrier at the same address in both CTAs.  Kernels
// using these run every tcgen05 instruction with cta_group::2 (TMEM allocation
// included) and are launched with cluster dimension 2.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The address in CTA `rank` of this cluster of the shared-memory word at
// `addr` (a shared::cta address of the calling CTA).
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrives on an mbarrier of any CTA of the cluster (address from mapa_shared),
// with the arrive's default release at CTA scope.  The pair kernels publish
// only data that lives in the arriving CTA itself -- its shared memory
// (after fence.proxy.async) or its Tensor Memory (after tcgen05.wait::st and
// tcgen05.fence::before_thread_sync) -- for tensor-core operations that the
// other CTA issues once it has seen the arrival; the same protocol as the
// CUTLASS sm100 pair pipelines.  A cluster-scope release would cost a
// cluster fence (~320 cycles per arrival, measured on B200; this arrive: ~6).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// Barrier over every thread of both CTAs of the cluster (each thread arrives
// once per use).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Pair allocation: the same warp index of both CTAs calls each of these, with
// the same destination address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D (+)= A * B over the CTA pair (M = 256), A from both CTAs' TMEM.
__device__ __forceinline__ void umma_tf32_ts_pair(uint32_t d_tmem, uint32_t a_tmem,
                                                  uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on the barrier at `bar` in both CTAs of the pair when all
// previously issued tcgen05 operations of the calling thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  const uint16_t both = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(both)
      : "memory");
}

// --------------------------------------------------------- TF32 helpers
// Round-to-nearest (ties away) to TF32; the low 13 bits of the result are 0.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// The same rounding for values known to be finite (softmax probabilities and
// score gradients): adding half of the dropped 13-bit field carries into the
// kept bits -- and on into the exponent -- exactly when the dropped part is at
// least half a TF32 ulp, ties going away from zero (sign-magnitude).  Two
// integer operations instead of a conversion, which shares its pipe with the
// exponentials.  Identical to cvt.rna.tf32.f32 on finite inputs (checked on
// the device bit for bit, ties, subnormals and the overflow edge included).
__device__ __forceinline__ float tf32_round_finite(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
// TF32 value the tensor core uses for an FP32 operand: the 13 low mantissa
// bits are dropped (truncation; checked on the device by the test-suite).
__device__ __forceinline__ float tf32_trunc(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}
// 3xTF32 split x = hi + lo: hi = tf32_trunc(x) is exact, lo = x - hi is exact
// in FP32 and loses at most 2^-21 |x| when the tensor core truncates it.
// Two ALU operations (no conversion instructions).
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
  hi = tf32_trunc(x);
  lo = x - hi;
}

// Packed pairs of FP32 operations (sm_100 f32x2): one instruction, two
// independent IEEE round-to-nearest results -- bit-identical to two scalar
// fmaf / + / - / * -- so row loops spend half the issue slots on them.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1,
                                      float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
#define CT_F32X2_BINOP(NAME, OP)                                                                 \
  __device__ __forceinline__ void NAME(float& d0, float& d1, float a0, float a1, float b0,       \
                                       float b1) {                                               \
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"                                                          \
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t" OP                                   \
        " rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"                                              \
        : "=f"(d0), "=f"(d1)                                                                     \
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));                                                   \
  }
CT_F32X2_BINOP(fadd2, "add.rn.f32x2")
CT_F32X2_BINOP(fsub2, "sub.rn.f32x2")
CT_F32X2_BINOP(fmul2, "mul.rn.f32x2")
#undef CT_F32X2_BINOP

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Read-only global load issued where it stands: an ordered (volatile) asm
// statement, so the compiler cannot sink it towards the first use of its
// result (used to prefetch one pipeline step ahead).
__device__ __forceinline__ float ldg_nc_early(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// 128-bit shared-memory accessors on 32-bit shared addresses.
__device__ __forceinline__ float4 lds128(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// Low parts x - tf32_trunc(x) of a float4 (3xTF32 split), subtractions packed.
__device__ __forceinline__ float4 tf32_lo4(float4 x) {
  float4 l;
  fsub2(l.x, l.y, x.x, x.y, tf32_trunc(x.x), tf32_trunc(x.y));
  fsub2(l.z, l.w, x.z, x.w, tf32_trunc(x.z), tf32_trunc(x.w));
  return l;
}

// Tile preparation by a group of NTHREADS threads, BYTES bytes per tile.
// Thread t handles the 16-byte words t, t + NTHREADS, ... (a warp covers 512
// contiguous bytes: no bank conflicts).  Words go in batches of up to 8: every
// load of a batch is issued before its first store (the accessors are ordered
// volatile asm), so the shared-memory latency is paid once per batch rather
// than once per word.
template <uint32_t BYTES, uint32_t NTHREADS>
struct TilePrep {
  static constexpr uint32_t PER = BYTES / (NTHREADS * 16u);  // words per thread
  static constexpr uint32_t U = PER < 8u ? PER : 8u;
  static_assert(PER >= 1 && PER % U == 0 && BYTES % (NTHREADS * 16u) == 0, "tile prep shape");
};

// 3xTF32 split of a shared-memory tile: lo + i receives x - tf32_trunc(x) for
// every fp32 word x at raw + i.  The raw tile itself is the "hi" operand,
// because the tensor core reads it truncated to tf32_trunc(x).  Both buffers
// share the same swizzled layout, so the element correspondence is positional.
template <uint32_t BYTES, uint32_t NTHREADS>
__device__ __forceinline__ void split_tile_smem(uint32_t raw, uint32_t lo, uint32_t tid) {
  using P = TilePrep<BYTES, NTHREADS>;
#pragma unroll 1
  for (uint32_t w0 = 0; w0 < P::PER; w0 += P::U) {
    float4 x[P::U];
#pragma unroll
    for (uint32_t u = 0; u < P::U; ++u) x[u] = lds128(raw + (tid + (w0 + u) * NTHREADS) * 16u);
#pragma unroll
    for (uint32_t u = 0; u < P::U; ++u)
      sts128(lo + (tid + (w0 + u) * NTHREADS) * 16u,
             tf32_lo4(x[u]));
  }
}

// 3xTF32 split of a tile stored as interleaved chunks: CHUNK raw bytes, then
// their CHUNK low-part bytes, repeated (BYTES raw bytes in all).  An MMA can
// then read a raw chunk and its low part as one operand of twice the rows.
template <uint32_t BYTES, uint32_t NTHREADS, uint32_t CHUNK>
__device__ __forceinline__ void split_tile_smem_il(uint32_t base, uint32_t tid) {
  using P = TilePrep<BYTES, NTHREADS>;
  static_assert(BYTES % CHUNK == 0 && CHUNK % 16u == 0, "chunk shape");
  auto raw_at = [&](uint32_t w) {
    const uint32_t byte = w * 16u;
    return base + (byte / CHUNK) * 2u * CHUNK + byte % CHUNK;
  };
#pragma unroll 1
  for (uint32_t w0 = 0; w0 < P::PER; w0 += P::U) {
    float4 x[P::U];
#pragma unroll
    for (uint32_t u = 0; u < P::U; ++u) x[u] = lds128(raw_at(tid + (w0 + u) * NTHREADS));
#pragma unroll
    for (uint32_t u = 0; u < P::U; ++u)
      sts128(raw_at(tid + (w0 + u) * NTHREADS) + CHUNK,
             tf32_lo4(x[u]));
  }
}

// Prepares a K-major tile landed by TMA -- per 32-column chunk (stride KCH)
// BN rows of 128 bytes in the 128-byte swizzle (16-byte unit u of row r at
// u ^ (r % 8)) -- and writes the same data as an MN-major tile at `mn` (chunk
// stride BN*128, 32-byte-atom swizzle: 32-byte unit a of row r at a ^ (r % 4)).
// SPLIT == 1 rounds both copies to the nearest TF32 (in place for the K-major
// one); SPLIT == 3 keeps the raw values and writes the low parts x - trunc(x)
// at +KLO (K-major) and +MLO (MN-major).  Each word moves within its row, so a
// warp's stores stay free of bank conflicts.  WRITE_K == false (SPLIT == 1):
// the K-major copy is already rounded and is only read (the tensor core may be
// reading it at the same time).
template <int SPLIT, uint32_t BYTES, uint32_t NTHREADS, uint32_t BN, uint32_t KCH, uint32_t KLO,
          uint32_t MLO, bool WRITE_K = true>
__device__ __forceinline__ void derive_tile_smem(uint32_t k, uint32_t mn, uint32_t tid) {
  using P = TilePrep<BYTES, NTHREADS>;
  constexpr uint32_t CH = BN * 128u;
  static_assert((CH & (CH - 1)) == 0, "chunk size");
#pragma unroll 1
  for (uint32_t w0 = 0; w0 < P::PER; w0 += P::U) {
    float4 x[P::U];
    uint32_t ka[P::U], ma[P::U];
#pragma unroll
    for (uint32_t u = 0; u < P::U; ++u) {
      const uint32_t o = (tid + (w0 + u) * NTHREADS) * 16u;
      const uint32_t c = o / CH, rem = o % CH, r = rem >> 7, pu = (rem >> 4) & 7u;
      const uint32_t lu = pu ^ (r & 7u);                                // logical 16-byte unit
      const uint32_t mu = ((((lu >> 1) ^ (r & 3u)) << 1) | (lu & 1u));  // its MN-major place
      ka[u] = k + c * KCH + rem;
      ma[u] = mn + c * CH + (r << 7) + (mu << 4);
      x[u] = lds128(ka[u]);
    }
#pragma unroll
    for (uint32_t u = 0; u < P::U; ++u) {
      if constexpr (SPLIT == 3) {
        const float4 lo = tf32_lo4(x[u]);
        sts128(ka[u] + KLO, lo);
        sts128(ma[u], x[u]);
        sts128(ma[u] + MLO, lo);
      } else {
        const float4 y = make_float4(tf32_round_finite(x[u].x), tf32_round_finite(x[u].y),
                                     tf32_round_finite(x[u].z), tf32_round_finite(x[u].w));
        if constexpr (WRITE_K) sts128(ka[u], y);
        sts128(ma[u], y);
      }
    }
  }
}

// TF32 mode: rounds a shared-memory tile in place to the nearest TF32 value
// (the tensor core itself truncates the 13 low mantissa bits).  The rounding
// is the two-integer-operation form of cvt.rna.tf32.f32 (tf32_round_finite),
// which keeps the conversion pipe free for the exponentials; it differs from
// cvt.rna only on NaNs whose payload lies entirely in the 13 dropped bits,
// which become infinities -- exactly what the tensor core's own truncation
// makes of them.
template <uint32_t BYTES, uint32_t NTHREADS>
__device__ __forceinline__ void round_tile_smem(uint32_t raw, uint32_t tid) {
  using P = TilePrep<BYTES, NTHREADS>;
#pragma unroll 1
  for (uint32_t w0 = 0; w0 < P::PER; w0 += P::U) {
    float4 x[P::U];
#pragma unroll
    for (uint32_t u = 0; u < P::U; ++u) x[u] = lds128(raw + (tid + (w0 + u) * NTHREADS) * 16u);
#pragma unroll
    for (uint32_t u = 0; u < P::U; ++u)
      sts128(raw + (tid + (w0 + u) * NTHREADS) * 16u,
             make_float4(tf32_round_finite(x[u].x), tf32_round_finite(x[u].y),
                         tf32_round_finite(x[u].z), tf32_round_finite(x[u].w)));
  }
}

// Byte offset of element (row, col) in a tile of `rows` rows written by TMA
// with 32-float boxes: column chunk c = col / 32 occupies rows * 128 bytes.
// K-major tiles (SWIZZLE_128B): the 16-byte unit index is XORed with row % 8.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t col,
                                                          uint32_t rows) {
  const uint32_t chunk = col >> 5;
  const uint32_t in_row = (col & 31u) * 4u;
  const uint32_t unit = (in_row >> 4) ^ (row & 7u);
  return chunk * rows * 128u + row * 128u + (unit << 4) + (in_row & 15u);
}
// MN-major tiles (SWIZZLE_128B_ATOM_32B): the 32-byte unit index is XORed
// with row % 4.
__host__ __device__ __forceinline__ uint32_t sw128_32b_offset(uint32_t row, uint32_t col,
                                                              uint32_t rows) {
  const uint32_t chunk = col >> 5;
  const uint32_t in_row = (col & 31u) * 4u;
  const uint32_t unit = (in_row >> 5) ^ (row & 3u);
  return chunk * rows * 128u + row * 128u + (unit << 5) + (in_row & 31u);
}

}  // namespace ct
