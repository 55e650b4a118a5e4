// watchdog.cu -- failure-detection self-test (ct_watchdog_selftest).
//
// Every bounded wait of the tensor-core kernels gives up after the device's
// wait limit, records CT_DEVSTAT_TIMEOUT, raises its CTA's abort flag and lets
// the CTA tear down: the MMA-issuing thread commits and drains its own work,
// all threads meet, TMEM is released.  This kernel exercises exactly that path
// without any fault: its warps wait on a barrier phase that nothing completes
// (the barrier expects one arrival that never comes), so the waits run out
// after the limit, and the CTA then takes the same teardown.  Nothing spins
// unbounded: the waits suspend in hardware between polls and stop at the
// limit; the drain is bounded too.
#include "ct_internal.h"
#include "fa2_common.cuh"

namespace ct {
namespace {

struct SelftestSmem {
  uint64_t never;      // one arrival expected, none ever made
  uint64_t mma_final;  // the teardown commit of the "MMA" thread
  CtaCtl ctl;
};

__global__ void __launch_bounds__(128, 1) watchdog_selftest_kernel(uint32_t* status) {
  __shared__ SelftestSmem sm;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&sm.never), 1);
    mbar_init(smem_u32(&sm.mma_final), 1);
    sm.ctl.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.ctl.tmem_base), 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.ctl.tmem_base;
  // Every warp waits for phase 0 of `never`; the first lane whose wait runs out
  // raises the abort flag and the status word, the others see the flag.
  fa2::warp_wait(smem_u32(&sm.never), 0, &sm.ctl, status);
  // Teardown as in the attention kernels: the MMA thread commits (nothing of it
  // is in flight) and waits, bounded, for that commit to arrive.
  if (warp == 1 && lane == 0) {
    umma_commit(smem_u32(&sm.mma_final));
    fa2::mbar_drain(smem_u32(&sm.mma_final), 0);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

}  // namespace

int launch_watchdog_selftest(const DeviceInfo& dev, cudaStream_t st) {
  watchdog_selftest_kernel<<<1, 128, 0, st>>>(dev.status);
  return check_launch();
}

}  // namespace ct
