// fa2_bwd_fused.cu -- one-kernel FlashAttention-2 backward on the sm_100a
// tensor cores (TF32 mode, head dim 64): ct_fa2_bwd_fused.
//
// The default backward (fa2_bwd_tc.cu) forms P and dS twice, once in the
// query-stationary dQ kernel and once in the key/value-stationary dK/dV kernel
// -- the split the reference uses to stay free of atomics
// (flash_attention.cuh:216-504).  Here one key/value-stationary CTA of 128 key
// rows forms, per 64-query tile i,
//   S^T = K Q_i^T, dP^T = V dO_i^T, P^T, dS^T       once (row warps, TMEM)
//   dV += P^T dO_i,  dK += dS^T Q_i                 TMEM accumulators
//   dQ_i(kt) = dS_i K                               an M = 64 MMA: A = dS from
//                                                   shared memory, B = K
// and adds its dQ contribution into dQ in global memory.  dK and dV come from
// the same MMA sequence as the dK/dV kernel's (bit-identical results).
//
// Deterministic dQ.  The contributions to a query tile are added in a fixed
// order of key tiles, highest first: the highest contributing key tile stores,
// each lower one adds once its predecessor's additions are visible.  One
// counter per (head, query tile, TMEM lane quadrant) counts the contributions
// made; a contributor waits (bounded) until the counter equals its rank, adds
// its 16 rows, fences, and increments it.  The sum is therefore the same
// sequence of round-to-nearest FP32 additions on every run.
//
// Progress.  A CTA takes its (key tile, head) from a ticket counter drawn at
// start, key tiles from the last to the first inside each head group, so it
// only ever waits for CTAs holding smaller tickets: those already run or have
// finished, and the waits cannot form a cycle.  With a causal mask, key tile kt
// starts at query tile 2 kt (its diagonal) and kt + 1 at 2 kt + 2, so kt + 1
// reaches a query tile two of its steps before kt does.
//
// Measured on B200 (B4 H32 N4096, causal): 3.3-3.4 ms against 2.5 ms for the
// two-kernel TF32 backward, which therefore stays the default.  The FP32
// additions into dQ (16 KB of red.global per CTA step) run into the L2's
// atomic throughput, and the row warps, which also store dS for the dQ MMA,
// take about twice as long per step as in the dK/dV kernel.
//
// Sequences longer than kSegLen run one launch per query segment; a segment's
// query tiles get all their dQ contributions inside its launch, dK / dV add
// into the previous segment's output.
#include <algorithm>

#include "fa2_bwd_parts.cuh"

namespace ct {
namespace {

using namespace fa2;

constexpr uint32_t kUpperLanes = 16u << 16;  // TMEM lane offset of a quadrant's upper half
constexpr int kFusedBN = 64;                 // queries per step (the dQ MMA's M)

// Five warpgroups (20 warps).  A warp reads and writes the TMEM lane quadrant
// warp % 4, so every group that touches the row-indexed TMEM spans all four.
//   WG0 (warps 0-3): 0 TMA producer, 1 S^T / dV issuer (and TMEM allocator),
//                    2 dP^T / dK issuer, 3 dQ issuer
//   WG1, WG2 (4-11): row warps, query columns [0, 32) and [32, 64) of a step
//   WG3 (12-15):     tile preparation (TF32 rounding, MN-major copies, LSE / delta)
//   WG4 (16-19):     dQ epilogue (TMEM -> ordered addition into dQ)
// 640 threads launch with 96 registers each; the row groups take 104 and the
// other three give up theirs down to 88 (setmaxnreg: 3 x 88 + 2 x 104 <=
// 5 x 96; the launch count is checked against the compiled kernel before the
// first launch).  ptxas fits every role in its share, but for a few words of
// the epilogue's two-step register queue that spill to local memory.
constexpr int kFusedThreads = 640;
constexpr int kFusedLaunchRegs = 96, kFusedLowRegs = 88, kFusedRowRegs = 104;
static_assert(3 * kFusedLowRegs + 2 * kFusedRowRegs <= 5 * kFusedLaunchRegs, "register split");
constexpr int kFusedPrepWarp0 = 12, kFusedEpiWarp0 = 16;
constexpr int kFusedIssuer1 = 1, kFusedIssuer2 = 2, kFusedIssuer3 = 3;

template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Shared memory: a 2 KB header (barriers, then the LSE / delta slots), then
// 1024-aligned tiles:
//   K MN-major (dQ's B, 128 keys x D) |
//   ring 1: NS1 slots [Q_i | dO_i] K-major (TMA lands them; rounded in place) |
//   ring 2: NS2 slots [Q_i | dO_i] MN-major (written by the preparation warps) |
//   dS MN-major (dQ's A: 128 keys x 64 queries).
// Ring 1 is read by S^T_i and dP^T_i, early in a step, and ring 2 by dV_i and
// dK_i, late: separate rings let the next tiles land while a step's MN-major
// copies are still in use (one 4-slot ring of both layouts does not fit).
template <int D_, int NS1_, int NS2_>
struct FusedCfg {
  static constexpr int D = D_, BN = kFusedBN, NS1 = NS1_, NS2 = NS2_;
  static constexpr uint32_t TILE = (uint32_t)BN * D_ * 4u;  // one Q or dO tile
  static constexpr uint32_t CH = (uint32_t)BN * 128u;      // one 32-column chunk of a tile
  static constexpr uint32_t SLOT = 2u * TILE;              // [Q | dO]
  static constexpr uint32_t KMN_BYTES = (uint32_t)kRows * D_ * 4u;
  static constexpr uint32_t DS_BYTES = (uint32_t)kRows * BN * 4u;
  static constexpr uint32_t OFF_KMN = 0, OFF_R1 = KMN_BYTES, OFF_R2 = OFF_R1 + NS1_ * SLOT,
                            OFF_DS = OFF_R2 + NS2_ * SLOT, TILE_BYTES = OFF_DS + DS_BYTES;
  static constexpr uint32_t KCHUNK = (uint32_t)kRows * 128u;  // one 32-column chunk of 128 rows
  static constexpr uint32_t HEADER = 2048, VEC_OFF = 512;
  static constexpr uint32_t TMEM_COLS = 512;
  // TMEM column map: K | V | dK | dV | S^T x 2 | dP^T | dQ x 2 (lane halves)
  static constexpr uint32_t TC_K = 0, TC_V = D_, TC_DK = 2 * D_, TC_DV = 3 * D_, TC_S = 4 * D_,
                            TC_DP = TC_S + 2 * BN, TC_DQ = TC_DP + BN;
  static_assert(TC_DQ + D_ <= TMEM_COLS, "TMEM budget");
  static_assert(D_ == 64, "the fused backward covers head dim 64");
  static_assert(VEC_OFF + NS2_ * 2 * BN * 4 <= HEADER, "header budget");
};

template <int NS1, int NS2>
struct FusedBars {
  uint64_t full1[NS1], rdy1[NS1], empty1[NS1];  // ring 1: landed, prepared, read (S^T, dP^T)
  uint64_t rdy2[NS2], empty2[NS2];              // ring 2 (+ LSE / delta): written, read (dV, dK)
  uint64_t s_full[2], p_full[2], dp_full, ds_full, dqd;
  uint64_t kmn_full, kmn_ready, dq_full[2], dq_free[2];
  uint64_t rows_ready, done, mma_final, mma_final2, mma_final3;
  CtaCtl ctl;
  uint32_t ticket;
};

struct FusedParams {
  BwdParams b;
  float* dq;            // dense [B,H,T,D]
  uint32_t* counters;   // [B*H][n_qt][4] contributions made, zero before the call
  uint32_t* ticket;     // this launch's ticket counter, zero before the launch
  int n_qt;             // query tiles of kFusedBN rows per head
};

template <class C>
constexpr size_t fused_smem_bytes() {
  static_assert(sizeof(FusedBars<C::NS1, C::NS2>) <= C::VEC_OFF, "barrier block");
  constexpr size_t b = C::HEADER + 1024 + (size_t)C::TILE_BYTES;  // 1024: alignment slack
  static_assert(b <= 227 * 1024, "shared memory budget");
  return b;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Warp-uniform bounded wait until *flag >= want (a counter written by other
// CTAs; every lane polls with acquire semantics).  Expiry records
// CT_DEVSTAT_TIMEOUT and raises the CTA's abort flag, like mbar_wait.
__device__ __noinline__ bool flag_wait_geq(const uint32_t* flag, uint32_t want, CtaCtl* ctl,
                                           uint32_t* status) {
  bool ok = true;
  if (ld_acquire_u32(flag) < want) {
    const uint64_t t0 = globaltimer_ns();
    const uint64_t limit = wait_limit_ns(status);
    for (uint32_t i = 1;; ++i) {
      __nanosleep(64);
      if (ld_acquire_u32(flag) >= want) break;
      if ((i & 15u) == 0u) {
        if (ctl->abort || *reinterpret_cast<volatile uint32_t*>(status) != 0u) {
          ctl->abort = 1u;
          ok = false;
          break;
        }
        if (globaltimer_ns() - t0 > limit) {
          ctl->abort = 1u;
          atomicOr(status, CT_DEVSTAT_TIMEOUT);
          ok = false;
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

template <class C>
__global__ void __launch_bounds__(kFusedThreads, 1)
    fa2_bwd_fused_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                            const __grid_constant__ CUtensorMap tmG,
                            const __grid_constant__ CUtensorMap tmK, const FusedParams fp) {
  constexpr int D = C::D, BN = C::BN, NS1 = C::NS1, NS2 = C::NS2;
  const BwdParams& p = fp.b;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (status_raised(p.status)) return;
  auto* bars = reinterpret_cast<FusedBars<NS1, NS2>*>(smem_raw);
  float* vec = reinterpret_cast<float*>(smem_raw + C::VEC_OFF);
  const uint32_t base = (smem_u32(smem_raw) + C::HEADER + 1023u) & ~1023u;
  const uint32_t kmn = base + C::OFF_KMN, ring1 = base + C::OFF_R1, ring2 = base + C::OFF_R2,
                 dsm = base + C::OFF_DS;
  CtaCtl* ctl = &bars->ctl;
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) bars->ticket = atomicAdd(fp.ticket, 1u);
  __syncthreads();
  int kt, bh;  // last key tile first inside each head group (see the file comment)
  cta_tile_at(bars->ticket, p.n_tiles, p.bh_total, p.head_group, true, kt, bh);
  const int b = bh / p.H, h = bh % p.H;
  const int k0 = kt * kRows, T = p.T;
  const int j0 = max(p.causal ? k0 / BN : 0, p.seg_lo / BN);
  const int j1 = min((T + BN - 1) / BN, (p.seg_hi + BN - 1) / BN);
  const int n = max(0, j1 - j0);
  if (n == 0 && p.accumulate_out) return;  // nothing to add (uniform exit)

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS1; ++s) {
      mbar_init(B(bars->full1[s]), 1);
      mbar_init(B(bars->rdy1[s]), kPrepWarps);
      mbar_init(B(bars->empty1[s]), 2);  // S^T_i, dP^T_i read it
    }
    for (int s = 0; s < NS2; ++s) {
      mbar_init(B(bars->rdy2[s]), kPrepWarps);
      mbar_init(B(bars->empty2[s]), 2);  // dV_i, dK_i read it
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(B(bars->s_full[i]), 1);
      mbar_init(B(bars->p_full[i]), 8);
      mbar_init(B(bars->dq_full[i]), 1);
      mbar_init(B(bars->dq_free[i]), 4);  // the epilogue warps
    }
    mbar_init(B(bars->dp_full), 1);
    mbar_init(B(bars->ds_full), 8);
    mbar_init(B(bars->dqd), 1);
    mbar_init(B(bars->kmn_full), 1);
    mbar_init(B(bars->kmn_ready), kPrepWarps);
    mbar_init(B(bars->rows_ready), 8);
    mbar_init(B(bars->done), 2);
    mbar_init(B(bars->mma_final), 1);
    mbar_init(B(bars->mma_final2), 1);
    mbar_init(B(bars->mma_final3), 1);
    ctl->abort = 0;
    fence_barrier_init();
  }
  if (warp == kFusedIssuer1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int wg = warp / 4;
  if (wg == 1 || wg == 2) regs_inc<kFusedRowRegs>();
  else regs_dec<kFusedLowRegs>();
  auto slot1 = [&](int i) { return ring1 + (uint32_t)(i % NS1) * C::SLOT; };
  auto slot2 = [&](int i) { return ring2 + (uint32_t)(i % NS2) * C::SLOT; };
  constexpr uint32_t idS = idesc_tf32(128, BN, false, false);
  constexpr uint32_t idO = idesc_tf32(128, D, false, true);
  constexpr uint32_t idQ = idesc_tf32(64, D, true, true);

  if (warp == 0) {
    // TMA producer (lane 0): K once (MN-major), then [Q_i | dO_i] K-major into ring 1.
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmG);
      tma_prefetch_desc(&tmK);
      mbar_arrive_expect_tx(B(bars->kmn_full), C::KMN_BYTES);
      tma_load_5d(kmn, &tmK, B(bars->kmn_full), 0, k0, 0, h, b);
      int last = -1;
      for (int i = 0; i < n; ++i) {
        const int s = i % NS1, r = i / NS1;
        if (r > 0 && !mbar_wait(B(bars->empty1[s]), (r - 1) & 1, ctl, p.status)) break;
        const uint32_t st = slot1(i), fb = B(bars->full1[s]);
        mbar_arrive_expect_tx(fb, C::SLOT);
        tma_load_5d(st, &tmQ, fb, 0, (j0 + i) * BN, 0, h, b);
        tma_load_5d(st + C::TILE, &tmG, fb, 0, (j0 + i) * BN, 0, h, b);
        last = i;
      }
      if (ctl->abort) {  // let issued copies land before the CTA exits
        mbar_drain(B(bars->kmn_full), 0);
        for (int i = max(0, last - NS1 + 1); i <= last; ++i)
          mbar_drain(B(bars->full1[i % NS1]), (i / NS1) & 1);
      }
    }
    __syncwarp();
  } else if (warp == kFusedIssuer1) {
    // Step i, S buffer i % 2:  [P_i ready, MN-major copies ready]  dV += P_i^T dO_i
    //   -> empty2;  [tiles i+2 rounded]  S^T_{i+2} -> s_full, empty1
    if (lane == 0) {
      auto issue_S = [&](int i) {
        mma_chain<1, D, false, BN, C::TILE>(tmem + C::TC_S + (uint32_t)(i & 1) * BN,
                                            tmem + C::TC_K, 0, sdesc_kmajor(slot1(i)), idS,
                                            false);
        umma_commit(B(bars->s_full[i & 1]));
        umma_commit(B(bars->empty1[i % NS1]));
      };
      bool ok = n > 0 && mbar_wait(B(bars->rows_ready), 0, ctl, p.status) &&
                mbar_wait(B(bars->rdy1[0]), 0, ctl, p.status);
      if (ok) {
        tc_fence_after();
        issue_S(0);
        if (n > 1 && (ok = mbar_wait(B(bars->rdy1[1 % NS1]), (1 / NS1) & 1, ctl, p.status))) {
          tc_fence_after();
          issue_S(1);
        }
        for (int i = 0; ok && i < n; ++i) {
          const int nx = i + 2;
          if (!(ok = mbar_wait(B(bars->p_full[i & 1]), (i >> 1) & 1, ctl, p.status))) break;
          if (!(ok = mbar_wait(B(bars->rdy2[i % NS2]), (i / NS2) & 1, ctl, p.status))) break;
          tc_fence_after();
          const uint32_t pb = tmem + C::TC_S + (uint32_t)(i & 1) * BN;
          mma_chain<1, BN, true, BN, C::TILE>(tmem + C::TC_DV, pb, 0,
                                              sdesc_mnmajor(slot2(i) + C::TILE, C::CH), idO,
                                              i > 0);
          umma_commit(B(bars->empty2[i % NS2]));
          if (nx < n) {
            if (!(ok = mbar_wait(B(bars->rdy1[nx % NS1]), (nx / NS1) & 1, ctl, p.status))) break;
            tc_fence_after();
            issue_S(nx);
          }
        }
        if (ok) umma_commit(B(bars->done));
      }
      umma_commit(B(bars->mma_final));
      mbar_drain(B(bars->mma_final), 0);
    }
    __syncwarp();
  } else if (warp == kFusedIssuer2) {
    // Step i (one dP buffer):  [dS_i ready, MN-major copies ready]  dK += dS_i^T Q_i
    //   -> empty2;  [tiles i+1 rounded]  dP^T_{i+1} -> dp_full, empty1
    //   (dP^T_{i+1} overwrites dS_i after dK_i in this thread's issue order)
    if (lane == 0) {
      auto issue_dP = [&](int i) {
        mma_chain<1, D, false, BN, C::TILE>(tmem + C::TC_DP, tmem + C::TC_V, 0,
                                            sdesc_kmajor(slot1(i) + C::TILE), idS, false);
        umma_commit(B(bars->dp_full));
        umma_commit(B(bars->empty1[i % NS1]));
      };
      bool ok = n > 0 && mbar_wait(B(bars->rows_ready), 0, ctl, p.status) &&
                mbar_wait(B(bars->rdy1[0]), 0, ctl, p.status);
      if (ok) {
        tc_fence_after();
        issue_dP(0);
        for (int i = 0; ok && i < n; ++i) {
          if (!(ok = mbar_wait(B(bars->ds_full), i & 1, ctl, p.status))) break;
          if (!(ok = mbar_wait(B(bars->rdy2[i % NS2]), (i / NS2) & 1, ctl, p.status))) break;
          tc_fence_after();
          mma_chain<1, BN, true, BN, C::TILE>(tmem + C::TC_DK, tmem + C::TC_DP, 0,
                                              sdesc_mnmajor(slot2(i), C::CH), idO, i > 0);
          umma_commit(B(bars->empty2[i % NS2]));
          if (i + 1 < n) {
            if (!(ok = mbar_wait(B(bars->rdy1[(i + 1) % NS1]), ((i + 1) / NS1) & 1, ctl,
                                 p.status)))
              break;
            tc_fence_after();
            issue_dP(i + 1);
          }
        }
        if (ok) umma_commit(B(bars->done));
      }
      umma_commit(B(bars->mma_final2));
      mbar_drain(B(bars->mma_final2), 0);
    }
    __syncwarp();
  } else if (warp == kFusedIssuer3) {
    // Step i, dQ buffer i % 2:  [dS_i in shared memory, buffer drained]
    //   dQ_i = dS_i K (M = 64, 16 MMAs over the 128 keys) -> dq_full; dqd: dS read
    if (lane == 0) {
      const uint64_t ad = sdesc_mnmajor(dsm, C::KCHUNK), bd = sdesc_mnmajor(kmn, C::KCHUNK);
      bool ok = n > 0 && mbar_wait(B(bars->kmn_ready), 0, ctl, p.status);
      for (int i = 0; ok && i < n; ++i) {
        const int bq = i & 1;
        if (!(ok = mbar_wait(B(bars->ds_full), i & 1, ctl, p.status))) break;
        if (i >= 2 && !(ok = mbar_wait(B(bars->dq_free[bq]), ((i >> 1) - 1) & 1, ctl, p.status)))
          break;
        tc_fence_after();
        const uint32_t d = tmem + C::TC_DQ + (bq ? kUpperLanes : 0u);
#pragma unroll
        for (int k = 0; k < kRows / 8; ++k)
          umma_tf32_ss(d, ad + (uint64_t)((k * 1024u) >> 4), bd + (uint64_t)((k * 1024u) >> 4),
                       idQ, k > 0 ? 1u : 0u);
        umma_commit(B(bars->dq_full[bq]));
        umma_commit(B(bars->dqd));
      }
      umma_commit(B(bars->mma_final3));
      mbar_drain(B(bars->mma_final3), 0);
    }
    __syncwarp();
  } else if (wg == kFusedPrepWarp0 / 4) {
    // Per step i: [tiles landed, ring-2 slot free]  round [Q_i | dO_i] in
    // place and write their MN-major copies into ring 2 (derive_tile_smem),
    // stage the step's LSE * -log2(e) and delta (one value per thread, loaded
    // a step ahead) -> rdy1, rdy2.
    const uint32_t tid = threadIdx.x - kFusedPrepWarp0 * 32;
    const int vsel = (int)(tid >> 6), vq = (int)(tid & 63u);  // 0: LSE, 1: delta; query
    const float* lse_bh = p.lse + b * p.l0 + h * p.l1;
    const float* del_bh = p.delta + (int64_t)bh * T;
    auto load_vec = [&](int i) -> float {
      const int q = (j0 + i) * BN + vq;
      if (i >= n || q >= T) return 0.0f;
      return vsel ? ldg_nc_early(del_bh + q) : ldg_nc_early(lse_bh + (int64_t)q * p.l2) * -kLog2e;
    };
    bool ok = n > 0;
    if (ok && (ok = warp_wait(B(bars->kmn_full), 0, ctl, p.status))) {
      round_tile_smem<C::KMN_BYTES, kSplitThreads>(kmn, tid);
      fence_proxy_async_smem();
      warp_arrive(B(bars->kmn_ready));
    }
    float vnext = ok ? load_vec(0) : 0.0f;
    for (int i = 0; ok && i < n; ++i) {
      const int s1 = i % NS1, s2 = i % NS2;
      if (!(ok = warp_wait(B(bars->full1[s1]), (i / NS1) & 1, ctl, p.status))) break;
      if (i >= NS2 && !(ok = warp_wait(B(bars->empty2[s2]), ((i / NS2) - 1) & 1, ctl, p.status)))
        break;
      const uint32_t k1 = slot1(i), m2 = slot2(i);
      derive_tile_smem<1, C::TILE, kSplitThreads, BN, C::CH, C::TILE, C::TILE>(k1, m2, tid);
      derive_tile_smem<1, C::TILE, kSplitThreads, BN, C::CH, C::TILE, C::TILE>(k1 + C::TILE,
                                                                             m2 + C::TILE, tid);
      vec[s2 * 2 * BN + vsel * BN + vq] = vnext;
      vnext = load_vec(i + 1);
      fence_proxy_async_smem();
      warp_arrive(B(bars->rdy1[s1]));
      warp_arrive(B(bars->rdy2[s2]));
    }
  } else if (wg == kFusedEpiWarp0 / 4) {
    // dQ epilogue.  Each step's accumulator is moved to registers (16 rows x
    // 64 columns per warp: threads 0-15 columns 0-31, 16-31 columns 32-63) as
    // soon as its MMAs complete, and its TMEM buffer released at once; up to
    // two steps wait there for their turn (the counter of their query tile
    // reaching this CTA's rank: the higher key tiles have added theirs), so
    // the ordering never holds up the MMAs.  Steps are written oldest first:
    // stored (rank 0) or added into dQ.  A written step is fenced and counted
    // on the next pass, when its additions have completed and the fence is
    // short.
    const int quad = warp & 3;
    float hva[32], hvb[32];
    int ea = -1, eb = -1, next = 0, unfenced = -1;
    auto cnt_of = [&](int e) {
      return fp.counters + ((size_t)bh * fp.n_qt + (j0 + e)) * 4u + quad;
    };
    auto rank_of = [&](int e) {
      const int last_q = min((j0 + e) * BN + BN - 1, T - 1);
      return (uint32_t)((p.causal ? last_q / kRows : p.n_tiles - 1) - kt);
    };
    auto release = [&]() {
      if (unfenced < 0) return;
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicAdd(cnt_of(unfenced), 1u);
      unfenced = -1;
    };
    auto turn = [&](int e) { return __all_sync(0xffffffffu, ld_acquire_u32(cnt_of(e)) >= rank_of(e)); };
    auto write = [&](const float (&hv)[32], int e) {
      release();
      const uint32_t rank = rank_of(e);
      const int q = (j0 + e) * BN + 16 * quad + (lane & 15);
      if (q < T) {
        float4* dst = reinterpret_cast<float4*>(fp.dq + ((int64_t)bh * T + q) * D + (lane >> 4) * 32);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 x = make_float4(hv[4 * u] * p.scale, hv[4 * u + 1] * p.scale,
                                       hv[4 * u + 2] * p.scale, hv[4 * u + 3] * p.scale);
          if (rank == 0) dst[u] = x;
          else atomicAdd(dst + u, x);
        }
      }
      unfenced = e;
    };
    auto load = [&](float (&hv)[32], int e) {
      const int bq = e & 1;
      tc_fence_after();
      tmem_ld_16x32bx2<32>(tmem_addr(tmem, 32u * quad + (bq ? 16u : 0u), C::TC_DQ), hv);
      tc_fence_before();
      warp_arrive(B(bars->dq_free[bq]));
    };
    auto full_done = [&](int e) {
      return __all_sync(0xffffffffu, mbar_test_wait(B(bars->dq_full[e & 1]), (e >> 1) & 1));
    };
    bool ok = n > 0;
    while (ok && (next < n || ea >= 0 || eb >= 0)) {
      // the oldest held step, written when its turn has come
      const bool a_old = ea >= 0 && (eb < 0 || ea < eb);
      const int eo = a_old ? ea : eb;
      if (eo >= 0 && turn(eo)) {
        if (a_old) {
          write(hva, ea);
          ea = -1;
        } else {
          write(hvb, eb);
          eb = -1;
        }
        continue;
      }
      // the next step's accumulator, into a free register slot
      if (next < n && (ea < 0 || eb < 0)) {
        if (eo < 0 || full_done(next)) {
          if (!(ok = warp_wait(B(bars->dq_full[next & 1]), (next >> 1) & 1, ctl, p.status))) break;
          if (ea < 0) {
            load(hva, next);
            ea = next++;
          } else {
            load(hvb, next);
            eb = next++;
          }
          continue;
        }
      }
      // nothing to do at once: wait for the oldest step's turn
      release();
      ok = flag_wait_geq(cnt_of(eo), rank_of(eo), ctl, p.status);
    }
    if (ok) release();
  } else if (wg == 1 || wg == 2) {
    // Row warps 4-7 (group 0) and 8-11 (group 1): thread (quad, lane) owns key
    // row quad*32 + lane; group g forms P^T and dS^T for the query columns
    // [32g, 32g + 32) of every step, loads K (g = 0) or V (g = 1) into TMEM, and
    // writes dK (g = 0) or dV (g = 1).  dS^T goes to TMEM (dK's A operand) and,
    // transposed by the layout, to shared memory as dQ's MN-major A operand:
    // key row r holds the group's 32 queries in chunk g.
    constexpr int HB = BN / 2;
    const int quad = warp & 3;
    const int grp = wg - 1;
    const int c0 = grp * HB;
    const int rl = quad * 32 + lane;  // key row within the tile
    const int row = k0 + rl;
    const bool valid = row < T;
    const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
    const uint32_t ds_row = dsm + (uint32_t)grp * C::KCHUNK + (uint32_t)rl * 128u;
    {
      const Ptr4& src = grp ? p.st1 : p.st0;
      const float* r = src.row(b, h, valid ? row : 0);
      const bool vr = src.s3 == 1 && ((reinterpret_cast<uintptr_t>(r) & 15u) == 0);
      row_to_tmem<D, 1>(src, r, valid, vr, lb, grp ? C::TC_V : C::TC_K);
      tmem_wait_st();
    }
    tc_fence_before();
    warp_arrive(B(bars->rows_ready));
    bool ok = n > 0;
    for (int i = 0; ok && i < n; ++i) {
      const int qs = (j0 + i) * BN + c0;
      const int bi = i & 1;
      const uint32_t sc = lb + C::TC_S + (uint32_t)bi * BN + c0;
      const uint32_t dc = lb + C::TC_DP + c0;
      // the step's LSE and delta (staged with the MN-major copies)
      if (!(ok = warp_wait(B(bars->rdy2[i % NS2]), (i / NS2) & 1, ctl, p.status))) break;
      const float* vl = vec + (i % NS2) * 2 * BN + c0;
      if (!(ok = warp_wait(B(bars->s_full[bi]), (i >> 1) & 1, ctl, p.status))) break;
      tc_fence_after();
      const bool need_mask = !valid || (qs + HB > T) || (p.causal && qs < k0 + kRows - 1);
      float pv[HB];
      {
        float t[HB], lv[HB];
        tmem_ldn<HB>(sc, t);
        load_vecn<HB>(vl, lv);  // -LSE * log2(e)
#pragma unroll
        for (int x = 0; x < HB; x += 2) {
          float a0, a1;
          ffma2(a0, a1, t[x], t[x + 1], p.scale_log2, p.scale_log2, lv[x], lv[x + 1]);
          t[x] = ex2_approx(a0);
          t[x + 1] = ex2_approx(a1);
        }
        if (need_mask) {
#pragma unroll
          for (int x = 0; x < HB; ++x) {
            const int q = qs + x;
            t[x] = (valid && q < T && (!p.causal || q >= row)) ? t[x] : 0.0f;
          }
        }
#pragma unroll
        for (int x = 0; x < HB; ++x) {
          pv[x] = t[x];
          t[x] = tf32_round_finite(t[x]);
        }
        tmem_stn<HB>(sc, t);
      }
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->p_full[bi]));  // S^T_i read, P^T_i in its place
      if (!(ok = warp_wait(B(bars->dp_full), i & 1, ctl, p.status))) break;
      tc_fence_after();
      float t[HB];
      {
        float dv[HB];
        tmem_ldn<HB>(dc, t);
        load_vecn<HB>(vl + BN, dv);
#pragma unroll
        for (int x = 0; x < HB; x += 2) {
          float u0, u1, d0, d1;
          fsub2(u0, u1, t[x], t[x + 1], dv[x], dv[x + 1]);
          fmul2(d0, d1, pv[x], pv[x + 1], u0, u1);  // dS^T = P^T (dP^T - delta)
          t[x] = tf32_round_finite(d0);
          t[x + 1] = tf32_round_finite(d1);
        }
      }
      tmem_stn<HB>(dc, t);
      // dQ_{i-1} has read the previous dS from shared memory
      if (i > 0 && !(ok = warp_wait(B(bars->dqd), (i - 1) & 1, ctl, p.status))) break;
      // 16-byte unit lu holds queries 4 lu .. 4 lu + 3, at 32-byte unit
      // (lu / 2) ^ (row % 4).  Rows r and r + 4 of a store phase (8 threads)
      // would hit the same banks: the second of them writes the two halves
      // of each 32-byte unit in the other order.
      const uint32_t flip = ((uint32_t)rl >> 2) & 1u;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int w = u ^ 1;
        const float4 x = flip ? make_float4(t[4 * w], t[4 * w + 1], t[4 * w + 2], t[4 * w + 3])
                              : make_float4(t[4 * u], t[4 * u + 1], t[4 * u + 2], t[4 * u + 3]);
        const uint32_t mu = ((((uint32_t)u >> 1) ^ ((uint32_t)rl & 3u)) << 1) | (((uint32_t)u & 1u) ^ flip);
        sts128(ds_row + (mu << 4), x);
      }
      fence_proxy_async_smem();
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->ds_full));
    }
    const int64_t orow = ((int64_t)bh * T + (valid ? row : 0)) * D;
    float* out = grp ? p.out1 : p.out0;
    if (n == 0) {  // no query of the first segment reaches these keys
      if (valid) {
        for (int d = 0; d < D; ++d) out[orow + d] = 0.0f;
      }
    } else if (ok && warp_wait(B(bars->done), 0, ctl, p.status)) {
      tc_fence_after();
      tmem_row_to_global<D>(lb, grp ? C::TC_DV : C::TC_DK, grp ? 1.0f : p.scale, out + orow, valid,
                            p.accumulate_out != 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <class C>
int run_fused(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
              const float* lse, const int64_t ls[3], const float* delta, float* dq, float* dk,
              float* dv, uint32_t* sync_words, const DeviceInfo& dev, cudaStream_t st) {
  static unsigned long long attr_done = 0;
  CUtensorMap tq, tg, tk;
  int rc = make_tmap_bhtd_whole(&tq, q, pr, C::BN);
  if (rc == CT_OK) rc = make_tmap_bhtd_whole(&tg, g, pr, C::BN);
  if (rc == CT_OK) rc = make_tmap_bhtd_whole(&tk, k, pr, kRows, true);
  if (rc != CT_OK) return rc;
  const size_t smem = fused_smem_bytes<C>();
  rc = ensure_smem_attr(fa2_bwd_fused_tc_kernel<C>, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  FusedParams fp;
  fp.b = make_params(pr, k, v, lse, ls, delta, dk, dv, dev);
  fp.dq = dq;
  fp.n_qt = (int)((pr.T + C::BN - 1) / C::BN);
  const size_t n_counters = (size_t)fp.b.bh_total * fp.n_qt * 4u;
  const int64_t n_seg = (pr.T + kSegLen - 1) / kSegLen;
  fp.counters = sync_words;
  if (cudaMemsetAsync(sync_words, 0, (n_counters + (size_t)n_seg) * sizeof(uint32_t), st) !=
      cudaSuccess)
    return CT_ERR_CUDA;
  const int64_t grid = (int64_t)fp.b.n_tiles * fp.b.bh_total;
  for (int64_t s0 = 0, si = 0; s0 < pr.T; s0 += kSegLen, ++si) {  // one launch per query segment
    fp.b.seg_lo = (int)s0;
    fp.b.seg_hi = (int)std::min<int64_t>(s0 + kSegLen, pr.T);
    fp.b.accumulate_out = s0 > 0;
    fp.ticket = sync_words + n_counters + si;
    fa2_bwd_fused_tc_kernel<C><<<(unsigned)grid, kFusedThreads, smem, st>>>(tq, tg, tk, fp);
    rc = check_launch();
    if (rc != CT_OK) return rc;
  }
  return CT_OK;
}

using FusedD64 = FusedCfg<64, 2, 3>;

// The register split (setmaxnreg) assumes the kernel launches with exactly
// kFusedLaunchRegs registers per thread; a build that compiled to another count
// never launches it (the two-kernel path runs instead).
bool fused_kernel_usable() {
  static const bool ok = [] {
    cudaFuncAttributes a;
    return cudaFuncGetAttributes(&a, fa2_bwd_fused_tc_kernel<FusedD64>) == cudaSuccess &&
           a.numRegs == kFusedLaunchRegs;
  }();
  return ok;
}

}  // namespace

size_t fa2_bwd_fused_sync_words(int64_t B, int64_t H, int64_t T) {
  const int64_t n_qt = (T + kFusedBN - 1) / kFusedBN, n_seg = (T + kSegLen - 1) / kSegLen;
  return (size_t)(B * H * n_qt * 4 + n_seg);
}

bool fa2_bwd_fused_supported(const Fa2Problem& p) {
  return p.precision == CT_PRECISION_TF32 && p.D == 64 && fa2_bwd_tc_supported(p) &&
         fused_kernel_usable();
}

int launch_fa2_bwd_fused_tc(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
                            const float* lse, const int64_t ls[3], const float* delta, float* dq,
                            float* dk, float* dv, uint32_t* sync_words, const DeviceInfo& dev,
                            cudaStream_t st) {
  if (!fa2_tma_ok(q) || !fa2_tma_ok(g) || !fa2_tma_ok(k)) return CT_ERR_UNSUPPORTED_LAYOUT;
  if (pr.D != 64 || pr.precision != CT_PRECISION_TF32) return CT_ERR_INVALID_ARGUMENT;
  if (!fused_kernel_usable()) return CT_ERR_INVALID_ARGUMENT;
  return run_fused<FusedD64>(pr, q, k, v, g, lse, ls, delta, dq, dk, dv, sync_words, dev, st);
}

}  // namespace ct
