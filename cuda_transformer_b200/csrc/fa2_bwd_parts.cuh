// fa2_bwd_parts.cuh -- pieces shared by the tensor-core backward kernels
// (fa2_bwd_tc.cu: the dQ and dK/dV kernels and the 64-row pass;
// fa2_bwd_fused.cu: the one-kernel TF32 backward): stage-tile layout, the
// barrier block, kernel parameters, the TMA producer warp and the tile
// preparation warps.
#pragma once

#include "fa2_common.cuh"

namespace ct {
namespace fa2 {

// ------------------------------------------------------------ configuration
// A stage holds the two streamed tiles of one step (dQ pass: K_j and V_j;
// dK/dV pass: Q_j and dO_j).  A tile the tensor core reads both K-major and
// MN-major is held in both shared-memory layouts (the TF32 MN-major operand
// layout differs from the K-major one): TMA lands the K-major copy and the
// preparation warps write the MN-major one from it.  Per stage, in order:
//   A K-major [raw, lo] | A MN-major [raw, lo] (LA == 2) | B K-major [raw, lo] |
//   B MN-major [raw, lo] (LB == 2), the lo copies present when SPLIT == 3.
// With KILA / KILB (3xTF32 only) the K-major copy of A / B interleaves instead:
// each 32-column chunk of BN raw rows is followed by its BN low-part rows (see
// mma_chain_kil).  With BMN, B is read only MN-major: TMA lands it in that
// layout and the preparation splits (or rounds) it in place -- no K-major copy.
template <int D_, int BN_, int SPLIT_, int NS_, int LA_, int LB_, bool KILA_ = false,
          bool KILB_ = false, bool BMN_ = false>
struct BwdTiles {
  static constexpr int D = D_, BN = BN_, SPLIT = SPLIT_, NS = NS_, LA = LA_, LB = LB_;
  static constexpr int NCOPY = SPLIT == 3 ? 2 : 1;
  static constexpr bool BMN = BMN_;
  static constexpr bool KILA = KILA_ && SPLIT == 3, KILB = KILB_ && SPLIT == 3 && !BMN_;
  static_assert(!BMN_ || LB_ == 1, "an MN-only B tile has one layout");
  static constexpr uint32_t TILE = (uint32_t)BN * D * 4u;
  // K-major chunk strides of A and B
  static constexpr uint32_t KCHA = (KILA ? 2u : 1u) * BN * 128u, KCHB = (KILB ? 2u : 1u) * BN * 128u;
  static constexpr uint32_t OFF_A0 = 0, OFF_A1 = NCOPY * TILE;
  static constexpr uint32_t OFF_B0 = LA * NCOPY * TILE,
                            OFF_B1 = BMN_ ? OFF_B0 : OFF_B0 + NCOPY * TILE;
  static constexpr uint32_t STAGE = (LA + LB) * NCOPY * TILE;
  static constexpr uint32_t TMEM_COLS = 512;
};

template <int NS>
struct BwdBars {
  // full_*: TMA landed (A / B tiles); ready_*: split or rounded; empty_*: no
  // longer read by the tensor core.  With MERGED stages (dK/dV pass) only the
  // _a barriers are used and cover both tiles.
  uint64_t full_a[NS], full_b[NS], ready_a[NS], ready_b[NS], empty_a[NS], empty_b[NS];
  uint64_t vec_full[NS];  // dK/dV pass: the step's LSE and delta are in shared memory
  // Indexed by S / dP TMEM buffer (the dQ pass and single-buffered dK/dV use [0]).
  uint64_t s_full[2], dp_full[2], p_full[2], ds_full[2], s_free[2];
  uint64_t dqd[2];  // dQ pass, two buffers: dQ_j has read dS_j from buffer j % 2
  uint64_t rows_ready, done, mma_final, mma_final2, mma_final3;
  CtaCtl ctl;
};

struct BwdParams {
  Ptr4 st0, st1;       // stationary operands (dQ: Q, dO; dK/dV: K, V)
  const float* lse;
  int64_t l0, l1, l2;
  const float* delta;  // contiguous [B,H,T]
  float* out0;         // dQ | dK
  float* out1;         // -  | dV
  int H, T, n_tiles, bh_total, head_group, causal;
  // This launch reduces over streamed rows [seg_lo, seg_hi) (keys in the dQ
  // pass, queries in the dK/dV pass; kSegLen long); accumulate_out: add into
  // the output written by the previous segment's launch instead of storing.
  int seg_lo, seg_hi, accumulate_out;
  float scale_log2, scale;
  uint32_t* status;
};

// Bytes of the per-stage vector slots (log-sum-exp and delta of BN queries).
template <class C>
constexpr size_t bwd_vec_bytes() {
  return (size_t)C::NS * 2 * C::BN * sizeof(float);
}
// Whether the row warps' write-out buffer fits beside the stage ring.
template <class C>
__host__ __device__ constexpr bool bwd_wbuf_fits() {
  return 1024 + 1024 + (size_t)C::NS * C::STAGE + (size_t)C::NS * 2 * C::BN * sizeof(float) +
             kRowWbufBytes <=
         227 * 1024;
}
template <class C>
constexpr size_t bwd_smem_bytes_wbuf() {  // with the row warps' write-out buffer
  static_assert(1024 + 1024 + (size_t)C::NS * C::STAGE + bwd_vec_bytes<C>() + kRowWbufBytes <=
                    227 * 1024,
                "shared memory budget");
  return 1024 + 1024 + (size_t)C::NS * C::STAGE + bwd_vec_bytes<C>() + kRowWbufBytes;
}
template <class C>
constexpr size_t bwd_smem_bytes() {
  static_assert(1024 + 1024 + (size_t)C::NS * C::STAGE + bwd_vec_bytes<C>() <= 227 * 1024,
                "shared memory budget");
  return 1024 + 1024 + (size_t)C::NS * C::STAGE + bwd_vec_bytes<C>();
}

// empty_count: MMA issuers that read a stage; done_count: issuers whose
// accumulators the epilogue reads; rows: the row warps (one arrival each).
template <class C>
__device__ __forceinline__ void init_bwd_bars(BwdBars<C::NS>* bars, int empty_count,
                                              int done_count, int rows) {
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  for (int s = 0; s < C::NS; ++s) {
    mbar_init(B(bars->full_a[s]), 1);
    mbar_init(B(bars->full_b[s]), 1);
    mbar_init(B(bars->ready_a[s]), kPrepWarps);
    mbar_init(B(bars->ready_b[s]), kPrepWarps);
    mbar_init(B(bars->empty_a[s]), empty_count);
    mbar_init(B(bars->empty_b[s]), 1);
    mbar_init(B(bars->vec_full[s]), 1);
  }
  for (int i = 0; i < 2; ++i) {
    mbar_init(B(bars->s_full[i]), 1);
    mbar_init(B(bars->dp_full[i]), 1);
    mbar_init(B(bars->p_full[i]), rows);
    mbar_init(B(bars->ds_full[i]), rows);
    mbar_init(B(bars->s_free[i]), rows);
  }
  mbar_init(B(bars->rows_ready), rows);
  mbar_init(B(bars->done), done_count);
  mbar_init(B(bars->mma_final), 1);
  mbar_init(B(bars->mma_final2), 1);
  mbar_init(B(bars->mma_final3), 1);
  mbar_init(B(bars->dqd[0]), 1);
  mbar_init(B(bars->dqd[1]), 1);
  bars->ctl.abort = 0;
  fence_barrier_init();
}

// Producer warp (all 32 lanes): lane 0 issues the TMA loads of tiles j0..j1-1
// of two [B,H,T,D] tensors into the stage ring (maps[0] = A, maps[1] = B, both
// as K-major tiles; the preparation warps derive the MN-major copies).  With
// VEC, all lanes then stage the step's per-query log-sum-exp (times log2 e) and
// delta into the stage's vector slot, so the row warps read them from shared
// memory.
template <class C, bool VEC, bool MERGED, bool B_FIRST = false>
__device__ __forceinline__ void bwd_producer(BwdBars<C::NS>* bars, uint32_t tiles, float* vec,
                                             const CUtensorMap* const* maps, int j0, int j1,
                                             int h, int b, const float* lse_bh, int64_t lse_t,
                                             const float* del_bh, int T, uint32_t* status) {
  constexpr int NS = C::NS, BN = C::BN, D = C::D;
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  CtaCtl* ctl = &bars->ctl;
  const int lane = threadIdx.x & 31;
  if (lane == 0)
    for (int m = 0; m < 2; ++m)
      tma_prefetch_desc(maps[m]);
  int last_a[NS], last_b[NS];
  for (int s = 0; s < NS; ++s) last_a[s] = last_b[s] = -1;
  // The vector values of step j + 1 are loaded into registers while step j is
  // staged, so the global-load latency stays off the stage turnaround.
  constexpr int NV = VEC ? BN / 32 : 1;
  float vl[NV], vd[NV];
  auto load_vec = [&](int j) {
#pragma unroll
    for (int u = 0; u < NV; ++u) {
      const int q = j * BN + 32 * u + lane;
      const bool in = VEC && j < j1 && q < T;
      vl[u] = in ? ldg_nc_early(lse_bh + (int64_t)q * lse_t) : 0.0f;
      vd[u] = in ? ldg_nc_early(del_bh + q) : 0.0f;
    }
  };
  if constexpr (VEC) load_vec(j0);
  for (int j = j0; j < j1; ++j) {
    const int i = j - j0, s = i % NS, r = i / NS;
    const uint32_t st = tiles + s * C::STAGE;
    // The tile copies go first: the vector values are needed only by the row
    // warps, much later, and signal their own barrier.  B_FIRST (separate
    // stage releases): B's copy, freed earlier by its single reader, first.
    auto load_a = [&]() -> bool {
      if (r > 0 && !warp_wait(B(bars->empty_a[s]), (r - 1) & 1, ctl, status)) return false;
      if (lane == 0) {
        const uint32_t fa = B(bars->full_a[s]);
        // only the K-major copy: the preparation warps write the MN-major one
        mbar_arrive_expect_tx(fa, C::TILE);
        tma_load_tile<!C::KILA, D>(st + C::OFF_A0, maps[0], fa, j * BN, h, b, C::KCHA);
      }
      last_a[s] = r;
      return true;
    };
    auto load_b = [&]() -> bool {
      if (!MERGED && r > 0 && !warp_wait(B(bars->empty_b[s]), (r - 1) & 1, ctl, status))
        return false;
      if (lane == 0) {
        const uint32_t fb = B(bars->full_b[s]);
        mbar_arrive_expect_tx(fb, C::TILE);
        tma_load_tile<!C::KILB, D>(st + C::OFF_B0, maps[1], fb, j * BN, h, b, C::KCHB);
      }
      last_b[s] = r;
      return true;
    };
    if (B_FIRST) {
      if (!load_b() || !load_a()) break;
    } else {
      if (!load_a() || !load_b()) break;
    }
    if constexpr (VEC) {
      float* vs = vec + s * 2 * BN;
#pragma unroll
      for (int u = 0; u < NV; ++u) {
        vs[32 * u + lane] = vl[u] * -kLog2e;  // rows add it in one FMA
        vs[BN + 32 * u + lane] = vd[u];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(B(bars->vec_full[s]));
      load_vec(j + 1);
    }
  }
  __syncwarp();
  if (ctl->abort && lane == 0) {
    for (int s = 0; s < NS; ++s) {
      if (last_a[s] >= 0) mbar_drain(B(bars->full_a[s]), last_a[s] & 1);
      if (last_b[s] >= 0) mbar_drain(B(bars->full_b[s]), last_b[s] & 1);
    }
  }
}

// Prepares tile A (is_b false) or B of a stage: its K-major copy in place and,
// for a tile the tensor core also reads MN-major (LA / LB == 2), the MN-major
// copy derived from it (derive_tile_smem), so TMA loads each tile once.
template <class C>
__device__ __forceinline__ void prep_tile(uint32_t st, bool is_b, uint32_t tid) {
  const uint32_t k = st + (is_b ? C::OFF_B0 : C::OFF_A0);
  const uint32_t mn = st + (is_b ? C::OFF_B1 : C::OFF_A1);
  const bool il = is_b ? C::KILB : C::KILA;
  const bool two = (is_b ? C::LB : C::LA) > 1;
  constexpr uint32_t CH = (uint32_t)C::BN * 128u;
  if (two) {
    if (il)
      derive_tile_smem<C::SPLIT, C::TILE, kSplitThreads, C::BN, 2u * CH, CH, C::TILE>(k, mn, tid);
    else
      derive_tile_smem<C::SPLIT, C::TILE, kSplitThreads, C::BN, CH, C::TILE, C::TILE>(k, mn, tid);
  } else if constexpr (C::SPLIT == 3) {
    if (il) split_tile_smem_il<C::TILE, kSplitThreads, CH>(k, tid);
    else split_tile_smem<C::TILE, kSplitThreads>(k, k + C::TILE, tid);
  } else {
    round_tile_smem<C::TILE, kSplitThreads>(k, tid);
  }
}

// Per stage: tile A prepared -> ready_a, tile B prepared -> ready_b.  In the
// dK/dV pass (MERGED) the issuers wait on ready_a for the K-major copies of
// both tiles (S^T, dP^T) and on ready_b for the MN-major ones (dV, dK); both
// complete once the two tiles are prepared.
template <class C, bool MERGED, bool B_FIRST = false>
__device__ __forceinline__ void bwd_splitter(BwdBars<C::NS>* bars, uint32_t tiles, int n,
                                             uint32_t* status) {
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  const uint32_t tid = prep_tid();
  for (int i = 0; i < n; ++i) {
    const int s = i % C::NS, r = i / C::NS;
    const uint32_t st = tiles + s * C::STAGE;
    if constexpr (B_FIRST) {  // separate stages: B, then A, each released as prepared
      if (!warp_wait(B(bars->full_b[s]), r & 1, &bars->ctl, status)) break;
      prep_tile<C>(st, true, tid);
      fence_proxy_async_smem();
      warp_arrive(B(bars->ready_b[s]));
      if (!warp_wait(B(bars->full_a[s]), r & 1, &bars->ctl, status)) break;
      prep_tile<C>(st, false, tid);
      fence_proxy_async_smem();
      warp_arrive(B(bars->ready_a[s]));
      continue;
    }
    if (!warp_wait(B(bars->full_a[s]), r & 1, &bars->ctl, status)) break;
    prep_tile<C>(st, false, tid);
    if (!MERGED) {
      fence_proxy_async_smem();
      warp_arrive(B(bars->ready_a[s]));
    }
    if (!warp_wait(B(bars->full_b[s]), r & 1, &bars->ctl, status)) break;
    prep_tile<C>(st, true, tid);
    fence_proxy_async_smem();
    if (MERGED) warp_arrive(B(bars->ready_a[s]));
    warp_arrive(B(bars->ready_b[s]));
  }
}

// Both backward kernels run two row warpgroups, warps 4-7 and 11-14, and a
// third MMA issuer, warp 15 (dQ pass with two dP buffers; idle otherwise):
// 16 warps, warps 0-3 and 8-10 keep the forward's roles.
constexpr int kBwdThreads = 512;
constexpr int kBwdRowWarp1 = 11;
constexpr int kIssuer3Warp = 15;

inline BwdParams make_params(const Fa2Problem& pr, Strided4 a, Strided4 b, const float* lse,
                      const int64_t ls[3], const float* delta, float* out0, float* out1,
                      const DeviceInfo& dev) {
  BwdParams p;
  p.st0 = Ptr4{a.ptr, a.s[0], a.s[1], a.s[2], a.s[3]};
  p.st1 = Ptr4{b.ptr, b.s[0], b.s[1], b.s[2], b.s[3]};
  p.lse = lse;
  p.l0 = ls[0];
  p.l1 = ls[1];
  p.l2 = ls[2];
  p.delta = delta;
  p.out0 = out0;
  p.out1 = out1;
  p.H = (int)pr.H;
  p.T = (int)pr.T;
  p.n_tiles = (int)((pr.T + kRows - 1) / kRows);
  p.bh_total = (int)(pr.B * pr.H);
  p.head_group = fa2_head_group(p.bh_total);
  p.causal = pr.causal ? 1 : 0;
  p.seg_lo = 0;
  p.seg_hi = (int)pr.T;
  p.accumulate_out = 0;
  p.scale = (float)(1.0 / std::sqrt((double)pr.D));
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)pr.D));
  p.status = dev.status;
  return p;
}

}  // namespace fa2
}  // namespace ct
