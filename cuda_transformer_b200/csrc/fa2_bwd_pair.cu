// fa2_bwd_pair.cu -- the TF32 dK/dV kernel at head dim 64 on CTA pairs
// (cta_group::2): the key/value-stationary pass of the FlashAttention-2
// backward (reference: Transformer_kernels/flash_attention.cuh:357-504,
// flash_attention_bwd_dk_dv), with each tensor-core product spanning 256 key
// rows over two SMs.
//
// A cluster of two CTAs owns keys [k0, k0 + 256): the even CTA keys k0..k0+127,
// the odd one k0+128..k0+255, each in its own Tensor Memory (K, V, dK, dV and
// two S^T / dP^T buffers, 512 columns, as in the one-CTA dK/dV kernel).  Per
// query tile j (64 queries) the even CTA's two issuing threads run
//   S^T  = K Q_j^T,  dP^T = V dO_j^T          (M = 256, N = 64, B K-major)
//   dV  += P^T dO_j, dK  += dS^T Q_j           (M = 256, N = 64, B MN-major)
// with B split along N: for S^T / dP^T each CTA holds 32 of the tile's 64
// query rows, for dV / dK each holds 32 of the 64 head-dim columns.  So each
// CTA lands, rounds and re-lays out half of every streamed tile, and one MMA
// instruction does the work two did: per 256 keys the issuers issue the
// instructions the one-CTA kernel issues per 128, and the rounding warps move
// half the shared-memory bytes per FLOP.
//
// Shared memory per stage and CTA (48 KB), for Q_j and dO_j each:
//   half 0 (8 KB): the CTA's own 32 query rows, both 32-column chunks
//                  ([chunk][32 rows][128 B], 128-byte swizzle, K-major);
//   half 1 (8 KB): the other 32 query rows, same layout;
//   MN (8 KB):     the CTA's 32-column chunk of all 64 rows, MN-major.
// Both CTAs keep their own rows at half 0, so one descriptor address serves
// the pair.  TMA lands both halves (two 8 KB copies of 32 rows); the
// preparation warps round half 0 to TF32 in place (the S^T / dP^T operand)
// and write the MN-major chunk from both halves (the dV / dK operand).
//
// Synchronisation across the pair: the preparation and row warps of both CTAs
// arrive on the even CTA's barriers (the odd CTA's by remote arrivals; what
// they publish lives in their own CTA's shared memory or TMEM, see
// mbar_arrive_remote), and every commit of the issuing threads arrives on the
// barrier at the same address in both CTAs.
// Every wait is bounded.  The two CTAs meet at a cluster barrier after the
// barrier set-up and TMEM allocation and again before the TMEM is released.
//
// Warp roles (16 warps, both CTAs): warp 0 TMA producer; warp 1 TMEM allocation
// and (even CTA) the S^T / dV issuer; warp 10 (even CTA) the dP^T / dK issuer;
// warps 2, 3, 8, 9 tile preparation; warps 4-7 and 11-14 the two row
// warpgroups (one key row per thread, each group half of a step's 64 query
// columns); warp 15 idle.
#include <algorithm>
#include <cstdlib>

#include "fa2_bwd_parts.cuh"

namespace ct {
namespace {

using namespace fa2;

template <int NS_>
struct PairCfg {
  static constexpr int D = 64, BN = 64, NS = NS_;
  static constexpr uint32_t CHUNK = 32u * 128u;      // 32 rows of 128 bytes
  static constexpr uint32_t HALF = 2u * CHUNK;       // 32 rows x 64 columns
  static constexpr uint32_t OFF_Q = 0, OFF_QM = 2u * HALF, OFF_G = 3u * HALF, OFF_GM = 5u * HALF;
  static constexpr uint32_t STAGE = 6u * HALF;       // 48 KB
  static constexpr uint32_t TX = 4u * HALF;          // bytes TMA lands per stage
  // TMEM columns (per CTA): K | V | dK | dV | S^T / P^T x2 | dP^T / dS^T x2
  static constexpr uint32_t TC_K = 0, TC_V = 64, TC_DK = 128, TC_DV = 192, TC_S = 256,
                            TC_DP = 384, SB = 64;
  static constexpr uint32_t TMEM_COLS = 512;
};

template <class C>
constexpr size_t pair_smem_bytes() {
  constexpr size_t bytes = 1024 + 1024 + (size_t)C::NS * C::STAGE + (size_t)C::NS * 2 * C::BN * 4 +
                           kRowWbufBytes;
  static_assert(bytes <= 227 * 1024, "shared memory budget");
  return bytes;
}

constexpr int kPairRowWarps = 16;  // both CTAs' row warps arrive on the even CTA's barriers

// full_a: TMA landed (local); ready_a: K-major halves rounded and MN-major
// chunks written (both CTAs' preparation warps, on the even CTA);
// empty_a: the stage's MMAs finished (both issuers' commits, in both CTAs).
template <class C>
__device__ __forceinline__ void init_pair_bars(BwdBars<C::NS>* bars) {
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  for (int s = 0; s < C::NS; ++s) {
    mbar_init(B(bars->full_a[s]), 1);
    mbar_init(B(bars->ready_a[s]), 2 * kPrepWarps);
    mbar_init(B(bars->empty_a[s]), 2);
    mbar_init(B(bars->vec_full[s]), 1);
  }
  for (int i = 0; i < 2; ++i) {
    mbar_init(B(bars->s_full[i]), 1);
    mbar_init(B(bars->dp_full[i]), 1);
    mbar_init(B(bars->p_full[i]), kPairRowWarps);
    mbar_init(B(bars->ds_full[i]), kPairRowWarps);
  }
  mbar_init(B(bars->rows_ready), kPairRowWarps);
  mbar_init(B(bars->done), 2);
  mbar_init(B(bars->mma_final), 1);
  mbar_init(B(bars->mma_final2), 1);
  bars->ctl.abort = 0;
  fence_barrier_init();
}

// Warp-uniform arrival on a barrier of the even CTA (cluster address).
__device__ __forceinline__ void warp_arrive_remote(uint32_t leader_bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_remote(leader_bar);
}

// S^T or dP^T: D[256 x 64] = X (TMEM, 64 head-dim columns) T^T, B = the own
// K-major half of tile T (32 query rows per CTA; chunk stride CHUNK).
template <class C>
__device__ __forceinline__ void pair_chain_k(uint32_t d, uint32_t a, uint64_t bd) {
  constexpr uint32_t id = idesc_tf32(256, 64, false, false);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t off = (uint32_t)(k / 4) * C::CHUNK + (uint32_t)(k % 4) * 32u;
    umma_tf32_ts_pair(d, a + 8u * k, bd + (off >> 4), id, k > 0 ? 1u : 0u);
  }
}
// dV or dK: D[256 x 64] += P^T or dS^T (TMEM, 64 query columns) times the
// MN-major chunk (32 head-dim columns per CTA, 64 query rows).
__device__ __forceinline__ void pair_chain_mn(uint32_t d, uint32_t a, uint64_t bd,
                                              bool accumulate) {
  constexpr uint32_t id = idesc_tf32(256, 64, false, true);
#pragma unroll
  for (int k = 0; k < 8; ++k)
    umma_tf32_ts_pair(d, a + 8u * k, bd + (((uint32_t)k * 1024u) >> 4), id,
                      (accumulate || k > 0) ? 1u : 0u);
}

// Writes the MN-major chunk `rank` of a landed tile at t (half 0: own rows,
// half 1: the other rows) to mn, rounded to TF32.  Source row s (half s / 32)
// holds query (s + 32 rank) % 64 of the tile, the MN-major row it lands in;
// each 16-byte word moves within its 128-byte row (K-major unit u of row r
// at u ^ (r % 8); MN-major 32-byte unit a of row r at a ^ (r % 4)).  Rows are
// moved by multiples of 32, so r % 8 is the same in source and destination.
__device__ __forceinline__ void pair_derive_mn(uint32_t t, uint32_t mn, uint32_t rank,
                                               uint32_t tid) {
  constexpr uint32_t PER = 4;  // 64 rows x 8 words / 128 threads
  float4 x[PER];
  uint32_t dst[PER];
#pragma unroll
  for (uint32_t u = 0; u < PER; ++u) {
    const uint32_t w = tid + u * kSplitThreads;
    const uint32_t s = w >> 3, pu = w & 7u;
    const uint32_t src = t + (s >> 5) * (2u * 32u * 128u) + rank * (32u * 128u) +
                         (s & 31u) * 128u + pu * 16u;
    const uint32_t lu = pu ^ (s & 7u);
    const uint32_t m = (s + 32u * rank) & 63u;
    const uint32_t mu = (((lu >> 1) ^ (m & 3u)) << 1) | (lu & 1u);
    dst[u] = mn + m * 128u + mu * 16u;
    x[u] = lds128(src);
  }
#pragma unroll
  for (uint32_t u = 0; u < PER; ++u) {
    const float4 y = make_float4(tf32_round_finite(x[u].x), tf32_round_finite(x[u].y),
                                 tf32_round_finite(x[u].z), tf32_round_finite(x[u].w));
    sts128(dst[u], y);
  }
}

// One 256-key tile of a persistent cluster: (head, keys [k0, k0 + 256)) and
// its query tiles [j0, j1) in this launch's segment.
struct PairTile {
  int b, h, bh, k0, kb, j0, j1, n;
  bool exists;
};
// The clusters' static schedule.  A unit is the tile pair (kp, NT-1-kp) of one
// head (NT tiles per head): under the causal mask their step counts add up to
// the same total for every kp, so units have equal work, and cluster c takes
// units c, c + G, c + 2G, ... (units in the head-grouped order of cta_tile_at,
// so the heads in flight share L2).  Tile m of cluster c is half m % 2 of its
// unit m / 2.  Returns false past the cluster's last unit; t.exists is false
// for the missing second half of the middle unit when NT is odd.
__device__ __forceinline__ bool pair_tile_at(const BwdParams& p, int c, int G, int m,
                                             uint32_t rank, PairTile& t) {
  constexpr int BN = 64;
  const int U = (p.n_tiles + 1) / 2;
  const int u = c + (m >> 1) * G;
  if (u >= U * p.bh_total) return false;
  int k;
  cta_tile_at((unsigned)u, U, p.bh_total, p.head_group, false, k, t.bh);
  const int kp = (m & 1) ? p.n_tiles - 1 - k : k;
  t.exists = !((m & 1) && kp == k);
  t.b = t.bh / p.H;
  t.h = t.bh % p.H;
  t.k0 = kp * 2 * kRows;
  t.kb = t.k0 + (int)rank * kRows;
  t.j0 = max(p.causal ? t.k0 / BN : 0, p.seg_lo / BN);
  t.j1 = min((p.T + BN - 1) / BN, (p.seg_hi + BN - 1) / BN);
  t.n = t.exists ? max(0, t.j1 - t.j0) : 0;
  return true;
}

// Persistent: each cluster loops over tiles.  The producer, preparation warps
// and issuers run on across tile boundaries (one step counter g for the stage
// ring and the S^T / dP^T buffers), so the next tile's tiles are landed and
// prepared while the current one finishes; per tile only the rows' dK / dV
// write-out and the load of the next K / V rows into TMEM sit between the
// last MMA of one tile and the first of the next.
template <class C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kBwdThreads, 1)
    fa2_bwd_dkdv_pair_kernel(const __grid_constant__ CUtensorMap tmQ,
                             const __grid_constant__ CUtensorMap tmG, const BwdParams p) {
  constexpr int D = C::D, BN = C::BN, NS = C::NS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  auto* bars = reinterpret_cast<BwdBars<NS>*>(smem_raw);
  const uint32_t tiles = (smem_u32(smem_raw) + (uint32_t)sizeof(BwdBars<NS>) + 1023u) & ~1023u;
  float* vec = reinterpret_cast<float*>(smem_raw + (tiles - smem_u32(smem_raw)) + NS * C::STAGE);
  CtaCtl* ctl = &bars->ctl;
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  auto L = [&](const uint64_t& x) { return mapa_shared(smem_u32(&x), 0); };  // even CTA's copy
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int T = p.T;
  const int G = (int)(gridDim.x / 2), cl = (int)(blockIdx.x / 2);

  if (threadIdx.x == 0) init_pair_bars<C>(bars);
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&ctl->tmem_base), C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  auto stg = [&](int g) { return (uint64_t)(((g % NS) * C::STAGE) >> 4); };

  if (warp == 0) {
    // Producer: per step, Q_j and dO_j (two 32-row copies each: own rows to
    // half 0), then the step's LSE * -log2(e) and delta into the stage's
    // vector slot (loaded before the stage wait, so the load overlaps it).
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmG);
    }
    int last[NS];
    for (int s = 0; s < NS; ++s) last[s] = -1;
    bool ok = true;
    int g = 0;
    PairTile t;
    for (int m = 0; ok && pair_tile_at(p, cl, G, m, rank, t); ++m) {
      const float* lse_bh = p.lse + t.b * p.l0 + t.h * p.l1;
      const float* del_bh = p.delta + (int64_t)t.bh * T;
      for (int i = 0; i < t.n; ++i) {
        const int gs = g + i, s = gs % NS, rr = gs / NS, j = t.j0 + i;
        float vl[BN / 32], vd[BN / 32];
#pragma unroll
        for (int u = 0; u < BN / 32; ++u) {
          const int q = j * BN + 32 * u + lane;
          vl[u] = q < T ? ldg_nc_early(lse_bh + (int64_t)q * p.l2) : 0.0f;
          vd[u] = q < T ? ldg_nc_early(del_bh + q) : 0.0f;
        }
        if (rr > 0 && !(ok = warp_wait(B(bars->empty_a[s]), (rr - 1) & 1, ctl, p.status))) break;
        const uint32_t st = tiles + s * C::STAGE;
        if (lane == 0) {
          const uint32_t fb = B(bars->full_a[s]);
          const int own = j * BN + 32 * (int)rank, other = j * BN + 32 * (int)(rank ^ 1u);
          mbar_arrive_expect_tx(fb, C::TX);
          tma_load_5d(st + C::OFF_Q, &tmQ, fb, 0, own, 0, t.h, t.b);
          tma_load_5d(st + C::OFF_Q + C::HALF, &tmQ, fb, 0, other, 0, t.h, t.b);
          tma_load_5d(st + C::OFF_G, &tmG, fb, 0, own, 0, t.h, t.b);
          tma_load_5d(st + C::OFF_G + C::HALF, &tmG, fb, 0, other, 0, t.h, t.b);
        }
        last[s] = rr;
        float* vs = vec + s * 2 * BN;
#pragma unroll
        for (int u = 0; u < BN / 32; ++u) {
          vs[32 * u + lane] = vl[u] * -kLog2e;
          vs[BN + 32 * u + lane] = vd[u];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(B(bars->vec_full[s]));
      }
      g += t.n;
    }
    __syncwarp();
    if (ctl->abort && lane == 0) {
      for (int s = 0; s < NS; ++s)
        if (last[s] >= 0) mbar_drain(B(bars->full_a[s]), last[s] & 1);
    }
  } else if (warp == 1 || warp == kIssuer2Warp) {
    // Even CTA.  Warp 1: S^T_i -> s_full; [P_i] dV += P_i^T dO_i; S^T_{i+2}
    // into P_i's buffer.  Warp 10: dP^T_i -> dp_full; [dS_i] dK += dS_i^T Q_i;
    // dP^T_{i+2} into dS_i's buffer.  Each reuses a buffer in its own issue
    // order; a stage is released after both issuers' last MMA reading it.
    // Per tile: wait until both CTAs' rows have written out the previous
    // tile's dK / dV and loaded this tile's K / V (rows_ready); commit `done`
    // after the tile's last MMAs.
    if (leader && lane == 0) {
      const bool first = warp == 1;
      const uint32_t tc_x = first ? C::TC_K : C::TC_V;        // stationary operand
      const uint32_t tc_b = first ? C::TC_S : C::TC_DP;       // S^T / dP^T buffers
      const uint32_t tc_acc = first ? C::TC_DV : C::TC_DK;    // accumulator
      const uint64_t kd0 = sdesc_kmajor(tiles + (first ? C::OFF_Q : C::OFF_G));
      const uint64_t md0 = sdesc_mnmajor(tiles + (first ? C::OFF_GM : C::OFF_QM), 64u * 128u);
      uint64_t* full = first ? bars->s_full : bars->dp_full;
      uint64_t* rows = first ? bars->p_full : bars->ds_full;
      auto issue_x = [&](int gs) {
        pair_chain_k<C>(tmem + tc_b + (uint32_t)(gs % 2) * C::SB, tmem + tc_x, kd0 + stg(gs));
        umma_commit_pair(B(full[gs % 2]));
      };
      bool ok = true;
      int g = 0, tn = 0;
      PairTile t;
      for (int m = 0; ok && pair_tile_at(p, cl, G, m, rank, t); ++m) {
        const int n = t.n;
        if (n == 0) continue;
        if (!(ok = mbar_wait(B(bars->rows_ready), tn & 1, ctl, p.status))) break;
        for (int i0 = 0; ok && i0 < 2 && i0 < n; ++i0) {
          const int gs = g + i0;
          if ((ok = mbar_wait(B(bars->ready_a[gs % NS]), (gs / NS) & 1, ctl, p.status))) {
            tc_fence_after();
            issue_x(gs);
          }
        }
        for (int i = 0; ok && i < n; ++i) {
          const int gi = g + i, bi = gi % 2, nx = i + 2, gx = gi + 2;
          // Both waits of the step together (a second wait on a completed
          // phase costs the issuing thread little more than the first; the
          // preparation runs steps ahead, so waiting for stage i+2 here does
          // not delay dV_i).  Stage i's MN-major chunk is covered by this
          // thread's wait on ready_a before S^T_i / dP^T_i.
          if (!(ok = mbar_wait(B(rows[bi]), (gi / 2) & 1, ctl, p.status))) break;
          if (nx < n &&
              !(ok = mbar_wait(B(bars->ready_a[gx % NS]), (gx / NS) & 1, ctl, p.status)))
            break;
          tc_fence_after();
          pair_chain_mn(tmem + tc_acc, tmem + tc_b + (uint32_t)bi * C::SB, md0 + stg(gi), i > 0);
          umma_commit_pair(B(bars->empty_a[gi % NS]));
          if (nx < n) issue_x(gx);
        }
        if (ok) umma_commit_pair(B(bars->done));
        g += n;
        ++tn;
      }
      const uint32_t fin = B(first ? bars->mma_final : bars->mma_final2);
      umma_commit_pair(fin);  // nothing of this thread in flight after this
      mbar_drain(fin, 0);
    }
    __syncwarp();
  } else if (warp == kIssuer3Warp) {
    // idle
  } else if (is_prep_warp(warp)) {
    // Per step: round the own halves of Q_j and dO_j in place (S^T / dP^T
    // operands) and write the MN-major chunks (dK / dV operands), then one
    // arrival on ready_a: each issuing thread waits once per step.  Rounding
    // is idempotent, so the MN pass may read half 0 before or after its
    // rounding.
    const uint32_t tid = prep_tid();
    bool ok = true;
    int g = 0;
    PairTile t;
    for (int m = 0; ok && pair_tile_at(p, cl, G, m, rank, t); ++m) {
      const int n = t.n;
      for (int i = 0; i < n; ++i) {
        const int gs = g + i, s = gs % NS;
        const uint32_t st = tiles + s * C::STAGE;
        if (!(ok = warp_wait(B(bars->full_a[s]), (gs / NS) & 1, ctl, p.status))) break;
        round_tile_smem<C::HALF, kSplitThreads>(st + C::OFF_Q, tid);
        round_tile_smem<C::HALF, kSplitThreads>(st + C::OFF_G, tid);
        pair_derive_mn(st + C::OFF_Q, st + C::OFF_QM, rank, tid);
        pair_derive_mn(st + C::OFF_G, st + C::OFF_GM, rank, tid);
        fence_proxy_async_smem();
        warp_arrive_remote(L(bars->ready_a[s]));
      }
      g += n;
    }
  } else {
    // Row warps 4-7 (group 0) and 11-14 (group 1): thread (quad, lane) owns key
    // row kb + quad*32 + lane; group g forms P^T and dS^T for query columns
    // [32g, 32g + 32) of every step, loads K (g = 0) or V (g = 1) into TMEM
    // and writes dK (g = 0) or dV (g = 1).
    constexpr int HB = BN / 2;
    const int quad = warp & 3;
    const int grp = warp >= kBwdRowWarp1 ? 1 : 0;
    const int c0 = grp * HB;
    const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
    const Ptr4& src = grp ? p.st1 : p.st0;
    float* out = grp ? p.out1 : p.out0;
    // Tile boundary: the next tile's K / V row goes into TMEM as soon as the
    // previous tile's last S^T and dP^T have completed, and rows_ready lets
    // the issuers start S^T_0 / dP^T_0 while the previous dV / dK MMAs drain;
    // the rows then wait for `done` and write out the previous dK / dV (the
    // first dV / dK MMAs, which overwrite the accumulators, wait for P_0 /
    // dS_0, formed after the write-out).
    bool ok = true, pending = false;
    int g = 0, tn = 0;
    // dK / dV rows leave through a per-warp shared-memory buffer
    // (warp_rows_to_global: coalesced stores).
    int64_t prev_row0 = 0;  // global row index (b h T + key) of this warp's first row
    int prev_nrows = 0;     // rows of the warp that lie inside the sequence
    float* wbuf = vec + NS * 2 * BN + (warp - 4 - (grp ? 3 : 0)) * kRowWbufFloats;
    auto write_out = [&]() {
      warp_rows_to_global<D>(lb + (grp ? C::TC_DV : C::TC_DK), grp ? 1.0f : p.scale, wbuf,
                             out + prev_row0 * D, prev_nrows, D, p.accumulate_out != 0);
      tc_fence_before();  // TMEM reads done before the next arrival
    };
    PairTile t;
    for (int m = 0; ok && pair_tile_at(p, cl, G, m, rank, t); ++m) {
      if (!t.exists) continue;
      const int row = t.kb + quad * 32 + lane;
      const bool valid = row < T;
      const int64_t orow = ((int64_t)t.bh * T + (valid ? row : 0)) * D;
      if (t.n == 0) {  // no query of the first segment reaches these keys
        if (valid && !p.accumulate_out) {
          for (int d = 0; d < D; ++d) out[orow + d] = 0.0f;
        }
        continue;
      }
      float x0[32], x1[32];
      {
        const float* rp = src.row(t.b, t.h, valid ? row : 0);
        const bool vr = src.s3 == 1 && ((reinterpret_cast<uintptr_t>(rp) & 15u) == 0);
        load_row32(src, rp, 0, valid, vr, x0);
        load_row32(src, rp, 32, valid, vr, x1);
      }
      // K / V are read only by the S^T / dP^T MMAs, which this warp saw
      // complete (s_full, dp_full of its last step): no wait for the previous
      // tile's `done` before replacing them.
      tc_fence_after();
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        x0[e] = tf32_round(x0[e]);
        x1[e] = tf32_round(x1[e]);
      }
      const uint32_t kv = lb + (grp ? C::TC_V : C::TC_K);
      tmem_st32(kv, x0);
      tmem_st32(kv + 32, x1);
      tmem_wait_st();
      tc_fence_before();
      warp_arrive_remote(L(bars->rows_ready));
      if (pending) {
        if (!(ok = warp_wait(B(bars->done), (tn - 1) & 1, ctl, p.status))) break;
        tc_fence_after();
        write_out();
      }
      {  // the next tile's K / V row into L2 while this tile runs
        PairTile nt;
        for (int m2 = m + 1; m2 <= m + 2; ++m2) {
          if (!pair_tile_at(p, cl, G, m2, rank, nt)) break;
          if (!nt.exists || nt.n == 0) continue;
          const int nrow = nt.kb + quad * 32 + lane;
          if (nrow < T && src.s3 == 1) {
            const float* np = src.row(nt.b, nt.h, nrow);
            asm volatile("prefetch.global.L2 [%0];" ::"l"(np));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(np + 32));
          }
          break;
        }
      }
      for (int i = 0; ok && i < t.n; ++i) {
        const int gi = g + i;
        const int qs = (t.j0 + i) * BN + c0;
        const int bi = gi % 2;
        const uint32_t par = (uint32_t)(gi / 2) & 1u;
        const uint32_t sc = lb + C::TC_S + (uint32_t)bi * C::SB + c0;
        const uint32_t dc = lb + C::TC_DP + (uint32_t)bi * C::SB + c0;
        if (!(ok = warp_wait(B(bars->vec_full[gi % NS]), (gi / NS) & 1, ctl, p.status))) break;
        const float* vl = vec + (gi % NS) * 2 * BN + c0;
        if (!(ok = warp_wait(B(bars->s_full[bi]), par, ctl, p.status))) break;
        tc_fence_after();
        const bool need_mask =
            !valid || (qs + HB > T) || (p.causal && qs < t.kb + kRows - 1);
        float pv[HB];
        {
          float x[HB], lv[HB];
          tmem_ldn<HB>(sc, x);
          load_vecn<HB>(vl, lv);  // -LSE * log2(e)
#pragma unroll
          for (int e = 0; e < HB; e += 2) {
            float a0, a1;
            ffma2(a0, a1, x[e], x[e + 1], p.scale_log2, p.scale_log2, lv[e], lv[e + 1]);
            x[e] = ex2_approx(a0);
            x[e + 1] = ex2_approx(a1);
          }
          if (need_mask) {
#pragma unroll
            for (int e = 0; e < HB; ++e) {
              const int q = qs + e;
              x[e] = (valid && q < T && (!p.causal || q >= row)) ? x[e] : 0.0f;
            }
          }
#pragma unroll
          for (int e = 0; e < HB; ++e) {
            pv[e] = x[e];
            x[e] = tf32_round_finite(x[e]);
          }
          tmem_stn<HB>(sc, x);
        }
        tmem_wait_st();
        tc_fence_before();
        warp_arrive_remote(L(bars->p_full[bi]));  // S^T_i read, P^T_i written
        if (!(ok = warp_wait(B(bars->dp_full[bi]), par, ctl, p.status))) break;
        tc_fence_after();
        {
          float x[HB], dv[HB];
          tmem_ldn<HB>(dc, x);
          load_vecn<HB>(vl + BN, dv);
#pragma unroll
          for (int e = 0; e < HB; e += 2) {
            float u0, u1, d0, d1;
            fsub2(u0, u1, x[e], x[e + 1], dv[e], dv[e + 1]);
            fmul2(d0, d1, pv[e], pv[e + 1], u0, u1);  // dS^T = P^T (dP^T - delta)
            x[e] = tf32_round_finite(d0);
            x[e + 1] = tf32_round_finite(d1);
          }
          tmem_stn<HB>(dc, x);
        }
        tmem_wait_st();
        tc_fence_before();
        warp_arrive_remote(L(bars->ds_full[bi]));
      }
      pending = ok;
      prev_row0 = (int64_t)t.bh * T + t.kb + quad * 32;
      prev_nrows = max(0, min(32, T - (t.kb + quad * 32)));
      g += t.n;
      ++tn;
    }
    if (ok && pending && warp_wait(B(bars->done), (tn - 1) & 1, ctl, p.status)) {
      tc_fence_after();
      write_out();
    }
  }

  tc_fence_before();
  cluster_sync_all();  // no MMA, copy or remote arrival of either CTA pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

template <class C>
int run_dkdv_pair(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
                  const float* lse, const int64_t ls[3], const float* delta, float* dk,
                  float* dv, const DeviceInfo& dev, cudaStream_t st) {
  static unsigned long long attr_done = 0;
  CUtensorMap tq, tg;  // 32-row whole-width copies: [chunk][32 rows][128 B]
  int rc = make_tmap_bhtd_whole(&tq, q, pr, 32);
  if (rc == CT_OK) rc = make_tmap_bhtd_whole(&tg, g, pr, 32);
  if (rc != CT_OK) return rc;
  const size_t smem = pair_smem_bytes<C>();
  rc = ensure_smem_attr(fa2_bwd_dkdv_pair_kernel<C>, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  BwdParams p = make_params(pr, k, v, lse, ls, delta, dk, dv, dev);
  p.n_tiles = (int)((pr.T + 2 * kRows - 1) / (2 * kRows));  // 256-key pair tiles
  const int64_t units = (int64_t)((p.n_tiles + 1) / 2) * p.bh_total;
  // persistent: one cluster per two SMs (one CTA per SM fits), at most one per unit
  const int64_t clusters = std::max<int64_t>(1, std::min<int64_t>(units, dev.sm_count / 2));
  for (int64_t s0 = 0; s0 < pr.T; s0 += kSegLen) {  // one launch per query segment
    p.seg_lo = (int)s0;
    p.seg_hi = (int)std::min<int64_t>(s0 + kSegLen, pr.T);
    p.accumulate_out = s0 > 0;
    fa2_bwd_dkdv_pair_kernel<C><<<(unsigned)(2 * clusters), kBwdThreads, smem, st>>>(tq, tg, p);
    rc = check_launch();
    if (rc != CT_OK) return rc;
  }
  return CT_OK;
}

}  // namespace

bool fa2_bwd_pair_supported(const Fa2Problem& p) {
  static const bool off = [] {
    const char* e = std::getenv("CT_FA2_PAIR_DKDV");
    return e && e[0] == '0';
  }();
  return !off && p.D == 64 && p.precision == CT_PRECISION_TF32 && p.T < (1ll << 31) &&
         2 * ((p.T + 2 * fa2::kRows - 1) / (2 * fa2::kRows)) * p.B * p.H < (1ll << 31);
}

int launch_fa2_bwd_dkdv_pair(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v,
                             Strided4 g, const float* lse, const int64_t ls[3],
                             const float* delta, float* dk, float* dv, const DeviceInfo& dev,
                             cudaStream_t st) {
  if (!fa2_tma_ok(q) || !fa2_tma_ok(g)) return CT_ERR_UNSUPPORTED_LAYOUT;
  if (!fa2_bwd_pair_supported(pr)) return CT_ERR_UNSUPPORTED_HEAD_DIM;
  return run_dkdv_pair<PairCfg<4>>(pr, q, k, v, g, lse, ls, delta, dk, dv, dev, st);
}

}  // namespace ct
