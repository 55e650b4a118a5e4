// fa2_bwd_tc.cu -- FlashAttention-2 backward on the sm_100a tensor cores,
// atomics-free like the reference (flash_attention.cuh:216-504): a
// query-stationary kernel produces dQ and a key/value-stationary kernel
// produces dK and dV, each recomputing P = exp(S - L) and dP = dO V^T.
// Unlike flash_attention_bwd_dk_dv (:409-411) the dK/dV pass starts at the
// causal diagonal instead of scanning every query tile.
//
// Warp roles (16 warps): warp 0 TMA producer, warp 1 TMEM allocator and first
// MMA issuer, warps 2, 3, 8, 9 TF32 hi/lo split or rounding of landed tiles
// (and the MN-major copies), warps 4-7 and 11-14 two row warpgroups (one
// stationary row per thread / TMEM lane, each group half of a step's
// columns), warp 10 the second MMA issuer, warp 15 a third.  dQ: warp 1 issues
// S, warp 10 dQ and dP -- dP on warp 15 when S / dP are double-buffered.
// dK/dV: warp 1 issues S^T and dV, warp 10 dP^T and dK.
//
// dQ kernel, per 128 query rows, per key tile j (BN keys):
//   S  = Q K_j^T     (A = Q in TMEM, B = K_j K-major)
//   dP = dO V_j^T    (A = dO in TMEM, B = V_j K-major)
//   dS = P * (dP - delta), P = exp2(S * log2e / sqrt(D) - L * log2e)   [row warps]
//   dQ += dS K_j     (A = dS in TMEM, B = K_j read MN-major)
// dK/dV kernel, per 128 key rows, per query tile j (BN queries):
//   S^T  = K Q_j^T,  dP^T = V dO_j^T,  P^T, dS^T in the row warps
//   dV += P^T dO_j,  dK += dS^T Q_j   (B = Q_j / dO_j read MN-major)
// The issuers run one step ahead of the row warps (S_{j+1} while dS_j is
// formed), two with double-buffered S / dP (TF32).  An S or dP buffer written
// and read by MMAs of one issuer is reused in that issuer's issue order; the
// dQ pass's third issuer waits on a barrier (dqd) for dQ_j before dP_{j+2}
// reuses dS_j's buffer.  3xTF32 interleaves the hi / lo copies of K-major
// tiles so one MMA forms hi*hi and hi*lo together (mma_chain_kil).
// Sequences longer than kSegLen run one launch per segment of the reduced
// dimension, each adding into the previous one's output (fa2_common.cuh).
#include <algorithm>

#include "fa2_bwd_parts.cuh"

namespace ct {
namespace {

using namespace fa2;

// dQ pass: A = K (K-major for S, MN-major for dQ), B = V (K-major for dP).
// NSB TMEM buffers each for S and dP / dS: with two, S_{j+1} and dP_{j+1} run
// on the tensor core while the row warps still form dS_j, and dP_{j+1} does
// not wait for dQ_j to finish reading dS_j.
// In 3xTF32 mode dP uses the interleaved K-major V tile: its hi/lo partial
// sums land side by side in the dP / dS buffer's 2*BN columns (mma_chain_kil).
template <int D_, int BN_, int SPLIT_, int NS_, int NSB_ = 1>
struct DqCfg : BwdTiles<D_, BN_, SPLIT_, NS_, 2, 1, false, true> {
  using T_ = BwdTiles<D_, BN_, SPLIT_, NS_, 2, 1, false, true>;
  static constexpr int NSB = NSB_;
  static constexpr uint32_t SB = T_::NCOPY * BN_;  // one dP / dS buffer: hi [| lo]
  static constexpr uint32_t TC_Q = 0, TC_G = T_::NCOPY * D_, TC_DQ = 2 * T_::NCOPY * D_;
  static constexpr uint32_t TC_S = TC_DQ + D_, TC_DP = TC_S + NSB * BN_;
  static_assert(NSB == 1 || NSB == 2, "S / dP buffering");
  static_assert(TC_DP + NSB * SB <= T_::TMEM_COLS, "TMEM budget");
};

template <class C>
__global__ void __launch_bounds__(kBwdThreads, 1)
    fa2_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const BwdParams p) {
  constexpr int D = C::D, BN = C::BN, NS = C::NS, SPLIT = C::SPLIT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (status_raised(p.status)) return;
  auto* bars = reinterpret_cast<BwdBars<NS>*>(smem_raw);
  const uint32_t tiles = (smem_u32(smem_raw) + (uint32_t)sizeof(BwdBars<NS>) + 1023u) & ~1023u;
  CtaCtl* ctl = &bars->ctl;
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  int qt, bh;  // head-major (L2 reuse of K/V), last query tiles of a head first
  cta_tile(p.n_tiles, p.bh_total, p.head_group, true, qt, bh);
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = qt * kRows, T = p.T;
  const int last_row = min(q0 + kRows - 1, T - 1);
  // key tiles [jb, jb + n_kv) of this launch's segment
  const int jb = p.seg_lo / BN;
  const int n_kv = max(0, min(p.causal ? last_row / BN + 1 : (T + BN - 1) / BN,
                              (p.seg_hi + BN - 1) / BN) - jb);
  if (n_kv == 0) {  // no key of the segment reaches these queries (uniform exit)
    if (!p.accumulate_out && threadIdx.x < kRows && q0 + (int)threadIdx.x < T) {
      float* o = p.out0 + ((int64_t)bh * T + q0 + threadIdx.x) * D;
      for (int d = 0; d < D; ++d) o[d] = 0.0f;
    }
    return;
  }

  // K_j is released by the dQ_j issuer alone: dQ_j waits for dS_j, formed
  // after the row warps read S_j, so S_j has completed by then.
  if (threadIdx.x == 0) init_bwd_bars<C>(bars, 1, 1, 8);
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    const CUtensorMap* maps[2] = {&tmK, &tmV};
    bwd_producer<C, false, false>(bars, tiles, nullptr, maps, jb, jb + n_kv, h, b, nullptr, 0,
                                  nullptr, T, p.status);
  } else if (warp == 1) {
    // S_j = Q K_j^T into S buffer j % NSB once the row warps hold S_{j-NSB}
    // (the buffer's previous contents) in registers.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_tf32(128, BN, false, false);
      const uint64_t kd0 = sdesc_kmajor(tiles + C::OFF_A0);  // stage-0 descriptor
      bool ok = mbar_wait(B(bars->rows_ready), 0, ctl, p.status);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int bj = j % C::NSB;
        if (j >= C::NSB &&
            !(ok = mbar_wait(B(bars->s_free[bj]), ((j - C::NSB) / C::NSB) & 1, ctl, p.status)))
          break;
        if (!(ok = mbar_wait(B(bars->ready_a[j % NS]), (j / NS) & 1, ctl, p.status))) break;
        tc_fence_after();
        mma_chain<SPLIT, D, false, BN, C::TILE>(tmem + C::TC_S + (uint32_t)bj * BN, tmem + C::TC_Q,
                                                tmem + C::TC_Q + D,
                                                kd0 + (uint64_t)(((j % NS) * C::STAGE) >> 4), idS,
                                                false);
        umma_commit(B(bars->s_full[bj]));
      }
      umma_commit(B(bars->mma_final));
      mbar_drain(B(bars->mma_final), 0);
    }
    __syncwarp();
  } else if (warp == kIssuer2Warp || warp == kIssuer3Warp) {
    // Warp 10 issues dQ += dS_j K_j.  With one dP buffer it also issues
    // dP_j = dO V_j^T, and dP_{j+1} overwrites dS_j only after dQ_j in its issue
    // order.  With two buffers warp 15 issues dP_j into buffer j % 2 once dQ_{j-2}
    // has finished reading dS_{j-2} from it (dqd), so dQ and dP do not queue
    // behind each other on one issuing thread.
    const bool dq_here = warp == kIssuer2Warp;
    const bool dp_here = C::NSB == 1 ? dq_here : warp == kIssuer3Warp;
    if (lane == 0 && (dq_here || dp_here)) {
      constexpr uint32_t idS = idesc_tf32(128, BN, false, false);
      constexpr uint32_t idQ = idesc_tf32(128, D, false, true);
      const uint64_t kmd0 = sdesc_mnmajor(tiles + C::OFF_A1, BN * 128);  // stage-0 descriptors
      const uint64_t vd0 = sdesc_kmajor(tiles + C::OFF_B0);
      auto stg = [&](int j) { return (uint64_t)(((j % NS) * C::STAGE) >> 4); };
      auto& rv = bars->ready_b;
      auto issue_dP = [&](int j) {
        const uint32_t db = tmem + C::TC_DP + (uint32_t)(j % C::NSB) * C::SB;
        if constexpr (C::KILB)
          mma_chain_kil<D, C::KCHB>(db, tmem + C::TC_G, tmem + C::TC_G + D, vd0 + stg(j),
                                    idesc_tf32(128, 2 * BN, false, false), idS);
        else
          mma_chain<SPLIT, D, false, BN, C::TILE>(db, tmem + C::TC_G, tmem + C::TC_G + D,
                                                  vd0 + stg(j), idS, false);
        umma_commit(B(bars->empty_b[j % NS]));  // V_j read for the last time
        umma_commit(B(bars->dp_full[j % C::NSB]));
      };
      auto issue_dQ = [&](int j) {
        const uint32_t db = tmem + C::TC_DP + (uint32_t)(j % C::NSB) * C::SB;
        mma_chain<SPLIT, BN, true, BN, C::TILE>(tmem + C::TC_DQ, db, db + BN, kmd0 + stg(j), idQ,
                                                j > 0);
        umma_commit(B(bars->empty_a[j % NS]));  // K_j read for the last time
      };
      bool ok = mbar_wait(B(bars->rows_ready), 0, ctl, p.status);
      if (ok && dq_here && dp_here) {  // one buffer: dP and dQ interleaved
        if ((ok = mbar_wait(B(rv[0]), 0, ctl, p.status))) {
          tc_fence_after();
          issue_dP(0);
        }
        for (int j = 0; ok && j < n_kv; ++j) {
          if (!(ok = mbar_wait(B(bars->ds_full[0]), j & 1, ctl, p.status))) break;
          tc_fence_after();
          issue_dQ(j);
          if (j + 1 < n_kv) {
            if (!(ok = mbar_wait(B(rv[(j + 1) % NS]), ((j + 1) / NS) & 1, ctl, p.status))) break;
            tc_fence_after();
            issue_dP(j + 1);
          }
        }
        if (ok) umma_commit(B(bars->done));
      } else if (ok && dq_here) {  // two buffers, warp 10: dQ only
        for (int j = 0; ok && j < n_kv; ++j) {
          const int bj = j % C::NSB;
          if (!(ok = mbar_wait(B(bars->ds_full[bj]), (j / C::NSB) & 1, ctl, p.status))) break;
          tc_fence_after();
          issue_dQ(j);
          umma_commit(B(bars->dqd[bj]));
        }
        if (ok) umma_commit(B(bars->done));
      } else if (ok) {  // two buffers, warp 15: dP only
        for (int j = 0; ok && j < n_kv; ++j) {
          if (j >= C::NSB && !(ok = mbar_wait(B(bars->dqd[j % C::NSB]),
                                              ((j - C::NSB) / C::NSB) & 1, ctl, p.status)))
            break;
          if (!(ok = mbar_wait(B(rv[j % NS]), (j / NS) & 1, ctl, p.status))) break;
          tc_fence_after();
          issue_dP(j);
        }
      }
      const uint32_t fin = B(dq_here ? bars->mma_final2 : bars->mma_final3);
      umma_commit(fin);  // nothing of this thread in flight after this
      mbar_drain(fin, 0);
    }
    __syncwarp();
  } else if (is_prep_warp(warp)) {
    bwd_splitter<C, false>(bars, tiles, n_kv, p.status);
  } else {
    // Row warps 4-7 (group 0) and 11-14 (group 1): thread (quad, lane) owns
    // query row quad*32 + lane in TMEM lane quarter quad; group g forms P and
    // dS for the key columns [g*BN/2, (g+1)*BN/2) of every step (both are
    // elementwise), loads Q (g = 0) or dO (g = 1) into TMEM, and writes dQ
    // columns [g*D/2, (g+1)*D/2).
    constexpr int HB = BN / 2, CW = HB < 32 ? HB : 32;
    const int quad = warp & 3;
    const int grp = warp >= kBwdRowWarp1 ? 1 : 0;
    const int c0 = grp * HB;
    const int row = q0 + quad * 32 + lane;
    const bool valid = row < T;
    const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
    float l2 = 0.0f, dl = 0.0f;
    {
      const Ptr4& src = grp ? p.st1 : p.st0;
      const float* r = src.row(b, h, valid ? row : 0);
      const bool vr = src.s3 == 1 && ((reinterpret_cast<uintptr_t>(r) & 15u) == 0);
      row_to_tmem<D, SPLIT>(src, r, valid, vr, lb, grp ? C::TC_G : C::TC_Q);
      if (valid) {
        l2 = __ldg(p.lse + b * p.l0 + h * p.l1 + (int64_t)row * p.l2) * kLog2e;
        dl = __ldg(p.delta + (int64_t)bh * T + row);
      }
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->rows_ready));
    }
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int bj = j % C::NSB;
      const uint32_t par = (uint32_t)(j / C::NSB) & 1u;
      const uint32_t dc = lb + C::TC_DP + (uint32_t)bj * C::SB + c0;
      if (!(ok = warp_wait(B(bars->s_full[bj]), par, ctl, p.status))) break;
      tc_fence_after();
      float pv[HB];
#pragma unroll
      for (int c = 0; c < HB / CW; ++c) {
        float t[CW];
        tmem_ldn<CW>(lb + C::TC_S + (uint32_t)bj * BN + c0 + CW * c, t);
#pragma unroll
        for (int i = 0; i < CW; ++i) pv[CW * c + i] = t[i];
      }
      tc_fence_before();
      warp_arrive(B(bars->s_free[bj]));
      const int kv0 = (jb + j) * BN + c0;
      const bool need_mask = !valid || (kv0 + HB > T) || (p.causal && kv0 + HB - 1 > q0);
      // straight-line exponentials, then the mask as a separate pass on the
      // few boundary tiles (a test per column would split the unrolled loop
      // into one basic block per column and serialise it)
      const float nl2 = -l2;
#pragma unroll
      for (int i = 0; i < HB; i += 2) {
        float a0, a1;
        ffma2(a0, a1, pv[i], pv[i + 1], p.scale_log2, p.scale_log2, nl2, nl2);
        pv[i] = ex2_approx(a0);
        pv[i + 1] = ex2_approx(a1);
      }
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < HB; ++i) {
          const int kv = kv0 + i;
          pv[i] = (valid && kv < T && (!p.causal || kv <= row)) ? pv[i] : 0.0f;
        }
      }
      if (!(ok = warp_wait(B(bars->dp_full[bj]), par, ctl, p.status))) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HB / CW; ++c) {
        float t[CW], lo[CW];
        tmem_ldn<CW>(dc + CW * c, t);
        if constexpr (C::KILB) {  // dP from its two partial sums
          tmem_ldn<CW>(dc + BN + CW * c, lo);
#pragma unroll
          for (int i = 0; i < CW; i += 2) fadd2(t[i], t[i + 1], t[i], t[i + 1], lo[i], lo[i + 1]);
        }
#pragma unroll
        for (int i = 0; i < CW; i += 2) {
          float u0, u1, d0, d1;
          fsub2(u0, u1, t[i], t[i + 1], dl, dl);
          fmul2(d0, d1, pv[CW * c + i], pv[CW * c + i + 1], u0, u1);  // dS = P (dP - delta)
          if constexpr (SPLIT == 3) {
            tf32_split2(d0, d1, t[i], t[i + 1], lo[i], lo[i + 1]);
          } else {
            t[i] = tf32_round_finite(d0);
            t[i + 1] = tf32_round_finite(d1);
          }
        }
        tmem_stn<CW>(dc + CW * c, t);
        if constexpr (SPLIT == 3) tmem_stn<CW>(dc + BN + CW * c, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->ds_full[bj]));
    }
    if (ok && warp_wait(B(bars->done), 0, ctl, p.status)) {
      tc_fence_after();
      // coalesced through the warp's shared-memory buffer
      float* wbuf = reinterpret_cast<float*>(smem_raw + (tiles - smem_u32(smem_raw)) +
                                             NS * C::STAGE + NS * 2 * BN * 4) +
                    (warp - 4 - (grp ? 3 : 0)) * kRowWbufFloats;
      const int r0 = q0 + quad * 32;
      warp_rows_to_global<D / 2>(lb + C::TC_DQ + grp * (D / 2), p.scale, wbuf,
                                 p.out0 + ((int64_t)bh * T + r0) * D + grp * (D / 2),
                                 max(0, min(32, T - r0)), D, p.accumulate_out != 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// -------------------------------------------------------------- dK/dV pass
// dK/dV pass: A = Q (K-major for S^T, MN-major for dK), B = dO (K-major for
// dP^T, MN-major for dV).
// In 3xTF32 mode S^T and dP^T use the interleaved K-major layout: their two
// hi/lo partial sums land side by side in the buffer's 2*BN columns and the
// row warps add them (mma_chain_kil).
//
// PASS selects what one launch accumulates: kDkvBoth (dK and dV), or, where K,
// V and both accumulators do not fit TMEM together (D = 128: 4 x 128 columns),
// kDkvOnlyDv (K, S^T -> P^T, dV; no V, dP^T or dK) followed by kDkvOnlyDk (K,
// V, S^T, dP^T -> dS^T, dK; no dV), each reading the same streamed tiles.
constexpr int kDkvBoth = 0, kDkvOnlyDv = 1, kDkvOnlyDk = 2;

// A single-gradient pass keeps only the layouts it reads: the dV pass no
// MN-major Q (dK's operand) and dO only MN-major (landed so by TMA), the dK
// pass no MN-major dO (dV's operand).
template <int D_, int BN_, int SPLIT_, int NS_, int NSB_ = 1, int PASS_ = kDkvBoth>
struct DkvCfg : BwdTiles<D_, BN_, SPLIT_, NS_, PASS_ == kDkvOnlyDv ? 1 : 2,
                         PASS_ == kDkvBoth ? 2 : 1, true, true, PASS_ == kDkvOnlyDv> {
  using T_ = BwdTiles<D_, BN_, SPLIT_, NS_, PASS_ == kDkvOnlyDv ? 1 : 2,
                      PASS_ == kDkvBoth ? 2 : 1, true, true, PASS_ == kDkvOnlyDv>;
  // NSB TMEM buffers each for S^T / P^T and dP^T / dS^T.  With two, S^T_{i+1}
  // and dP^T_{i+1} run on the tensor core while the row warps still form P_i
  // and dS_i, so the rows go from one step to the next without waiting.
  static constexpr int NSB = NSB_, PASS = PASS_;
  static constexpr bool DO_DV = PASS != kDkvOnlyDk, DO_DK = PASS != kDkvOnlyDv;
  static constexpr uint32_t SB = T_::NCOPY * BN_;  // columns of one buffer: hi [| lo]
  // column map: K [| V] [| dK] [| dV] | S^T buffers [| dP^T buffers]
  static constexpr uint32_t TC_K = 0, TC_V = T_::NCOPY * D_;
  static constexpr uint32_t TC_DK = TC_V + (DO_DK ? T_::NCOPY * D_ : 0);
  static constexpr uint32_t TC_DV = TC_DK + (DO_DK ? D_ : 0);
  static constexpr uint32_t TC_S = TC_DV + (DO_DV ? D_ : 0), TC_DP = TC_S + NSB * SB;
  static_assert(NSB == 1 || NSB == 2, "S / dP buffering");
  static_assert((DO_DK ? TC_DP + NSB * SB : TC_S + NSB * SB) <= T_::TMEM_COLS, "TMEM budget");
};

template <class C>
__global__ void __launch_bounds__(kBwdThreads, 1)
    fa2_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                           const __grid_constant__ CUtensorMap tmG,
                           const BwdParams p) {
  constexpr int D = C::D, BN = C::BN, NS = C::NS, SPLIT = C::SPLIT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (status_raised(p.status)) return;
  auto* bars = reinterpret_cast<BwdBars<NS>*>(smem_raw);
  const uint32_t tiles = (smem_u32(smem_raw) + (uint32_t)sizeof(BwdBars<NS>) + 1023u) & ~1023u;
  float* vec = reinterpret_cast<float*>(smem_raw + (tiles - smem_u32(smem_raw)) + NS * C::STAGE);
  CtaCtl* ctl = &bars->ctl;
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  int kt_, bh;  // head-major (L2 reuse of Q/dO); causal: low key tiles are heaviest
  cta_tile(p.n_tiles, p.bh_total, p.head_group, false, kt_, bh);
  const int b = bh / p.H, h = bh % p.H;
  const int k0 = kt_ * kRows, T = p.T;
  // query tiles [j0, j1) of this launch's segment
  const int j0 = max(p.causal ? k0 / BN : 0, p.seg_lo / BN);
  const int j1 = min((T + BN - 1) / BN, (p.seg_hi + BN - 1) / BN);
  const int n = max(0, j1 - j0);
  if (n == 0 && p.accumulate_out) return;  // nothing to add (uniform exit)

  // Q_i / dO_i are read by both issuers (S^T_i, dV_i by warp 1; dP^T_i, dK_i
  // by warp 10; in the dV pass S^T_i by warp 1, dV_i by warp 10): the merged
  // stage is free after both have committed.
  if (threadIdx.x == 0) init_bwd_bars<C>(bars, 2, 2, 8);
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  auto stg = [&](int i) { return (uint64_t)(((i % NS) * C::STAGE) >> 4); };
  auto& rdy = bars->ready_a;     // K-major copies of Q_i and dO_i prepared
  auto& rdy_mn = bars->ready_b;  // MN-major copies prepared
  constexpr uint32_t idS = idesc_tf32(128, BN, false, false);
  constexpr uint32_t idS2 = idesc_tf32(128, 2 * BN, false, false);  // [hi | lo] rows (KIL)
  constexpr uint32_t idO = idesc_tf32(128, D, false, true);

  if (warp == 0) {
    const CUtensorMap* maps[2] = {&tmQ, &tmG};
    bwd_producer<C, true, true>(bars, tiles, vec, maps, j0, j1, h, b, p.lse + b * p.l0 + h * p.l1,
                          p.l2, p.delta + (int64_t)bh * T, T, p.status);
  } else if (C::PASS == kDkvOnlyDv && (warp == 1 || warp == kIssuer2Warp)) {
    // dV pass, two issuing threads.  Warp 1: S^T_{i+NSB} into buffer i % NSB
    // once dV_i has read P_i from it (dqd[b], committed by warp 10).  Warp 10:
    // [P_i ready, dO_i MN-major ready]  dV += P_i^T dO_i -> dqd[b].
    if (lane == 0) {
      auto issue_S = [&](int i) {
        const uint32_t sb = (uint32_t)(i % C::NSB) * C::SB;
        if constexpr (C::KILA)
          mma_chain_kil<D, C::KCHA>(tmem + C::TC_S + sb, tmem + C::TC_K, tmem + C::TC_K + D,
                                   sdesc_kmajor(tiles + C::OFF_A0) + stg(i), idS2, idS);
        else
          mma_chain<SPLIT, D, false, BN, C::TILE>(tmem + C::TC_S + sb, tmem + C::TC_K,
                                                  tmem + C::TC_K + D,
                                                  sdesc_kmajor(tiles + C::OFF_A0) + stg(i), idS,
                                                  false);
        umma_commit(B(bars->s_full[i % C::NSB]));
      };
      const uint32_t fin = B(warp == 1 ? bars->mma_final : bars->mma_final2);
      bool ok = n > 0 && mbar_wait(B(bars->rows_ready), 0, ctl, p.status);
      if (warp == 1) {
        for (int i = 0; ok && i < C::NSB && i < n; ++i) {
          if ((ok = mbar_wait(B(rdy[i % NS]), (i / NS) & 1, ctl, p.status))) {
            tc_fence_after();
            issue_S(i);
          }
        }
        for (int i = 0; ok && i < n; ++i) {
          const int bi = i % C::NSB, nx = i + C::NSB;
          umma_commit(B(bars->empty_a[i % NS]));  // S^T_i, issued earlier, read Q_i
          if (nx < n) {
            if (!(ok = mbar_wait(B(bars->dqd[bi]), (i / C::NSB) & 1, ctl, p.status))) break;
            if (!(ok = mbar_wait(B(rdy[nx % NS]), (nx / NS) & 1, ctl, p.status))) break;
            tc_fence_after();
            issue_S(nx);
          }
        }
      } else {
        const uint64_t gmd0 = sdesc_mnmajor(tiles + C::OFF_B1, BN * 128);
        for (int i = 0; ok && i < n; ++i) {
          const int bi = i % C::NSB;
          if (!(ok = mbar_wait(B(bars->p_full[bi]), (i / C::NSB) & 1, ctl, p.status))) break;
          if (!(ok = mbar_wait(B(rdy_mn[i % NS]), (i / NS) & 1, ctl, p.status))) break;
          tc_fence_after();
          const uint32_t pb = tmem + C::TC_S + (uint32_t)bi * C::SB;
          mma_chain<SPLIT, BN, true, BN, C::TILE>(  // dV += P^T dO_i
              tmem + C::TC_DV, pb, pb + BN, gmd0 + stg(i), idO, i > 0);
          umma_commit(B(bars->dqd[bi]));
          umma_commit(B(bars->empty_a[i % NS]));
        }
      }
      if (ok) umma_commit(B(bars->done));
      umma_commit(fin);  // nothing of this thread in flight after this
      mbar_drain(fin, 0);
    }
    __syncwarp();
  } else if (warp == 1) {
    // Step i of buffer b = i % NSB:  [P_i ready, tiles i+NSB prepared]
    //   dV += P_i^T dO_i;  S^T_{i+NSB} -> s_full[b]
    // S^T_{i+NSB} overwrites P_i after dV_i in this thread's issue order.
    if (lane == 0) {
      const uint64_t qd0 = sdesc_kmajor(tiles + C::OFF_A0);  // stage-0 descriptors
      const uint64_t gmd0 = sdesc_mnmajor(tiles + C::OFF_B1, BN * 128);
      auto issue_S = [&](int i) {
        const uint32_t sb = (uint32_t)(i % C::NSB) * C::SB;
        if constexpr (C::KILA)
          mma_chain_kil<D, C::KCHA>(tmem + C::TC_S + sb, tmem + C::TC_K, tmem + C::TC_K + D,
                                   qd0 + stg(i), idS2, idS);
        else
          mma_chain<SPLIT, D, false, BN, C::TILE>(tmem + C::TC_S + sb, tmem + C::TC_K,
                                                  tmem + C::TC_K + D, qd0 + stg(i), idS, false);
        umma_commit(B(bars->s_full[i % C::NSB]));
      };
      bool ok = n > 0 && mbar_wait(B(bars->rows_ready), 0, ctl, p.status) &&
                mbar_wait(B(rdy[0]), 0, ctl, p.status);
      if (ok) {
        tc_fence_after();
        issue_S(0);
        if (C::NSB == 2 && n > 1) {
          ok = mbar_wait(B(rdy[1 % NS]), (1 / NS) & 1, ctl, p.status);
          if (ok) {
            tc_fence_after();
            issue_S(1);
          }
        }
        for (int i = 0; ok && i < n; ++i) {
          const int bi = i % C::NSB, nx = i + C::NSB;
          if (!(ok = mbar_wait(B(bars->p_full[bi]), (i / C::NSB) & 1, ctl, p.status))) break;
          // One buffer: the next S^T is needed by the rows right away, so both
          // waits are taken together and the MMA groups issue back to back.
          // Two buffers: stage i is released right after dV_i (the ring holds
          // steps i .. i+2 at once) and S^T_{i+2} waits for its own tiles.
          if (C::NSB == 1 && nx < n &&
              !(ok = mbar_wait(B(rdy[nx % NS]), (nx / NS) & 1, ctl, p.status)))
            break;
          if constexpr (C::DO_DV) {
            // dO_i's MN-major copy (prepared right after the K-major ones)
            if (!(ok = mbar_wait(B(rdy_mn[i % NS]), (i / NS) & 1, ctl, p.status))) break;
            tc_fence_after();
            const uint32_t pb = tmem + C::TC_S + (uint32_t)bi * C::SB;
            mma_chain<SPLIT, BN, true, BN, C::TILE>(  // dV += P^T dO_i
                tmem + C::TC_DV, pb, pb + BN, gmd0 + stg(i), idO, i > 0);
          }
          if (C::NSB == 1 && nx < n) issue_S(nx);
          umma_commit(B(bars->empty_a[i % NS]));
          if (C::NSB == 2 && nx < n) {
            if (!(ok = mbar_wait(B(rdy[nx % NS]), (nx / NS) & 1, ctl, p.status))) break;
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
  } else if (warp == kIssuer2Warp) {
    // Step i of buffer b:  [dS_i ready]  dK += dS_i^T Q_i -> empty_i;
    //   [tiles i+NSB prepared]  dP^T_{i+NSB} -> dp_full[b]
    // dP^T_{i+NSB} overwrites dS_i after dK_i in this thread's issue order.
    if (C::DO_DK && lane == 0) {
      const uint64_t gd0 = sdesc_kmajor(tiles + C::OFF_B0);  // stage-0 descriptors
      const uint64_t qmd0 = sdesc_mnmajor(tiles + C::OFF_A1, BN * 128);
      auto issue_dP = [&](int i) {
        const uint32_t sb = (uint32_t)(i % C::NSB) * C::SB;
        if constexpr (C::KILB)
          mma_chain_kil<D, C::KCHB>(tmem + C::TC_DP + sb, tmem + C::TC_V, tmem + C::TC_V + D,
                                   gd0 + stg(i), idS2, idS);
        else
          mma_chain<SPLIT, D, false, BN, C::TILE>(tmem + C::TC_DP + sb, tmem + C::TC_V,
                                                  tmem + C::TC_V + D, gd0 + stg(i), idS, false);
        umma_commit(B(bars->dp_full[i % C::NSB]));
      };
      bool ok = n > 0 && mbar_wait(B(bars->rows_ready), 0, ctl, p.status) &&
                mbar_wait(B(rdy[0]), 0, ctl, p.status);
      if (ok) {
        tc_fence_after();
        issue_dP(0);
        if (C::NSB == 2 && n > 1) {
          ok = mbar_wait(B(rdy[1 % NS]), (1 / NS) & 1, ctl, p.status);
          if (ok) {
            tc_fence_after();
            issue_dP(1);
          }
        }
        for (int i = 0; ok && i < n; ++i) {
          const int bi = i % C::NSB, nx = i + C::NSB;
          if (!(ok = mbar_wait(B(bars->ds_full[bi]), (i / C::NSB) & 1, ctl, p.status))) break;
          if (!(ok = mbar_wait(B(rdy_mn[i % NS]), (i / NS) & 1, ctl, p.status))) break;
          tc_fence_after();
          const uint32_t db = tmem + C::TC_DP + (uint32_t)bi * C::SB;
          mma_chain<SPLIT, BN, true, BN, C::TILE>(  // dK += dS^T Q_i
              tmem + C::TC_DK, db, db + BN, qmd0 + stg(i), idO, i > 0);
          umma_commit(B(bars->empty_a[i % NS]));  // Q_i, dO_i read for the last time
          if (nx < n) {
            if (!(ok = mbar_wait(B(rdy[nx % NS]), (nx / NS) & 1, ctl, p.status))) break;
            tc_fence_after();
            issue_dP(nx);
          }
        }
        if (ok) umma_commit(B(bars->done));
      }
      umma_commit(B(bars->mma_final2));
      mbar_drain(B(bars->mma_final2), 0);
    }
    __syncwarp();
  } else if (warp == kIssuer3Warp) {
    // unused in this pass
  } else if (is_prep_warp(warp)) {
    bwd_splitter<C, true>(bars, tiles, n, p.status);
  } else {
    // Row warps 4-7 (group 0) and 11-14 (group 1): thread (quad, lane) owns key
    // row quad*32 + lane in TMEM lane quarter quad; group g forms P^T and dS^T
    // for the query columns [g*BN/2, (g+1)*BN/2) of every step (both are
    // elementwise), loads K (g = 0) or V (g = 1) into TMEM, and writes dK
    // (g = 0) or dV (g = 1).
    constexpr int HB = BN / 2, CW = HB < 32 ? HB : 32;
    const int quad = warp & 3;
    const int grp = warp >= kBwdRowWarp1 ? 1 : 0;
    const int c0 = grp * HB;
    const int row = k0 + quad * 32 + lane;  // key row
    const bool valid = row < T;
    const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
    if (grp == 0 || C::DO_DK) {  // V is read only by dP^T
      const Ptr4& src = grp ? p.st1 : p.st0;
      const float* r = src.row(b, h, valid ? row : 0);
      const bool vr = src.s3 == 1 && ((reinterpret_cast<uintptr_t>(r) & 15u) == 0);
      row_to_tmem<D, SPLIT>(src, r, valid, vr, lb, grp ? C::TC_V : C::TC_K);
      tmem_wait_st();
    }
    tc_fence_before();
    warp_arrive(B(bars->rows_ready));
    bool ok = n > 0;
    for (int i = 0; ok && i < n; ++i) {
      const int qs = (j0 + i) * BN + c0;
      const int bi = i % C::NSB;
      const uint32_t par = (uint32_t)(i / C::NSB) & 1u;
      const uint32_t sc = lb + C::TC_S + (uint32_t)bi * C::SB + c0;
      const uint32_t dc = lb + C::TC_DP + (uint32_t)bi * C::SB + c0;
      // the step's log-sum-exp * log2(e) and delta, staged by the producer warp
      if (!(ok = warp_wait(B(bars->vec_full[i % NS]), (i / NS) & 1, ctl, p.status))) break;
      const float* vl = vec + (i % NS) * 2 * BN + c0;
      if (!(ok = warp_wait(B(bars->s_full[bi]), par, ctl, p.status))) break;
      tc_fence_after();
      const bool need_mask = !valid || (qs + HB > T) || (p.causal && qs < k0 + kRows - 1);
      float pv[HB];
#pragma unroll
      for (int c = 0; c < HB / CW; ++c) {
        float t[CW], lo[CW], lv[CW];
        tmem_ldn<CW>(sc + CW * c, t);
        if constexpr (C::KILA) {  // S^T = [hi-hi + lo-hi part] + [hi-lo part]
          tmem_ldn<CW>(sc + BN + CW * c, lo);
#pragma unroll
          for (int x = 0; x < CW; x += 2) fadd2(t[x], t[x + 1], t[x], t[x + 1], lo[x], lo[x + 1]);
        }
        load_vecn<CW>(vl + CW * c, lv);  // -LSE * log2(e)
        // straight-line exponentials; the mask is a separate pass on the few
        // boundary tiles (a test per column would serialise the loop)
#pragma unroll
        for (int x = 0; x < CW; x += 2) {
          float a0, a1;
          ffma2(a0, a1, t[x], t[x + 1], p.scale_log2, p.scale_log2, lv[x], lv[x + 1]);
          t[x] = ex2_approx(a0);
          t[x + 1] = ex2_approx(a1);
        }
        if (need_mask) {
#pragma unroll
          for (int x = 0; x < CW; ++x) {
            const int q = qs + CW * c + x;
            t[x] = (valid && q < T && (!p.causal || q >= row)) ? t[x] : 0.0f;
          }
        }
#pragma unroll
        for (int x = 0; x < CW; x += 2) {
          pv[CW * c + x] = t[x];
          pv[CW * c + x + 1] = t[x + 1];
          if constexpr (SPLIT == 3) {
            tf32_split2(t[x], t[x + 1], t[x], t[x + 1], lo[x], lo[x + 1]);
          } else {
            t[x] = tf32_round_finite(t[x]);
            t[x + 1] = tf32_round_finite(t[x + 1]);
          }
        }
        if constexpr (C::DO_DV) {  // P^T is the A operand of dV only
          tmem_stn<CW>(sc + CW * c, t);
          if constexpr (SPLIT == 3) tmem_stn<CW>(sc + BN + CW * c, lo);
        }
      }
      if constexpr (C::DO_DV) tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->p_full[bi]));  // S^T_i read: its buffer may be reused
      if constexpr (!C::DO_DK) continue;
      if (!(ok = warp_wait(B(bars->dp_full[bi]), par, ctl, p.status))) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HB / CW; ++c) {
        float t[CW], lo[CW], dv[CW];
        tmem_ldn<CW>(dc + CW * c, t);
        if constexpr (C::KILB) {  // dP^T from its two partial sums
          tmem_ldn<CW>(dc + BN + CW * c, lo);
#pragma unroll
          for (int x = 0; x < CW; x += 2) fadd2(t[x], t[x + 1], t[x], t[x + 1], lo[x], lo[x + 1]);
        }
        load_vecn<CW>(vl + BN + CW * c, dv);
#pragma unroll
        for (int x = 0; x < CW; x += 2) {
          const int cc = CW * c + x;
          float u0, u1, d0, d1;
          fsub2(u0, u1, t[x], t[x + 1], dv[x], dv[x + 1]);
          fmul2(d0, d1, pv[cc], pv[cc + 1], u0, u1);  // dS^T = P^T (dP^T - delta)
          if constexpr (SPLIT == 3) {
            tf32_split2(d0, d1, t[x], t[x + 1], lo[x], lo[x + 1]);
          } else {
            t[x] = tf32_round_finite(d0);
            t[x + 1] = tf32_round_finite(d1);
          }
        }
        tmem_stn<CW>(dc + CW * c, t);
        if constexpr (SPLIT == 3) tmem_stn<CW>(dc + BN + CW * c, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->ds_full[bi]));
    }
    const int64_t orow = ((int64_t)bh * T + (valid ? row : 0)) * D;
    float* out = grp ? p.out1 : p.out0;
    if (grp == 0 ? !C::DO_DK : !C::DO_DV) {
      // this pass does not produce the group's gradient
    } else if (n == 0) {  // no query of the first segment reaches these keys
      if (valid) {
        for (int d = 0; d < D; ++d) out[orow + d] = 0.0f;
      }
    } else if (ok && warp_wait(B(bars->done), 0, ctl, p.status)) {
      tc_fence_after();
      if constexpr (bwd_wbuf_fits<C>()) {  // coalesced through the warp's buffer
        float* wbuf = reinterpret_cast<float*>(smem_raw + (tiles - smem_u32(smem_raw)) +
                                               NS * C::STAGE + NS * 2 * BN * 4) +
                      (warp - 4 - (grp ? 3 : 0)) * kRowWbufFloats;
        const int r0 = k0 + quad * 32;
        warp_rows_to_global<D>(lb + (grp ? C::TC_DV : C::TC_DK), grp ? 1.0f : p.scale, wbuf,
                               out + ((int64_t)bh * T + r0) * D, max(0, min(32, T - r0)), D,
                               p.accumulate_out != 0);
      } else {
        tmem_row_to_global<D>(lb, grp ? C::TC_DV : C::TC_DK, grp ? 1.0f : p.scale, out + orow,
                              valid, p.accumulate_out != 0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}


// ------------------------------------------------------- 64-row (M = 64) pass
// Head dim 128 in 3xTF32: the hi / lo copies of two stationary 128-column
// operands alone fill the 512 TMEM columns of a 128-row tile.  An M = 64 MMA
// keeps its rows in 16 lanes of each warp's lane quadrant (row r in lane
// 32 * (r / 16) + r % 16, plus 16 in the quadrant's upper half; the A operand
// read from TMEM sits in the same lanes as the accumulator), so a 64-row tile
// gives each stationary operand its own half of the lanes:
//   lower halves: X hi | X lo | 2 x S (two partial sums)
//   upper halves: Y hi | Y lo | 2 x dP (two partial sums, then dS hi | lo) | gradient
//   S = X A_j^T,  dP = Y B_j^T,  dS = P * (dP - delta),  grad += dS A_j
// QSTAT (dQ pass): X = Q, Y = dO, A = K, B = V, grad = dQ, P and delta per row.
// !QSTAT (dK pass): X = K, Y = V, A = Q, B = dO, grad = dK, P and delta per
// column (staged in shared memory by the producer warp).
// P = exp2(S * log2e / sqrt(D) - LSE * log2e) and delta = rowsum(O * dO) are
// per query (flash_attention.cuh:318-326 for dQ, :452-476 for dK).  The row
// warps read both halves with the 16-lane 16x32bx2 shape, so one thread sees
// S and dP of the same element: row 16 * quad + lane % 16, a quarter of the
// step's columns (lane half x row warpgroup).
// S and dP are double-buffered (step j in buffer j % 2), so S_{j+1} and
// dP_{j+1} run on the tensor core while the rows form dS_j.
// Staging in two rings, so the early readers of a step do not wait for its
// late one: ring 1 holds the K-major tiles A_j and B_j (read by S_j and dP_j,
// hi / lo interleaved) and is released as soon as both MMAs complete; ring 2
// holds A_j MN-major (read by grad_j), landed in that layout by TMA and split
// in place, released by grad_j.  In the dK pass every row thread loads the
// LSE and delta of its step's columns itself, one step ahead (the same
// addresses across half a warp: broadcast L2 hits).
// Warps: 0 TMA producer (lane 0 ring 1, lane 1 ring 2), 1 TMEM allocator and
// S issuer, 2, 3, 8, 9 tile preparation (3xTF32 split), 10 gradient issuer,
// 15 dP issuer, 4-7 and 11-14 row warps.
constexpr int kRows64 = 64;
constexpr uint32_t kUpperLanes = 16u << 16;  // TMEM lane offset of a quadrant's upper half

template <int D_, int BN_, int NS1_, int NS2_>
struct Half64Cfg {
  static constexpr int D = D_, BN = BN_, NS1 = NS1_, NS2 = NS2_, NSB = 2;
  static constexpr uint32_t TILE = (uint32_t)BN_ * D_ * 4u;
  static constexpr uint32_t CH = (uint32_t)BN_ * 128u;  // one 32-column chunk of BN rows
  static constexpr uint32_t KCH = 2u * CH;              // interleaved hi | lo chunk stride
  // ring 1 slot: A K-major (hi | lo interleaved) | B K-major (the same)
  static constexpr uint32_t OFF_A = 0, OFF_B = 2u * TILE, SLOT1 = 4u * TILE;
  // ring 2 slot: A MN-major raw | its low parts
  static constexpr uint32_t SLOT2 = 2u * TILE, RING2 = NS1 * SLOT1, TILE_BYTES = RING2 + NS2 * SLOT2;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t SB = 2u * BN_;  // one S / dP buffer
  static constexpr uint32_t TC_X = 0, TC_S = 2u * D_;                           // lower halves
  static constexpr uint32_t TC_Y = 0, TC_DP = 2u * D_, TC_G = 2u * D_ + NSB * SB;  // upper halves
  static constexpr int CT = BN_ / 4;  // score columns per row thread per step
  static_assert(D_ == 128, "the 64-row pass is the head-dim-128 3xTF32 path");
  static_assert(CT == 8 || CT == 16, "16x32bx2 access width");
  static_assert(TC_G + D_ <= TMEM_COLS && TC_S + NSB * SB <= TMEM_COLS, "TMEM budget");
};

template <int NS1, int NS2>
struct M64Bars {
  uint64_t full_a[NS1], full_b[NS1], ready_a[NS1], ready_b[NS1], empty1[NS1];
  uint64_t full_c[NS2], ready_c[NS2], empty2[NS2];
  uint64_t s_full[2], s_free[2], dp_full[2], ds_full[2], dqd[2];
  uint64_t rows_ready, done, mma_final, mma_final2, mma_final3;
  CtaCtl ctl;
};

template <class C>
constexpr size_t m64_smem_bytes() {
  constexpr size_t b = 1024 + 1024 + (size_t)C::TILE_BYTES;
  static_assert(sizeof(M64Bars<C::NS1, C::NS2>) <= 1024, "barrier block");
  static_assert(b <= 227 * 1024, "shared memory budget");
  return b;
}

template <class C, bool QSTAT>
__global__ void __launch_bounds__(kBwdThreads, 1)
    fa2_bwd_m64_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmAm, const BwdParams p) {
  constexpr int D = C::D, BN = C::BN, NS1 = C::NS1, NS2 = C::NS2, CT = C::CT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (status_raised(p.status)) return;
  auto* bars = reinterpret_cast<M64Bars<NS1, NS2>*>(smem_raw);
  const uint32_t tiles = (smem_u32(smem_raw) + (uint32_t)sizeof(M64Bars<NS1, NS2>) + 1023u) & ~1023u;
  CtaCtl* ctl = &bars->ctl;
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  int tile, bh;  // head-major; dQ: late (heavy) query tiles first
  cta_tile(p.n_tiles, p.bh_total, p.head_group, QSTAT, tile, bh);
  const int b = bh / p.H, h = bh % p.H;
  const int r0 = tile * kRows64, T = p.T;
  // streamed tiles [j0, j0 + n) of this launch's segment
  int j0, n;
  if constexpr (QSTAT) {
    const int last_row = min(r0 + kRows64 - 1, T - 1);
    j0 = p.seg_lo / BN;
    n = max(0, min(p.causal ? last_row / BN + 1 : (T + BN - 1) / BN, (p.seg_hi + BN - 1) / BN) -
                   j0);
  } else {
    j0 = max(p.causal ? r0 / BN : 0, p.seg_lo / BN);
    n = max(0, min((T + BN - 1) / BN, (p.seg_hi + BN - 1) / BN) - j0);
  }
  if (n == 0) {  // nothing of the segment reaches these rows (uniform exit)
    if (!p.accumulate_out && threadIdx.x < kRows64 && r0 + (int)threadIdx.x < T) {
      float* o = p.out0 + ((int64_t)bh * T + r0 + threadIdx.x) * D;
      for (int d = 0; d < D; ++d) o[d] = 0.0f;
    }
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS1; ++s) {
      mbar_init(B(bars->full_a[s]), 1);
      mbar_init(B(bars->full_b[s]), 1);
      mbar_init(B(bars->ready_a[s]), kPrepWarps);
      mbar_init(B(bars->ready_b[s]), kPrepWarps);
      mbar_init(B(bars->empty1[s]), 2);  // S_j and dP_j
    }
    for (int s = 0; s < NS2; ++s) {
      mbar_init(B(bars->full_c[s]), 1);
      mbar_init(B(bars->ready_c[s]), kPrepWarps);
      mbar_init(B(bars->empty2[s]), 1);  // grad_j
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(B(bars->s_full[i]), 1);
      mbar_init(B(bars->s_free[i]), 8);
      mbar_init(B(bars->dp_full[i]), 1);
      mbar_init(B(bars->ds_full[i]), 8);
      mbar_init(B(bars->dqd[i]), 1);
    }
    mbar_init(B(bars->rows_ready), 8);
    mbar_init(B(bars->done), 1);
    mbar_init(B(bars->mma_final), 1);
    mbar_init(B(bars->mma_final2), 1);
    mbar_init(B(bars->mma_final3), 1);
    bars->ctl.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  auto slot1 = [&](int i) { return tiles + (uint32_t)(i % NS1) * C::SLOT1; };
  auto slot2 = [&](int i) { return tiles + C::RING2 + (uint32_t)(i % NS2) * C::SLOT2; };
  constexpr uint32_t idS2 = idesc_tf32(64, 2 * BN, false, false);  // [hi | lo] rows (kil)
  constexpr uint32_t idS = idesc_tf32(64, BN, false, false);
  constexpr uint32_t idG = idesc_tf32(64, D, false, true);

  if (warp == 0) {
    // Lane 0: ring 1 (K-major A_j, B_j; B first); lane 1: ring 2 (MN-major A_j).
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int last = -1;
      for (int i = 0; i < n; ++i) {
        const int j = j0 + i, s = i % NS1, r = i / NS1;
        if (r > 0 && !mbar_wait(B(bars->empty1[s]), (r - 1) & 1, ctl, p.status)) break;
        const uint32_t st = slot1(i);
        mbar_arrive_expect_tx(B(bars->full_b[s]), C::TILE);
        tma_load_tile<false, D>(st + C::OFF_B, &tmB, B(bars->full_b[s]), j * BN, h, b, C::KCH);
        mbar_arrive_expect_tx(B(bars->full_a[s]), C::TILE);
        tma_load_tile<false, D>(st + C::OFF_A, &tmA, B(bars->full_a[s]), j * BN, h, b, C::KCH);
        last = i;
      }
      if (ctl->abort) {  // drain this lane's copies in flight
        for (int i = max(0, last - NS1 + 1); i <= last; ++i) {
          mbar_drain(B(bars->full_b[i % NS1]), (i / NS1) & 1);
          mbar_drain(B(bars->full_a[i % NS1]), (i / NS1) & 1);
        }
      }
    } else if (lane == 1) {
      tma_prefetch_desc(&tmAm);
      int last = -1;
      for (int i = 0; i < n; ++i) {
        const int j = j0 + i, s = i % NS2, r = i / NS2;
        if (r > 0 && !mbar_wait(B(bars->empty2[s]), (r - 1) & 1, ctl, p.status)) break;
        mbar_arrive_expect_tx(B(bars->full_c[s]), C::TILE);
        tma_load_5d(slot2(i), &tmAm, B(bars->full_c[s]), 0, j * BN, 0, h, b);
        last = i;
      }
      if (ctl->abort) {
        for (int i = max(0, last - NS2 + 1); i <= last; ++i)
          mbar_drain(B(bars->full_c[i % NS2]), (i / NS2) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // S_j = X A_j^T (lower halves) into buffer j % 2 once the rows hold
    // S_{j-2} in registers.
    if (lane == 0) {
      bool ok = mbar_wait(B(bars->rows_ready), 0, ctl, p.status);
      for (int j = 0; ok && j < n; ++j) {
        const int bj = j & 1;
        if (j >= 2 && !(ok = mbar_wait(B(bars->s_free[bj]), ((j - 2) >> 1) & 1, ctl, p.status)))
          break;
        if (!(ok = mbar_wait(B(bars->ready_a[j % NS1]), (j / NS1) & 1, ctl, p.status))) break;
        tc_fence_after();
        mma_chain_kil<D, C::KCH>(tmem + C::TC_S + bj * C::SB, tmem + C::TC_X, tmem + C::TC_X + D,
                                 sdesc_kmajor(slot1(j) + C::OFF_A), idS2, idS);
        umma_commit(B(bars->s_full[bj]));
        umma_commit(B(bars->empty1[j % NS1]));  // A_j K-major read
      }
      umma_commit(B(bars->mma_final));
      mbar_drain(B(bars->mma_final), 0);
    }
    __syncwarp();
  } else if (warp == kIssuer2Warp) {
    // grad += dS_j A_j (upper halves) once the rows formed dS_j in buffer j % 2.
    if (lane == 0) {
      const uint32_t up = tmem + kUpperLanes;
      bool ok = true;
      for (int j = 0; ok && j < n; ++j) {
        const int bj = j & 1;
        if (!(ok = mbar_wait(B(bars->ds_full[bj]), (j >> 1) & 1, ctl, p.status))) break;
        if (!(ok = mbar_wait(B(bars->ready_c[j % NS2]), (j / NS2) & 1, ctl, p.status))) break;
        tc_fence_after();
        const uint32_t db = up + C::TC_DP + bj * C::SB;
        mma_chain<3, BN, true, BN, C::TILE>(up + C::TC_G, db, db + BN,
                                            sdesc_mnmajor(slot2(j), BN * 128), idG, j > 0);
        umma_commit(B(bars->empty2[j % NS2]));  // A_j MN-major read
        umma_commit(B(bars->dqd[bj]));          // dS_j read: dP_{j+2} may overwrite it
      }
      if (ok) umma_commit(B(bars->done));
      umma_commit(B(bars->mma_final2));
      mbar_drain(B(bars->mma_final2), 0);
    }
    __syncwarp();
  } else if (warp == kIssuer3Warp) {
    // dP_j = Y B_j^T (upper halves) into buffer j % 2 once grad_{j-2} has read
    // dS_{j-2} from it.
    if (lane == 0) {
      const uint32_t up = tmem + kUpperLanes;
      bool ok = mbar_wait(B(bars->rows_ready), 0, ctl, p.status);
      for (int j = 0; ok && j < n; ++j) {
        const int bj = j & 1;
        if (j >= 2 && !(ok = mbar_wait(B(bars->dqd[bj]), ((j - 2) >> 1) & 1, ctl, p.status)))
          break;
        if (!(ok = mbar_wait(B(bars->ready_b[j % NS1]), (j / NS1) & 1, ctl, p.status))) break;
        tc_fence_after();
        mma_chain_kil<D, C::KCH>(up + C::TC_DP + bj * C::SB, up + C::TC_Y, up + C::TC_Y + D,
                                 sdesc_kmajor(slot1(j) + C::OFF_B), idS2, idS);
        umma_commit(B(bars->dp_full[bj]));
        umma_commit(B(bars->empty1[j % NS1]));  // B_j read
      }
      umma_commit(B(bars->mma_final3));
      mbar_drain(B(bars->mma_final3), 0);
    }
    __syncwarp();
  } else if (is_prep_warp(warp)) {
    // Per step: B_j, then A_j K-major (both interleaved hi | lo), then A_j
    // MN-major (split in place), each released to its readers when done.
    const uint32_t tid = prep_tid();
    for (int i = 0; i < n; ++i) {
      const int s = i % NS1, r = i / NS1, s2 = i % NS2, r2 = i / NS2;
      if (!warp_wait(B(bars->full_b[s]), r & 1, ctl, p.status)) break;
      split_tile_smem_il<C::TILE, kSplitThreads, C::CH>(slot1(i) + C::OFF_B, tid);
      fence_proxy_async_smem();
      warp_arrive(B(bars->ready_b[s]));
      if (!warp_wait(B(bars->full_a[s]), r & 1, ctl, p.status)) break;
      split_tile_smem_il<C::TILE, kSplitThreads, C::CH>(slot1(i) + C::OFF_A, tid);
      fence_proxy_async_smem();
      warp_arrive(B(bars->ready_a[s]));
      if (!warp_wait(B(bars->full_c[s2]), r2 & 1, ctl, p.status)) break;
      split_tile_smem<C::TILE, kSplitThreads>(slot2(i), slot2(i) + C::TILE, tid);
      fence_proxy_async_smem();
      warp_arrive(B(bars->ready_c[s2]));
    }
  } else {
    // Row warps 4-7 (group 0) and 11-14 (group 1) of lane quadrant q = warp % 4.
    const int quad = warp & 3;
    const int grp = warp >= kBwdRowWarp1 ? 1 : 0;
    const int hl = lane >> 4;                 // lane half: which columns of a 16x32bx2 access
    const int row = r0 + 16 * quad + (lane & 15);
    const bool valid = row < T;
    const uint32_t qlo = tmem + ((32u * quad) << 16);  // the quadrant's lower half
    const uint32_t qup = qlo + kUpperLanes;            // and upper half
    // Stationary rows into TMEM (32x32b: each thread its own lane): lanes
    // 0-15 X's row into the lower half, lanes 16-31 Y's row into the upper
    // half; group g writes head-dim columns [g D/2, (g + 1) D/2), hi and lo.
    {
      const Ptr4& src = hl ? p.st1 : p.st0;
      const float* rp = src.row(b, h, valid ? row : 0);
      const bool vr = src.s3 == 1 && ((reinterpret_cast<uintptr_t>(rp) & 15u) == 0);
      const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        const int col = grp * (D / 2) + 32 * c;
        float x[32], lo[32];
        load_row32(src, rp, col, valid, vr, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float hi;
          tf32_split(x[i], hi, lo[i]);
          x[i] = hi;
        }
        tmem_st32(lb + C::TC_X + col, x);  // TC_X == TC_Y: the lane picks the operand
        tmem_st32(lb + C::TC_X + D + col, lo);
      }
      tmem_wait_st();
    }
    float l2 = 0.0f, dl = 0.0f;  // per-row LSE * log2e and delta (dQ pass)
    if constexpr (QSTAT) {
      if (valid) {
        l2 = __ldg(p.lse + b * p.l0 + h * p.l1 + (int64_t)row * p.l2) * kLog2e;
        dl = __ldg(p.delta + (int64_t)bh * T + row);
      }
    }
    tc_fence_before();
    warp_arrive(B(bars->rows_ready));
    const int cs = grp * (BN / 2) + hl * CT;  // this thread's first column of a step
    // dK pass: LSE and delta of this thread's columns, loaded one step ahead
    const float* lse_bh = p.lse + b * p.l0 + h * p.l1;
    const float* del_bh = p.delta + (int64_t)bh * T;
    float nl[CT], nd[CT];
    auto fetch_cols = [&](int j) {
#pragma unroll
      for (int x = 0; x < CT; ++x) {
        const int q = (j0 + j) * BN + cs + x;
        const bool in = !QSTAT && j < n && q < T;
        nl[x] = in ? ldg_nc_early(lse_bh + (int64_t)q * p.l2) : 0.0f;
        nd[x] = in ? ldg_nc_early(del_bh + q) : 0.0f;
      }
    };
    if constexpr (!QSTAT) fetch_cols(0);
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int col0 = (j0 + j) * BN + cs;  // its key (dQ) or query (dK) index
      const int bj = j & 1;
      const uint32_t par = (uint32_t)(j >> 1) & 1u;
      float lv[CT], dv[CT];
      if constexpr (!QSTAT) {  // this step's -LSE * log2e and delta, per column
#pragma unroll
        for (int x = 0; x < CT; ++x) {
          lv[x] = nl[x] * -kLog2e;
          dv[x] = nd[x];
        }
        fetch_cols(j + 1);
      } else {
#pragma unroll
        for (int x = 0; x < CT; ++x) {
          lv[x] = -l2;
          dv[x] = dl;
        }
      }
      if (!(ok = warp_wait(B(bars->s_full[bj]), par, ctl, p.status))) break;
      tc_fence_after();
      float pv[CT];
      {
        const uint32_t sb = qlo + C::TC_S + bj * C::SB + grp * (BN / 2);
        float t1[CT];
        tmem_ld_16x32bx2<CT>(sb, pv);
        tmem_ld_16x32bx2<CT>(sb + BN, t1);
#pragma unroll
        for (int x = 0; x < CT; x += 2) fadd2(pv[x], pv[x + 1], pv[x], pv[x + 1], t1[x], t1[x + 1]);
      }
      tc_fence_before();
      warp_arrive(B(bars->s_free[bj]));  // S_j read: S_{j+2} may overwrite it
#pragma unroll
      for (int x = 0; x < CT; x += 2) {
        float a0, a1;
        ffma2(a0, a1, pv[x], pv[x + 1], p.scale_log2, p.scale_log2, lv[x], lv[x + 1]);
        pv[x] = ex2_approx(a0);
        pv[x + 1] = ex2_approx(a1);
      }
      const bool need_mask =
          !valid || (col0 + CT > T) ||
          (p.causal && (QSTAT ? (col0 + CT - 1 > row) : (col0 < row)));
      if (need_mask) {
#pragma unroll
        for (int x = 0; x < CT; ++x) {
          const int c = col0 + x;
          const bool keep = valid && c < T && (!p.causal || (QSTAT ? c <= row : c >= row));
          pv[x] = keep ? pv[x] : 0.0f;
        }
      }
      if (!(ok = warp_wait(B(bars->dp_full[bj]), par, ctl, p.status))) break;
      tc_fence_after();
      const uint32_t dpb = qup + C::TC_DP + bj * C::SB + grp * (BN / 2);
      float d0[CT], d1[CT];
      tmem_ld_16x32bx2<CT>(dpb, d0);
      tmem_ld_16x32bx2<CT>(dpb + BN, d1);
#pragma unroll
      for (int x = 0; x < CT; x += 2) {
        float u0, u1, s0, s1;
        fadd2(u0, u1, d0[x], d0[x + 1], d1[x], d1[x + 1]);        // dP from its partial sums
        fsub2(u0, u1, u0, u1, dv[x], dv[x + 1]);
        fmul2(s0, s1, pv[x], pv[x + 1], u0, u1);                  // dS = P (dP - delta)
        tf32_split2(s0, s1, d0[x], d0[x + 1], d1[x], d1[x + 1]);  // hi | lo
      }
      tmem_st_16x32bx2<CT>(dpb, d0);
      tmem_st_16x32bx2<CT>(dpb + BN, d1);
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->ds_full[bj]));
    }
    if (ok && warp_wait(B(bars->done), 0, ctl, p.status)) {
      tc_fence_after();
      // gradient rows (upper halves): group g, lane half -> columns [g D/2 + 32 hl, +32)
      float v[32];
      tmem_ld_16x32bx2<32>(qup + C::TC_G + grp * (D / 2), v);
      if (valid) {
        float4* d4 =
            reinterpret_cast<float4*>(p.out0 + ((int64_t)bh * T + row) * D + grp * (D / 2) + 32 * hl);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 a = make_float4(v[4 * i] * p.scale, v[4 * i + 1] * p.scale,
                                 v[4 * i + 2] * p.scale, v[4 * i + 3] * p.scale);
          if (p.accumulate_out) {
            const float4 o = d4[i];
            a = make_float4(o.x + a.x, o.y + a.y, o.z + a.z, o.w + a.w);
          }
          d4[i] = a;
        }
      }
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
int run_dq(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, Strided4 g, const float* lse,
           const int64_t ls[3], const float* delta, float* dq, const DeviceInfo& dev,
           cudaStream_t st) {
  static unsigned long long attr_done = 0;
  CUtensorMap tk, tv;
  // K-major copies of interleaved (KIL) tiles load chunk by chunk, every other
  // tile in one copy
  int rc = C::KILA ? make_tmap_bhtd(&tk, k, pr, C::BN) : make_tmap_bhtd_whole(&tk, k, pr, C::BN);
  if (rc == CT_OK)
    rc = C::KILB ? make_tmap_bhtd(&tv, v, pr, C::BN) : make_tmap_bhtd_whole(&tv, v, pr, C::BN);
  if (rc != CT_OK) return rc;
  const size_t smem = bwd_smem_bytes_wbuf<C>();
  rc = ensure_smem_attr(fa2_bwd_dq_tc_kernel<C>, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  BwdParams p = make_params(pr, q, g, lse, ls, delta, dq, nullptr, dev);
  const int64_t grid = (int64_t)p.n_tiles * p.bh_total;
  for (int64_t s0 = 0; s0 < pr.T; s0 += kSegLen) {  // one launch per key segment
    p.seg_lo = (int)s0;
    p.seg_hi = (int)std::min<int64_t>(s0 + kSegLen, pr.T);
    p.accumulate_out = s0 > 0;
    fa2_bwd_dq_tc_kernel<C><<<(unsigned)grid, kBwdThreads, smem, st>>>(tk, tv, p);
    rc = check_launch();
    if (rc != CT_OK) return rc;
  }
  return CT_OK;
}

template <class C>
int run_dkdv(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
             const float* lse, const int64_t ls[3], const float* delta, float* dk, float* dv,
             const DeviceInfo& dev, cudaStream_t st) {
  static unsigned long long attr_done = 0;
  CUtensorMap tq, tg;
  int rc = C::KILA ? make_tmap_bhtd(&tq, q, pr, C::BN) : make_tmap_bhtd_whole(&tq, q, pr, C::BN);
  if (rc == CT_OK)
    rc = C::KILB ? make_tmap_bhtd(&tg, g, pr, C::BN)
                 : make_tmap_bhtd_whole(&tg, g, pr, C::BN, C::BMN);
  if (rc != CT_OK) return rc;
  size_t smem = bwd_smem_bytes<C>();
  if constexpr (bwd_wbuf_fits<C>()) smem = bwd_smem_bytes_wbuf<C>();
  rc = ensure_smem_attr(fa2_bwd_dkdv_tc_kernel<C>, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  BwdParams p = make_params(pr, k, v, lse, ls, delta, dk, dv, dev);
  const int64_t grid = (int64_t)p.n_tiles * p.bh_total;
  for (int64_t s0 = 0; s0 < pr.T; s0 += kSegLen) {  // one launch per query segment
    p.seg_lo = (int)s0;
    p.seg_hi = (int)std::min<int64_t>(s0 + kSegLen, pr.T);
    p.accumulate_out = s0 > 0;
    fa2_bwd_dkdv_tc_kernel<C><<<(unsigned)grid, kBwdThreads, smem, st>>>(tq, tg, p);
    rc = check_launch();
    if (rc != CT_OK) return rc;
  }
  return CT_OK;
}

// The 64-row pass: streamed tiles a (A: S and the gradient) and bb (B: dP),
// stationary x (X) and y (Y); the gradient into grad.
template <class C, bool QSTAT>
int run_m64(const Fa2Problem& pr, Strided4 a, Strided4 bb, Strided4 x, Strided4 y,
            const float* lse, const int64_t ls[3], const float* delta, float* grad,
            const DeviceInfo& dev, cudaStream_t st) {
  static unsigned long long attr_done = 0;
  // K-major tiles interleave hi / lo and load chunk by chunk; A's MN-major
  // copy loads whole
  CUtensorMap ta, tb, tam;
  int rc = make_tmap_bhtd(&ta, a, pr, C::BN);
  if (rc == CT_OK) rc = make_tmap_bhtd(&tb, bb, pr, C::BN);
  if (rc == CT_OK) rc = make_tmap_bhtd_whole(&tam, a, pr, C::BN, true);
  if (rc != CT_OK) return rc;
  const size_t smem = m64_smem_bytes<C>();
  rc = ensure_smem_attr(fa2_bwd_m64_tc_kernel<C, QSTAT>, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  BwdParams p = make_params(pr, x, y, lse, ls, delta, grad, nullptr, dev);
  p.n_tiles = (int)((pr.T + kRows64 - 1) / kRows64);
  const int64_t grid = (int64_t)p.n_tiles * p.bh_total;
  for (int64_t s0 = 0; s0 < pr.T; s0 += kSegLen) {  // one launch per segment
    p.seg_lo = (int)s0;
    p.seg_hi = (int)std::min<int64_t>(s0 + kSegLen, pr.T);
    p.accumulate_out = s0 > 0;
    fa2_bwd_m64_tc_kernel<C, QSTAT><<<(unsigned)grid, kBwdThreads, smem, st>>>(ta, tb, tam, p);
    rc = check_launch();
    if (rc != CT_OK) return rc;
  }
  return CT_OK;
}

}  // namespace

bool fa2_bwd_tc_supported(const Fa2Problem& p) {
  // D = 128 in 3xTF32 runs the 64-row pass (the hi / lo copies of two
  // stationary 128-column operands fill the TMEM of a 128-row tile).
  return (p.D == 32 || p.D == 64 || p.D == 128) &&
         (p.precision == CT_PRECISION_3XTF32 || p.precision == CT_PRECISION_TF32) &&
         p.T < (1ll << 31) && ((p.T + kRows - 1) / kRows) * p.B * p.H < (1ll << 31);
}

int launch_fa2_bwd_dq_tc(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
                         const float* lse, const int64_t ls[3], const float* delta, float* dq,
                         const DeviceInfo& dev, cudaStream_t st) {
  if (!fa2_tma_ok(k) || !fa2_tma_ok(v)) return CT_ERR_UNSUPPORTED_LAYOUT;
  const bool split = pr.precision == CT_PRECISION_3XTF32;
  if (fa2_bwd_dq_persist_supported(pr))  // TF32, D = 64: persistent CTAs
    return launch_fa2_bwd_dq_persist(pr, q, k, v, g, lse, ls, delta, dq, dev, st);
  if (pr.D == 64)
    return split ? run_dq<DqCfg<64, 64, 3, 2>>(pr, q, k, v, g, lse, ls, delta, dq, dev, st)
                 : run_dq<DqCfg<64, 64, 1, 4, 2>>(pr, q, k, v, g, lse, ls, delta, dq, dev, st);
  if (pr.D == 32)
    return split ? run_dq<DqCfg<32, 64, 3, 4>>(pr, q, k, v, g, lse, ls, delta, dq, dev, st)
                 : run_dq<DqCfg<32, 128, 1, 4>>(pr, q, k, v, g, lse, ls, delta, dq, dev, st);
  if (pr.D == 128)
    return split ? run_m64<Half64Cfg<128, 32, 2, 2>, true>(pr, k, v, q, g, lse, ls, delta, dq, dev, st)
                 : run_dq<DqCfg<128, 64, 1, 2>>(pr, q, k, v, g, lse, ls, delta, dq, dev, st);
  return CT_ERR_UNSUPPORTED_HEAD_DIM;
}

int launch_fa2_bwd_dkdv_tc(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, Strided4 g,
                           const float* lse, const int64_t ls[3], const float* delta, float* dk,
                           float* dv, const DeviceInfo& dev, cudaStream_t st) {
  if (!fa2_tma_ok(q) || !fa2_tma_ok(g)) return CT_ERR_UNSUPPORTED_LAYOUT;
  const bool split = pr.precision == CT_PRECISION_3XTF32;
  if (fa2_bwd_pair_supported(pr))  // TF32, D = 64: 256-key tiles on CTA pairs
    return launch_fa2_bwd_dkdv_pair(pr, q, k, v, g, lse, ls, delta, dk, dv, dev, st);
  if (pr.D == 64)
    return split ? run_dkdv<DkvCfg<64, 32, 3, 3>>(pr, q, k, v, g, lse, ls, delta, dk, dv, dev, st)
                 : run_dkdv<DkvCfg<64, 64, 1, 3, 2>>(pr, q, k, v, g, lse, ls, delta, dk, dv, dev, st);
  if (pr.D == 32)
    return split ? run_dkdv<DkvCfg<32, 64, 3, 3>>(pr, q, k, v, g, lse, ls, delta, dk, dv, dev, st)
                 : run_dkdv<DkvCfg<32, 128, 1, 3>>(pr, q, k, v, g, lse, ls, delta, dk, dv, dev, st);
  if (pr.D == 128 && !split) {  // dV, then dK: one pass does not fit TMEM
    const int rc =
        run_dkdv<DkvCfg<128, 32, 1, 6, 2, kDkvOnlyDv>>(pr, q, k, v, g, lse, ls, delta, dk, dv, dev, st);
    if (rc != CT_OK) return rc;
    return run_dkdv<DkvCfg<128, 32, 1, 4, 2, kDkvOnlyDk>>(pr, q, k, v, g, lse, ls, delta, dk, dv,
                                                          dev, st);
  }
  if (pr.D == 128) {  // 3xTF32: dV on 128-row tiles, then dK on 64-row tiles (K, V in lane halves)
    const int rc =
        run_dkdv<DkvCfg<128, 32, 3, 3, 2, kDkvOnlyDv>>(pr, q, k, v, g, lse, ls, delta, dk, dv, dev, st);
    if (rc != CT_OK) return rc;
    return run_m64<Half64Cfg<128, 32, 2, 2>, false>(pr, q, g, k, v, lse, ls, delta, dk, dev, st);
  }
  return CT_ERR_UNSUPPORTED_HEAD_DIM;
}

}  // namespace ct
