// fa2_fwd_tc.cu -- FlashAttention-2 forward on the sm_100a tensor cores.
//
// Computes what flash_attention_fwd_kernel computes
// (Transformer_kernels/flash_attention.cuh:27-170): S = Q K^T / sqrt(D) with
// the mask (!causal || q >= k) && q < T && k < T (:117), an online softmax
// (:124-141), O = sum P V rescaled (:150), then O /= l and L = m + ln(l)
// (:163, :167).
//
// Per CTA: one (batch, head) and 128 query rows.  Warp roles (15 warps):
//   warp 0      TMA producer of K/V tiles (NS-stage ring)
//   warp 1      TMEM allocator + issuer of S = Q K^T (one thread)
//   warps 2,3,8,9  TF32 hi/lo split (SPLIT == 3) or rounding (SPLIT == 1) of
//               each landed K/V tile
//   warps 4-7, 11-14  two row warpgroups: thread r of a group <-> query row r
//               <-> TMEM lane r; each group takes half of a step's score
//               columns (softmax with the pair's maxima exchanged, O
//               correction and epilogue of half of O); group 0 loads Q
//   warp 10     issuer of O += P V (one thread)
// K tiles use the K-major tile layout, V tiles the MN-major one.
// TMEM columns: Q (hi[,lo]) | O | two or three S/P buffers (S overwritten by P
// hi, then P lo).  S_{j+1} (and S_{j+2} with three buffers) runs on the tensor
// core while the row warps turn S_j into P_j.  O is rescaled only when a row
// maximum grows by more than 2^8 (exact: l and O always share the stale
// maximum).  3xTF32 forms hi*hi and hi*lo of S, and of P V, with one MMA
// (mma_chain_kil, mma_chain_mn2).
// TF32 mode at head dims 32 and 64 runs fa2_fwd_pair_kernel instead: two
// query tiles per CTA, one row warpgroup and one issuing thread per tile
// (see there).
#include "fa2_common.cuh"

namespace ct {
namespace {

using namespace fa2;

// NSB S/P buffers in TMEM: S_{j+NSB-1} is computed while the row warps turn
// S_j into P_j and the tensor core runs O += P_{j-1} V_{j-1}.
template <int D_, int BN_, int SPLIT_, int NS_, int NSB_ = 2>
struct FwdCfg {
  static constexpr int D = D_, BN = BN_, SPLIT = SPLIT_, NS = NS_, NSB = NSB_;
  static constexpr int NCOPY = SPLIT == 3 ? 2 : 1;
  static constexpr uint32_t TILE = (uint32_t)BN * D * 4u;  // one K or V tile
  // 3xTF32: the K tile interleaves each 32-column chunk of BN raw rows with its
  // BN low-part rows, so S lands as two partial sums in the S buffer's 2*BN
  // columns (mma_chain_kil); the row warps add them.
  static constexpr bool KIL = SPLIT == 3;
  static constexpr uint32_t KCH = (KIL ? 2u : 1u) * BN * 128u;  // K chunk stride
  static constexpr uint32_t STAGE = 2u * NCOPY * TILE;
  static constexpr uint32_t OFF_K = 0, OFF_V = NCOPY * TILE;  // lo copy at +TILE
  static constexpr uint32_t TC_Q = 0;
  // 3xTF32 with room in TMEM: O += P V from one N = 2D MMA on [V_hi | V_lo]
  // and one N = D MMA per k-step (mma_chain_mn2); O then spans 2D columns
  // whose halves the epilogue adds.
  static constexpr bool PVM = SPLIT == 3 && NCOPY * D + 2 * D + NSB * NCOPY * BN <= 512;
  static constexpr uint32_t OW = PVM ? 2 * D : D;  // O accumulator columns
  static constexpr uint32_t TC_O = NCOPY * D;
  static constexpr uint32_t TC_S = TC_O + OW;
  static constexpr uint32_t SBUF = NCOPY * BN;
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(TC_S + NSB * SBUF <= TMEM_COLS, "TMEM budget");
  static_assert(NSB == 2 || NSB == 3, "S buffering");
  static_assert(NS >= 3 && NS >= NSB, "K_{j+NSB} is needed before V_j is released");
  static_assert(D % 32 == 0 && BN % 32 == 0, "tile shape");
};

// Two row warpgroups, warps 4-7 and 11-14 (15 warps); warps 0-3 and 8-10 keep
// their roles.
constexpr int kFwdThreads = 480;
constexpr int kFwdRowWarp1 = 11;

template <int NS>
struct FwdBars {  // (p_full: one per S/P buffer, at most 3)
  // full_*: TMA landed; ready_*: split or rounded; empty_*: free again.  K and V
  // keep separate barriers: K_j is released when S_j is done, well before V_j,
  // which gives the producer more lead on the next K tiles.
  uint64_t full_k[NS], full_v[NS], ready_k[NS], ready_v[NS], empty_k[NS], empty_v[NS];
  // The row warps learn that S_j is done from empty_k of its stage and that
  // O += P_j V_j is done from empty_v (both complete exactly then); a stage's
  // barrier cannot run a phase ahead of the row warps, whose P feeds it.
  uint64_t p_full[3], q_ready, mma_final, mma_final_pv;
  CtaCtl ctl;
  // The two row warps of a TMEM lane quarter (one per row group) exchange each
  // row's partial maximum (two slots, alternating by step) and, at the end,
  // its partial sum; xchg / xfin (one arrival per warp) tell each warp that its
  // partner's value is in place (bounded waits, unlike a named barrier).
  uint64_t xchg[4][2], xfin[4];
  float xmax[2][2][kRows];
  float xsum[2][kRows];
};

struct FwdParams {
  Ptr4 q;
  float* o;
  float* lse;
  int H, T, n_qt, bh_total, head_group;
  int causal;
  float scale_log2;  // log2(e) / sqrt(D)
  uint32_t* status;
};

template <class C>
constexpr size_t fwd_smem_bytes() {
  constexpr size_t head = (sizeof(FwdBars<C::NS>) + 1023) / 1024 * 1024 + 1024;
  static_assert(head + (size_t)C::NS * C::STAGE <= 227 * 1024, "shared memory budget");
  return head + (size_t)C::NS * C::STAGE;
}

template <class C>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fa2_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  constexpr int D = C::D, BN = C::BN, NS = C::NS, SPLIT = C::SPLIT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (status_raised(p.status)) return;
  auto* bars = reinterpret_cast<FwdBars<NS>*>(smem_raw);
  const uint32_t tiles = (smem_u32(smem_raw) + (uint32_t)sizeof(FwdBars<NS>) + 1023u) & ~1023u;
  CtaCtl* ctl = &bars->ctl;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // Head-major order (L2 reuse of K/V), last query tiles of a head first.
  int qt, bh;
  cta_tile(p.n_qt, p.bh_total, p.head_group, true, qt, bh);
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = qt * kRows;
  const int T = p.T;
  const int last_row = min(q0 + kRows - 1, T - 1);
  const int n_kv = p.causal ? last_row / BN + 1 : (T + BN - 1) / BN;

  auto B = [&](const uint64_t& x) { return smem_u32(&x); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(B(bars->full_k[s]), 1);
      mbar_init(B(bars->full_v[s]), 1);
      mbar_init(B(bars->ready_k[s]), kPrepWarps);
      mbar_init(B(bars->ready_v[s]), kPrepWarps);
      mbar_init(B(bars->empty_k[s]), 1);
      mbar_init(B(bars->empty_v[s]), 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(B(bars->p_full[i]), 8);  // row warps
    }
    mbar_init(B(bars->q_ready), 4);  // row group 0's warps
    for (int i = 0; i < 4; ++i) {
      mbar_init(B(bars->xchg[i][0]), 2);  // the two warps of a lane quarter
      mbar_init(B(bars->xchg[i][1]), 2);
      mbar_init(B(bars->xfin[i]), 2);
    }
    mbar_init(B(bars->mma_final), 1);
    mbar_init(B(bars->mma_final_pv), 1);
    ctl->abort = 0;
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int last_k[NS], last_v[NS];
      for (int s = 0; s < NS; ++s) last_k[s] = last_v[s] = -1;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % NS, r = j / NS;
        const uint32_t st = tiles + s * C::STAGE;
        if (r > 0 && !mbar_wait(B(bars->empty_k[s]), (r - 1) & 1, ctl, p.status)) break;
        mbar_arrive_expect_tx(B(bars->full_k[s]), C::TILE);
        tma_load_tile<!C::KIL, D>(st + C::OFF_K, &tmK, B(bars->full_k[s]), j * BN, h, b, C::KCH);
        last_k[s] = r;
        if (r > 0 && !mbar_wait(B(bars->empty_v[s]), (r - 1) & 1, ctl, p.status)) break;
        mbar_arrive_expect_tx(B(bars->full_v[s]), C::TILE);
        tma_load_tile<true, D>(st + C::OFF_V, &tmV, B(bars->full_v[s]), j * BN, h, b, BN * 128u);
        last_v[s] = r;
      }
      if (ctl->abort) {  // let every issued copy land before the CTA exits
        for (int s = 0; s < NS; ++s) {
          if (last_k[s] >= 0) mbar_drain(B(bars->full_k[s]), last_k[s] & 1);
          if (last_v[s] >= 0) mbar_drain(B(bars->full_v[s]), last_v[s] & 1);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------ Q.K^T MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_tf32(128, BN, false, false);
      constexpr uint32_t idS2 = idesc_tf32(128, 2 * BN, false, false);  // [hi | lo] rows (KIL)
      const uint64_t kd0 = sdesc_kmajor(tiles + C::OFF_K);  // stage-0 descriptor
      // S_j = Q K_j^T into S buffer j % NSB; before S_j overwrites the buffer
      // of P_{j-NSB}, the P.V issuer must have finished O += P_{j-NSB} V_{j-NSB}
      // (empty_v of its stage completes exactly then).  empty_k tells the row
      // warps that S_j is ready.
      bool ok = mbar_wait(B(bars->q_ready), 0, ctl, p.status);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j % NS, bb = j % C::NSB;
        if (j >= C::NSB) {
          const int jj = j - C::NSB;
          if (!(ok = mbar_wait(B(bars->empty_v[jj % NS]), (jj / NS) & 1, ctl, p.status))) break;
        }
        if (!(ok = mbar_wait(B(bars->ready_k[s]), (j / NS) & 1, ctl, p.status))) break;
        tc_fence_after();
        if constexpr (C::KIL)
          mma_chain_kil<D, C::KCH>(tmem + C::TC_S + bb * C::SBUF, tmem + C::TC_Q,
                                   tmem + C::TC_Q + D, kd0 + (s * C::STAGE >> 4), idS2, idS);
        else
          mma_chain<SPLIT, D, false, BN, C::TILE>(tmem + C::TC_S + bb * C::SBUF, tmem + C::TC_Q,
                                                  tmem + C::TC_Q + D, kd0 + (s * C::STAGE >> 4),
                                                  idS, false);
        umma_commit(B(bars->empty_k[s]));  // also tells the row warps S_j is ready
      }
      umma_commit(B(bars->mma_final));  // nothing of ours in flight after this
      mbar_drain(B(bars->mma_final), 0);
    }
    __syncwarp();
  } else if (warp == kIssuer2Warp) {
    // ------------------------------------------------- P.V MMA issuer
    if (lane == 0) {
      constexpr uint32_t idO = idesc_tf32(128, D, false, true);
      constexpr uint32_t idO2 = idesc_tf32(128, 2 * D, false, true);  // [V_hi | V_lo] (PVM)
      const uint64_t vd0 = sdesc_mnmajor(tiles + C::OFF_V, BN * 128);
      bool ok = true;
      for (int jj = 0; ok && jj < n_kv; ++jj) {
        const int s = jj % NS, bb = jj % C::NSB;
        if (!(ok = mbar_wait(B(bars->p_full[bb]), (jj / C::NSB) & 1, ctl, p.status))) break;
        if (!(ok = mbar_wait(B(bars->ready_v[s]), (jj / NS) & 1, ctl, p.status))) break;
        tc_fence_after();
        const uint32_t pA = tmem + C::TC_S + bb * C::SBUF;
        if constexpr (C::PVM)
          mma_chain_mn2<BN>(tmem + C::TC_O, pA, pA + BN, vd0 + (s * C::STAGE >> 4), idO2, idO,
                            jj > 0);
        else
          mma_chain<SPLIT, BN, true, BN, C::TILE>(tmem + C::TC_O, pA, pA + BN,
                                                  vd0 + (s * C::STAGE >> 4), idO, jj > 0);
        umma_commit(B(bars->empty_v[s]));  // also: O += P_jj V_jj is done
      }
      umma_commit(B(bars->mma_final_pv));  // nothing of this thread in flight after this
      mbar_drain(B(bars->mma_final_pv), 0);
    }
    __syncwarp();
  } else if (is_prep_warp(warp)) {
    // ---------------------------------------- split / rounding warps
    const uint32_t tid = prep_tid();
    auto prep = [&](uint32_t t, bool is_k) {
      if constexpr (SPLIT == 3) {
        if (is_k) split_tile_smem_il<C::TILE, kSplitThreads, (uint32_t)BN * 128u>(t, tid);
        else split_tile_smem<C::TILE, kSplitThreads>(t, t + C::TILE, tid);
      } else {
        round_tile_smem<C::TILE, kSplitThreads>(t, tid);
      }
    };
    for (int j = 0; j < n_kv; ++j) {
      const int s = j % NS, r = j / NS;
      const uint32_t st = tiles + s * C::STAGE;
      if (!warp_wait(B(bars->full_k[s]), r & 1, ctl, p.status)) break;
      prep(st + C::OFF_K, true);
      fence_proxy_async_smem();
      warp_arrive(B(bars->ready_k[s]));
      if (!warp_wait(B(bars->full_v[s]), r & 1, ctl, p.status)) break;
      prep(st + C::OFF_V, false);
      fence_proxy_async_smem();
      warp_arrive(B(bars->ready_v[s]));
    }
  } else {
    // --------------------------------------------------------- row warps
    // Warps 4-7 (group 0) and 11-14 (group 1): thread (quad, lane) owns query
    // row quad*32 + lane (TMEM lane quarter quad); group g takes the score
    // columns [g*BN/2, (g+1)*BN/2) of every step.  The pair of warps sharing a
    // quarter exchange partial row maxima through shared memory, so both apply
    // the same maximum; each keeps its partial row sum and rescales / writes
    // its half of the O columns.  Group 0 loads Q.
    constexpr int HB = BN / 2, CW = HB < 32 ? HB : 32;
    constexpr int OH = (int)C::OW / 2, OCW = OH < 32 ? OH : 32;  // O columns rescaled per group
    const int quad = warp & 3;
    const int grp = warp >= kFwdRowWarp1 ? 1 : 0;
    const int c0 = grp * HB;
    const int r = quad * 32 + lane;
    const int row = q0 + r;
    const bool valid = row < T;
    const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
    if (grp == 0) {
      const float* qrow = p.q.row(b, h, valid ? row : 0);
      const bool vec = p.q.s3 == 1 && ((reinterpret_cast<uintptr_t>(qrow) & 15u) == 0);
      row_to_tmem<D, SPLIT>(p.q, qrow, valid, vec, lb, C::TC_Q);
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->q_ready));
    }
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int bb = j % C::NSB;
      if (!(ok = warp_wait(B(bars->empty_k[j % NS]), (j / NS) & 1, ctl, p.status))) break;
      tc_fence_after();
      const uint32_t sc = lb + C::TC_S + bb * C::SBUF + c0;
      const int kv0 = j * BN + c0;
      const bool need_mask = (kv0 + HB > T) || (p.causal && kv0 + HB - 1 > q0);
      // This group's masked scores (with KIL the sum of the two partial sums),
      // kept in registers for the exponentials, and their maximum.
      float sv[HB];
      float mraw = -INFINITY;
#pragma unroll
      for (int c = 0; c < HB / CW; ++c) {
        float t[CW];
        tmem_ldn<CW>(sc + CW * c, t);
        if constexpr (C::KIL) {
          float t2[CW];
          tmem_ldn<CW>(sc + BN + CW * c, t2);
#pragma unroll
          for (int i = 0; i < CW; i += 2) fadd2(t[i], t[i + 1], t[i], t[i + 1], t2[i], t2[i + 1]);
        }
        if (need_mask) mask_cols<CW>(t, kv0 + CW * c, T, p.causal, row);
        mraw = fmaxf(mraw, maxn<CW>(t));
#pragma unroll
        for (int i = 0; i < CW; ++i) sv[CW * c + i] = t[i];
      }
      bars->xmax[j & 1][grp][r] = mraw;
      warp_arrive(B(bars->xchg[quad][j & 1]));
      if (!(ok = warp_wait(B(bars->xchg[quad][j & 1]), (j >> 1) & 1, ctl, p.status))) break;
      mraw = fmaxf(mraw, bars->xmax[j & 1][grp ^ 1][r]);
      // scale_log2 > 0, so scaling after the maximum is exact
      const float m_new = fmaxf(m_used, mraw * p.scale_log2);
      const bool resc = m_new > m_used + 8.0f;
      if (__any_sync(0xffffffffu, resc)) {
        const float alpha = resc ? ex2_approx(m_used - m_new) : 1.0f;
        if (resc) m_used = m_new;
        l *= alpha;
        if (j > 0) {
          const int jj = j - 1;
          if (!(ok = warp_wait(B(bars->empty_v[jj % NS]), (jj / NS) & 1, ctl, p.status))) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < OH / OCW; ++c) {
            float ov[OCW];
            tmem_ldn<OCW>(lb + C::TC_O + grp * OH + OCW * c, ov);
#pragma unroll
            for (int i = 0; i < OCW; ++i) ov[i] *= alpha;
            tmem_stn<OCW>(lb + C::TC_O + grp * OH + OCW * c, ov);
          }
        }
      }
      // P = exp2(s * scale_log2 - m), written over S (hi) and next to it (lo).
      const float neg_m = -m_used;
      float ls0 = 0.0f, ls1 = 0.0f;
#pragma unroll
      for (int c = 0; c < HB / CW; ++c) {
        float t[CW], lo[CW];
#pragma unroll
        for (int i = 0; i < CW; i += 2) {
          float a0, a1;
          ffma2(a0, a1, sv[CW * c + i], sv[CW * c + i + 1], p.scale_log2, p.scale_log2, neg_m,
                neg_m);
          const float e0 = ex2_approx(a0), e1 = ex2_approx(a1);
          fadd2(ls0, ls1, ls0, ls1, e0, e1);  // even / odd column sums
          if constexpr (SPLIT == 3) {
            tf32_split2(e0, e1, t[i], t[i + 1], lo[i], lo[i + 1]);
          } else {
            t[i] = tf32_round_finite(e0);
            t[i + 1] = tf32_round_finite(e1);
          }
        }
        tmem_stn<CW>(sc + CW * c, t);
        if constexpr (SPLIT == 3) tmem_stn<CW>(sc + BN + CW * c, lo);
      }
      l += ls0 + ls1;
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->p_full[bb]));
    }
    if (ok) {
      const int jj = n_kv - 1;
      const bool done = warp_wait(B(bars->empty_v[jj % NS]), (jj / NS) & 1, ctl, p.status);
      bars->xsum[grp][r] = l;
      warp_arrive(B(bars->xfin[quad]));
      if (warp_wait(B(bars->xfin[quad]), 0, ctl, p.status) && done) {
        tc_fence_after();
        const float lt = l + bars->xsum[grp ^ 1][r];
        const float inv_l = 1.0f / lt;
        constexpr int DH = D / 2;  // output columns written per group
        float* orow = p.o + ((int64_t)bh * T + (valid ? row : 0)) * D + grp * DH;
        if constexpr (C::PVM) {
#pragma unroll
          for (int c = 0; c < DH / 16; ++c) {
            float v[16], w[16];
            tmem_ld16(lb + C::TC_O + grp * DH + 16 * c, v);
            tmem_ld16(lb + C::TC_O + D + grp * DH + 16 * c, w);
            if (valid) {
              float4* d4 = reinterpret_cast<float4*>(orow + 16 * c);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                d4[i] = make_float4((v[4 * i] + w[4 * i]) * inv_l, (v[4 * i + 1] + w[4 * i + 1]) * inv_l,
                                    (v[4 * i + 2] + w[4 * i + 2]) * inv_l,
                                    (v[4 * i + 3] + w[4 * i + 3]) * inv_l);
            }
          }
        } else {
          tmem_cols_to_global<DH>(lb, C::TC_O + grp * DH, inv_l, orow, valid);
        }
        if (valid && grp == 0) p.lse[(int64_t)bh * T + row] = (m_used + log2f(lt)) * kLn2;
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
int run_fwd(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, float* o, float* lse,
            const DeviceInfo& dev, cudaStream_t st) {
  static unsigned long long attr_done = 0;
  CUtensorMap tmK, tmV;
  int rc = C::KIL ? make_tmap_bhtd(&tmK, k, pr, C::BN) : make_tmap_bhtd_whole(&tmK, k, pr, C::BN);
  if (rc != CT_OK) return rc;
  rc = make_tmap_bhtd_whole(&tmV, v, pr, C::BN, /*mn_major=*/true);
  if (rc != CT_OK) return rc;
  const size_t smem = fwd_smem_bytes<C>();
  rc = ensure_smem_attr(fa2_fwd_tc_kernel<C>, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  FwdParams p;
  p.q = Ptr4{q.ptr, q.s[0], q.s[1], q.s[2], q.s[3]};
  p.o = o;
  p.lse = lse;
  p.H = (int)pr.H;
  p.T = (int)pr.T;
  p.n_qt = (int)((pr.T + kRows - 1) / kRows);
  p.bh_total = (int)(pr.B * pr.H);
  p.head_group = fa2_head_group(p.bh_total);
  p.causal = pr.causal ? 1 : 0;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)pr.D));
  p.status = dev.status;
  const int64_t grid = (int64_t)p.n_qt * p.bh_total;
  fa2_fwd_tc_kernel<C><<<(unsigned)grid, kFwdThreads, smem, st>>>(tmK, tmV, p);
  return check_launch();
}

// ------------------------------------------- TF32: two query tiles per CTA
// The TF32 forward at head dims 32 and 64 keeps two 128-row query tiles (A,
// B) per CTA instead of splitting one tile's score columns between the two
// row warpgroups.  Each warpgroup owns a whole tile: it takes every column of
// its S, so no row maximum is exchanged between warps, and the K / V tiles a
// stage lands serve 256 query rows.  Each tile has its own issuing thread
// (warp 1: tile A, warp 10: tile B) and two S / P buffers:
//   S_t(j+1) = Q_t K_{j+1}^T runs while the rows turn S_t(j) into P_t(j);
//   O_t += P_t(j) V_j, then S_t(j+2) into P_t(j)'s buffer (same thread, in
//   order), so while one group forms P the tensor core works for the other.
// TMEM: Q_A | Q_B | O_A | O_B | S_A x 2 | S_B x 2.  The rows rescale O_t (when
// the maximum grows by more than 2^8) once O_t += P_t(j-1) V_{j-1} is done
// (pv_done).
template <int D_, int BN_, int NS_>
struct FwdPairCfg {
  static constexpr int D = D_, BN = BN_, NS = NS_;
  static constexpr uint32_t TILE = (uint32_t)BN * D_ * 4u;
  static constexpr uint32_t STAGE = 2u * TILE, OFF_K = 0, OFF_V = TILE;
  // Q_t at t * D, O_t at 2D + t * D, S buffer bb of tile t at 4D + (2t + bb) * BN
  static constexpr uint32_t TC_Q = 0, TC_O = 2u * D_, TC_S = 4u * D_;
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(TC_S + 4u * BN <= TMEM_COLS, "TMEM budget");
  static_assert(BN == 64, "the row warps keep a step's 64 scores in registers");
};

template <int NS>
struct FwdPairBars {
  uint64_t full_k[NS], full_v[NS], ready_k[NS], ready_v[NS], empty_k[NS], empty_v[NS];
  uint64_t s_full[2][2], p_full[2][2], pv_done[2], o_done[2], q_ready[2], mma_final[2];
  CtaCtl ctl;
};

template <class C>
constexpr size_t fwd_pair_smem_bytes() {  // with the row warps' write-out buffer
  constexpr size_t head = (sizeof(FwdPairBars<C::NS>) + 1023) / 1024 * 1024 + 1024;
  static_assert(head + (size_t)C::NS * C::STAGE + kRowWbufBytes <= 227 * 1024,
                "shared memory budget");
  return head + (size_t)C::NS * C::STAGE + kRowWbufBytes;
}

// One unit tile of a persistent CTA: query-tile pair qp of head bh (tiles A
// and B, rows q0 .. q0 + 255), with n_a / n_b key tiles each and n_kv the
// larger.
struct FwdUnitTile {
  int b, h, bh, q0, n_a, n_b, n_kv;
};
// Tile m of CTA c (of G): half m % 2 of unit c + (m / 2) G, a unit being the
// tile pairs (qp, NQ-1-qp) of one head (NQ pairs per head), whose causal key
// counts add up to the same total for every qp.  Returns false past the CTA's
// last unit and skips the missing half of the middle unit when NQ is odd.
__device__ __forceinline__ bool fwd_tile_at(const FwdParams& p, int c, int G, int& m,
                                            FwdUnitTile& u) {
  constexpr int BN = 64;
  const int U = (p.n_qt + 1) / 2;
  for (;; ++m) {
    const int un = c + (m >> 1) * G;
    if (un >= U * p.bh_total) return false;
    int k;
    cta_tile_at((unsigned)un, U, p.bh_total, p.head_group, false, k, u.bh);
    const int qp = (m & 1) ? p.n_qt - 1 - k : k;
    if ((m & 1) && qp == k) continue;
    u.b = u.bh / p.H;
    u.h = u.bh % p.H;
    u.q0 = qp * 2 * kRows;
    auto steps = [&](int t) {
      const int last = min(u.q0 + (t + 1) * kRows - 1, p.T - 1);
      return p.causal ? last / BN + 1 : (p.T + BN - 1) / BN;
    };
    u.n_a = steps(0);
    u.n_b = steps(1);
    u.n_kv = max(u.n_a, u.n_b);
    return true;
  }
}

// Persistent: each CTA loops over unit tiles; the producer and rounding warps
// run across tile boundaries (one step counter for the stage ring).
template <class C>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fa2_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  constexpr int D = C::D, BN = C::BN, NS = C::NS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  auto* bars = reinterpret_cast<FwdPairBars<NS>*>(smem_raw);
  const uint32_t tiles = (smem_u32(smem_raw) + (uint32_t)sizeof(FwdPairBars<NS>) + 1023u) & ~1023u;
  CtaCtl* ctl = &bars->ctl;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int T = p.T, G = (int)gridDim.x, cta = (int)blockIdx.x;

  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      // one landing, one readiness and one release barrier per stage (K_j, V_j)
      mbar_init(B(bars->full_k[s]), 1);
      mbar_init(B(bars->ready_k[s]), kPrepWarps);
      mbar_init(B(bars->empty_k[s]), 2);  // both tiles' S and P.V MMAs read the stage
    }
    for (int t = 0; t < 2; ++t) {
      for (int bb = 0; bb < 2; ++bb) {
        mbar_init(B(bars->s_full[t][bb]), 1);
        mbar_init(B(bars->p_full[t][bb]), 4);  // the tile's row warps
      }
      mbar_init(B(bars->pv_done[t]), 1);
      mbar_init(B(bars->o_done[t]), 1);
      mbar_init(B(bars->mma_final[t]), 1);
      mbar_init(B(bars->q_ready[t]), 4);  // the tile's row warps
    }
    ctl->abort = 0;
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int last_k[NS];
      for (int s = 0; s < NS; ++s) last_k[s] = -1;
      bool ok = true;
      int g = 0;
      FwdUnitTile u;
      for (int m = 0; ok && fwd_tile_at(p, cta, G, m, u); ++m) {
        for (int j = 0; j < u.n_kv; ++j) {
          const int gs = g + j, s = gs % NS, r = gs / NS;
          const uint32_t st = tiles + s * C::STAGE;
          // K_j and V_j share one stage release and one landing barrier
          if (r > 0 && !(ok = mbar_wait(B(bars->empty_k[s]), (r - 1) & 1, ctl, p.status))) break;
          mbar_arrive_expect_tx(B(bars->full_k[s]), 2 * C::TILE);
          tma_load_tile<true, D>(st + C::OFF_K, &tmK, B(bars->full_k[s]), j * BN, u.h, u.b,
                                 BN * 128u);
          tma_load_tile<true, D>(st + C::OFF_V, &tmV, B(bars->full_k[s]), j * BN, u.h, u.b,
                                 BN * 128u);
          last_k[s] = r;
        }
        g += u.n_kv;
      }
      if (ctl->abort) {  // let every issued copy land before the CTA exits
        for (int s = 0; s < NS; ++s)
          if (last_k[s] >= 0) mbar_drain(B(bars->full_k[s]), last_k[s] & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1 || warp == kIssuer2Warp) {
    // ------------------------------------- tile t's issuer: S, then P.V
    // One readiness wait per step (ready_k covers K_j and V_j; S(j) waits on
    // it, P.V(j) follows on the same thread) and one stage release (empty_k,
    // committed after P.V(j), so it also covers S(j)).  Past its last key
    // tile a tile still releases the stages (commits with nothing new in
    // flight, after the stage has landed), so the producer's two-issuer count
    // holds.  g counts the CTA's key steps (stage ring), gt this tile's own
    // steps (S / P buffers, pv_done); per unit tile: wait for the rows' Q
    // (q_ready), commit o_done after the last P.V.
    if (lane == 0) {
      const int t = warp == 1 ? 0 : 1;
      constexpr uint32_t idS = idesc_tf32(128, BN, false, false);
      constexpr uint32_t idO = idesc_tf32(128, D, false, true);
      const uint64_t kd0 = sdesc_kmajor(tiles + C::OFF_K);
      const uint64_t vd0 = sdesc_mnmajor(tiles + C::OFF_V, BN * 128);
      const uint32_t sb0 = tmem + C::TC_S + (uint32_t)(2 * t) * BN;
      bool ok = true;
      int g = 0, gt = 0, tn = 0;
      FwdUnitTile u;
      for (int m = 0; ok && fwd_tile_at(p, cta, G, m, u); ++m) {
        const int n_mine = t ? u.n_b : u.n_a, n_kv = u.n_kv;
        // Past its last key tile a tile still releases each stage, but only
        // once the stage holds that step's tiles (the wait on ready_k below,
        // two steps before the release): an early release would count toward
        // the stage's previous round, which the other tile may still be
        // reading.
        auto issue_S = [&](int j) -> bool {  // S_t(j) into buffer (gt + j) % 2
          const int gs = g + j, s = gs % NS;
          if (!mbar_wait(B(bars->ready_k[s]), (gs / NS) & 1, ctl, p.status)) return false;
          if (j < n_mine) {
            tc_fence_after();
            mma_chain<1, D, false, BN, C::TILE>(sb0 + (uint32_t)((gt + j) & 1) * BN,
                                                tmem + C::TC_Q + (uint32_t)t * D, 0,
                                                kd0 + (s * C::STAGE >> 4), idS, false);
            umma_commit(B(bars->s_full[t][(gt + j) & 1]));
          }
          return true;
        };
        ok = mbar_wait(B(bars->q_ready[t]), tn & 1, ctl, p.status) && issue_S(0) &&
             (n_kv < 2 || issue_S(1));
        for (int j = 0; ok && j < n_kv; ++j) {
          const int gs = g + j, s = gs % NS;
          if (j < n_mine) {
            const int gb = gt + j;
            if (!(ok = mbar_wait(B(bars->p_full[t][gb & 1]), (gb >> 1) & 1, ctl, p.status))) break;
            tc_fence_after();
            mma_chain<1, BN, true, BN, C::TILE>(tmem + C::TC_O + (uint32_t)t * D,
                                                sb0 + (uint32_t)(gb & 1) * BN, 0,
                                                vd0 + (s * C::STAGE >> 4), idO, j > 0);
            umma_commit(B(bars->pv_done[t]));
          }
          umma_commit(B(bars->empty_k[s]));  // K_j and V_j read for the last time
          if (j + 2 < n_kv && !(ok = issue_S(j + 2))) break;
        }
        if (ok) umma_commit(B(bars->o_done[t]));
        g += n_kv;
        gt += n_mine;
        ++tn;
      }
      umma_commit(B(bars->mma_final[t]));  // nothing of this thread in flight after this
      mbar_drain(B(bars->mma_final[t]), 0);
    }
    __syncwarp();
  } else if (is_prep_warp(warp)) {
    // ----------------------------------------------- TF32 rounding warps
    const uint32_t tid = prep_tid();
    bool ok = true;
    int g = 0;
    FwdUnitTile u;
    for (int m = 0; ok && fwd_tile_at(p, cta, G, m, u); ++m) {
      for (int j = 0; j < u.n_kv; ++j) {
        const int gs = g + j, s = gs % NS, r = gs / NS;
        const uint32_t st = tiles + s * C::STAGE;
        if (!(ok = warp_wait(B(bars->full_k[s]), r & 1, ctl, p.status))) break;
        round_tile_smem<C::TILE, kSplitThreads>(st + C::OFF_K, tid);
        round_tile_smem<C::TILE, kSplitThreads>(st + C::OFF_V, tid);
        fence_proxy_async_smem();
        warp_arrive(B(bars->ready_k[s]));  // K_j and V_j
      }
      g += u.n_kv;
    }
  } else {
    // --------------------------------------------------------- row warps
    // Warps 4-7 own tile A, warps 11-14 tile B: thread (quad, lane) owns
    // query row quad*32 + lane of its tile (TMEM lane quarter quad) and all
    // BN score columns of a step, kept in registers between the maximum and
    // the exponentials.
    // Unit-tile boundary: the next Q row goes into TMEM as soon as the
    // previous tile's last S has completed, and q_ready lets the tile's issuer
    // start S while the previous P.V drains; the rows then wait for o_done and
    // write out the previous O_t and LSE (the first P.V, which overwrites the
    // accumulator, waits for P(0), formed after the write-out).
    const int t = warp >= kFwdRowWarp1 ? 1 : 0;
    const int quad = warp & 3;
    const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
    float* wbuf = reinterpret_cast<float*>(smem_raw + (tiles - smem_u32(smem_raw)) +
                                           NS * C::STAGE) +
                  (t * 4 + quad) * kRowWbufFloats;
    bool ok = true, pending = false;
    int gt = 0, tn = 0;
    int64_t prev_row0 = 0;
    int prev_nrows = 0;
    bool prev_valid = false;
    int64_t prev_lse = 0;
    float prev_inv_l = 0.0f, prev_lse_val = 0.0f;
    auto write_out = [&]() {
      warp_rows_to_global<D>(lb + C::TC_O + (uint32_t)t * D, prev_inv_l, wbuf,
                             p.o + prev_row0 * D, prev_nrows, D, false);
      if (prev_valid) p.lse[prev_lse] = prev_lse_val;
      tc_fence_before();  // TMEM reads done before the next arrival
    };
    FwdUnitTile u;
    for (int m = 0; ok && fwd_tile_at(p, cta, G, m, u); ++m) {
      const int n_mine = t ? u.n_b : u.n_a;
      const int qt0 = u.q0 + t * kRows;
      const int row = qt0 + quad * 32 + lane;
      const bool valid = row < T;
      const uint32_t sc0 = lb + C::TC_S + (uint32_t)(2 * t) * BN;
      const uint32_t oc = lb + C::TC_O + (uint32_t)t * D;
      {
        const float* qrow = p.q.row(u.b, u.h, valid ? row : 0);
        const bool vec = p.q.s3 == 1 && ((reinterpret_cast<uintptr_t>(qrow) & 15u) == 0);
        float xq[D / 32][32];
#pragma unroll
        for (int c = 0; c < D / 32; ++c) load_row32(p.q, qrow, 32 * c, valid, vec, xq[c]);
        // Q_t is read only by the S MMAs, which this warp saw complete
        // (s_full of its last step): no wait for o_done before replacing it.
        tc_fence_after();
        const uint32_t qa = lb + C::TC_Q + (uint32_t)t * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
#pragma unroll
          for (int e = 0; e < 32; ++e) xq[c][e] = tf32_round(xq[c][e]);
          tmem_st32(qa + 32 * c, xq[c]);
        }
        tmem_wait_st();
        tc_fence_before();
        warp_arrive(B(bars->q_ready[t]));
      }
      if (pending) {
        if (!(ok = warp_wait(B(bars->o_done[t]), (tn - 1) & 1, ctl, p.status))) break;
        tc_fence_after();
        write_out();
      }
      float m_used = -INFINITY, l = 0.0f;
      for (int j = 0; ok && j < n_mine; ++j) {
        const int gb = gt + j, bb = gb & 1;
        const uint32_t sc = sc0 + (uint32_t)bb * BN;
        if (!(ok = warp_wait(B(bars->s_full[t][bb]), (gb >> 1) & 1, ctl, p.status))) break;
        tc_fence_after();
        const int kv0 = j * BN;
        const bool need_mask = (kv0 + BN > T) || (p.causal && kv0 + BN - 1 > qt0);
        float sv[BN];
        float mraw = -INFINITY;
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          float x[32];
          tmem_ld32(sc + 32 * c, x);
          if (need_mask) mask_cols32(x, kv0 + 32 * c, T, p.causal, row);
          mraw = fmaxf(mraw, max32(x));
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[32 * c + i] = x[i];
        }
        // scale_log2 > 0, so scaling after the maximum is exact
        const float m_new = fmaxf(m_used, mraw * p.scale_log2);
        const bool resc = m_new > m_used + 8.0f;
        const bool any_resc = __any_sync(0xffffffffu, resc);
        const float alpha = resc ? ex2_approx(m_used - m_new) : 1.0f;
        if (resc) m_used = m_new;
        l *= alpha;
        const float neg_m = -m_used;
        float ls0 = 0.0f, ls1 = 0.0f;
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          float x[32];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float a0, a1;
            ffma2(a0, a1, sv[32 * c + i], sv[32 * c + i + 1], p.scale_log2, p.scale_log2, neg_m,
                  neg_m);
            const float e0 = ex2_approx(a0), e1 = ex2_approx(a1);
            fadd2(ls0, ls1, ls0, ls1, e0, e1);
            x[i] = tf32_round_finite(e0);
            x[i + 1] = tf32_round_finite(e1);
          }
          tmem_st32(sc + 32 * c, x);
        }
        l += ls0 + ls1;
        // O_t rescaled to the new maximum once O_t += P_t(j-1) V_{j-1} is done
        // (the scores are out of the registers by now)
        if (any_resc && j > 0) {
          if (!(ok = warp_wait(B(bars->pv_done[t]), (gb - 1) & 1, ctl, p.status))) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float ov[32];
            tmem_ld32(oc + 32 * c, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_st32(oc + 32 * c, ov);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        warp_arrive(B(bars->p_full[t][bb]));
      }
      pending = ok;
      prev_row0 = (int64_t)u.bh * T + qt0 + quad * 32;
      prev_nrows = max(0, min(32, T - (qt0 + quad * 32)));
      prev_valid = valid;
      prev_lse = (int64_t)u.bh * T + row;
      prev_inv_l = 1.0f / l;
      prev_lse_val = (m_used + log2f(l)) * kLn2;
      gt += n_mine;
      ++tn;
    }
    if (ok && pending && warp_wait(B(bars->o_done[t]), (tn - 1) & 1, ctl, p.status)) {
      tc_fence_after();
      write_out();
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
int run_fwd_pair(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, float* o, float* lse,
                 const DeviceInfo& dev, cudaStream_t st) {
  static unsigned long long attr_done = 0;
  CUtensorMap tmK, tmV;
  int rc = make_tmap_bhtd_whole(&tmK, k, pr, C::BN);
  if (rc != CT_OK) return rc;
  rc = make_tmap_bhtd_whole(&tmV, v, pr, C::BN, /*mn_major=*/true);
  if (rc != CT_OK) return rc;
  const size_t smem = fwd_pair_smem_bytes<C>();
  rc = ensure_smem_attr(fa2_fwd_pair_kernel<C>, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  FwdParams p;
  p.q = Ptr4{q.ptr, q.s[0], q.s[1], q.s[2], q.s[3]};
  p.o = o;
  p.lse = lse;
  p.H = (int)pr.H;
  p.T = (int)pr.T;
  p.n_qt = (int)((pr.T + 2 * kRows - 1) / (2 * kRows));  // query-tile pairs
  p.bh_total = (int)(pr.B * pr.H);
  p.head_group = fa2_head_group(p.bh_total);
  p.causal = pr.causal ? 1 : 0;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)pr.D));
  p.status = dev.status;
  // persistent: one CTA per SM (one fits), at most one per unit
  const int64_t units = (int64_t)((p.n_qt + 1) / 2) * p.bh_total;
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(units, dev.sm_count));
  fa2_fwd_pair_kernel<C><<<(unsigned)grid, kFwdThreads, smem, st>>>(tmK, tmV, p);
  return check_launch();
}

}  // namespace

bool fa2_fwd_tc_supported(const Fa2Problem& p) {
  return (p.D == 32 || p.D == 64 || p.D == 128) &&
         (p.precision == CT_PRECISION_3XTF32 || p.precision == CT_PRECISION_TF32) &&
         p.T < (1ll << 31) && p.B * p.H < (1ll << 31) &&
         ((p.T + kRows - 1) / kRows) * p.B * p.H < (1ll << 31);
}

int launch_fa2_fwd_tc(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v, float* o,
                      float* lse, const DeviceInfo& dev, cudaStream_t st) {
  if (!fa2_tma_ok(k) || !fa2_tma_ok(v)) return CT_ERR_UNSUPPORTED_LAYOUT;
  const bool split = pr.precision == CT_PRECISION_3XTF32;
  switch (pr.D) {
    case 32:
      return split ? run_fwd<FwdCfg<32, 64, 3, 4, 3>>(pr, q, k, v, o, lse, dev, st)
                   : run_fwd_pair<FwdPairCfg<32, 64, 8>>(pr, q, k, v, o, lse, dev, st);
    case 64:
      return split ? run_fwd<FwdCfg<64, 64, 3, 3, 2>>(pr, q, k, v, o, lse, dev, st)
                   : run_fwd_pair<FwdPairCfg<64, 64, 6>>(pr, q, k, v, o, lse, dev, st);
    case 128:
      return split ? run_fwd<FwdCfg<128, 32, 3, 3, 2>>(pr, q, k, v, o, lse, dev, st)
                   : run_fwd<FwdCfg<128, 64, 1, 3, 3>>(pr, q, k, v, o, lse, dev, st);
    default:
      return CT_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

}  // namespace ct
