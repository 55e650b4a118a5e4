// fa2_bwd_dq_persist.cu -- the TF32 dQ kernel at head dim 64 as a persistent
// kernel: the query-stationary pass of the FlashAttention-2 backward
// (reference: Transformer_kernels/flash_attention.cuh:216-354,
// flash_attention_bwd_dq), per 128 query rows and key tile j (64 keys):
//   S  = Q K_j^T,  dP = dO V_j^T,  dS = P (dP - delta)  (row warps),
//   dQ += dS K_j   (K_j read MN-major)
// with the same tile layout, TMEM map and warp roles as the one-CTA dQ kernel
// (fa2_bwd_tc.cu), but each CTA loops over query tiles.  The producer and the
// preparation warps run across tile boundaries (one step counter g for the
// stage ring and the S / dP buffers), so the next tile's K / V tiles are
// landed and prepared while the current one finishes; per tile only the row
// warps' dQ write-out and the load of the next Q / dO rows into TMEM sit
// between the last MMA of one tile and the first of the next.
//
// Schedule: a unit is the query-tile pair (qt, NT-1-qt) of one head (NT tiles
// per head); under the causal mask their key-tile counts add up to the same
// total for every qt, so units have equal work.  CTA c takes units c, c + G,
// ... in the head-grouped order of cta_tile_at (heads in flight share K / V
// in L2).
//
// Warp roles (16 warps): 0 TMA producer (K_j, V_j); 1 S issuer and TMEM
// allocator; 10 dQ issuer; 15 dP issuer; 2, 3, 8, 9 tile preparation (K_j
// rounded in place plus its MN-major copy, V_j rounded); 4-7 and 11-14 the two
// row warpgroups (one query row per thread, each half of a step's 64 keys).
#include <algorithm>
#include <cstdlib>

#include "fa2_bwd_parts.cuh"

namespace ct {
namespace {

using namespace fa2;

// A = K (K-major for S, MN-major for dQ), B = V (K-major for dP).
struct DqpCfg : BwdTiles<64, 64, 1, 4, 2, 1> {
  static constexpr int NSB = 2;
  static constexpr uint32_t SB = 64;
  static constexpr uint32_t TC_Q = 0, TC_G = 64, TC_DQ = 128, TC_S = 192, TC_DP = 320;
  static_assert(TC_DP + NSB * SB <= TMEM_COLS, "TMEM budget");
};

struct DqTile {
  int b, h, bh, q0, jb, n;
  bool exists;
};
// Tile m of CTA c (of G): half m % 2 of unit c + (m / 2) G.  Returns false past
// the CTA's last unit; t.exists is false for the missing half of the middle
// unit when NT is odd.
__device__ __forceinline__ bool dq_tile_at(const BwdParams& p, int c, int G, int m, DqTile& t) {
  constexpr int BN = 64;
  const int U = (p.n_tiles + 1) / 2;
  const int u = c + (m >> 1) * G;
  if (u >= U * p.bh_total) return false;
  int k;
  cta_tile_at((unsigned)u, U, p.bh_total, p.head_group, false, k, t.bh);
  const int qt = (m & 1) ? p.n_tiles - 1 - k : k;
  t.exists = !((m & 1) && qt == k);
  t.b = t.bh / p.H;
  t.h = t.bh % p.H;
  t.q0 = qt * kRows;
  const int last_row = min(t.q0 + kRows - 1, p.T - 1);
  t.jb = p.seg_lo / BN;
  t.n = t.exists ? max(0, min(p.causal ? last_row / BN + 1 : (p.T + BN - 1) / BN,
                              (p.seg_hi + BN - 1) / BN) - t.jb)
                 : 0;
  return true;
}

__global__ void __launch_bounds__(kBwdThreads, 1)
    fa2_bwd_dq_persist_kernel(const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const BwdParams p) {
  using C = DqpCfg;
  constexpr int D = C::D, BN = C::BN, NS = C::NS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  auto* bars = reinterpret_cast<BwdBars<NS>*>(smem_raw);
  const uint32_t tiles = (smem_u32(smem_raw) + (uint32_t)sizeof(BwdBars<NS>) + 1023u) & ~1023u;
  CtaCtl* ctl = &bars->ctl;
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int T = p.T, G = (int)gridDim.x, cta = (int)blockIdx.x;
  auto stg = [&](int g) { return (uint64_t)(((g % NS) * C::STAGE) >> 4); };

  // empty_a: K_j released by the dQ issuer; empty_b: V_j by the dP issuer;
  // done: the dQ issuer's last MMA of a tile.
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
    // Producer: K_j then V_j into stage g % NS (lane 0), once each is released.
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
    }
    int last_a[NS], last_b[NS];
    for (int s = 0; s < NS; ++s) last_a[s] = last_b[s] = -1;
    bool ok = true;
    int g = 0;
    DqTile t;
    for (int m = 0; ok && dq_tile_at(p, cta, G, m, t); ++m) {
      for (int i = 0; i < t.n; ++i) {
        const int gs = g + i, s = gs % NS, r = gs / NS, j = t.jb + i;
        const uint32_t st = tiles + s * C::STAGE;
        if (r > 0 && !(ok = warp_wait(B(bars->empty_a[s]), (r - 1) & 1, ctl, p.status))) break;
        if (lane == 0) {
          const uint32_t fa = B(bars->full_a[s]);
          mbar_arrive_expect_tx(fa, C::TILE);
          tma_load_tile<true, D>(st + C::OFF_A0, &tmK, fa, j * BN, t.h, t.b, C::KCHA);
        }
        last_a[s] = r;
        if (r > 0 && !(ok = warp_wait(B(bars->empty_b[s]), (r - 1) & 1, ctl, p.status))) break;
        if (lane == 0) {
          const uint32_t fb = B(bars->full_b[s]);
          mbar_arrive_expect_tx(fb, C::TILE);
          tma_load_tile<true, D>(st + C::OFF_B0, &tmV, fb, j * BN, t.h, t.b, C::KCHB);
        }
        last_b[s] = r;
      }
      g += t.n;
    }
    __syncwarp();
    if (ctl->abort && lane == 0) {
      for (int s = 0; s < NS; ++s) {
        if (last_a[s] >= 0) mbar_drain(B(bars->full_a[s]), last_a[s] & 1);
        if (last_b[s] >= 0) mbar_drain(B(bars->full_b[s]), last_b[s] & 1);
      }
    }
  } else if (warp == 1) {
    // S_g = Q K_g^T into buffer g % 2 once the rows hold S_{g-2} in registers
    // (s_free); per tile, the first waits until the rows have loaded Q.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_tf32(128, BN, false, false);
      const uint64_t kd0 = sdesc_kmajor(tiles + C::OFF_A0);
      bool ok = true;
      int g = 0, tn = 0;
      DqTile t;
      for (int m = 0; ok && dq_tile_at(p, cta, G, m, t); ++m) {
        if (t.n == 0) continue;
        if (!(ok = mbar_wait(B(bars->rows_ready), tn & 1, ctl, p.status))) break;
        for (int i = 0; ok && i < t.n; ++i) {
          const int gs = g + i, bj = gs % 2, gp = gs - 2;
          if (gp >= 0 &&
              !(ok = mbar_wait(B(bars->s_free[bj]), (gp / 2) & 1, ctl, p.status)))
            break;
          if (!(ok = mbar_wait(B(bars->ready_a[gs % NS]), (gs / NS) & 1, ctl, p.status))) break;
          tc_fence_after();
          mma_chain<1, D, false, BN, C::TILE>(tmem + C::TC_S + (uint32_t)bj * BN, tmem + C::TC_Q,
                                              tmem + C::TC_Q + D, kd0 + stg(gs), idS, false);
          umma_commit(B(bars->s_full[bj]));
        }
        g += t.n;
        ++tn;
      }
      umma_commit(B(bars->mma_final));
      mbar_drain(B(bars->mma_final), 0);
    }
    __syncwarp();
  } else if (warp == kIssuer2Warp) {
    // dQ += dS_g K_g (K_g MN-major) once the rows have written dS_g; releases
    // K_g (empty_a) and dS_g's buffer (dqd); `done` after a tile's last step.
    if (lane == 0) {
      constexpr uint32_t idQ = idesc_tf32(128, D, false, true);
      const uint64_t kmd0 = sdesc_mnmajor(tiles + C::OFF_A1, BN * 128);
      bool ok = true;
      int g = 0;
      DqTile t;
      for (int m = 0; ok && dq_tile_at(p, cta, G, m, t); ++m) {
        if (t.n == 0) continue;
        for (int i = 0; ok && i < t.n; ++i) {
          const int gs = g + i, bj = gs % 2;
          if (!(ok = mbar_wait(B(bars->ds_full[bj]), (gs / 2) & 1, ctl, p.status))) break;
          tc_fence_after();
          const uint32_t db = tmem + C::TC_DP + (uint32_t)bj * C::SB;
          mma_chain<1, BN, true, BN, C::TILE>(tmem + C::TC_DQ, db, db + BN, kmd0 + stg(gs), idQ,
                                              i > 0);
          umma_commit(B(bars->empty_a[gs % NS]));
          umma_commit(B(bars->dqd[bj]));
        }
        if (ok) umma_commit(B(bars->done));
        g += t.n;
      }
      umma_commit(B(bars->mma_final2));
      mbar_drain(B(bars->mma_final2), 0);
    }
    __syncwarp();
  } else if (warp == kIssuer3Warp) {
    // dP_g = dO V_g^T into buffer g % 2 once dQ_{g-2} has read dS_{g-2} from
    // it (dqd); per tile, the first waits until the rows have loaded dO.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_tf32(128, BN, false, false);
      const uint64_t vd0 = sdesc_kmajor(tiles + C::OFF_B0);
      bool ok = true;
      int g = 0, tn = 0;
      DqTile t;
      for (int m = 0; ok && dq_tile_at(p, cta, G, m, t); ++m) {
        if (t.n == 0) continue;
        if (!(ok = mbar_wait(B(bars->rows_ready), tn & 1, ctl, p.status))) break;
        for (int i = 0; ok && i < t.n; ++i) {
          const int gs = g + i, bj = gs % 2, gp = gs - 2;
          if (gp >= 0 && !(ok = mbar_wait(B(bars->dqd[bj]), (gp / 2) & 1, ctl, p.status))) break;
          if (!(ok = mbar_wait(B(bars->ready_b[gs % NS]), (gs / NS) & 1, ctl, p.status))) break;
          tc_fence_after();
          mma_chain<1, D, false, BN, C::TILE>(tmem + C::TC_DP + (uint32_t)bj * C::SB,
                                              tmem + C::TC_G, tmem + C::TC_G + D, vd0 + stg(gs),
                                              idS, false);
          umma_commit(B(bars->empty_b[gs % NS]));  // V_g read for the last time
          umma_commit(B(bars->dp_full[bj]));
        }
        g += t.n;
        ++tn;
      }
      umma_commit(B(bars->mma_final3));
      mbar_drain(B(bars->mma_final3), 0);
    }
    __syncwarp();
  } else if (is_prep_warp(warp)) {
    // K_g rounded in place plus its MN-major copy -> ready_a; V_g rounded ->
    // ready_b.
    const uint32_t tid = prep_tid();
    bool ok = true;
    int g = 0;
    DqTile t;
    for (int m = 0; ok && dq_tile_at(p, cta, G, m, t); ++m) {
      for (int i = 0; i < t.n; ++i) {
        const int gs = g + i, s = gs % NS, r = gs / NS;
        const uint32_t st = tiles + s * C::STAGE;
        if (!(ok = warp_wait(B(bars->full_a[s]), r & 1, ctl, p.status))) break;
        prep_tile<C>(st, false, tid);
        fence_proxy_async_smem();
        warp_arrive(B(bars->ready_a[s]));
        if (!(ok = warp_wait(B(bars->full_b[s]), r & 1, ctl, p.status))) break;
        prep_tile<C>(st, true, tid);
        fence_proxy_async_smem();
        warp_arrive(B(bars->ready_b[s]));
      }
      g += t.n;
    }
  } else {
    // Row warps 4-7 (group 0) and 11-14 (group 1): thread (quad, lane) owns
    // query row q0 + quad*32 + lane; group g forms P and dS for key columns
    // [32g, 32g + 32) of every step, loads Q (g = 0) or dO (g = 1) into TMEM,
    // and writes dQ columns [32g, 32g + 32).
    // Tile boundary: the next tile's Q / dO row (and the row's LSE and delta)
    // goes into TMEM as soon as the previous tile's last S and dP have
    // completed, and rows_ready lets the S and dP issuers start while the
    // previous tile's dQ MMAs drain; the rows then wait for its `done` and
    // write out the previous dQ (the first dQ MMA, which overwrites the
    // accumulator, waits for dS_0, formed after the write-out).
    constexpr int HB = BN / 2;
    const int quad = warp & 3;
    const int grp = warp >= kBwdRowWarp1 ? 1 : 0;
    const int c0 = grp * HB;
    const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
    const Ptr4& src = grp ? p.st1 : p.st0;
    float* wbuf = reinterpret_cast<float*>(smem_raw + (tiles - smem_u32(smem_raw)) +
                                           NS * C::STAGE + NS * 2 * BN * 4) +
                  (warp - 4 - (grp ? 3 : 0)) * kRowWbufFloats;
    bool ok = true, pending = false;
    int g = 0, tn = 0;
    int64_t prev_row0 = 0;
    int prev_nrows = 0;
    auto write_out = [&]() {
      warp_rows_to_global<D / 2>(lb + C::TC_DQ + grp * (D / 2), p.scale, wbuf,
                                 p.out0 + prev_row0 * D + grp * (D / 2), prev_nrows, D,
                                 p.accumulate_out != 0);
      tc_fence_before();  // TMEM reads done before the next arrival
    };
    DqTile t;
    for (int m = 0; ok && dq_tile_at(p, cta, G, m, t); ++m) {
      if (!t.exists) continue;
      const int row = t.q0 + quad * 32 + lane;
      const bool valid = row < T;
      if (t.n == 0) {  // no key of the segment reaches these queries
        if (valid && !p.accumulate_out) {
          float* o = p.out0 + ((int64_t)t.bh * T + row) * D + grp * (D / 2);
          for (int d = 0; d < D / 2; ++d) o[d] = 0.0f;
        }
        continue;
      }
      const float* rp = src.row(t.b, t.h, valid ? row : 0);
      const bool vr = src.s3 == 1 && ((reinterpret_cast<uintptr_t>(rp) & 15u) == 0);
      float x0[32], x1[32];
      load_row32(src, rp, 0, valid, vr, x0);
      load_row32(src, rp, 32, valid, vr, x1);
      float l2 = 0.0f, dl = 0.0f;
      if (valid) {
        l2 = ldg_nc_early(p.lse + t.b * p.l0 + t.h * p.l1 + (int64_t)row * p.l2);
        dl = ldg_nc_early(p.delta + (int64_t)t.bh * T + row);
      }
      // No wait for the previous tile's `done` here: only its S and dP MMAs read
      // Q / dO, and this warp saw them complete (s_full, dp_full of its last
      // step); the previous dQ accumulator is written out after rows_ready.
      tc_fence_after();
      l2 *= kLog2e;
      const uint32_t qa = lb + (grp ? C::TC_G : C::TC_Q);
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        x0[e] = tf32_round(x0[e]);
        x1[e] = tf32_round(x1[e]);
      }
      tmem_st32(qa, x0);
      tmem_st32(qa + 32, x1);
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B(bars->rows_ready));
      if (pending) {
        if (!(ok = warp_wait(B(bars->done), (tn - 1) & 1, ctl, p.status))) break;
        tc_fence_after();
        write_out();
      }
      {  // the next tile's row into L2 while this tile runs
        DqTile nt;
        for (int m2 = m + 1; m2 <= m + 2; ++m2) {
          if (!dq_tile_at(p, cta, G, m2, nt)) break;
          if (!nt.exists || nt.n == 0) continue;
          const int nrow = nt.q0 + quad * 32 + lane;
          if (nrow < T && src.s3 == 1) {
            const float* np = src.row(nt.b, nt.h, nrow);
            asm volatile("prefetch.global.L2 [%0];" ::"l"(np));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(np + 32));
          }
          break;
        }
      }
      for (int i = 0; ok && i < t.n; ++i) {
        const int gs = g + i, bj = gs % 2;
        const uint32_t par = (uint32_t)(gs / 2) & 1u;
        const uint32_t dc = lb + C::TC_DP + (uint32_t)bj * C::SB + c0;
        if (!(ok = warp_wait(B(bars->s_full[bj]), par, ctl, p.status))) break;
        tc_fence_after();
        float pv[HB];
        tmem_ldn<HB>(lb + C::TC_S + (uint32_t)bj * BN + c0, pv);
        tc_fence_before();
        warp_arrive(B(bars->s_free[bj]));
        const int kv0 = (t.jb + i) * BN + c0;
        const bool need_mask = !valid || (kv0 + HB > T) || (p.causal && kv0 + HB - 1 > t.q0);
        const float nl2 = -l2;
#pragma unroll
        for (int e = 0; e < HB; e += 2) {
          float a0, a1;
          ffma2(a0, a1, pv[e], pv[e + 1], p.scale_log2, p.scale_log2, nl2, nl2);
          pv[e] = ex2_approx(a0);
          pv[e + 1] = ex2_approx(a1);
        }
        if (need_mask) {
#pragma unroll
          for (int e = 0; e < HB; ++e) {
            const int kv = kv0 + e;
            pv[e] = (valid && kv < T && (!p.causal || kv <= row)) ? pv[e] : 0.0f;
          }
        }
        if (!(ok = warp_wait(B(bars->dp_full[bj]), par, ctl, p.status))) break;
        tc_fence_after();
        {
          float x[HB];
          tmem_ldn<HB>(dc, x);
#pragma unroll
          for (int e = 0; e < HB; e += 2) {
            float u0, u1, d0, d1;
            fsub2(u0, u1, x[e], x[e + 1], dl, dl);
            fmul2(d0, d1, pv[e], pv[e + 1], u0, u1);  // dS = P (dP - delta)
            x[e] = tf32_round_finite(d0);
            x[e + 1] = tf32_round_finite(d1);
          }
          tmem_stn<HB>(dc, x);
        }
        tmem_wait_st();
        tc_fence_before();
        warp_arrive(B(bars->ds_full[bj]));
      }
      pending = ok;
      prev_row0 = (int64_t)t.bh * T + t.q0 + quad * 32;
      prev_nrows = max(0, min(32, T - (t.q0 + quad * 32)));
      g += t.n;
      ++tn;
    }
    if (ok && pending && warp_wait(B(bars->done), (tn - 1) & 1, ctl, p.status)) {
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

}  // namespace

bool fa2_bwd_dq_persist_supported(const Fa2Problem& p) {
  static const bool off = [] {
    const char* e = std::getenv("CT_FA2_PERSIST_DQ");
    return e && e[0] == '0';
  }();
  return !off && p.D == 64 && p.precision == CT_PRECISION_TF32 && p.T < (1ll << 31) &&
         ((p.T + fa2::kRows - 1) / fa2::kRows) * p.B * p.H < (1ll << 31);
}

int launch_fa2_bwd_dq_persist(const Fa2Problem& pr, Strided4 q, Strided4 k, Strided4 v,
                              Strided4 g, const float* lse, const int64_t ls[3],
                              const float* delta, float* dq, const DeviceInfo& dev,
                              cudaStream_t st) {
  using C = DqpCfg;
  if (!fa2_tma_ok(k) || !fa2_tma_ok(v)) return CT_ERR_UNSUPPORTED_LAYOUT;
  if (!fa2_bwd_dq_persist_supported(pr)) return CT_ERR_UNSUPPORTED_HEAD_DIM;
  static unsigned long long attr_done = 0;
  CUtensorMap tk, tv;
  int rc = make_tmap_bhtd_whole(&tk, k, pr, C::BN);
  if (rc == CT_OK) rc = make_tmap_bhtd_whole(&tv, v, pr, C::BN);
  if (rc != CT_OK) return rc;
  const size_t smem = bwd_smem_bytes_wbuf<C>();
  rc = ensure_smem_attr(fa2_bwd_dq_persist_kernel, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  BwdParams p = make_params(pr, q, g, lse, ls, delta, dq, nullptr, dev);
  const int64_t units = (int64_t)((p.n_tiles + 1) / 2) * p.bh_total;
  // persistent: one CTA per SM (one fits), at most one per unit
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(units, dev.sm_count));
  for (int64_t s0 = 0; s0 < pr.T; s0 += kSegLen) {  // one launch per key segment
    p.seg_lo = (int)s0;
    p.seg_hi = (int)std::min<int64_t>(s0 + kSegLen, pr.T);
    p.accumulate_out = s0 > 0;
    fa2_bwd_dq_persist_kernel<<<(unsigned)ctas, kBwdThreads, smem, st>>>(tk, tv, p);
    rc = check_launch();
    if (rc != CT_OK) return rc;
  }
  return CT_OK;
}

}  // namespace ct
