// gemm_tc.cu -- linear layer out[b] = x[b] @ W[b | 0] + bias on the sm_100a
// tensor cores (tcgen05, kind::tf32, accumulators in TMEM).
//
// Computes what fused_multiply_add computes
// (Transformer_kernels/fused_multiply_add.cuh:10-93, launched by
// Transformer_launchers/linear_layer.cu:28-70): for every batch b and output
// element (i, j), out[b][i][j] = sum_k x[b][i][k] * W[b or 0][k][j] + bias[j].
//
// Persistent kernel, one CTA per SM.  Work units are (128 x BN output tile,
// K slice), taken in the order (batch, tile row, tile column, slice) so that
// the CTAs running at the same time share the x row block in L2.  Warp roles:
//   warp 0      TMA producer (NS-stage ring of 32-deep K blocks of x and W)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-3   TF32 hi/lo split of each stage (3xTF32 mode)
//   warps 4-7   epilogue: thread r <-> tile row r <-> TMEM lane r
// TF32 mode feeds the tiles to the tensor core as loaded: it reads an FP32
// operand as its TF32 truncation (the 13 low mantissa bits dropped), a
// relative bias near 7e-4 on a product, inside the TF32 tolerance.  Rounding
// the tiles in shared memory first would cost about as long as the MMAs.
// Either operand may be K-major (the reduction index is contiguous: x as the
// forward passes it, W^T views) or MN-major (rows/columns contiguous: W as
// stored, x^T views); the layout is picked per call from the strides, so the
// three GEMMs of the linear layer's forward and backward need no copies.
//
// Accumulation.  The tensor core's FP32 accumulator drops the bits below its
// 24-bit mantissa on every addition (round toward zero), a bias that grows
// with the number of MMAs folded into one accumulator.  The K loop is
// therefore cut into chunks of at most chunk_kb(precision) K blocks: 256
// values of K in 3xTF32 (which issues three MMAs per K step; about 5e-6
// relative bias even when every product is positive), 1024 in TF32 (its
// tolerance is 2e-3):
// each chunk accumulates in one of two TMEM buffers and the epilogue warps
// add the chunks with round-to-nearest FP32 additions into a running sum kept
// in a third TMEM region (BN = 128 only; the wider BN = 256 tiles are used
// when K fits one chunk).  The two TMEM buffers also let the epilogue of one
// unit overlap the main loop of the next.
//
// Split K.  When the output has fewer tiles than the GPU has SMs (weight
// gradients, x^T dy over batch*seq rows) and the caller passes a workspace,
// the K range is cut into `slices` and each slice is a work unit.  The slices
// of a tile add into the output in slice order (deterministic): slice s waits
// until the tile's counter in the workspace reads s, adds its partial sum to
// what slices 0..s-1 stored, and sets the counter to s + 1.  Every slice of a
// tile sits in the same round of the persistent loop (the grid is a multiple
// of `slices`), on CTAs of increasing index, so each wait is on a CTA that is
// already running; all waits are bounded.
//
// Fused neighbours (ct_linear_fwd_ex).  The epilogue can apply the MLP's GELU
// to the tile (writing the pre-activation and gelu of it) or multiply by the
// GELU derivative at a given pre-activation (the input gradient through the
// activation; the pre-activation of the next 32 columns is loaded while the
// current ones are finished), and can add into the output.  The column sums
// of the W operand (the bias gradient when W is dY) are formed by the
// preparation warps from the W tiles the units stage anyway: the units of a
// tile column share the K blocks between them (unit of tile row tm: blocks
// kb % tiles_m == tm).  A unit adds its partial sums into its tile row's slot
// of the workspace (the slices of a tile in slice order, like the output);
// the last tile of a column to finish (an atomic counter per tile column)
// adds the slots in tile-row order into the result -- deterministic, and no
// unit waits for another tile.
#include <cstring>

#include "act.cuh"
#include "fa2_common.cuh"

namespace ct {
namespace {

using fa2::mbar_drain;
using fa2::status_raised;
using fa2::warp_wait;

constexpr int kBM = 128;
constexpr int kBK = 32;
// K blocks per TMEM accumulation chunk
__host__ __device__ constexpr int chunk_kb(int split) { return split == 3 ? 8 : 32; }
constexpr int kThreadsG = 256;
constexpr int kPrepWarp0 = 2, kPrepThreads = 64, kEpiWarp0 = 4;

// EPI_: the epilogue (CT_EPILOGUE_*) compiled into this instance, so the plain
// GEMM carries none of the activation code and each variant gets its own
// register allocation.
template <int BN_, int SPLIT_, int NS_, int EPI_ = CT_EPILOGUE_NONE>
struct GemmCfg {
  static constexpr int BN = BN_, SPLIT = SPLIT_, NS = NS_, EPI = EPI_;
  static constexpr uint32_t A_TILE = kBM * kBK * 4u;      // 16 KB
  static constexpr uint32_t B_TILE = (uint32_t)BN * kBK * 4u;
  static constexpr uint32_t RAW = A_TILE + B_TILE;         // bytes TMA writes per stage
  static constexpr uint32_t OFF_A = 0, OFF_B = A_TILE;
  static constexpr uint32_t LO = RAW;                      // 3xTF32 low parts, same layout
  static constexpr uint32_t STAGE = (SPLIT == 3 ? 2u : 1u) * RAW;
  // TMEM: two accumulator buffers, then (BN = 128) the running sum of chunks
  static constexpr uint32_t TC_SUM = 2u * BN;
  static constexpr bool FOLD = BN <= 128;  // multi-chunk K allowed
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(BN == 128 || BN == 256, "tile width");
  static_assert(!FOLD || TC_SUM + BN <= TMEM_COLS, "TMEM budget");
  static_assert(STAGE % 1024 == 0, "stage alignment");
};

struct GemmBars {
  uint64_t full[8], ready[8], empty[8];
  uint64_t acc_full[2], acc_empty[2], stored, mma_final;
  uint64_t db_ready[2], db_free[2], db_stored;  // column-sum partials (w_colsum)
  uint32_t cs_last;
  CtaCtl ctl;
};

struct GemmParams {
  int m, n, batch;
  int tiles_m, tiles_n, units;
  int kb_total;  // number of 32-deep K blocks
  int slices, kb_per_slice;
  int a_mn, b_mn, w_batched;
  const float* bias;
  int64_t bias_s;
  float* out;
  uint32_t* sem;     // one counter per tile (slices > 1)
  uint32_t* cs_cnt;  // one counter per tile column (colsum: finished tiles)
  float* cs_part;    // [tiles_m][n] partial column sums (colsum)
  uint32_t* status;
  int tma_out;    // epilogue stores through TMA (tmO, tmO2) instead of per-thread rows
  int epi;        // CT_EPILOGUE_*
  float* out_act;        // CT_EPILOGUE_GELU: gelu(out)
  const float* act_in;   // CT_EPILOGUE_GELU_GRAD: pre-activation [batch, m, n]
  float* colsum;         // column sums of the W operand (batch == 1, BN == 128), or null
  int accumulate;        // out (and colsum) += instead of =
};

// Epilogue staging: two 32 x 32 FP32 tiles (4 KB each, 128-byte swizzle) per
// epilogue warp, after the stage ring; then (BN = 128) two BN-float buffers
// of column-sum partials.
constexpr uint32_t kStageOut = 4u * 2u * 4096u;
template <class C>
constexpr uint32_t db_bytes() { return C::BN == 128 ? 2u * 128u * 4u : 0u; }

template <class C>
constexpr size_t gemm_smem_bytes() {
  static_assert(sizeof(GemmBars) <= 1024, "barrier block");
  static_assert(1024 + 1024 + (size_t)C::NS * C::STAGE + kStageOut + db_bytes<C>() <= 227 * 1024,
                "shared memory budget");
  return 1024 + 1024 + (size_t)C::NS * C::STAGE + kStageOut + db_bytes<C>();
}

struct Unit {
  int tile, slice, b, m0, n0, kb0, kb1;
};
__device__ __forceinline__ Unit decode_unit(int u, const GemmParams& p, int bn) {
  Unit w;
  w.slice = u % p.slices;
  w.tile = u / p.slices;
  const int tn = w.tile % p.tiles_n;
  const int t = w.tile / p.tiles_n;
  w.b = t / p.tiles_m;
  w.m0 = (t % p.tiles_m) * kBM;
  w.n0 = tn * bn;
  w.kb0 = w.slice * p.kb_per_slice;
  w.kb1 = min(p.kb_total, w.kb0 + p.kb_per_slice);
  return w;
}

__device__ __forceinline__ int n_chunks(int kbs, int ckb) { return (kbs + ckb - 1) / ckb; }

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *sem == want (split-K slice order).
__device__ __forceinline__ bool sem_wait(const uint32_t* sem, uint32_t want, CtaCtl* ctl,
                                         uint32_t* status) {
  if (ld_acquire_gpu(sem) == want) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(status);
  for (uint32_t i = 1;; ++i) {
    __nanosleep(128);
    if (ld_acquire_gpu(sem) == want) return true;
    if ((i & 15u) == 0u) {
      if (ctl->abort || status_raised(status)) {
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

// v[i] += bias[col0 + i] for the columns inside the output.
__device__ __forceinline__ void add_bias32(float (&v)[32], const GemmParams& p, int col0) {
  const int n = p.n;
  if (col0 + 32 <= n && p.bias_s == 1 && ((reinterpret_cast<uintptr_t>(p.bias + col0) & 15u) == 0)) {
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 bb = __ldg(b4 + i);
      v[4 * i] += bb.x; v[4 * i + 1] += bb.y; v[4 * i + 2] += bb.z; v[4 * i + 3] += bb.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < n) v[i] += __ldg(p.bias + (int64_t)(col0 + i) * p.bias_s);
  }
}

// Per-thread epilogue of one 32-column slice of a tile row (outputs TMA
// cannot address): adds what the output holds (later split-K slices, or
// accumulate), then stores the row.
__device__ __forceinline__ void store_row32(float (&v)[32], const GemmParams& p, float* orow,
                                            int col0, bool vec_ok, bool add_existing) {
  const int n = p.n;
  if (col0 >= n) return;
  const bool full = col0 + 32 <= n;
  if (add_existing) {
    if (full && vec_ok) {
      const float4* o4 = reinterpret_cast<const float4*>(orow + col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 q = __ldcg(o4 + i);  // written by another SM: read from L2
        v[4 * i] += q.x; v[4 * i + 1] += q.y; v[4 * i + 2] += q.z; v[4 * i + 3] += q.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < n) v[i] += __ldcg(orow + col0 + i);
    }
  }
  if (full && vec_ok) {
    float4* d4 = reinterpret_cast<float4*>(orow + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < n) orow[col0 + i] = v[i];
  }
}

__device__ __forceinline__ float lds32(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}

// Adds the column sums of one staged W tile (32 K rows) into cs: thread t of
// the 64 preparation threads owns columns t + 64 i.  MN-major tiles are 32-
// column chunks of 32 rows x 128 bytes with 32-byte units XORed with row % 4;
// K-major tiles are BN rows (one per column) of 32 values, 16-byte units
// XORed with row % 8 (summed in stored order).
template <int BN>
__device__ __forceinline__ void colsum_tile(uint32_t b, bool b_mn, uint32_t tid,
                                            float (&cs)[BN / 64]) {
#pragma unroll
  for (int i = 0; i < BN / 64; ++i) {
    const uint32_t col = tid + 64u * i;
    float acc = 0.0f;
    if (b_mn) {
      const uint32_t base = b + (col >> 5) * 4096u + (col & 7u) * 4u, u = (col & 31u) >> 3;
#pragma unroll 8
      for (uint32_t kr = 0; kr < 32; ++kr) acc += lds32(base + kr * 128u + ((u ^ (kr & 3u)) << 5));
    } else {
#pragma unroll
      for (uint32_t u = 0; u < 8; ++u) {
        const float4 x = lds128(b + col * 128u + u * 16u);
        acc += (x.x + x.y) + (x.z + x.w);
      }
    }
    cs[i] += acc;
  }
}

template <class C>
__global__ void __launch_bounds__(kThreadsG, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO,
                     const __grid_constant__ CUtensorMap tmO2, const GemmParams p) {
  constexpr int BN = C::BN, NS = C::NS, SPLIT = C::SPLIT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (status_raised(p.status)) return;
  // the host never launches a multi-chunk unit without TMEM for the sum
  // the host launches multi-chunk BN = 256 tiles only with TMA stores and no split
  if (!C::FOLD && n_chunks(min(p.kb_per_slice, p.kb_total), chunk_kb(SPLIT)) > 1 &&
      (!p.tma_out || p.slices > 1))
    return;
  auto* bars = reinterpret_cast<GemmBars*>(smem_raw);
  const uint32_t tiles = (smem_u32(smem_raw) + (uint32_t)sizeof(GemmBars) + 1023u) & ~1023u;
  CtaCtl* ctl = &bars->ctl;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  auto B = [&](const uint64_t& x) { return smem_u32(&x); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(B(bars->full[s]), 1);
      mbar_init(B(bars->ready[s]), kPrepThreads);
      mbar_init(B(bars->empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(B(bars->acc_full[i]), 1);
      mbar_init(B(bars->acc_empty[i]), 128);
    }
    mbar_init(B(bars->stored), 128);
    mbar_init(B(bars->mma_final), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(B(bars->db_ready[i]), kPrepThreads);
      mbar_init(B(bars->db_free[i]), 128);
    }
    mbar_init(B(bars->db_stored), 128);
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
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int last[NS];
      for (int s = 0; s < NS; ++s) last[s] = -1;
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        const Unit w = decode_unit(u, p, BN);
        const int wb = p.w_batched ? w.b : 0;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = (int)(it % NS), r = (int)(it / NS);
          const uint32_t st = tiles + s * C::STAGE;
          if (r > 0 && !mbar_wait(B(bars->empty[s]), (r - 1) & 1, ctl, p.status)) {
            ok = false;
            break;
          }
          const uint32_t bar = B(bars->full[s]);
          mbar_arrive_expect_tx(bar, C::RAW);
          const int k0 = kb * kBK;
          if (p.a_mn) {
#pragma unroll
            for (int c = 0; c < kBM / 32; ++c)
              tma_load_3d(st + C::OFF_A + c * 4096u, &tmA, bar, w.m0 + 32 * c, k0, w.b);
          } else {
            tma_load_3d(st + C::OFF_A, &tmA, bar, k0, w.m0, w.b);
          }
          if (p.b_mn) {
#pragma unroll
            for (int c = 0; c < BN / 32; ++c)
              tma_load_3d(st + C::OFF_B + c * 4096u, &tmB, bar, w.n0 + 32 * c, k0, wb);
          } else {
            tma_load_3d(st + C::OFF_B, &tmB, bar, k0, w.n0, wb);
          }
          last[s] = r;
        }
      }
      if (ctl->abort) {  // let every issued copy land before the CTA exits
        for (int s = 0; s < NS; ++s)
          if (last[s] >= 0) mbar_drain(B(bars->full[s]), last[s] & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32(kBM, BN, p.a_mn != 0, p.b_mn != 0);
      // stage-0 descriptors; MN-major tiles are 32-element chunks of 32 K rows
      const uint64_t ad0 = p.a_mn ? sdesc_mnmajor(tiles + C::OFF_A, 4096u) : sdesc_kmajor(tiles + C::OFF_A);
      const uint64_t bd0 = p.b_mn ? sdesc_mnmajor(tiles + C::OFF_B, 4096u) : sdesc_kmajor(tiles + C::OFF_B);
      const uint32_t astep = p.a_mn ? 1024u >> 4 : 32u >> 4;  // per 8-deep k step
      const uint32_t bstep = p.b_mn ? 1024u >> 4 : 32u >> 4;
      // the preparation warps release a stage (3xTF32 split, column sums)
      const bool use_ready = SPLIT == 3 || p.colsum != nullptr;
      uint32_t it = 0, ci = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        const Unit w = decode_unit(u, p, BN);
        for (int kc = w.kb0; ok && kc < w.kb1; kc += chunk_kb(SPLIT), ++ci) {
          const int acc = (int)(ci & 1);
          if (ci >= 2 && !mbar_wait(B(bars->acc_empty[acc]), ((ci >> 1) - 1) & 1, ctl, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + acc * BN;
          const int kce = min(w.kb1, kc + chunk_kb(SPLIT));
          for (int kb = kc; kb < kce; ++kb, ++it) {
            const int s = (int)(it % NS), r = (int)(it / NS);
            const uint32_t rbar = use_ready ? B(bars->ready[s]) : B(bars->full[s]);
            if (!mbar_wait(rbar, r & 1, ctl, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = ad0 + ((s * C::STAGE) >> 4);
            const uint64_t bd = bd0 + ((s * C::STAGE) >> 4);
#pragma unroll
            for (int j = 0; j < kBK / 8; ++j) {
              const uint64_t a = ad + j * astep, b = bd + j * bstep;
              umma_tf32_ss(d, a, b, idesc, (kb > kc || j > 0) ? 1u : 0u);
              if constexpr (SPLIT == 3) {
                umma_tf32_ss(d, a, b + (C::LO >> 4), idesc, 1u);
                umma_tf32_ss(d, a + (C::LO >> 4), b, idesc, 1u);
              }
            }
            umma_commit(B(bars->empty[s]));
          }
          if (ok) umma_commit(B(bars->acc_full[acc]));
        }
      }
      umma_commit(B(bars->mma_final));  // nothing of ours in flight after this
      mbar_drain(B(bars->mma_final), 0);
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ---------------------------- 3xTF32 split warps, W column sums
    if (SPLIT == 3 || p.colsum != nullptr) {
      const uint32_t tid = threadIdx.x - kPrepWarp0 * 32;
      float* dbs = reinterpret_cast<float*>(smem_raw + (tiles - smem_u32(smem_raw)) +
                                            NS * C::STAGE + kStageOut);
      uint32_t it = 0, n_db = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        const Unit w = decode_unit(u, p, BN);
        const bool sums = BN == 128 && p.colsum != nullptr;
        const int tm = w.m0 / kBM;  // this unit sums the K blocks kb % tiles_m == tm
        float cs[BN / 64];
#pragma unroll
        for (int i = 0; i < BN / 64; ++i) cs[i] = 0.0f;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = (int)(it % NS), r = (int)(it / NS);
          const uint32_t st = tiles + s * C::STAGE;
          if (!mbar_wait(B(bars->full[s]), r & 1, ctl, p.status)) {
            ok = false;
            break;
          }
          if (sums && kb % p.tiles_m == tm) colsum_tile<BN>(st + C::OFF_B, p.b_mn != 0, tid, cs);
          if constexpr (SPLIT == 3) split_tile_smem<C::RAW, kPrepThreads>(st, st + C::LO, tid);
          fence_proxy_async_smem();
          mbar_arrive(B(bars->ready[s]));
        }
        if (ok && sums) {  // hand the unit's partial column sums to the epilogue
          const uint32_t buf = n_db & 1u;
          if (n_db >= 2 && !mbar_wait(B(bars->db_free[buf]), ((n_db >> 1) - 1) & 1, ctl, p.status))
            break;
#pragma unroll
          for (int i = 0; i < BN / 64; ++i) dbs[buf * 128u + tid + 64u * i] = cs[i];
          mbar_arrive(B(bars->db_ready[buf]));
          ++n_db;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp q owns tile rows 32q..32q+31.  With tma_out each 32 x 32 piece is
    // staged in this warp's swizzled buffer (thread = row) and written by one
    // TMA store -- or, for split-K slices after the first, one TMA add.
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lb = tmem_addr(tmem, 32u * quad, 0);
    const bool vec_ok = (p.n & 3) == 0 && ((reinterpret_cast<uintptr_t>(p.out) & 15u) == 0);
    const uint32_t stg = tiles + NS * C::STAGE + (uint32_t)quad * 2u * 4096u;
    const float* dbs = reinterpret_cast<const float*>(smem_raw + (tiles - smem_u32(smem_raw)) +
                                                      NS * C::STAGE + kStageOut);
    volatile uint32_t* ctl_last = &bars->cs_last;  // "this was the column's last tile"
    if (p.tma_out && lane == 0) {
      tma_prefetch_desc(&tmO);
      if (C::EPI == CT_EPILOGUE_GELU) tma_prefetch_desc(&tmO2);
    }
    uint32_t ci = 0, n_split = 0, n_out = 0, n_db = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      const Unit w = decode_unit(u, p, BN);
      const int row = w.m0 + r;
      const bool valid = row < p.m;
      const bool rows_in = w.m0 + 32 * quad < p.m;  // warp-uniform
      const int64_t row_off = ((int64_t)w.b * p.m + (valid ? row : 0)) * p.n;
      float* orow = p.out + row_off;
      const int nch = n_chunks(w.kb1 - w.kb0, chunk_kb(SPLIT));
      for (int c = 0; c < nch; ++c, ++ci) {
        const int acc = (int)(ci & 1);
        const bool last = c == nch - 1;
        // FOLD (BN = 128): chunks add into the TMEM running sum, the last one
        // writes.  Otherwise (BN = 256, no TMEM left for a sum) every chunk
        // writes: the first stores, later ones add in L2 by TMA, each after
        // this warp's previous writes have completed (fixed order).
        const bool writes = last || !C::FOLD;
        const bool first_write = C::FOLD ? last : c == 0;
        const bool add_mode = p.accumulate || w.slice > 0 || (!C::FOLD && c > 0);
        const bool with_bias = w.slice == 0 && first_write;
        if (!warp_wait(B(bars->acc_full[acc]), (ci >> 1) & 1, ctl, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (first_write && w.slice > 0) {
          if (sem_wait(p.sem + w.tile, (uint32_t)w.slice, ctl, p.status))
            fence_proxy_async_global();  // the TMA add below follows the acquire
          else
            ok = false;  // finish the protocol (free the accumulator), write nothing
        }
        if (!C::FOLD && c > 0 && p.tma_out) {
          if (lane == 0) {
            bulk_wait_group<0>();  // the previous chunk's rows of this warp have landed
            fence_proxy_async_global();
          }
          __syncwarp();
        }
        // GELU-gradient epilogue: the pre-activation of column slice q + 1 is
        // loaded as soon as slice q has used its own (the latency overlaps
        // slice q's staging and store)
        float hnext[32];
        auto load_act = [&](int q) {
          const int col0 = w.n0 + 32 * q;
          const float* arow = p.act_in + row_off;
          if (valid && col0 + 32 <= p.n && vec_ok) {
            const float4* a4 = reinterpret_cast<const float4*>(arow + col0);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 a = __ldg(a4 + i);
              hnext[4 * i] = a.x; hnext[4 * i + 1] = a.y; hnext[4 * i + 2] = a.z; hnext[4 * i + 3] = a.w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              hnext[i] = (valid && col0 + i < p.n) ? __ldg(arow + col0 + i) : 0.0f;
          }
        };
        const bool gelu_grad = C::EPI == CT_EPILOGUE_GELU_GRAD && writes;
        if (gelu_grad) load_act(0);
#pragma unroll 1
        for (int q = 0; q < BN / 32; ++q) {
          float v[32];
          tmem_ld32(lb + acc * BN + 32 * q, v);
          if (C::FOLD && c > 0) {  // running sum of the earlier chunks, round-to-nearest adds
            float s[32];
            tmem_ld32(lb + C::TC_SUM + 32 * q, s);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += s[i];
          }
          const int col0 = w.n0 + 32 * q;
          if (!writes) {
            tmem_st32(lb + C::TC_SUM + 32 * q, v);
          } else if (!__all_sync(0xffffffffu, ok)) {
            // a wait of this unit failed: nothing is written
          } else {
            const bool live = p.tma_out ? (rows_in && col0 < p.n) : valid;
            if (live && with_bias) add_bias32(v, p, col0);
            if (gelu_grad) {  // times gelu'(pre-activation), then fetch the next slice's
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] *= gelu_d(hnext[i]);
              if (q + 1 < BN / 32) load_act(q + 1);
            }
            if (p.tma_out) {
              if (live) {
                // one 32 x 32 piece: stage it, then one TMA store (or add)
                auto put = [&](const CUtensorMap* map, bool add) {
                  const uint32_t buf = stg + (n_out & 1u) * 4096u;
                  if (lane == 0) bulk_wait_group_read<1>();  // the store two pieces back has read buf
                  __syncwarp();
#pragma unroll
                  for (int j = 0; j < 8; ++j)
                    sts128(buf + (uint32_t)lane * 128u + ((uint32_t)(j ^ (lane & 7)) << 4),
                           make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
                  fence_proxy_async_smem();
                  __syncwarp();
                  if (lane == 0) {
                    if (!add) tma_store_3d(map, buf, col0, w.m0 + 32 * quad, w.b);
                    else tma_reduce_add_3d(map, buf, col0, w.m0 + 32 * quad, w.b);
                    bulk_commit_group();
                  }
                  ++n_out;
                };
                put(&tmO, add_mode);
                if (C::EPI == CT_EPILOGUE_GELU) {  // then the activation of the same piece
#pragma unroll
                  for (int i = 0; i < 32; ++i) v[i] = gelu_f(v[i]);
                  put(&tmO2, false);
                }
              }
            } else if (valid) {
              store_row32(v, p, orow, col0, vec_ok, p.accumulate || w.slice > 0);
              if (C::EPI == CT_EPILOGUE_GELU) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = gelu_f(v[i]);
                store_row32(v, p, p.out_act + row_off, col0,
                            vec_ok && ((reinterpret_cast<uintptr_t>(p.out_act) & 15u) == 0), false);
              }
            }
          }
        }
        if (!last) tmem_wait_st();
        tc_fence_before();
        mbar_arrive(B(bars->acc_empty[acc]));
      }
      if (!__all_sync(0xffffffffu, ok)) break;
      if (BN == 128 && p.colsum != nullptr) {
        // the unit's partial W column sums into its tile row's slot (the
        // slices of this tile add in slice order: this slice holds the tile's
        // counter here); the tile column's last tile adds the slots up
        const uint32_t buf = n_db & 1u;
        const int tn = w.n0 / BN, tm = w.m0 / kBM;
        if (!warp_wait(B(bars->db_ready[buf]), (n_db >> 1) & 1, ctl, p.status)) break;
        const int col = r, j = w.n0 + col;
        const bool in = col < BN && j < p.n;
        float* slot = p.cs_part + (int64_t)tm * p.n;
        if (in) slot[j] = w.slice > 0 ? __ldcg(slot + j) + dbs[buf * 128u + col] : dbs[buf * 128u + col];
        mbar_arrive(B(bars->db_free[buf]));
        if (w.slice == p.slices - 1) {  // this tile's column sums are complete
          __threadfence();
          mbar_arrive(B(bars->db_stored));
          if (!mbar_wait(B(bars->db_stored), n_db & 1, ctl, p.status)) {
            ok = false;
          } else if (r == 0) {
            *ctl_last = atomicAdd(p.cs_cnt + tn, 1u) == (uint32_t)(p.tiles_m - 1) ? 1u : 0u;
          }
          // every epilogue thread learns whether this was the column's last tile
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (ok && *ctl_last && in) {
            __threadfence();
            float sum = p.accumulate ? p.colsum[j] : 0.0f;
            for (int t = 0; t < p.tiles_m; ++t) sum += __ldcg(p.cs_part + (int64_t)t * p.n + j);
            p.colsum[j] = sum;
          }
        }
        ++n_db;
      }
      if (p.slices > 1) {  // publish this slice: counter = slice + 1
        if (p.tma_out && lane == 0) {
          bulk_wait_group<0>();  // this warp's TMA writes are done
          fence_proxy_async_global();
        }
        __syncwarp();
        __threadfence();
        mbar_arrive(B(bars->stored));
        if (r == 0) {
          if (mbar_wait(B(bars->stored), n_split & 1, ctl, p.status))
            st_release_gpu(p.sem + w.tile, (uint32_t)w.slice + 1u);
          else
            ok = false;
        }
        ++n_split;
      }
    }
    if (p.tma_out && lane == 0) bulk_wait_group<0>();  // staging buffers are read before exit
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Operand layout of x (A) and W (B) from their strides: K-major when the
// reduction index is contiguous, MN-major when the row (x) / column (W) index
// is.  Returns false when neither holds.
bool a_layout(const GemmProblem& g, bool* mn) {
  if (g.xs[2] == 1) { *mn = false; return true; }
  if (g.xs[1] == 1) { *mn = true; return true; }
  return false;
}
bool b_layout(const GemmProblem& g, bool* mn) {
  if (g.ws[2] == 1) { *mn = true; return true; }
  if (g.ws[1] == 1) { *mn = false; return true; }
  return false;
}

// Byte stride of a TMA dimension; a dimension of extent 1 gets a stride that
// is never used but satisfies the encoder (a non-zero multiple of 16 that
// spans the dimensions inside it).
uint64_t dim_stride(int64_t elems, int64_t extent, uint64_t fallback) {
  return extent > 1 ? (uint64_t)elems * 4u : fallback;
}
uint64_t row_bytes16(int64_t inner) { return ((uint64_t)inner * 4u + 15u) & ~15ull; }

int make_maps(const GemmProblem& g, bool a_mn, bool b_mn, int bn, CUtensorMap* ta,
              CUtensorMap* tb) {
  const int64_t wb = g.ws[0] == 0 ? 1 : g.batch;
  {
    const int64_t inner = a_mn ? g.m : g.k, outer = a_mn ? g.k : g.m;
    const int64_t os = a_mn ? g.xs[2] : g.xs[1];
    const uint64_t s1 = dim_stride(os, outer, row_bytes16(inner));
    const uint64_t dims[3] = {(uint64_t)inner, (uint64_t)outer, (uint64_t)g.batch};
    const uint64_t strides[2] = {s1, dim_stride(g.xs[0], g.batch, s1 * (uint64_t)outer)};
    const uint32_t box[3] = {32u, a_mn ? (uint32_t)kBK : (uint32_t)kBM, 1u};
    const int rc = make_tmap_f32(ta, g.x, 3, dims, strides, box, a_mn);
    if (rc != CT_OK) return rc;
  }
  {
    const int64_t inner = b_mn ? g.n : g.k, outer = b_mn ? g.k : g.n;
    const int64_t os = b_mn ? g.ws[1] : g.ws[2];
    const uint64_t s1 = dim_stride(os, outer, row_bytes16(inner));
    const uint64_t dims[3] = {(uint64_t)inner, (uint64_t)outer, (uint64_t)wb};
    const uint64_t strides[2] = {s1, dim_stride(g.ws[0], wb, s1 * (uint64_t)outer)};
    const uint32_t box[3] = {32u, b_mn ? (uint32_t)kBK : (uint32_t)bn, 1u};
    return make_tmap_f32(tb, g.w, 3, dims, strides, box, b_mn);
  }
}

int64_t tile_count(const GemmProblem& g, int bn) {
  return g.batch * ((g.m + kBM - 1) / kBM) * ((g.n + bn - 1) / bn);
}

// K split: slices of whole accumulation chunks, enough to give every SM a
// unit, each slice at least two chunks deep.
void pick_split(const GemmProblem& g, int bn, int sms, bool have_ws, int ckb, int* slices,
                int* kbps) {
  const int kb_total = (int)((g.k + kBK - 1) / kBK);
  *slices = 1;
  *kbps = kb_total;
  const int64_t tiles = tile_count(g, bn);
  // a GELU epilogue needs the whole sum of a tile at once
  if (!have_ws || tiles * 2 > sms || g.epilogue != CT_EPILOGUE_NONE) return;
  int s = (int)(sms / tiles);
  const int max_s = kb_total / (2 * ckb);
  if (s > max_s) s = max_s;
  if (s < 2) return;
  int per = (kb_total + s - 1) / s;
  per = (per + ckb - 1) / ckb * ckb;
  *kbps = per;
  *slices = (kb_total + per - 1) / per;
}

// TMA map of a dense [batch, m, n] output with 32 x 32 boxes (epilogue);
// false when TMA cannot address it (n not a multiple of 4, unaligned base).
bool make_out_map(const GemmProblem& g, float* out, CUtensorMap* to) {
  if ((g.n & 3) != 0 || (reinterpret_cast<uintptr_t>(out) & 15u) != 0) return false;
  const uint64_t s1 = (uint64_t)g.n * 4u;
  const uint64_t dims[3] = {(uint64_t)g.n, (uint64_t)g.m, (uint64_t)g.batch};
  const uint64_t strides[2] = {s1, s1 * (uint64_t)g.m};
  const uint32_t box[3] = {32u, 32u, 1u};
  return make_tmap_f32(to, out, 3, dims, strides, box, false) == CT_OK;
}

template <class C>
int run_linear(const GemmProblem& g, bool a_mn, bool b_mn, void* ws, size_t ws_bytes,
               const DeviceInfo& dev, cudaStream_t st) {
  static unsigned long long attr_done = 0;
  CUtensorMap ta, tb, to, to2;
  int rc = make_maps(g, a_mn, b_mn, C::BN, &ta, &tb);
  if (rc != CT_OK) return rc;
  std::memset(&to2, 0, sizeof(to2));
  bool tma_out = make_out_map(g, g.out, &to);
  if (tma_out && g.epilogue == CT_EPILOGUE_GELU) tma_out = make_out_map(g, g.out_act, &to2);
  if (!tma_out) std::memset(&to, 0, sizeof(to));
  const size_t smem = gemm_smem_bytes<C>();
  rc = ensure_smem_attr(linear_tc_kernel<C>, smem, dev.device, &attr_done);
  if (rc != CT_OK) return rc;
  GemmParams p;
  p.m = (int)g.m;
  p.n = (int)g.n;
  p.batch = (int)g.batch;
  p.tiles_m = (int)((g.m + kBM - 1) / kBM);
  p.tiles_n = (int)((g.n + C::BN - 1) / C::BN);
  p.kb_total = (int)((g.k + kBK - 1) / kBK);
  const int64_t tiles = tile_count(g, C::BN);
  // counters: one per tile (split-K order), then one per tile column (column
  // sums); then the column sums' [tiles_m][n] partial slots
  const size_t sem_bytes = (size_t)(tiles + (g.n + C::BN - 1) / C::BN) * 4u;
  const size_t cs_part_off = (sem_bytes + 255) / 256 * 256;
  const size_t need = g.w_colsum ? cs_part_off + (size_t)((g.m + kBM - 1) / kBM) * g.n * 4u
                                 : sem_bytes;
  const bool have_ws = ws != nullptr && ws_bytes >= need;
  if (g.w_colsum && !have_ws) return CT_ERR_WORKSPACE_TOO_SMALL;
  pick_split(g, C::BN, dev.sm_count, have_ws, chunk_kb(C::SPLIT), &p.slices, &p.kb_per_slice);
  if (!C::FOLD && p.kb_per_slice > chunk_kb(C::SPLIT) && (!tma_out || p.slices > 1))
    return CT_ERR_UNSUPPORTED_LAYOUT;  // the L2 fold needs TMA stores (caller falls back)
  p.units = (int)(tiles * p.slices);
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.w_batched = g.ws[0] != 0;
  p.bias = g.bias;
  p.bias_s = g.bias_s;
  p.out = g.out;
  p.sem = static_cast<uint32_t*>(ws);
  p.cs_cnt = p.sem + tiles;
  p.cs_part = reinterpret_cast<float*>(static_cast<char*>(ws) + cs_part_off);
  p.status = dev.status;
  p.tma_out = tma_out ? 1 : 0;
  p.epi = C::EPI;
  p.out_act = g.out_act;
  p.act_in = g.act_in;
  p.colsum = g.w_colsum;
  p.accumulate = g.accumulate ? 1 : 0;
  if ((g.epilogue != C::EPI) || ((C::EPI != CT_EPILOGUE_NONE || p.colsum) && (!C::FOLD || C::BN != 128)))
    return CT_ERR_UNSUPPORTED_LAYOUT;  // (pick_bn picks 128-wide tiles for these)
  int grid = p.units < dev.sm_count ? p.units : dev.sm_count;
  if (p.slices > 1) grid = grid / p.slices * p.slices;  // whole tiles per round
  if ((p.slices > 1 || p.colsum) && cudaMemsetAsync(ws, 0, sem_bytes, st) != cudaSuccess)
    return CT_ERR_CUDA;
  linear_tc_kernel<C><<<grid, kThreadsG, smem, st>>>(ta, tb, to, to2, p);
  return check_launch();
}

// Tile width: BN = 256 has no TMEM left for a running sum, so K beyond one
// accumulation chunk is folded in L2 (at most four chunks, TMA-storable
// output, no split-K); otherwise the choice minimises (waves of tiles) x (tile
// cost), a 128-wide tile costing a little more than half a 256-wide one (x
// re-read, per-tile overhead).  The
// environment variable CT_GEMM_BN (128 or 256) overrides it (tuning).
int pick_bn(const GemmProblem& g, int sms) {
  const int64_t kb = (g.k + kBK - 1) / kBK;
  const int ckb = chunk_kb(g.precision == CT_PRECISION_3XTF32 ? 3 : 1);
  // fused epilogues and W column sums run on 128-wide tiles (the TMEM running
  // sum holds the whole K before the epilogue; room for the sum buffers)
  if (g.n <= 128 || g.epilogue != CT_EPILOGUE_NONE || g.w_colsum) return 128;
  if (kb > ckb) {  // several chunks: BN = 256 folds them in L2 (TMA stores, no split-K)
    const bool tma_out = (g.n & 3) == 0 && (reinterpret_cast<uintptr_t>(g.out) & 15u) == 0;
    if (!tma_out || g.accumulate || kb > 4 * ckb || tile_count(g, 256) * 2 <= sms) return 128;
  }
  static const int env = [] {
    const char* e = std::getenv("CT_GEMM_BN");
    return e ? std::atoi(e) : 0;
  }();
  if (env == 128 || env == 256) return env;
  auto cost = [&](int bn, double rel) {
    const int64_t waves = (tile_count(g, bn) + sms - 1) / sms;
    return (double)waves * rel;
  };
  // Relative cost of a 128-wide tile, measured on the linear layer's shapes
  // (M = 16384, K = 384 / 1536): 3xTF32's BN = 256 ring holds only two stages,
  // so there the narrow tile costs relatively less.
  const double rel128 = g.precision == CT_PRECISION_3XTF32 ? 0.53 : 0.59;
  return cost(256, 1.0) <= cost(128, rel128) ? 256 : 128;
}

}  // namespace

size_t linear_workspace_bytes(int64_t batch, int64_t m, int64_t n) {
  if (batch <= 0 || m <= 0 || n <= 0) return 0;
  // counters (split-K, column sums), then (batch 1) the column sums' partial slots
  const int64_t tiles = batch * ((m + kBM - 1) / kBM) * ((n + 127) / 128) + (n + 127) / 128;
  const int64_t slots = batch == 1 ? ((m + kBM - 1) / kBM) * n : 0;
  return (size_t)((tiles * 4 + 255) / 256 * 256 + slots * 4);
}

bool linear_tc_supported(const GemmProblem& g) {
  if (g.precision != CT_PRECISION_3XTF32 && g.precision != CT_PRECISION_TF32) return false;
  if (g.m <= 0 || g.n <= 0 || g.k <= 0 || g.batch <= 0) return false;
  if (g.m >= (1ll << 31) || g.n >= (1ll << 31) || g.k >= (1ll << 31) || g.batch >= (1ll << 31))
    return false;
  if (tile_count(g, 128) >= (1ll << 26)) return false;  // units (tiles x slices) fit an int
  bool amn, bmn;
  if (!a_layout(g, &amn) || !b_layout(g, &bmn)) return false;
  const int64_t a_outer[2] = {amn ? g.xs[2] : g.xs[1], g.xs[0]};
  const int64_t b_outer[2] = {bmn ? g.ws[1] : g.ws[2], g.ws[0]};
  auto ok = [](const void* base, const int64_t* outer, int64_t ext1, int64_t ext2) {
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
    if (ext1 > 1 && (outer[0] <= 0 || (outer[0] * 4) % 16 != 0)) return false;
    if (ext2 > 1 && (outer[1] <= 0 || (outer[1] * 4) % 16 != 0)) return false;
    return true;
  };
  const int64_t wb = g.ws[0] == 0 ? 1 : g.batch;
  return ok(g.x, a_outer, amn ? g.k : g.m, g.batch) && ok(g.w, b_outer, bmn ? g.k : g.n, wb);
}

int launch_linear_tc(const GemmProblem& g, void* ws, size_t ws_bytes, const DeviceInfo& dev,
                     cudaStream_t st) {
  if (!linear_tc_supported(g)) return CT_ERR_UNSUPPORTED_LAYOUT;
  bool amn = false, bmn = false;
  a_layout(g, &amn);
  b_layout(g, &bmn);
  const bool split = g.precision == CT_PRECISION_3XTF32;
  if (g.epilogue == CT_EPILOGUE_GELU)
    return split ? run_linear<GemmCfg<128, 3, 3, CT_EPILOGUE_GELU>>(g, amn, bmn, ws, ws_bytes, dev, st)
                 : run_linear<GemmCfg<128, 1, 6, CT_EPILOGUE_GELU>>(g, amn, bmn, ws, ws_bytes, dev, st);
  if (g.epilogue == CT_EPILOGUE_GELU_GRAD)
    return split ? run_linear<GemmCfg<128, 3, 3, CT_EPILOGUE_GELU_GRAD>>(g, amn, bmn, ws, ws_bytes,
                                                                          dev, st)
                 : run_linear<GemmCfg<128, 1, 6, CT_EPILOGUE_GELU_GRAD>>(g, amn, bmn, ws, ws_bytes,
                                                                          dev, st);
  if (pick_bn(g, dev.sm_count) == 256)
    return split ? run_linear<GemmCfg<256, 3, 2>>(g, amn, bmn, ws, ws_bytes, dev, st)
                 : run_linear<GemmCfg<256, 1, 4>>(g, amn, bmn, ws, ws_bytes, dev, st);
  return split ? run_linear<GemmCfg<128, 3, 3>>(g, amn, bmn, ws, ws_bytes, dev, st)
               : run_linear<GemmCfg<128, 1, 6>>(g, amn, bmn, ws, ws_bytes, dev, st);
}

}  // namespace ct
