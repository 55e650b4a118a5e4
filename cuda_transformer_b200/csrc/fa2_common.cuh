// fa2_common.cuh -- pieces shared by the tcgen05 FlashAttention-2 kernels.
//
// Conventions of every FA2 tensor-core kernel here:
//  * 128-row stationary tile per CTA (M = 128 MMAs); row r of the tile lives
//    in TMEM lane r and is owned by thread r of the 4-warp "row" warpgroup
//    (warps 4..7, warp w reading lanes 32*(w%4) .. +31).
//  * Streamed tiles (K/V in the forward and dQ pass, Q/dO in the dK/dV pass)
//    arrive by TMA into 1024-byte aligned shared memory in the 128-byte swizzle
//    with 32-float boxes, and are read by the tensor core either K-major (the
//    head dim is the reduction) or MN-major (the sequence is the reduction).
//  * Precision: SPLIT == 3 stores every operand as a TF32 hi/lo pair and issues
//    hi*hi + hi*lo + lo*hi; SPLIT == 1 issues one TF32 MMA per product on
//    operands rounded to the nearest TF32 (the tensor core truncates raw FP32).
//  * Warps 2, 3, 8, 9 prepare every landed tile before the MMA reads it: the hi/lo
//    split (SPLIT == 3) or the in-place rounding (SPLIT == 1).
#pragma once

#include <cmath>
#include <cstdlib>

#include "ct_internal.h"
#include "tc_ptx.cuh"

namespace ct {
namespace fa2 {

constexpr int kRows = 128;        // stationary rows per CTA
constexpr int kThreads = 352;     // 11 warps
constexpr int kRowWarp0 = 4;      // first warp of the row warpgroup (4 warps)
// Warp w runs on SM sub-partition w % 4.  The four tile-preparation warps
// (2, 3, 8, 9) sit one per sub-partition, so the split / rounding work of a
// landed tile spreads over all four schedulers instead of competing with two
// of the row warps for issue slots.  (ptxas sizes registers for 12 warps
// whether the block has 9 or 11, so the two extra warps cost no registers.)
constexpr int kSplitThreads = 128;
constexpr int kPrepWarps = 4;
// Warp 1 issues one group of tcgen05.mma chains and warp 10 the other.  An
// issuing thread waits for each MMA to be accepted, so one thread drives the
// tensor pipe at ~45 cycles per N <= 64 MMA at best and idles it whenever it
// waits on a barrier; two threads feeding independent accumulators
// interleave and reach the pipe's full rate (measured on B200).
constexpr int kIssuer2Warp = 10;
__device__ __forceinline__ bool is_prep_warp(int w) { return w == 2 || w == 3 || w == 8 || w == 9; }
// Index 0..127 of this thread among the preparation warps.
__device__ __forceinline__ uint32_t prep_tid() {
  const int w = threadIdx.x / 32;
  return (uint32_t)((((w & 1) + (w >= 8 ? 2 : 0)) * 32) + (threadIdx.x & 31));
}
constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kLog2e = 1.44269504088896340736f;

struct Ptr4 {
  const float* p;
  int64_t s0, s1, s2, s3;
  __device__ __forceinline__ const float* row(int64_t b, int64_t h, int64_t t) const {
    return p + b * s0 + h * s1 + t * s2;
  }
};

// Loads 32 consecutive head-dim values of one row (zeros when !valid).
__device__ __forceinline__ void load_row32(const Ptr4& t, const float* rowp, int c0, bool valid,
                                           bool vec, float (&x)[32]) {
  if (!valid) {
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = 0.0f;
    return;
  }
  if (vec) {
    const float4* p4 = reinterpret_cast<const float4*>(rowp + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = __ldg(p4 + i);
      x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = __ldg(rowp + (int64_t)(c0 + i) * t.s3);
  }
}

// Writes one D-wide row into TMEM columns [col, col + D): the TF32 hi part and
// its low part into [col + D, col + 2D) when SPLIT == 3, the value rounded to
// the nearest TF32 when SPLIT == 1.  Caller waits/fences.
template <int D, int SPLIT>
__device__ __forceinline__ void row_to_tmem(const Ptr4& t, const float* rowp, bool valid,
                                            bool vec, uint32_t lane_base, uint32_t col) {
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    float x[32];
    load_row32(t, rowp, 32 * c, valid, vec, x);
    if constexpr (SPLIT == 3) {
      float lo[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float h, l;
        tf32_split(x[i], h, l);
        x[i] = h;
        lo[i] = l;
      }
      tmem_st32(lane_base + col + D + 32 * c, lo);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = tf32_round(x[i]);
    }
    tmem_st32(lane_base + col + 32 * c, x);
  }
}

// 3xTF32 split of two values (tf32_split with the subtraction packed).
__device__ __forceinline__ void tf32_split2(float x0, float x1, float& h0, float& h1, float& l0,
                                            float& l1) {
  const float a = tf32_trunc(x0), b = tf32_trunc(x1);
  fsub2(l0, l1, x0, x1, a, b);
  h0 = a;
  h1 = b;
}

// Causal / ragged mask of 32 consecutive score columns starting at key kv0:
// column kv stays iff kv < T and (!causal || kv <= row); others become -inf.
__device__ __forceinline__ void mask_cols32(float (&t)[32], int kv0, int T, int causal, int row) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int kv = kv0 + i;
    if (!(kv < T && (!causal || kv <= row))) t[i] = -INFINITY;
  }
}

// mask_cols32 and max32 for N (16 or 32) columns.
template <int N>
__device__ __forceinline__ void mask_cols(float (&t)[N], int kv0, int T, int causal, int row) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int kv = kv0 + i;
    if (!(kv < T && (!causal || kv <= row))) t[i] = -INFINITY;
  }
}
template <int N>
__device__ __forceinline__ float maxn(const float (&t)[N]) {
  float m = t[0];
#pragma unroll
  for (int i = 1; i < N; ++i) m = fmaxf(m, t[i]);
  return m;
}

// 32 consecutive floats from 16-byte aligned shared memory (every lane of a
// warp reads the same address: broadcast).
__device__ __forceinline__ void load_vec32(const float* src, float (&v)[32]) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 x = s4[i];
    v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
  }
}

// N = 16 or 32 columns of one TMEM lane quarter (load waits, store does not).
template <int N>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, float (&v)[N]) {
  static_assert(N == 16 || N == 32, "TMEM access width");
  if constexpr (N == 32) tmem_ld32(taddr, v);
  else tmem_ld16(taddr, v);
}
template <int N>
__device__ __forceinline__ void tmem_stn(uint32_t taddr, const float (&v)[N]) {
  static_assert(N == 16 || N == 32, "TMEM access width");
  if constexpr (N == 32) tmem_st32(taddr, v);
  else tmem_st16(taddr, v);
}
// N consecutive floats (N % 4 == 0) from 16-byte aligned shared memory (broadcast).
template <int N>
__device__ __forceinline__ void load_vecn(const float* src, float (&v)[N]) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    const float4 x = s4[i];
    v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
  }
}

__device__ __forceinline__ float max32(const float (&t)[32]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(fmaxf(t[4 * i], t[4 * i + 1]), fmaxf(t[4 * i + 2], t[4 * i + 3]));
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}

// Stores NC (16 or a multiple of 32) TMEM columns [col, col+NC) of this
// thread's lane times `scale` to dense global memory.  With `add_partial`,
// dst already holds the previous segments' sum (kSegLen): the result is
// dst + TMEM * scale.
template <int NC>
__device__ __forceinline__ void tmem_cols_to_global(uint32_t lane_base, uint32_t col, float scale,
                                                    float* dst, bool valid,
                                                    bool add_partial = false) {
  constexpr int CW = NC < 32 ? NC : 32;
  static_assert(NC % CW == 0, "column count");
#pragma unroll
  for (int c = 0; c < NC / CW; ++c) {
    float v[CW];
    tmem_ldn<CW>(lane_base + col + CW * c, v);
    if (valid) {
      float4* d4 = reinterpret_cast<float4*>(dst + CW * c);
#pragma unroll
      for (int i = 0; i < CW / 4; ++i) {
        float4 a = make_float4(v[4 * i] * scale, v[4 * i + 1] * scale, v[4 * i + 2] * scale,
                               v[4 * i + 3] * scale);
        if (add_partial) {
          const float4 o = d4[i];
          a = make_float4(o.x + a.x, o.y + a.y, o.z + a.z, o.w + a.w);
        }
        d4[i] = a;
      }
    }
  }
}
// A D-wide row: tmem_cols_to_global over D columns.
template <int D>
__device__ __forceinline__ void tmem_row_to_global(uint32_t lane_base, uint32_t col, float scale,
                                                   float* dst, bool valid,
                                                   bool add_partial = false) {
  tmem_cols_to_global<D>(lane_base, col, scale, dst, valid, add_partial);
}

// Row warps' write-out buffer: 32 rows x 16 columns per warp, rows padded to
// 17 floats (conflict-free column writes and row reads); eight row warps.
constexpr uint32_t kRowWbufFloats = 32 * 17;
constexpr size_t kRowWbufBytes = 8 * (size_t)kRowWbufFloats * 4;

// Writes TMEM columns [col, col + NC) of a row warp's 32 lanes (lane r = row
// r), times `scale`, to rows 0 .. nrows-1 of `out` (row stride ld floats),
// 16 columns at a time through the warp's buffer: each store instruction then
// writes two 64-byte row segments, where a thread storing its own row would
// scatter 16-byte pieces over 32 rows.  `accumulate` adds to what out holds.
// `scale` may differ per lane (row).  All 32 lanes call it.
template <int NC>
__device__ __forceinline__ void warp_rows_to_global(uint32_t col, float scale, float* wbuf,
                                                    float* out, int nrows, int64_t ld,
                                                    bool accumulate) {
  static_assert(NC % 16 == 0, "column count");
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < NC / 16; ++c) {
    float x[16];
    tmem_ld16(col + 16 * c, x);
#pragma unroll
    for (int e = 0; e < 16; ++e) wbuf[lane * 17 + e] = x[e] * scale;
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int r = 2 * k + (lane >> 4), cc = lane & 15;
      if (r < nrows) {
        float* dst = out + (int64_t)r * ld + 16 * c + cc;
        const float v = wbuf[r * 17 + cc];
        *dst = accumulate ? *dst + v : v;
      }
    }
    __syncwarp();
  }
}

// Long reductions.  The tensor core adds each MMA's products into its FP32
// accumulator with a rounding biased toward zero: the relative error of a
// gradient grows with the reduction length (measured in 3xTF32: ~4e-5 at
// 4096 keys, 1.5e-4 at 16384).  The backward therefore reduces over at most
// kSegLen keys (dQ) or queries (dK, dV) per launch: longer sequences run one
// launch per segment, each adding its FP32 partial gradient into the output
// written by the previous one (round-to-nearest adds, fixed order:
// deterministic), which keeps the error at the one-segment level at any
// length.  The step loops are the same for every segment.
constexpr int kSegLen = 4096;

// D (+)= A x B over K = KDIM in steps of 8: A from TMEM columns a_hi (+ a_lo
// for the 3xTF32 low part), B from a shared-memory tile whose k-step-0
// descriptor is `bd` (its low copy TILE bytes further).  Descriptors advance
// by compile-time offsets (start address field counts 16-byte units):
//   K-major tile of BN rows: k-step k at (k/4)*BN*128 + (k%4)*32 bytes
//   MN-major tile:           k-step k at k*1024 bytes
template <int SPLIT, int KDIM, bool MN_MAJOR, int BN, uint32_t TILE>
__device__ __forceinline__ void mma_chain(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint64_t bd,
                                          uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int k = 0; k < KDIM / 8; ++k) {
    const uint32_t off = MN_MAJOR ? (uint32_t)k * 1024u
                                  : (uint32_t)(k / 4) * BN * 128u + (uint32_t)(k % 4) * 32u;
    const uint64_t bh = bd + (off >> 4);
    umma_tf32_ts(d, a_hi + 8 * k, bh, idesc, (accumulate || k > 0) ? 1u : 0u);
    if constexpr (SPLIT == 3) {
      umma_tf32_ts(d, a_hi + 8 * k, bh + (TILE >> 4), idesc, 1u);
      umma_tf32_ts(d, a_lo + 8 * k, bh, idesc, 1u);
    }
  }
}

// 3xTF32 product D = A x B over K = KDIM into 2*BN accumulator columns, B a
// K-major tile whose 32-column chunks (stride KCH bytes) each hold BN raw rows
// followed by the BN rows of their low parts.  Per k-step, one MMA of N = 2*BN
// gives [a_hi*b_hi | a_hi*b_lo] and one of N = BN adds a_lo*b_hi to the first
// half: the product is the sum of the two halves, and N = 2*BN costs the
// tensor pipe's issue no more than N = BN does when BN <= 32.
template <int KDIM, uint32_t KCH>
__device__ __forceinline__ void mma_chain_kil(uint32_t d, uint32_t a_hi, uint32_t a_lo,
                                              uint64_t bd, uint32_t id_wide, uint32_t id_narrow) {
#pragma unroll
  for (int k = 0; k < KDIM / 8; ++k) {
    const uint32_t off = (uint32_t)(k / 4) * KCH + (uint32_t)(k % 4) * 32u;
    const uint64_t bh = bd + (off >> 4);
    umma_tf32_ts(d, a_hi + 8 * k, bh, id_wide, k > 0 ? 1u : 0u);
    umma_tf32_ts(d, a_lo + 8 * k, bh, id_narrow, 1u);
  }
}

// 3xTF32 product D (+)= A x B over K = KDIM with B an MN-major tile of N
// columns whose low parts follow it at the same chunk stride, i.e. [B_hi | B_lo]
// is one MN-major operand of 2N columns.  Per k-step, one MMA of N = 2N gives
// [a_hi*b_hi | a_hi*b_lo] and one of N adds a_lo*b_hi to the first half: the
// product is the sum of the accumulator's two halves.
template <int KDIM>
__device__ __forceinline__ void mma_chain_mn2(uint32_t d, uint32_t a_hi, uint32_t a_lo,
                                              uint64_t bd, uint32_t id_wide, uint32_t id_narrow,
                                              bool accumulate) {
#pragma unroll
  for (int k = 0; k < KDIM / 8; ++k) {
    const uint64_t bh = bd + (((uint32_t)k * 1024u) >> 4);
    umma_tf32_ts(d, a_hi + 8 * k, bh, id_wide, (accumulate || k > 0) ? 1u : 0u);
    umma_tf32_ts(d, a_lo + 8 * k, bh, id_narrow, 1u);
  }
}

// Maps a linear CTA index to (tile, batch*head).  Heads are taken in groups of
// `group` (the last group may be smaller): all tiles of a group run before the
// next group, so resident CTAs share a few heads' streamed operands in L2,
// and inside a group consecutive CTAs alternate between its heads, so they do
// not all stream the same tile at the same moment.  `heavy_first_desc` lists a
// head's tiles from the last to the first (causal forward / dQ do the most
// work on late query tiles; dK/dV on early key tiles keep ascending order).
// cta_tile_at takes the linear index explicitly (a ticket drawn at run time).
__device__ __forceinline__ void cta_tile_at(unsigned idx, int n_tiles, int bh_total, int group,
                                            bool heavy_first_desc, int& tile, int& bh) {
  const int per_group = group * n_tiles;
  const int g = (int)(idx / per_group);
  const int r = (int)(idx % per_group);
  const int gsize = min(group, bh_total - g * group);
  const int t = r / gsize;
  bh = g * group + r % gsize;
  tile = heavy_first_desc ? n_tiles - 1 - t : t;
}
__device__ __forceinline__ void cta_tile(int n_tiles, int bh_total, int group,
                                         bool heavy_first_desc, int& tile, int& bh) {
  cta_tile_at(blockIdx.x, n_tiles, bh_total, group, heavy_first_desc, tile, bh);
}

// Loads tile row block `r0` of head (h, b) into `dst`: one copy through a
// whole-tile map (WHOLE), else one copy per 32-column chunk at chunk stride
// `chunk` bytes (interleaved hi/lo layouts leave room between the chunks).
template <bool WHOLE, int D>
__device__ __forceinline__ void tma_load_tile(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                              int r0, int h, int b, uint32_t chunk) {
  if constexpr (WHOLE) {
    tma_load_5d(dst, map, bar, 0, r0, 0, h, b);
  } else {
#pragma unroll
    for (int c = 0; c < D / 32; ++c) tma_load_4d(dst + c * chunk, map, bar, 32 * c, r0, h, b);
  }
}

// Drain-wait used on teardown: ignores the CTA abort flag, bounded by time.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > CT_WAIT_TIMEOUT_NS) return;
  }
}

// Warp-uniform bounded wait (all 32 lanes must call it).  Every lane polls:
// a warp with only lane 0 suspended in try_wait wakes much later (measured).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, CtaCtl* ctl,
                                          uint32_t* status) {
  const bool ok = mbar_wait(bar, parity, ctl, status);
  return __all_sync(0xffffffffu, ok);
}

// Warp-uniform arrive (all 32 lanes must call it): the warp synchronises,
// which orders every lane's earlier writes (and, after
// tcgen05.fence::before_thread_sync, its tensor-memory stores) before lane 0's
// single arrival.  Barriers armed with warp_arrive count warps, not threads.
__device__ __forceinline__ void warp_arrive(uint32_t bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ bool status_raised(const uint32_t* status) {
  return *reinterpret_cast<const volatile uint32_t*>(status) != 0u;
}

}  // namespace fa2

// Host helper: TMA map for an FP32 [B,H,T,D] tensor with a {32, rows} box, in
// the K-major (SWIZZLE_128B) or MN-major (SWIZZLE_128B_ATOM_32B) tile layout.
inline int make_tmap_bhtd(CUtensorMap* map, const Strided4& t, const Fa2Problem& p, int rows,
                          bool mn_major = false) {
  const uint64_t dims[4] = {(uint64_t)p.D, (uint64_t)p.T, (uint64_t)p.H, (uint64_t)p.B};
  const uint64_t strides[3] = {(uint64_t)t.s[2] * 4u, (uint64_t)t.s[1] * 4u, (uint64_t)t.s[0] * 4u};
  const uint32_t box[4] = {32u, (uint32_t)rows, 1u, 1u};
  return make_tmap_f32(map, t.ptr, 4, dims, strides, box, mn_major);
}

// Host helper: TMA map that loads a whole `rows` x D tile of an FP32 [B,H,T,D]
// tensor (unit head-dim stride) with one copy: dims {32, T, D/32, H, B}, the
// third dimension stepping 128 bytes to the next 32-column chunk.  The box
// lands as D/32 chunks of `rows` 128-byte rows each -- the same shared-memory
// tile as D/32 copies of make_tmap_bhtd's box.
inline int make_tmap_bhtd_whole(CUtensorMap* map, const Strided4& t, const Fa2Problem& p,
                                int rows, bool mn_major = false) {
  const uint64_t dims[5] = {32u, (uint64_t)p.T, (uint64_t)(p.D / 32), (uint64_t)p.H,
                            (uint64_t)p.B};
  const uint64_t strides[4] = {(uint64_t)t.s[2] * 4u, 128u, (uint64_t)t.s[1] * 4u,
                               (uint64_t)t.s[0] * 4u};
  const uint32_t box[5] = {32u, (uint32_t)rows, (uint32_t)(p.D / 32), 1u, 1u};
  return make_tmap_f32(map, t.ptr, 5, dims, strides, box, mn_major);
}

// Number of (b,h) heads interleaved per CTA-order group (see fa2::cta_tile).
// The environment variable CT_FA2_HEAD_GROUP overrides the default (tuning).
inline int fa2_head_group(int bh_total) {
  static const int env = [] {
    const char* e = std::getenv("CT_FA2_HEAD_GROUP");
    return e ? std::atoi(e) : 0;
  }();
  int g = env > 0 ? env : 16;
  return g < 1 ? 1 : (g > bh_total ? (bh_total > 0 ? bh_total : 1) : g);
}

inline bool fa2_tma_ok(const Strided4& t) {
  return tma_compatible(t.ptr, t.s[3], t.s, 3);
}

// Enables large dynamic shared memory once per (kernel, device).
template <typename K>
inline int ensure_smem_attr(K kernel, size_t bytes, int device, unsigned long long* done_mask) {
  const unsigned long long bit = 1ull << (device & 63);
  if (__atomic_load_n(done_mask, __ATOMIC_ACQUIRE) & bit) return CT_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
      cudaSuccess)
    return CT_ERR_CUDA;
  __atomic_fetch_or(done_mask, bit, __ATOMIC_RELEASE);
  return CT_OK;
}

}  // namespace ct
