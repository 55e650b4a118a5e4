/*
 * ct_diag.h -- TEST-ONLY diagnostics (tests/diag/libct_diag.so), not part of
 * the product C ABI (include/ct_b200.h).  Return 0 on success, 1 for an
 * invalid argument, 4 for a failed launch, 6 for another CUDA error.
 */
#ifndef CT_DIAG_H
#define CT_DIAG_H

#ifdef __cplusplus
extern "C" {
#endif

/* One 128 x n x 32 TF32 tensor-core product on a single CTA, checking operand
 * layouts and rounding on the device:
 *   mode 0: A smem K-major,  B smem K-major      (b is [n,32])
 *   mode 1: A smem K-major,  B smem MN-major     (b is [32,n])
 *   mode 2: A TMEM,          B smem K-major      (b is [n,32])
 *   mode 3: A TMEM,          B smem MN-major     (b is [32,n])
 *   mode 4: A smem MN-major, B smem MN-major     (a is [32,128], b is [32,n])
 * a is [128,32] row-major for modes 0-3; d is [128,n] row-major.  n in {32,64,128}. */
int ct_diag_umma_tf32(int mode, const float* a, const float* b, float* d, int n, void* stream);

/* One M = 64 TF32 product D[64 x n] = A[64 x 32] B[n x 32]^T on a single CTA,
 * checking the M = 64 data-path layout of Tensor Memory (row r of D in lane
 * 32 * (r / 16) + r % 16 + L).  mode bit 0: A from TMEM (else shared memory);
 * bit 1: L = 16 (else 0); bit 2: D read with the 16-lane 16x32bx2 shape
 * (n = 32 only); bit 3: A and B from shared memory MN-major (not with bit 0;
 * a is then [32,64] = A^T and b [32,n] = B^T).  a is [64,32] row-major, b
 * [n,32], d [64,n]; n in {32, 64}. */
int ct_diag_umma_m64(int mode, const float* a, const float* b, float* d, int n, void* stream);

/* One M = 256 TF32 product D[256 x n] = A[256 x 64] B^T on a CTA pair
 * (cluster of two, cta_group::2).  A from Tensor Memory (CTA r: rows
 * 128r..128r+127); B split along N between the two CTAs' shared memory:
 * mode 0 K-major (b is [n,64]), mode 1 MN-major (b is [64,n]).  a is [256,64]
 * row-major, d [256,n]; n in {64, 128}. */
int ct_diag_umma_pair(int mode, const float* a, const float* b, float* d, int n, void* stream);

/* Tensor-pipe throughput of kind::tf32 MMAs, M = 128, N in {32, 64, 128, 256}.
 * `flags`: bit 0 A from TMEM (else shared memory), bit 1 B MN-major (else
 * K-major), bit 2 two issuing threads in different warps, each with its own
 * accumulator (N <= 128).  `blocks` CTAs (at most one per SM) each issue
 * reps x 4 MMAs per issuing thread back to back and write the clock64 cycles
 * from first issue to the first thread's completion into the device array
 * cycles[blocks] (-1 if the completion wait timed out). */
int ct_diag_mma_rate(int n, int flags, int reps, int blocks, long long* cycles, void* stream);

/* Watchdog word of this library's own bounded waits (0 = none expired). */
int ct_diag_status(unsigned int* flag_out);

#ifdef __cplusplus
}
#endif

#endif /* CT_DIAG_H */
