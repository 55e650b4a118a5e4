/*
 * ct_b200.h -- C ABI of the B200 (sm_100a) attention hot path.
 *
 * Every entry point takes caller-owned device pointers, explicit element
 * strides and sizes, and a cudaStream_t passed as `void*` (NULL = legacy
 * default stream).  Nothing here allocates device memory: operations that need
 * scratch space take a `workspace` pointer whose minimum size is reported by
 * the matching *_workspace_size() query.  All launches are asynchronous on the
 * given stream; the return value reports argument validation and launch
 * errors only.  Device-side watchdog failures (a bounded wait that ran out)
 * are recorded in a per-device status word read by ct_device_status().
 *
 * Tensors are FP32.  Four-dimensional attention tensors are indexed
 * [batch, head, seq, head_dim]; strides are in elements.  Outputs are written
 * densely (contiguous) exactly as the reference launchers allocate them.
 *
 * Each declaration names the reference interface it replaces
 * (AnshSachinkumarArora/CUDA_Transformer, path:line).
 */
#ifndef CT_B200_H
#define CT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
  CT_OK = 0,
  CT_ERR_INVALID_ARGUMENT = 1,     /* null pointer, negative size, size mismatch        */
  CT_ERR_UNSUPPORTED_HEAD_DIM = 2, /* FA2 head_dim not in {32, 64, 128}                 */
  CT_ERR_UNSUPPORTED_LAYOUT = 3,   /* strides the selected kernel cannot address (TMA)  */
  CT_ERR_LAUNCH_FAILED = 4,        /* cudaGetLastError() after a launch                 */
  CT_ERR_DEVICE_TIMEOUT = 5,       /* a device-side bounded wait expired                */
  CT_ERR_CUDA = 6,                 /* any other CUDA runtime error                      */
  CT_ERR_UNSUPPORTED_DEVICE = 7,   /* not an sm_100 device                              */
  CT_ERR_WORKSPACE_TOO_SMALL = 8   /* workspace_bytes below the *_workspace_size()      */
};

/* ---- precision modes for the tensor-core kernels ----------------------- */
enum {
  CT_PRECISION_3XTF32 = 0, /* FP32-accurate: hi/lo TF32 split, three MMAs per product   */
  CT_PRECISION_TF32 = 1,   /* one TF32 MMA per product (looser tolerance)               */
  CT_PRECISION_FP32 = 2    /* CUDA-core FP32 FFMA kernels (no tensor cores)             */
};

const char* ct_status_string(int status);
int ct_version(void);

/* Reads (and optionally clears) the device watchdog word of `device`.
 * *flag_out is 0 when no bounded wait has expired since the last clear.
 * While the word is non-zero, the tensor-core kernels of this library (FA2
 * forward, dQ, dK/dV, linear layer) return at entry without writing their
 * outputs: a failed wait stops the device's queue of tensor-core work until
 * the caller has seen the failure and cleared the word.  No reference
 * counterpart: the reference kernels have no failure detection. */
int ct_device_status(int device, int clear, unsigned int* flag_out);

/* Limit of every bounded device-side wait (barrier phases, split-K ordering)
 * on `device`, in nanoseconds; 2 s by default.  Legitimate waits last
 * microseconds, so the limit only decides how long a stuck kernel takes to
 * give up, report CT_DEVSTAT_TIMEOUT and tear down.  Accepted range
 * [CT_WAIT_LIMIT_MIN_NS, CT_WAIT_LIMIT_MAX_NS].  The setter copies
 * synchronously; set it while no kernel of this library runs on the device.
 * No reference counterpart. */
#define CT_WAIT_LIMIT_MIN_NS 100000ull         /* 0.1 ms */
#define CT_WAIT_LIMIT_MAX_NS 60000000000ull    /* 60 s   */
int ct_set_wait_limit_ns(int device, unsigned long long limit_ns);
int ct_get_wait_limit_ns(int device, unsigned long long* limit_ns);

/* Failure-detection self-test: launches, on the current device and `stream`,
 * one CTA whose warps wait on a barrier phase that nothing ever completes.
 * The waits run out after the device's wait limit and the CTA takes the same
 * abort teardown as the attention and GEMM kernels (MMA commit and bounded
 * drain, TMEM release); the kernel then returns, leaving CT_DEVSTAT_TIMEOUT
 * in the device's status word for ct_device_status to report.  Set a short
 * limit first (ct_set_wait_limit_ns) and clear the word afterwards.  No
 * reference counterpart. */
int ct_watchdog_selftest(void* stream);

/* ======================================================================== */
/* FlashAttention-2                                                          */
/* ======================================================================== */

/* Forward: O = softmax(Q K^T / sqrt(D) [causal mask q >= k]) V and
 * LSE = rowmax + ln(rowsum) (natural log, scaled-score domain).
 * O is written contiguous [B,H,T,D]; lse contiguous [B,H,T].
 * Replaces cuda_transformer::flash_attention_fwd
 * (Transformer_launchers/flash_attn_launcher.cu:22-65) and the kernel
 * flash_attention_fwd_kernel (Transformer_kernels/flash_attention.cuh:27-170). */
int ct_fa2_fwd(const float* q, const int64_t q_stride[4],
               const float* k, const int64_t k_stride[4],
               const float* v, const int64_t v_stride[4],
               float* o, float* lse,
               int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
               int causal, int precision, void* stream);

/* delta[b,h,t] = sum_d O[b,h,t,d] * dO[b,h,t,d]; delta contiguous [B,H,T].
 * Replaces flash_attention_bwd_delta (Transformer_kernels/flash_attention.cuh:175-213). */
int ct_fa2_bwd_delta(const float* o, const int64_t o_stride[4],
                     const float* d_o, const int64_t do_stride[4],
                     float* delta,
                     int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                     void* stream);

/* dQ = sum_j dS_ij K_j / sqrt(D) with P = exp(S - L), dS = P * (dP - delta).
 * lse_stride has three entries ([B,H,T]); delta is contiguous [B,H,T].
 * Replaces flash_attention_bwd_dq (Transformer_kernels/flash_attention.cuh:216-354). */
int ct_fa2_bwd_dq(const float* q, const int64_t q_stride[4],
                  const float* k, const int64_t k_stride[4],
                  const float* v, const int64_t v_stride[4],
                  const float* d_o, const int64_t do_stride[4],
                  const float* lse, const int64_t lse_stride[3],
                  const float* delta, float* dq,
                  int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                  int causal, int precision, void* stream);

/* dV = sum_i P_ij^T dO_i ; dK = sum_i dS_ij^T Q_i / sqrt(D).
 * Replaces flash_attention_bwd_dk_dv (Transformer_kernels/flash_attention.cuh:357-504);
 * unlike the reference it skips fully masked causal tiles. */
int ct_fa2_bwd_dkdv(const float* q, const int64_t q_stride[4],
                    const float* k, const int64_t k_stride[4],
                    const float* v, const int64_t v_stride[4],
                    const float* d_o, const int64_t do_stride[4],
                    const float* lse, const int64_t lse_stride[3],
                    const float* delta, float* dk, float* dv,
                    int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                    int causal, int precision, void* stream);

/* Bytes of workspace ct_fa2_bwd and ct_fa2_bwd_fused need: the delta vector,
 * then (from a 256-byte boundary) the one-kernel backward's ordering counters
 * and launch tickets. */
size_t ct_fa2_bwd_workspace_size(int64_t batch, int64_t heads, int64_t seq_len,
                                 int64_t head_dim);

/* Full backward: delta, dQ, dK, dV (three launches on `stream`).
 * Replaces cuda_transformer::flash_attention_bwd
 * (Transformer_launchers/flash_attn_launcher.cu:67-142), which allocates delta
 * itself; here delta lives in the caller's workspace. */
int ct_fa2_bwd(const float* q, const int64_t q_stride[4],
               const float* k, const int64_t k_stride[4],
               const float* v, const int64_t v_stride[4],
               const float* o, const int64_t o_stride[4],
               const float* d_o, const int64_t do_stride[4],
               const float* lse, const int64_t lse_stride[3],
               float* dq, float* dk, float* dv,
               void* workspace, size_t workspace_bytes,
               int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
               int causal, int precision, void* stream);

/* The same backward as ct_fa2_bwd in one key/value-stationary kernel after
 * delta: P and dS are formed once per (key tile, query tile) and each CTA adds
 * its dQ contribution into dQ in a fixed order of key tiles (per-tile counters
 * in the workspace; bit-identical run to run).  TF32 precision and head dim 64
 * only (CT_ERR_INVALID_ARGUMENT / CT_ERR_UNSUPPORTED_HEAD_DIM otherwise).  Not
 * the default: on B200 it measures slower than ct_fa2_bwd's two kernels.  No
 * reference counterpart (the reference's backward is two atomics-free kernels,
 * Transformer_kernels/flash_attention.cuh:216-504). */
int ct_fa2_bwd_fused(const float* q, const int64_t q_stride[4],
                     const float* k, const int64_t k_stride[4],
                     const float* v, const int64_t v_stride[4],
                     const float* o, const int64_t o_stride[4],
                     const float* d_o, const int64_t do_stride[4],
                     const float* lse, const int64_t lse_stride[3],
                     float* dq, float* dk, float* dv,
                     void* workspace, size_t workspace_bytes,
                     int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                     int causal, int precision, void* stream);

/* Largest batch * heads * seq_len ct_fa2_bwd_noalloc accepts. */
#define CT_FA2_BWD_NOALLOC_MAX_ROWS 2097152

/* The full backward of ct_fa2_bwd for callers that cannot allocate device
 * memory (for example a plugin given only tensor pointers by a host whose
 * allocator it cannot reach, or a service that allows no cudaMalloc after
 * start-up).  This entry point has no counterpart in the reference, whose
 * launcher allocates the delta temporary with torch::empty.  Delta lives in a
 * fixed array inside this library (8 MiB held on every GPU that loads it
 * until the process exits); the call itself allocates nothing.  Returns
 * CT_ERR_WORKSPACE_TOO_SMALL when batch * heads * seq_len exceeds
 * CT_FA2_BWD_NOALLOC_MAX_ROWS.  The first call on a device looks up the
 * array's device address, so make it before any stream capture.  All calls
 * share the array: calls that overlap on the GPU race, so order them on one
 * stream (or with events). */
int ct_fa2_bwd_noalloc(const float* q, const int64_t q_stride[4],
                       const float* k, const int64_t k_stride[4],
                       const float* v, const int64_t v_stride[4],
                       const float* o, const int64_t o_stride[4],
                       const float* d_o, const int64_t do_stride[4],
                       const float* lse, const int64_t lse_stride[3],
                       float* dq, float* dk, float* dv,
                       int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                       int causal, int precision, void* stream);

/* ======================================================================== */
/* Linear layer                                                              */
/* ======================================================================== */

/* out[b] = x[b] @ W[w_batch == 1 ? 0 : b] + bias, out contiguous [batch,m,n].
 * x is [batch,m,k] with strides x_stride; W is [w_batch,k,n] with strides
 * w_stride (w_stride[0] ignored when w_batch == 1); bias is [n] with stride
 * bias_stride.  Replaces cuda_transformer::cuda_fma
 * (Transformer_launchers/linear_layer.cu:28-70) and fused_multiply_add
 * (Transformer_kernels/fused_multiply_add.cuh:10-93). */
int ct_linear_fwd(const float* x, const int64_t x_stride[3],
                  const float* w, const int64_t w_stride[3],
                  const float* bias, int64_t bias_stride,
                  float* out,
                  int64_t batch, int64_t m, int64_t k, int64_t n, int64_t w_batch,
                  int precision, void* stream);

/* Device workspace (bytes, possibly 0) that ct_linear_fwd_ws may use to split
 * the K reduction across SMs when the output has few tiles (the weight
 * gradient x^T dy over batch*seq rows). */
size_t ct_linear_workspace_size(int64_t batch, int64_t m, int64_t k, int64_t n);

/* ct_linear_fwd with a caller-owned device workspace of workspace_bytes
 * (>= ct_linear_workspace_size for the split-K schedule; smaller or NULL
 * disables it).  The slices of a split reduction are added in a fixed order,
 * so results are deterministic.  The workspace must not be used by another
 * call that can run concurrently.  Same reference counterpart as
 * ct_linear_fwd (Transformer_launchers/linear_layer.cu:28-70). */
int ct_linear_fwd_ws(const float* x, const int64_t x_stride[3],
                     const float* w, const int64_t w_stride[3],
                     const float* bias, int64_t bias_stride,
                     float* out,
                     int64_t batch, int64_t m, int64_t k, int64_t n, int64_t w_batch,
                     int precision, void* workspace, size_t workspace_bytes, void* stream);

/* Fused epilogues of ct_linear_fwd_ex. */
enum {
  CT_EPILOGUE_NONE = 0,      /* out = x W + bias                                        */
  CT_EPILOGUE_GELU = 1,      /* out = x W + bias and act_out = gelu(out) (erf form)     */
  CT_EPILOGUE_GELU_GRAD = 2  /* out = (x W + bias) * gelu'(act_in), act_in [batch,m,n]  */
};

/* ct_linear_fwd_ws with the linear layer's neighbours fused in:
 *  - `epilogue` applies GELU (gelu/gelu_bwd of Transformer_kernels/GeLU.cuh:7-29)
 *    to the GEMM's output tile before it leaves the chip: CT_EPILOGUE_GELU
 *    also writes act_out = gelu(out) (the MLP's fc1 and activation,
 *    gpt/gpt.py:134-135), CT_EPILOGUE_GELU_GRAD multiplies by the GELU
 *    derivative at act_in (the fc2 input gradient times gelu', the same
 *    MLP's backward);
 *  - `w_colsum` (batch == 1), when not NULL, receives the column sums of the
 *    W operand over the reduction index: with W = dY this is the bias
 *    gradient db, formed from the dY tiles the weight-gradient GEMM
 *    dW = x^T dY already stages (cuda_autograd_fns/cuda_linear_layer.py:25-27,
 *    Transformer_kernels/warp_sum_kernel.cuh:13-51);
 *  - `accumulate` != 0 adds into out (and w_colsum) instead of storing
 *    (CT_EPILOGUE_NONE only).
 * On the tensor cores w_colsum needs workspace_bytes >= ct_linear_workspace_size
 * (CT_ERR_WORKSPACE_TOO_SMALL otherwise): the units that share a tile column
 * add their partial sums in a fixed order through counters kept there.
 * Deterministic: split-K slices and the column sums add in a fixed order.
 * Same reference counterpart as ct_linear_fwd (linear_layer.cu:28-70). */
int ct_linear_fwd_ex(const float* x, const int64_t x_stride[3],
                     const float* w, const int64_t w_stride[3],
                     const float* bias, int64_t bias_stride,
                     float* out,
                     int64_t batch, int64_t m, int64_t k, int64_t n, int64_t w_batch,
                     int precision, int epilogue, float* act_out, const float* act_in,
                     float* w_colsum, int accumulate,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace ct_bias_grad needs. */
size_t ct_bias_grad_workspace_size(int64_t batch, int64_t m, int64_t n);

/* db[j] = sum_{b,i} dy[b,i,j].  Replaces cuda_transformer::db_calculation
 * (Transformer_launchers/linear_layer.cu:74-97) and warp_sum_kernel
 * (Transformer_kernels/warp_sum_kernel.cuh:13-51).  Deterministic two-stage
 * column reduction; the partial sums live in `workspace`. */
int ct_bias_grad(const float* dy, const int64_t dy_stride[3], float* db,
                 int64_t batch, int64_t m, int64_t n,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ======================================================================== */
/* Row-wise kernels                                                          */
/* ======================================================================== */

/* y = softmax(x) along the last dimension of a contiguous [rows, n] tensor.
 * Replaces cuda_transformer::cuda_softmax (Transformer_launchers/softmax_layer.cu:22-50)
 * and naive_softmax (Transformer_kernels/softmax.cuh:25-106). */
int ct_softmax_fwd(const float* x, float* y, int64_t rows, int64_t n, void* stream);

/* dx = p * (dp - sum(p * dp)) per row.  Replaces cuda_softmax_bwd
 * (Transformer_launchers/softmax_layer.cu:52-80) and naive_softmax_bwd
 * (Transformer_kernels/softmax.cuh:108-159). */
int ct_softmax_bwd(const float* p, const float* dp, float* dx, int64_t rows, int64_t n,
                   void* stream);

/* Exact (erf) GELU y = x * Phi(x).  Replaces gelu_activation
 * (Transformer_launchers/gelu_activation.cu:22-47) and gelu (Transformer_kernels/GeLU.cuh:7-16). */
int ct_gelu_fwd(const float* x, float* y, int64_t numel, void* stream);

/* dx = dy * (Phi(x) + x * phi(x)).  Replaces gelu_activation_bwd
 * (Transformer_launchers/gelu_activation.cu:49-77) and gelu_bwd (Transformer_kernels/GeLU.cuh:19-29). */
int ct_gelu_bwd(const float* x, const float* dy, float* dx, int64_t numel, void* stream);

/* LayerNorm over the last dimension of a contiguous [rows, n] tensor:
 * y = (x - mean) / sqrt(var_biased + eps) * gamma + beta (n <= 8192); mean and rstd
 * ([rows], may be NULL) are saved for the backward.  The reference has no
 * CUDA LayerNorm: this restates the PyTorch module in gpt/gpt.py:47-59. */
int ct_layernorm_fwd(const float* x, const float* gamma, const float* beta,
                     float* y, float* mean, float* rstd,
                     int64_t rows, int64_t n, float eps, void* stream);

size_t ct_layernorm_bwd_workspace_size(int64_t rows, int64_t n);

/* Gradients of ct_layernorm_fwd: dx [rows,n], dgamma [n], dbeta [n]
 * (autograd of gpt/gpt.py:55-58).  Column sums are reduced
 * deterministically through `workspace`. */
int ct_layernorm_bwd(const float* x, const float* gamma, const float* mean,
                     const float* rstd, const float* dy,
                     float* dx, float* dgamma, float* dbeta,
                     int64_t rows, int64_t n,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Cross entropy of `rows` logit rows of length `vocab` (row stride ld),
 * forward and backward together:
 *   loss_rows[r] = logsumexp(logits[r]) - logits[r][targets[r]]
 *   logits[r][:] <- softmax(logits[r]) - onehot(targets[r])   (in place)
 * A target equal to ignore_index gives loss 0 and a zero gradient row; one
 * outside [0, vocab) gives NaN for that row.  With mean reduction the caller
 * divides the summed loss and the gradient by the number of counted rows.
 * The reference applies torch's F.cross_entropy to the lm_head logits
 * (gpt/gpt.py:167-175); this lets the lm_head GEMM and the loss run chunk by
 * chunk without materialising every row of logits. */
int ct_cross_entropy_fwd_bwd(float* logits, int64_t ld, int64_t rows, int64_t vocab,
                             const int64_t* targets, int64_t ignore_index, float* loss_rows,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CT_B200_H */
