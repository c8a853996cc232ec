/*
 * b200_kernels.h — thin C ABI over the hand-written sm_100a kernels.
 *
 * Plain pointers (device memory), sizes and a cudaStream_t passed as void*.
 * No torch or C++ types cross this boundary.  Every entry point returns 0 on
 * success or a nonzero B200_ERR_* code; b200_last_error() gives the message of
 * the calling thread's last failure.  Launches are asynchronous on `stream`.
 *
 * The PJRT plugin (libb200_pjrt.so) calls these from its executables; tests and
 * bench.py call them directly through ctypes.
 */
#ifndef B200_KERNELS_H_
#define B200_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

#ifndef B200_API
#define B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  B200_OK = 0,
  B200_ERR_INVALID = 1,     /* bad argument: shape, alignment, dtype */
  B200_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  B200_ERR_UNSUPPORTED = 3, /* shape/dtype combination without a kernel */
  B200_ERR_TIMEOUT = 4      /* a bounded device-side wait ran out */
};

/* Element types, numbered as PJRT_Buffer_Type (S32=4, F32=11, BF16=13). */
enum { B200_DT_PRED = 1, B200_DT_S32 = 4, B200_DT_U32 = 8, B200_DT_F32 = 11, B200_DT_BF16 = 13 };

B200_API const char* b200_last_error(void);
/* Library version string "b200-kernels <semver> sm_100a". */
B200_API const char* b200_kernels_version(void);
/* How many kernels this library has launched in this process, every kernel an
 * entry point below starts counted (a split-K GEMM counts its partial-sum
 * reduction too).  For counting the launches of a timed region: read it before
 * and after.  The reference has no counterpart (MLX launches its own kernels
 * inside mx::eval). */
B200_API uint64_t b200_kernel_launches(void);

/* Fused residual-add + LayerNorm / RMSNorm forward over the last axis.
 *   h = x + residual        (residual may be NULL: h = x)
 *   y = norm(h) * gamma + beta   (gamma/beta may be NULL: 1 / 0)
 *   norm = (h - mean) * rsqrt(var + eps)   for kind 0 (LayerNorm)
 *        = h * rsqrt(mean(h^2) + eps)      for kind 1 (RMSNorm)
 * x, residual, y, h_out: [rows, cols] row-major of `dtype` (F32 or BF16);
 * gamma, beta: [cols] of `dtype`.  h_out may be NULL.  mean_out/rstd_out
 * (f32 [rows], may be NULL) keep the statistics for the backward pass.
 * Replaces reference src/jax_mlx_pjrt.cpp:4430-4437 (mlx.layer_norm /
 * mlx.rms_norm) and :8208-8236 (custom_call mlx_layer_norm), whose residual add
 * and affine stayed separate MLX ops. */
B200_API int b200_ln_residual_fwd(const void* x, const void* residual, const void* gamma,
                         const void* beta, void* y, void* h_out, float* mean_out,
                         float* rstd_out, int64_t rows, int64_t cols, float eps,
                         int dtype, int kind, void* stream);

/* LayerNorm backward (kind 0) given the saved statistics:
 *   dx[r,:], and column sums dgamma = sum_r dy*xhat, dbeta = sum_r dy.
 * dgamma/dbeta are f32 [cols] (zeroed and written by the call); `ws` is a
 * caller-provided f32 scratch of b200_ln_bwd_workspace(rows, cols) bytes.
 * Replaces reference src/jax_mlx_pjrt.cpp:8238-8281 (mlx_layer_norm_bwd via
 * mx::vjp) and src/jax_mlx/layer_norm.py:59-76 (its math). */
B200_API int64_t b200_ln_bwd_workspace(int64_t rows, int64_t cols);
B200_API int b200_ln_bwd(const void* x, const void* gamma, const float* mean, const float* rstd,
                const void* dy, void* dx, float* dgamma, float* dbeta, void* ws,
                int64_t rows, int64_t cols, int dtype, void* stream);

/* Scaled dot-product attention forward, layout BTNH (batch, seq, heads, dim):
 *   O[b,t,n,:] = softmax_s(scale * Q[b,t,n,:].K[b,s,n,:] + mask) V[b,s,n,:]
 * with mask = -0.7*FLT_MAX where causal and s > t (JAX's large-negative fill).
 * q: [B,T,N,D]; k, v: [B,S,N,D]; o: [B,T,N,D]; dtype F32 (each f32 operand
 * split into bf16 hi + lo parts and every product taken as hi*hi + hi*lo +
 * lo*hi in kind::f16 MMAs with f32 accumulation; softmax in f32) or BF16 (one
 * kind::f16 MMA per product, f32 accumulate).  D must be 64.
 * Replaces reference src/jax_mlx_pjrt.cpp:4440-4446 / :8111-8150
 * (mlx::fast::scaled_dot_product_attention) and src/jax_mlx/sdpa.py:19-31. */
B200_API int b200_sdpa_fwd(const void* q, const void* k, const void* v, void* o, int64_t B,
                  int64_t T, int64_t S, int64_t N, int64_t D, float scale, int causal,
                  int dtype, void* stream);

/* Same computation with explicit element strides (head dim contiguous):
 * strides[0..2] = q (b,t,n), [3..5] = k (b,s,n), [6..8] = v (b,s,n),
 * [9..11] = o (b,t,n).  The plugin uses it for attention matched out of a
 * dot_general -> softmax -> dot_general chain, whose operands may be BTNH or
 * BNTH views; every stride must be a multiple of 4 elements (16 bytes). */
B200_API int b200_sdpa_fwd_strided(const void* q, const void* k, const void* v, void* o,
                                   int64_t B, int64_t T, int64_t S, int64_t N, int64_t D,
                                   const int64_t* strides, float scale, int causal, int dtype,
                                   void* stream);

/* b200_sdpa_fwd_strided that also writes each query row's softmax statistic
 * lse2[b, n, t] = log2(sum_s 2^(scale * log2(e) * q_t.k_s)) (masked keys
 * excluded), f32 [B, N, T] contiguous, for b200_sdpa_bwd.  Tensor-core path
 * only: D == 64, scale > 0, 16-byte aligned operands and strides; anything
 * else returns B200_ERR_UNSUPPORTED. */
B200_API int b200_sdpa_fwd_lse(const void* q, const void* k, const void* v, void* o, float* lse2,
                               int64_t B, int64_t T, int64_t S, int64_t N, int64_t D,
                               const int64_t* strides, float scale, int causal, int dtype,
                               void* stream);

/* Attention backward for O = softmax(scale * Q K^T + mask) V (S == T):
 *   dV = P^T dO,  dS = P * (dO V^T - rowsum(dO * O)) * scale,
 *   dQ = dS K,    dK = dS^T Q,
 * with P recomputed from lse2 (b200_sdpa_fwd_lse) and never stored.  All of
 * q, k, v, o, dout, dq, dk, dv are bf16 with the head dim contiguous; strides
 * (elements) are (b, t, n) for q, k, v, o, dout, dq, dk, dv in that order (24
 * values, each a multiple of 8).  Needs D == 64 and T <= 256; other shapes
 * and dtypes return B200_ERR_UNSUPPORTED.  P enters the tensor-core products
 * as bf16 (as jax.nn.dot_product_attention rounds the probabilities), dS as
 * bf16 hi + lo parts (about 16 significant bits); accumulation is f32.  Replaces reference
 * src/jax_mlx_pjrt.cpp:8152-8206 (mlx_sdpa_bwd through mx::vjp) and the math
 * of src/jax_mlx/sdpa.py:65-87. */
B200_API int b200_sdpa_bwd(const void* q, const void* k, const void* v, const void* o,
                           const void* dout, const float* lse2, void* dq, void* dk, void* dv,
                           int64_t B, int64_t T, int64_t N, int64_t D, const int64_t* strides,
                           float scale, int causal, int dtype, void* stream);

/* Batched GEMM on tcgen05: for b in [0,batch):
 *   C_b[m,n] = alpha * sum_k A_b[m,k] * B_b[k,n]  (+ bias[n]) (+ relu)
 * A element (b,m,k) at a + b*sAb + m*sAm + k*sAk (strides in elements), one of
 * sAm/sAk must be 1; same for B with (b,k,n).  C is dense row-major [batch,M,N]
 * unless ldc (elements between rows) says otherwise.  in_dtype F32 (operands
 * split into bf16 hi + lo planes, three kind::f16 MMAs per step; 3xTF32 where
 * no plane workspace can be had) or BF16; out_dtype F32 or BF16; accumulation
 * in f32.  epilogue: 0 none, 1 bias,
 * 2 bias+relu, 3 relu.  M == 0 or N == 0: nothing is written; K == 0: C is
 * set to zero (epilogue 0 or 3; a bias epilogue with K == 0 is rejected).
 * Replaces reference src/jax_mlx_pjrt.cpp:4577-4666 (dot_general ->
 * transpose/reshape -> mlx::core::matmul). */
B200_API int b200_gemm(const void* a, const void* b, void* c, const void* bias, int64_t batch,
              int64_t M, int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk,
              int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, float alpha,
              int in_dtype, int out_dtype, int epilogue, void* stream);

/* b200_gemm that allocates no device memory, for callers that cannot allocate:
 *  - a host program whose device memory belongs to another allocator, such as
 *    a JAX/XLA process whose PJRT client has reserved most of HBM up front, so a
 *    library-side cudaMallocAsync either fails or takes memory that allocator
 *    was counting on;
 *  - code that must not let a library grow or touch the CUDA memory pool
 *    behind its back (a fixed memory budget, or a pool owned by someone else).
 * b200_gemm takes its split-K partial sums from cudaMallocAsync on `stream`;
 * this variant keeps them in one fixed 8 MiB device array inside the library
 * (every GPU that loads the library holds it until the process exits), and its
 * bounded-wait error word is a fixed device variable too (b200_device_error
 * reports it).  It calls no cudaMalloc, cudaMallocAsync, cudaFree or other
 * allocating routine.
 * Limit: a call whose split-K plan needs more than 8 MiB of partial sums
 * (splits x batch x M x N x 4 bytes) returns B200_ERR_INVALID and
 * b200_last_error() names both sizes; shapes that need no split use no scratch.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current, so make that first call
 * before any stream capture.  All calls on a device share the array, which
 * keeps the last call's contents: two calls that overlap on the GPU (different
 * streams, or host threads that do not order their calls) race on it.  Each
 * call writes every partial sum it reads, so nothing needs clearing between
 * calls.  in_dtype must be B200_DT_F32 or B200_DT_BF16: the mixed F32 x BF16
 * codes need a widened or split copy of one operand, so they are refused with
 * B200_ERR_UNSUPPORTED (as is any path that would need a buffer other than the
 * fixed array).  b200_device_error reads this entry point's error word without
 * allocating.  Arguments, results and error codes are otherwise those of
 * b200_gemm.
 * No counterpart in the reference: it has no split-K scratch and allocates
 * through MLX. */
B200_API int b200_gemm_noalloc(const void* a, const void* b, void* c, const void* bias,
                               int64_t batch, int64_t M, int64_t N, int64_t K, int64_t sAb,
                               int64_t sAm, int64_t sAk, int64_t sBb, int64_t sBk, int64_t sBn,
                               int64_t ldc, float alpha, int in_dtype, int out_dtype, int epilogue,
                               void* stream);

/* 1 when b200_gemm would take the tcgen05/TMA path for these arguments, 0 when
 * it falls back to the SIMT kernel (rows not 16-byte aligned, tiny K, ...). */
B200_API int b200_gemm_uses_tensor_cores(const void* a, const void* b, int64_t batch, int64_t K,
                                         int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                                         int64_t sBk, int64_t sBn, int in_dtype);

/* Site code recorded by the last bounded device-side wait that ran out on the
 * current device (0 = none, -1 = could not be read); clear != 0 resets it.
 * Synchronizes with the device. */
B200_API int b200_device_error(int clear);

#ifdef __cplusplus
}
#endif
#endif /* B200_KERNELS_H_ */
