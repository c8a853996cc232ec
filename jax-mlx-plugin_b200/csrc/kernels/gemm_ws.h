// GEMM entry points used by the PJRT runtime (not part of the public kernel
// ABI): the runtime asks how much workspace a b200_gemm call needs and lends it
// from its caching allocator, so a jitted step never reaches cudaMallocAsync.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "b200_kernels.h"

#ifdef __cplusplus
extern "C" {
#endif

// Extra in_dtype values accepted by the entry points below (and by b200_gemm):
// one f32 and one bf16 operand, as JAX's transpose rule emits for a bf16
// dot_general with an f32 result.  The f32 operand is split into bf16 hi + lo
// planes and the bf16 one is read as it is: two bf16 MMAs per K step, the
// accuracy of three-plane f32 (the bf16 operand's lo plane is zero).
#define B200_GEMM_DT_A_F32_B_BF16 100
#define B200_GEMM_DT_A_BF16_B_F32 101

// Bytes of workspace b200_gemm_ws needs for these arguments (same meaning as
// b200_gemm's); 0 when none, -1 when the arguments are rejected.  Launches
// nothing.
B200_API int64_t b200_gemm_workspace_bytes(const void* a, const void* b, void* c, const void* bias,
                                           int64_t batch, int64_t M, int64_t N, int64_t K,
                                           int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                                           int64_t sBk, int64_t sBn, int64_t ldc, float alpha,
                                           int in_dtype, int out_dtype, int epilogue, void* stream);

// b200_gemm with the workspace lent by the caller (`ws` of `ws_bytes`, which
// must stay untouched until the call's kernels have run in stream order).
B200_API int b200_gemm_ws(const void* a, const void* b, void* c, const void* bias, int64_t batch,
                          int64_t M, int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk,
                          int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, float alpha,
                          int in_dtype, int out_dtype, int epilogue, void* stream, void* ws,
                          size_t ws_bytes);

// b200_gemm_ws / b200_gemm_workspace_bytes for f32 operands that arrive
// already split into bf16 planes: when a_lo (b_lo) is not null, a (b) points
// at the operand's bf16 hi plane and a_lo (b_lo) at its lo plane, both with the
// operand's element strides (x ~= hi + lo, each rounded to nearest), so a
// producer such as an im2col kernel can write the planes directly.  in_dtype
// gives the logical types (B200_DT_F32 or a mixed code).
B200_API int64_t b200_gemm_planes_workspace_bytes(
    const void* a, const void* a_lo, const void* b, const void* b_lo, void* c, const void* bias,
    int64_t batch, int64_t M, int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk,
    int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int in_dtype, int out_dtype,
    int epilogue, void* stream);
B200_API int b200_gemm_planes_ws(const void* a, const void* a_lo, const void* b, const void* b_lo,
                                 void* c, const void* bias, int64_t batch, int64_t M, int64_t N,
                                 int64_t K, int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                                 int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int in_dtype,
                                 int out_dtype, int epilogue, void* stream, void* ws,
                                 size_t ws_bytes);

#ifdef __cplusplus
}
#endif
