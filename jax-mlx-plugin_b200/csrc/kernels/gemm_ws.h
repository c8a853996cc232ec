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

#ifdef __cplusplus
}
#endif
