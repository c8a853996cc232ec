"""ctypes binding of ``libb200_kernels.so`` (include/b200_kernels.h).

Arguments are raw device pointers (ints) and a CUDA stream handle; callers
holding torch tensors pass ``t.data_ptr()`` and
``torch.cuda.current_stream().cuda_stream``.  Every call raises on a nonzero
status with the library's error message.  There is no CPU fallback: without the
built library this module fails at import of the library.
"""
from __future__ import annotations

import ctypes as C
import os

from .pjrt import LIB_DIR

KERNELS_LIB = os.path.join(LIB_DIR, "libb200_kernels.so")

DT_PRED, DT_S32, DT_U32, DT_F32, DT_BF16 = 1, 4, 8, 11, 13

EXPORTS = {
    "b200_last_error": (C.c_char_p, []),
    "b200_kernels_version": (C.c_char_p, []),
    "b200_ln_residual_fwd": (C.c_int, [C.c_void_p] * 8 + [C.c_int64, C.c_int64, C.c_float, C.c_int,
                                                          C.c_int, C.c_void_p]),
    "b200_ln_bwd_workspace": (C.c_int64, [C.c_int64, C.c_int64]),
    "b200_ln_bwd": (C.c_int, [C.c_void_p] * 9 + [C.c_int64, C.c_int64, C.c_int, C.c_void_p]),
    "b200_sdpa_fwd": (C.c_int, [C.c_void_p] * 4 + [C.c_int64] * 5 + [C.c_float, C.c_int, C.c_int,
                                                                    C.c_void_p]),
    "b200_sdpa_fwd_strided": (C.c_int, [C.c_void_p] * 4 + [C.c_int64] * 5 +
                              [C.POINTER(C.c_int64), C.c_float, C.c_int, C.c_int, C.c_void_p]),
    "b200_sdpa_fwd_lse": (C.c_int, [C.c_void_p] * 5 + [C.c_int64] * 5 +
                          [C.POINTER(C.c_int64), C.c_float, C.c_int, C.c_int, C.c_void_p]),
    "b200_sdpa_bwd": (C.c_int, [C.c_void_p] * 9 + [C.c_int64] * 4 +
                      [C.POINTER(C.c_int64), C.c_float, C.c_int, C.c_int, C.c_void_p]),
    "b200_gemm": (C.c_int, [C.c_void_p] * 4 + [C.c_int64] * 11 + [C.c_float, C.c_int, C.c_int,
                                                                  C.c_int, C.c_void_p]),
    "b200_gemm_noalloc": (C.c_int, [C.c_void_p] * 4 + [C.c_int64] * 11 +
                          [C.c_float, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "b200_gemm_uses_tensor_cores": (C.c_int, [C.c_void_p, C.c_void_p] + [C.c_int64] * 8 + [C.c_int]),
    "b200_device_error": (C.c_int, [C.c_int]),
    "b200_kernel_launches": (C.c_uint64, []),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(KERNELS_LIB):
            raise FileNotFoundError(f"{KERNELS_LIB} not built (run __graft_entry__.build())")
        l = C.CDLL(KERNELS_LIB)
        for name, (res, args) in EXPORTS.items():
            f = getattr(l, name)
            f.restype, f.argtypes = res, args
        _lib = l
    return _lib


class KernelError(RuntimeError):
    pass


def _check(rc: int, what: str):
    if rc != 0:
        raise KernelError(f"{what} failed ({rc}): {lib().b200_last_error().decode()}")


def ln_residual_fwd(x, residual, gamma, beta, y, h_out, mean_out, rstd_out, rows, cols, eps,
                    dtype, kind, stream):
    _check(lib().b200_ln_residual_fwd(x, residual, gamma, beta, y, h_out, mean_out, rstd_out, rows,
                                      cols, eps, dtype, kind, stream), "ln_residual_fwd")


def ln_bwd_workspace(rows, cols) -> int:
    return lib().b200_ln_bwd_workspace(rows, cols)


def ln_bwd(x, gamma, mean, rstd, dy, dx, dgamma, dbeta, ws, rows, cols, dtype, stream):
    _check(lib().b200_ln_bwd(x, gamma, mean, rstd, dy, dx, dgamma, dbeta, ws, rows, cols, dtype,
                             stream), "ln_bwd")


def sdpa_fwd(q, k, v, o, B, T, S, N, D, scale, causal, dtype, stream):
    _check(lib().b200_sdpa_fwd(q, k, v, o, B, T, S, N, D, scale, int(causal), dtype, stream),
           "sdpa_fwd")


def sdpa_fwd_strided(q, k, v, o, B, T, S, N, D, strides, scale, causal, dtype, stream):
    arr = (C.c_int64 * 12)(*strides)
    _check(lib().b200_sdpa_fwd_strided(q, k, v, o, B, T, S, N, D, arr, scale, int(causal), dtype,
                                       stream), "sdpa_fwd_strided")


def sdpa_fwd_lse(q, k, v, o, lse2, B, T, S, N, D, strides, scale, causal, dtype, stream):
    """sdpa_fwd_strided that also writes the rows' log2-sum-exp2 statistic
    (f32 [B, N, T]) for sdpa_bwd."""
    arr = (C.c_int64 * 12)(*strides)
    _check(lib().b200_sdpa_fwd_lse(q, k, v, o, lse2, B, T, S, N, D, arr, scale, int(causal), dtype,
                                   stream), "sdpa_fwd_lse")


def sdpa_bwd(q, k, v, o, dout, lse2, dq, dk, dv, B, T, N, D, strides, scale, causal, dtype, stream):
    """dQ, dK, dV of attention (bf16, D == 64, T <= 256); strides: (b, t, n) of
    q, k, v, o, dout, dq, dk, dv (24 values)."""
    arr = (C.c_int64 * 24)(*strides)
    _check(lib().b200_sdpa_bwd(q, k, v, o, dout, lse2, dq, dk, dv, B, T, N, D, arr, scale,
                               int(causal), dtype, stream), "sdpa_bwd")


def gemm(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, in_dtype,
         out_dtype, epilogue, stream):
    _check(lib().b200_gemm(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha,
                           in_dtype, out_dtype, epilogue, stream), "gemm")


def gemm_noalloc(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha,
                 in_dtype, out_dtype, epilogue, stream):
    """b200_gemm_noalloc: same call as gemm(), but the library allocates no device
    memory (split-K partials live in its fixed 8 MiB per-device array)."""
    _check(lib().b200_gemm_noalloc(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn,
                                   ldc, alpha, in_dtype, out_dtype, epilogue, stream),
           "gemm_noalloc")


def gemm_uses_tensor_cores(a, b, batch, K, sAb, sAm, sAk, sBb, sBk, sBn, in_dtype) -> bool:
    return bool(lib().b200_gemm_uses_tensor_cores(a, b, batch, K, sAb, sAm, sAk, sBb, sBk, sBn,
                                                  in_dtype))


def device_error(clear: bool = True) -> int:
    return lib().b200_device_error(int(clear))
