"""GPU: the allocation-free GEMM entry point, b200_gemm_noalloc.

Some callers of this library cannot let it allocate device memory: a JAX/XLA
process whose PJRT client has already reserved most of HBM for its own
allocator, or any program with a fixed memory budget or a memory pool that it
owns.  For them b200_gemm_noalloc keeps its split-K partial sums in one fixed
8 MiB array inside the library instead of calling cudaMallocAsync.  These tests
call it through the C ABI and check it against b200_gemm on the same inputs,
twice in a row (the array keeps the previous call's contents, which must not
leak into the next result), and check that a call needing more than the array
is refused with a clear error.  Tolerances are the ones the GEMM tests use:
2e-3 relative for f32 operands (3xTF32 tensor-core path), 1e-2 for bf16.

The file name sorts last so that pytest collects it after the other tests; it
also passes when run on its own in a fresh process."""
import numpy as np
import pytest

from helpers import assert_close
from jax_b200 import kernels

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SCRATCH_BYTES = 8 << 20  # the array size b200_gemm_noalloc documents


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _operands(M, N, K, a_t, b_t, dt, seed):
    """Device A [M,K] (stored [K,M] when a_t), B [K,N] (stored [N,K] when b_t),
    bias [N], plus the strides b200_gemm takes."""
    rng = np.random.default_rng(seed)
    tdt = torch.bfloat16 if dt == kernels.DT_BF16 else torch.float32
    a = rng.standard_normal((K, M) if a_t else (M, K)).astype(np.float32)
    b = rng.standard_normal((N, K) if b_t else (K, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    A, B, BIAS = (torch.from_numpy(v).to("cuda", tdt) for v in (a, b, bias))
    strides = (M * K, 1 if a_t else K, M if a_t else 1, K * N, 1 if b_t else N, K if b_t else 1)
    return A, B, BIAS, strides


def _call(fn, A, B, BIAS, strides, M, N, K, dt, epi):
    C = torch.full((M, N), float("nan"), device="cuda",
                   dtype=torch.bfloat16 if dt == kernels.DT_BF16 else torch.float32)
    sAb, sAm, sAk, sBb, sBk, sBn = strides
    fn(A.data_ptr(), B.data_ptr(), C.data_ptr(), BIAS.data_ptr(), 1, M, N, K, sAb, sAm, sAk,
       sBb, sBk, sBn, N, 1.0, dt, dt, epi, _stream())
    torch.cuda.synchronize()
    return C.float().cpu().numpy()


# Shapes whose split-K plan uses the scratch array: conv weight gradients and
# tall-skinny dense gradients on the tcgen05 path, a narrow output on the SIMT
# path, and one shape that needs no split at all.
CASES = [
    (288, 64, 50176, False, False, kernels.DT_F32, 0),
    (3136, 256, 256, True, False, kernels.DT_F32, 2),
    (256, 64, 16384, False, True, kernels.DT_BF16, 0),
    (1024, 10, 4096, False, False, kernels.DT_F32, 1),
    (2048, 2048, 256, False, False, kernels.DT_F32, 3),
]


@pytest.mark.parametrize("M,N,K,a_t,b_t,dt,epi", CASES)
def test_noalloc_matches_gemm_two_calls(M, N, K, a_t, b_t, dt, epi):
    tol = 2e-3 if dt == kernels.DT_F32 else 1e-2
    for call, seed in enumerate((M + K, M + K + 1)):  # two calls in a row, new inputs each
        A, B, BIAS, strides = _operands(M, N, K, a_t, b_t, dt, seed)
        want = _call(kernels.gemm, A, B, BIAS, strides, M, N, K, dt, epi)
        got = _call(kernels.gemm_noalloc, A, B, BIAS, strides, M, N, K, dt, epi)
        assert np.isfinite(got).all()
        assert_close(got, want, tol, f"gemm_noalloc {M}x{N}x{K} call {call}")
    assert kernels.device_error(clear=True) == 0


def test_noalloc_rejects_split_beyond_scratch():
    """1024x1024x4096 f32 splits K three ways: 12 MiB of partial sums, more than
    the 8 MiB array.  The call is refused before anything is launched, and the
    next call that fits still works."""
    M, N, K = 1024, 1024, 4096
    A, B, BIAS, strides = _operands(M, N, K, False, False, kernels.DT_F32, 7)
    assert 3 * M * N * 4 > SCRATCH_BYTES
    with pytest.raises(kernels.KernelError, match="scratch") as e:
        _call(kernels.gemm_noalloc, A, B, BIAS, strides, M, N, K, kernels.DT_F32, 0)
    assert str(SCRATCH_BYTES) in str(e.value)
    M, N, K = 288, 64, 50176
    A, B, BIAS, strides = _operands(M, N, K, False, False, kernels.DT_F32, 8)
    want = _call(kernels.gemm, A, B, BIAS, strides, M, N, K, kernels.DT_F32, 0)
    got = _call(kernels.gemm_noalloc, A, B, BIAS, strides, M, N, K, kernels.DT_F32, 0)
    assert_close(got, want, 2e-3, "gemm_noalloc after a refused call")
