"""GPU: the allocation-free GEMM entry point, b200_gemm_noalloc.

Some callers of this library cannot let it allocate device memory: a JAX/XLA
process whose PJRT client has already reserved most of HBM for its own
allocator, or any program with a fixed memory budget or a memory pool that it
owns.  For them b200_gemm_noalloc keeps its split-K partial sums in one fixed
8 MiB array inside the library instead of calling cudaMallocAsync.  These tests
call it through the C ABI and check:

* its result against a numpy float64 product of the same operands, and against
  b200_gemm, twice in a row with new inputs (the array keeps the previous
  call's contents, which must not leak into the next result), within the GEMM
  tests' tolerances: 2e-3 relative for f32 operands, 1e-2 for bf16;
* that a call allocates nothing: the device's free memory (cudaMemGetInfo) and
  the default memory pool's high-water marks of reserved and used bytes
  (which any cudaMallocAsync would raise) stay where they were across the calls;
* that a call needing more than the array, or a mixed f32 x bf16 operand pair
  (which would need a widened copy of one operand), is refused with a clear
  error before anything is launched.

The file name sorts last so that pytest collects it after the other tests; it
also passes when run on its own in a fresh process."""
import numpy as np
import pytest

from helpers import assert_close
from jax_b200 import kernels

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SCRATCH_BYTES = 8 << 20  # the array size b200_gemm_noalloc documents
MIXED_CODES = (100, 101)  # f32 A x bf16 B and bf16 A x f32 B (b200_gemm accepts them)


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _operands(M, N, K, a_t, b_t, dt, seed):
    """Device A [M,K] (stored [K,M] when a_t), B [K,N] (stored [N,K] when b_t),
    bias [N], the strides b200_gemm takes, and the host values the device
    operands hold (after rounding to bf16 where dt is bf16)."""
    rng = np.random.default_rng(seed)
    tdt = torch.bfloat16 if dt == kernels.DT_BF16 else torch.float32
    a = rng.standard_normal((K, M) if a_t else (M, K)).astype(np.float32)
    b = rng.standard_normal((N, K) if b_t else (K, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    A, B, BIAS = (torch.from_numpy(v).to("cuda", tdt) for v in (a, b, bias))
    strides = (M * K, 1 if a_t else K, M if a_t else 1, K * N, 1 if b_t else N, K if b_t else 1)
    host = [t.float().cpu().numpy().astype(np.float64) for t in (A, B, BIAS)]
    ha = host[0].T if a_t else host[0]
    hb = host[1].T if b_t else host[1]
    return A, B, BIAS, strides, (ha, hb, host[2])


def _reference(host, epi):
    """float64 product with the epilogue: 0 none, 1 +bias, 2 relu(+bias), 3 relu."""
    a, b, bias = host
    c = a @ b
    if epi in (1, 2):
        c = c + bias
    if epi in (2, 3):
        c = np.maximum(c, 0.0)
    return c


def _call(fn, A, B, BIAS, strides, M, N, K, dt, epi, C=None):
    if C is None:
        C = torch.full((M, N), float("nan"), device="cuda",
                       dtype=torch.bfloat16 if dt == kernels.DT_BF16 else torch.float32)
    sAb, sAm, sAk, sBb, sBk, sBn = strides
    fn(A.data_ptr(), B.data_ptr(), C.data_ptr(), BIAS.data_ptr(), 1, M, N, K, sAb, sAm, sAk,
       sBb, sBk, sBn, N, 1.0, dt, dt, epi, _stream())
    torch.cuda.synchronize()
    return C


_HIGH_MARKS = ("cudaMemPoolAttrReservedMemHigh", "cudaMemPoolAttrUsedMemHigh")


def _pool_high_marks():
    """High-water marks of the current device's default memory pool (the pool
    cudaMallocAsync draws from): reserved bytes and bytes in use."""
    from cuda.bindings import runtime as rt
    err, dev = rt.cudaGetDevice()
    assert err == rt.cudaError_t.cudaSuccess
    err, pool = rt.cudaDeviceGetDefaultMemPool(dev)
    assert err == rt.cudaError_t.cudaSuccess
    marks = []
    for name in _HIGH_MARKS:
        err, v = rt.cudaMemPoolGetAttribute(pool, getattr(rt.cudaMemPoolAttr, name))
        assert err == rt.cudaError_t.cudaSuccess
        marks.append(int(v))
    return marks, pool


def _reset_pool_high_marks(pool):
    """Both marks back to the pool's current levels (zero is the only value
    the runtime accepts, and it means "reset")."""
    from cuda.bindings import runtime as rt
    from cuda.bindings.driver import cuuint64_t
    for name in _HIGH_MARKS:
        err, = rt.cudaMemPoolSetAttribute(pool, getattr(rt.cudaMemPoolAttr, name), cuuint64_t(0))
        assert err == rt.cudaError_t.cudaSuccess


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
def test_noalloc_matches_reference_two_calls(M, N, K, a_t, b_t, dt, epi):
    tol = 2e-3 if dt == kernels.DT_F32 else 1e-2
    for call, seed in enumerate((M + K, M + K + 1)):  # two calls in a row, new inputs each
        A, B, BIAS, strides, host = _operands(M, N, K, a_t, b_t, dt, seed)
        got = _call(kernels.gemm_noalloc, A, B, BIAS, strides, M, N, K, dt, epi)
        got = got.float().cpu().numpy()
        assert np.isfinite(got).all()
        ref = _reference(host, epi)
        if dt == kernels.DT_BF16:
            ref = torch.from_numpy(ref.astype(np.float32)).bfloat16().float().numpy()
        assert_close(got, ref, tol, f"gemm_noalloc {M}x{N}x{K} call {call} vs float64")
        want = _call(kernels.gemm, A, B, BIAS, strides, M, N, K, dt, epi).float().cpu().numpy()
        assert_close(got, want, tol, f"gemm_noalloc {M}x{N}x{K} call {call} vs b200_gemm")
    assert kernels.device_error(clear=True) == 0


@pytest.mark.parametrize("M,N,K,a_t,b_t,dt,epi", [CASES[0], CASES[2], CASES[3]])
def test_noalloc_allocates_nothing(M, N, K, a_t, b_t, dt, epi):
    """With operands and output allocated beforehand and torch's allocator
    idle, calls leave the device's free memory and the default pool's
    high-water marks unchanged.  One call first loads the kernels
    (module loading is the driver's, not the call's)."""
    A, B, BIAS, strides, host = _operands(M, N, K, a_t, b_t, dt, 11)
    C = torch.empty((M, N), device="cuda",
                    dtype=torch.bfloat16 if dt == kernels.DT_BF16 else torch.float32)
    _call(kernels.gemm_noalloc, A, B, BIAS, strides, M, N, K, dt, epi, C)
    torch.cuda.synchronize()
    _, pool = _pool_high_marks()
    _reset_pool_high_marks(pool)
    high0, _ = _pool_high_marks()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _call(kernels.gemm_noalloc, A, B, BIAS, strides, M, N, K, dt, epi, C)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    high1, _ = _pool_high_marks()
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes"
    assert high1 == high0, f"default pool high-water marks (reserved, used) rose {high0} -> {high1}"
    ref = _reference(host, epi)
    tol = 2e-3 if dt == kernels.DT_F32 else 1e-2
    if dt == kernels.DT_BF16:
        ref = torch.from_numpy(ref.astype(np.float32)).bfloat16().float().numpy()
    assert_close(C.float().cpu().numpy(), ref, tol, "gemm_noalloc result after the memory check")


def test_noalloc_rejects_split_beyond_scratch():
    """1024x1024x4096 f32 splits K three ways: 12 MiB of partial sums, more than
    the 8 MiB array.  The call is refused before anything is launched, and the
    next call that fits still works."""
    M, N, K = 1024, 1024, 4096
    A, B, BIAS, strides, _ = _operands(M, N, K, False, False, kernels.DT_F32, 7)
    assert 3 * M * N * 4 > SCRATCH_BYTES
    with pytest.raises(kernels.KernelError, match="scratch") as e:
        _call(kernels.gemm_noalloc, A, B, BIAS, strides, M, N, K, kernels.DT_F32, 0)
    assert str(SCRATCH_BYTES) in str(e.value)
    M, N, K = 288, 64, 50176
    A, B, BIAS, strides, host = _operands(M, N, K, False, False, kernels.DT_F32, 8)
    got = _call(kernels.gemm_noalloc, A, B, BIAS, strides, M, N, K, kernels.DT_F32, 0)
    assert_close(got.cpu().numpy(), _reference(host, 0), 2e-3, "gemm_noalloc after a refused call")


@pytest.mark.parametrize("code", MIXED_CODES)
def test_noalloc_refuses_mixed_operand_types(code):
    """b200_gemm serves an f32 x bf16 pair by widening or splitting one operand
    into a workspace; the allocation-free entry point has none, so it refuses
    the pair (UNSUPPORTED) and leaves the output untouched."""
    M, N, K = 256, 256, 512
    a32 = code == 100
    A = torch.randn(M, K, device="cuda", dtype=torch.float32 if a32 else torch.bfloat16)
    B = torch.randn(K, N, device="cuda", dtype=torch.bfloat16 if a32 else torch.float32)
    C = torch.full((M, N), 7.0, device="cuda", dtype=torch.float32)
    with pytest.raises(kernels.KernelError, match=r"\(3\).*in_dtype must be F32 or BF16"):
        kernels.gemm_noalloc(A.data_ptr(), B.data_ptr(), C.data_ptr(), 0, 1, M, N, K, M * K, K, 1,
                             K * N, N, 1, N, 1.0, code, kernels.DT_F32, 0, _stream())
    torch.cuda.synchronize()
    assert bool((C == 7.0).all())
