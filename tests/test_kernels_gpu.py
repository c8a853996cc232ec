"""GPU: the hand-written sm_100a kernels, called through their C ABI
(include/b200_kernels.h), against the float64 oracle.

Tolerances (written per test): fp32 non-contraction ops 1e-5 relative, with an
error floor of 1e-5 * rms(reference); contractions 2e-3 relative with a floor of
2e-3 * rms(reference) (TF32 / bf16 tensor-core inputs); bf16 outputs 1e-2."""
import numpy as np
import pytest

from helpers import assert_close
from jax_b200 import kernels
from oracle import restate

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream():
    return torch.cuda.current_stream().cuda_stream


def normwise(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-300))


def bf16_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(torch.bfloat16)


def host(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


@pytest.fixture(autouse=True)
def no_device_error():
    kernels.device_error(clear=True)
    yield
    assert kernels.device_error(clear=True) == 0, "a bounded device-side wait gave up"


# ------------------------------------------------------------------ LayerNorm
@pytest.mark.parametrize("rows,cols", [(4096, 1024), (7, 1000), (33, 128), (5, 4096), (3, 50)])
def test_ln_residual_f32(rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    x, r = (rng.standard_normal((rows, cols)).astype(np.float32) for _ in range(2))
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    b = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    X, R, G, B = dev(x), dev(r), dev(g), dev(b)
    Y = torch.empty_like(X)
    H = torch.empty_like(X)
    mean = torch.empty(rows, device="cuda")
    rstd = torch.empty(rows, device="cuda")
    kernels.ln_residual_fwd(X.data_ptr(), R.data_ptr(), G.data_ptr(), B.data_ptr(), Y.data_ptr(),
                            H.data_ptr(), mean.data_ptr(), rstd.data_ptr(), rows, cols, 1e-5,
                            kernels.DT_F32, 0, stream())
    ref = restate.layer_norm_ref(x, r, g, b)
    assert_close(host(Y), ref, 1e-5, "ln y", atol_rms=1.0)
    np.testing.assert_array_equal(host(H), x + r)  # the residual sum is exact in f32
    h64 = x.astype(np.float64) + r
    assert_close(host(mean), h64.mean(-1), 1e-5, "mean")
    assert_close(host(rstd), 1 / np.sqrt(h64.var(-1) + 1e-5), 1e-5, "rstd")


def test_ln_no_residual_no_affine_and_rms():
    rng = np.random.default_rng(11)
    x = rng.standard_normal((64, 512)).astype(np.float32)
    X = dev(x)
    Y = torch.empty_like(X)
    kernels.ln_residual_fwd(X.data_ptr(), 0, 0, 0, Y.data_ptr(), 0, 0, 0, 64, 512, 1e-6,
                            kernels.DT_F32, 0, stream())
    assert_close(host(Y), restate.layer_norm_ref(x, None, None, None, 1e-6), 1e-5, "ln")
    kernels.ln_residual_fwd(X.data_ptr(), 0, 0, 0, Y.data_ptr(), 0, 0, 0, 64, 512, 1e-6,
                            kernels.DT_F32, 1, stream())
    xd = x.astype(np.float64)
    rms_ref = xd / np.sqrt((xd * xd).mean(-1, keepdims=True) + 1e-6)
    assert_close(host(Y), rms_ref, 1e-5, "rms")


def test_ln_bf16():
    rng = np.random.default_rng(12)
    rows, cols = 256, 512
    x, r = (rng.standard_normal((rows, cols)).astype(np.float32) for _ in range(2))
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    b = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    X, R, G, B = bf16_dev(x), bf16_dev(r), bf16_dev(g), bf16_dev(b)
    Y = torch.empty_like(X)
    kernels.ln_residual_fwd(X.data_ptr(), R.data_ptr(), G.data_ptr(), B.data_ptr(), Y.data_ptr(),
                            0, 0, 0, rows, cols, 1e-5, kernels.DT_BF16, 0, stream())
    xr = [host(t) for t in (X, R, G, B)]
    assert_close(host(Y), restate.layer_norm_ref(*xr), 1e-2, "ln bf16")


def test_ln_bwd_f32():
    rng = np.random.default_rng(13)
    rows, cols = 100, 256
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    dy = rng.standard_normal((rows, cols)).astype(np.float32)
    X, Gd, DY = dev(x), dev(g), dev(dy)
    Y = torch.empty_like(X)
    mean = torch.empty(rows, device="cuda")
    rstd = torch.empty(rows, device="cuda")
    kernels.ln_residual_fwd(X.data_ptr(), 0, Gd.data_ptr(), 0, Y.data_ptr(), 0, mean.data_ptr(),
                            rstd.data_ptr(), rows, cols, 1e-5, kernels.DT_F32, 0, stream())
    DX = torch.empty_like(X)
    dg = torch.empty(cols, device="cuda")
    db = torch.empty(cols, device="cuda")
    ws = torch.empty(kernels.ln_bwd_workspace(rows, cols) // 4, device="cuda")
    kernels.ln_bwd(X.data_ptr(), Gd.data_ptr(), mean.data_ptr(), rstd.data_ptr(), DY.data_ptr(),
                   DX.data_ptr(), dg.data_ptr(), db.data_ptr(), ws.data_ptr(), rows, cols,
                   kernels.DT_F32, stream())
    rdx, rdg, rdb = restate.layer_norm_bwd_ref(x, g, dy)
    assert_close(host(DX), rdx, 1e-4, "dx")
    assert_close(host(dg), rdg, 1e-4, "dgamma")
    assert_close(host(db), rdb, 1e-4, "dbeta")


# ----------------------------------------------------------------------- SDPA
@pytest.mark.parametrize("B,T,N,causal", [(8, 512, 8, True), (8, 512, 8, False), (2, 200, 3, True),
                                          (1, 128, 1, True), (2, 384, 2, False), (1, 1, 1, True),
                                          (1, 1024, 2, True), (1, 1000, 2, False)])
def test_sdpa_f32(B, T, N, causal):
    rng = np.random.default_rng(B * 1000 + T + N)
    q, k, v = (rng.standard_normal((B, T, N, 64)).astype(np.float32) for _ in range(3))
    Q, K, V = dev(q), dev(k), dev(v)
    O = torch.empty_like(Q)
    kernels.sdpa_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, T, T, N, 64,
                     0.125, causal, kernels.DT_F32, stream())
    assert_close(host(O), restate.sdpa_ref(q, k, v, 0.125, causal), 2e-3, "sdpa f32")


def test_sdpa_cross_lengths_non_causal():
    rng = np.random.default_rng(21)
    B, T, S, N = 2, 130, 300, 2
    q = rng.standard_normal((B, T, N, 64)).astype(np.float32)
    k, v = (rng.standard_normal((B, S, N, 64)).astype(np.float32) for _ in range(2))
    Q, K, V = dev(q), dev(k), dev(v)
    O = torch.empty_like(Q)
    kernels.sdpa_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, T, S, N, 64,
                     0.125, False, kernels.DT_F32, stream())
    assert_close(host(O), restate.sdpa_ref(q, k, v, 0.125, False), 2e-3, "sdpa T!=S")


@pytest.mark.parametrize("causal", [True, False])
def test_sdpa_bf16(causal):
    rng = np.random.default_rng(22)
    B, T, N = 4, 256, 8
    q, k, v = (rng.standard_normal((B, T, N, 64)).astype(np.float32) for _ in range(3))
    Q, K, V = bf16_dev(q), bf16_dev(k), bf16_dev(v)
    O = torch.empty_like(Q)
    kernels.sdpa_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, T, T, N, 64,
                     0.125, causal, kernels.DT_BF16, stream())
    ref = restate.sdpa_ref(host(Q), host(K), host(V), 0.125, causal)
    assert_close(host(O), ref, 2e-2, "sdpa bf16")


@pytest.mark.parametrize("B,T,N,causal", [(2, 256, 3, True), (2, 256, 3, False), (3, 128, 2, True),
                                          (2, 200, 2, True), (1, 77, 2, False), (1, 1, 1, True)])
def test_sdpa_bwd_bf16(B, T, N, causal):
    """Forward with row statistics, then the fused backward, against the float64
    closed form of the kernel's formula on the same bf16 inputs: P rounded to
    bf16 in dV (as jax.nn.dot_product_attention rounds the probabilities) and
    the row term rowsum(dO * O) taken from the forward's bf16 O.  bf16
    outputs: 2e-2 relative with a floor of 2e-2 * rms(reference).  Against
    the exact closed form the gradients stay within 1e-2 normwise."""
    rng = np.random.default_rng(B * 100 + T + N + causal)
    q, k, v, g = (rng.standard_normal((B, T, N, 64)).astype(np.float32) for _ in range(4))
    Q, K, V, G = (bf16_dev(a) for a in (q, k, v, g))
    O = torch.empty_like(Q)
    lse = torch.empty((B, N, T), device="cuda")
    dense = [T * N * 64, N * 64, 64]
    kernels.sdpa_fwd_lse(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), lse.data_ptr(), B, T,
                         T, N, 64, dense * 4, 0.125, causal, kernels.DT_BF16, stream())
    qh, kh, vh, gh = (host(a) for a in (Q, K, V, G))
    assert_close(host(O), restate.sdpa_ref(qh, kh, vh, 0.125, causal), 2e-2, "sdpa fwd")
    s = np.einsum("btnh,bsnh->bnts", qh.astype(np.float64), kh.astype(np.float64)) * 0.125
    if causal:
        s = np.where(np.tril(np.ones((T, T), bool)), s, -np.inf)
    mx = s.max(-1, keepdims=True)
    ref_lse = (mx[..., 0] + np.log(np.exp(s - mx).sum(-1))) / np.log(2.0)
    assert_close(host(lse), ref_lse, 1e-5, "lse2")
    dQ, dK, dV = (torch.empty_like(Q) for _ in range(3))
    kernels.sdpa_bwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), G.data_ptr(), lse.data_ptr(),
                     dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), B, T, N, 64, dense * 8, 0.125, causal,
                     kernels.DT_BF16, stream())
    rq, rk, rv = restate.sdpa_bwd_ref(qh, kh, vh, gh, 0.125, causal, probs_bf16=True, o=host(O))
    assert_close(host(dV), rv, 2e-2, "dv")
    assert_close(host(dK), rk, 2e-2, "dk")
    assert_close(host(dQ), rq, 2e-2, "dq")
    for got, ref, nm in zip((dQ, dK, dV), restate.sdpa_bwd_ref(qh, kh, vh, gh, 0.125, causal), "qkv"):
        assert normwise(host(got), ref) <= 1e-2, f"d{nm} vs the exact closed form"


def test_sdpa_bwd_bnth_strides():
    """BNTH inputs and BTNH outputs through the strides (the plugin's layouts)."""
    rng = np.random.default_rng(31)
    B, N, T = 2, 4, 256
    qb, kb, vb, gb = (rng.standard_normal((B, N, T, 64)).astype(np.float32) for _ in range(4))
    Q, K, V, G = (bf16_dev(a) for a in (qb, kb, vb, gb))
    O = torch.empty((B, N, T, 64), device="cuda", dtype=torch.bfloat16)
    lse = torch.empty((B, N, T), device="cuda")
    bnth, btnh = [N * T * 64, 64, T * 64], [T * N * 64, N * 64, 64]
    kernels.sdpa_fwd_lse(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), lse.data_ptr(), B, T,
                         T, N, 64, bnth * 4, 0.125, True, kernels.DT_BF16, stream())
    dQ, dK, dV = (torch.empty((B, T, N, 64), device="cuda", dtype=torch.bfloat16) for _ in range(3))
    kernels.sdpa_bwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), G.data_ptr(), lse.data_ptr(),
                     dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), B, T, N, 64, bnth * 5 + btnh * 3, 0.125,
                     True, kernels.DT_BF16, stream())
    tr = lambda a: np.transpose(a, (0, 2, 1, 3))
    rq, rk, rv = restate.sdpa_bwd_ref(*(tr(host(a)) for a in (Q, K, V, G)), 0.125, True,
                                      probs_bf16=True, o=tr(host(O)))
    assert_close(host(dV), rv, 2e-2, "dv")
    assert_close(host(dK), rk, 2e-2, "dk")
    assert_close(host(dQ), rq, 2e-2, "dq")


def test_sdpa_bnth_strides_and_simt_fallback():
    """BNTH views through the strided entry point, and head dim 32 (SIMT path)."""
    rng = np.random.default_rng(23)
    B, N, T = 2, 4, 256
    qb, kb, vb = (rng.standard_normal((B, N, T, 64)).astype(np.float32) for _ in range(3))
    Q, K, V = dev(qb), dev(kb), dev(vb)
    O = torch.empty((B, T, N, 64), device="cuda")
    st = [N * T * 64, 64, T * 64] * 3 + [T * N * 64, N * 64, 64]
    kernels.sdpa_fwd_strided(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, T, T, N, 64,
                             st, 0.125, True, kernels.DT_F32, stream())
    tr = lambda a: np.transpose(a, (0, 2, 1, 3))
    assert_close(host(O), restate.sdpa_ref(tr(qb), tr(kb), tr(vb), 0.125, True), 2e-3, "bnth")
    q, k, v = (rng.standard_normal((1, 64, 2, 32)).astype(np.float32) for _ in range(3))
    Q, K, V = dev(q), dev(k), dev(v)
    O = torch.empty_like(Q)
    kernels.sdpa_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), 1, 64, 64, 2, 32,
                     0.2, True, kernels.DT_F32, stream())
    assert_close(host(O), restate.sdpa_ref(q, k, v, 0.2, True), 1e-5, "simt")


# ----------------------------------------------------------------------- GEMM
def _gemm_case(M, N, K, a_t, b_t, dt, batch=1, epi=0, seed=0, out_dt=None):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((batch, M, K)).astype(np.float32)
    b = rng.standard_normal((batch, K, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    conv = bf16_dev if dt == kernels.DT_BF16 else dev
    # physical layouts: a_t -> stored [batch, K, M]; b_t -> stored [batch, N, K]
    A = conv(np.swapaxes(a, 1, 2).copy() if a_t else a)
    Bm = conv(np.swapaxes(b, 1, 2).copy() if b_t else b)
    if dt == kernels.DT_BF16:
        a = host(A) if not a_t else np.swapaxes(host(A), 1, 2)
        b = host(Bm) if not b_t else np.swapaxes(host(Bm), 1, 2)
    sAb, sAm, sAk = M * K, (1 if a_t else K), (M if a_t else 1)
    sBb, sBk, sBn = K * N, (1 if b_t else N), (K if b_t else 1)
    out_dt = dt if out_dt is None else out_dt
    out_t = torch.bfloat16 if out_dt == kernels.DT_BF16 else torch.float32
    C = torch.empty((batch, M, N), device="cuda", dtype=out_t)
    BIAS = (bf16_dev if out_dt == kernels.DT_BF16 else dev)(bias)  # bias has the output's type
    tc = kernels.gemm_uses_tensor_cores(A.data_ptr(), Bm.data_ptr(), batch, K, sAb, sAm, sAk, sBb,
                                        sBk, sBn, dt)
    kernels.gemm(A.data_ptr(), Bm.data_ptr(), C.data_ptr(), BIAS.data_ptr(), batch, M, N, K, sAb, sAm,
                 sAk, sBb, sBk, sBn, N, 1.0, dt, out_dt, epi, stream())
    ref = np.einsum("bmk,bkn->bmn", a.astype(np.float64), b.astype(np.float64))
    if epi in (1, 2):
        ref = ref + host(BIAS)
    if epi >= 2:
        ref = np.maximum(ref, 0)
    return host(C), ref, tc


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("dt", [kernels.DT_F32, kernels.DT_BF16])
def test_gemm_layouts(a_t, b_t, dt):
    got, ref, tc = _gemm_case(296, 264, 200, a_t, b_t, dt, seed=a_t * 2 + b_t)
    assert tc, "expected the tcgen05 path"
    assert_close(got, ref, 2e-3 if dt == kernels.DT_F32 else 1e-2, f"gemm a_t={a_t} b_t={b_t}")


def _kernel_names(fn):
    """Names of the CUDA kernels `fn` launches (CUPTI sees every kernel of the
    process, ones launched from this package's libraries included)."""
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}


@pytest.mark.parametrize("out_dt", [kernels.DT_BF16, kernels.DT_F32])
@pytest.mark.parametrize("M,N,K,a_t,b_t,batch,epi", [(2520, 2376, 200, False, False, 1, 0),
                                                     (2520, 2376, 200, False, True, 1, 1),
                                                     (2520, 2376, 200, True, False, 1, 2),
                                                     (2520, 2376, 200, True, True, 1, 0),
                                                     (1000, 744, 128, False, True, 8, 1),
                                                     (4200, 4160, 72, False, True, 1, 0),
                                                     (512, 512, 8192, True, False, 1, 0),
                                                     (600, 520, 3000, True, False, 1, 2),
                                                     (256, 512, 2048, False, True, 4, 1)])
def test_gemm_two_sm_pairs(M, N, K, a_t, b_t, batch, epi, out_dt):
    """bf16 GEMMs run on the two-SM kernel (one 256-row MMA per SM pair,
    cta_group::2): with at least 74 tiles of 256 x 256 whole, with fewer (the
    last three shapes: weight-gradient-like, long K) as K splits whose f32
    partials are summed afterwards.  Ragged M, N and K, every operand layout,
    a batch, the bias and bias+relu epilogues and the grouped tile order
    (17 x 17 tiles).  vs f64 on the bf16 values, 1e-2 relative."""
    res = {}

    def run():
        res["v"] = _gemm_case(M, N, K, a_t, b_t, kernels.DT_BF16, batch=batch, epi=epi,
                              seed=M + N + K + 2 * a_t + b_t, out_dt=out_dt)

    n0 = kernels.lib().b200_kernel_launches()
    names = _kernel_names(run)
    launched = kernels.lib().b200_kernel_launches() - n0
    got, ref, tc = res["v"]
    assert tc
    if names:
        assert any("gemm_tc_pair" in n for n in names), sorted(names)
    split = -(-M // 256) * -(-N // 256) * batch < 74  # fewer tiles than SM pairs: K splits + their sum
    assert launched == (2 if split else 1), launched
    assert_close(got, ref, 1e-2, f"pair gemm {batch}x{M}x{N}x{K} a_t={a_t} b_t={b_t} epi={epi}")


# in_dtype codes for one f32 and one bf16 operand (csrc/kernels/gemm_ws.h)
GEMM_DT_A_F32_B_BF16, GEMM_DT_A_BF16_B_F32 = 100, 101


@pytest.mark.parametrize("a32", [True, False])
@pytest.mark.parametrize("M,N,K,a_t,b_t,batch", [(296, 264, 200, False, False, 1),
                                                 (256, 256, 64, True, False, 16),
                                                 (256, 64, 256, False, True, 8),
                                                 (100, 37, 12, False, False, 1)])
def test_gemm_mixed_f32_bf16(a32, M, N, K, a_t, b_t, batch):
    """One f32 and one bf16 operand (JAX's transpose rule for a bf16 dot with
    an f32 result): the f32 side as bf16 hi + lo planes, the bf16 side read as
    it is (the last shape takes the widen-to-f32 fallback: 12-element rows are
    not 16-byte strided in bf16).  vs f64 on the same values, 2e-3 relative."""
    rng = np.random.default_rng(M + N + K + a32)
    a = rng.standard_normal((batch, M, K)).astype(np.float32)
    b = rng.standard_normal((batch, K, N)).astype(np.float32)
    A_phys = np.swapaxes(a, 1, 2).copy() if a_t else a
    B_phys = np.swapaxes(b, 1, 2).copy() if b_t else b
    A = dev(A_phys) if a32 else bf16_dev(A_phys)
    Bm = bf16_dev(B_phys) if a32 else dev(B_phys)
    a_val = host(A) if not a_t else np.swapaxes(host(A), 1, 2)
    b_val = host(Bm) if not b_t else np.swapaxes(host(Bm), 1, 2)
    sAb, sAm, sAk = M * K, (1 if a_t else K), (M if a_t else 1)
    sBb, sBk, sBn = K * N, (1 if b_t else N), (K if b_t else 1)
    C = torch.full((batch, M, N), float("nan"), device="cuda", dtype=torch.float32)
    code = GEMM_DT_A_F32_B_BF16 if a32 else GEMM_DT_A_BF16_B_F32
    kernels.gemm(A.data_ptr(), Bm.data_ptr(), C.data_ptr(), 0, batch, M, N, K, sAb, sAm, sAk, sBb,
                 sBk, sBn, N, 1.0, code, kernels.DT_F32, 0, stream())
    ref = np.einsum("bmk,bkn->bmn", a_val.astype(np.float64), b_val.astype(np.float64))
    assert_close(host(C), ref, 2e-3, f"mixed gemm a32={a32} {batch}x{M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K,b_t", [(512, 96, 288, False), (300, 40, 576, True), (100, 37, 12, False)])
def test_gemm_with_given_planes(M, N, K, b_t):
    """An f32 A handed over as bf16 hi + lo planes (what the im2col kernels of
    f32 convolutions write) with f32 B: the persistent kernel reads them
    directly; K = 12 (rows not 16-byte strided in bf16) joins them back into
    f32 for the fallback path.  vs f64 on hi + lo, 2e-3 relative."""
    import ctypes as C
    rng = np.random.default_rng(M + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N)).astype(np.float32)
    hi = torch.from_numpy(a).to("cuda", torch.bfloat16)
    lo = (torch.from_numpy(a).cuda() - hi.float()).to(torch.bfloat16)
    Bm = dev(b.T.copy() if b_t else b)
    sBk, sBn = (1, K) if b_t else (N, 1)
    C_ = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
    lib = kernels.lib()
    f = lib.b200_gemm_planes_ws
    f.restype = C.c_int
    f.argtypes = [C.c_void_p] * 6 + [C.c_int64] * 11 + [C.c_float, C.c_int, C.c_int, C.c_int,
                                                         C.c_void_p, C.c_void_p, C.c_size_t]
    q = lib.b200_gemm_planes_workspace_bytes
    q.restype = C.c_int64
    q.argtypes = f.argtypes[:-2]
    args = [hi.data_ptr(), lo.data_ptr(), Bm.data_ptr(), None, C_.data_ptr(), None, 1, M, N, K, 0, K, 1,
            0, sBk, sBn, N, 1.0, kernels.DT_F32, kernels.DT_F32, 0, stream()]
    wsb = q(*args)
    assert wsb >= 0
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device="cuda")
    kernels._check(f(*args, ws.data_ptr(), wsb), "gemm_planes_ws")
    torch.cuda.synchronize()
    ref = (hi.double() + lo.double()).cpu().numpy() @ b.astype(np.float64)
    assert_close(host(C_), ref, 2e-3, f"gemm planes {M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 784), (1024, 1024, 1024), (128, 128, 32), (1, 64, 16),
                                   (200704, 32, 12)])
def test_gemm_config_shapes_f32(M, N, K):
    got, ref, tc = _gemm_case(M, N, K, False, False, kernels.DT_F32, seed=M + N + K)
    assert tc
    assert_close(got, ref, 2e-3, f"gemm {M}x{N}x{K}")


def test_gemm_batched_and_epilogues():
    for epi in (1, 2, 3):
        got, ref, tc = _gemm_case(256, 192, 96, False, True, kernels.DT_F32, batch=3, epi=epi, seed=epi)
        assert tc
        assert_close(got, ref, 2e-3, f"epi {epi}")


@pytest.mark.parametrize("M,N,K,a_t,b_t", [(288, 64, 50176, False, False), (9, 32, 200704, False, False),
                                           (3136, 256, 256, True, False), (1024, 1024, 1024, True, False)])
def test_gemm_split_k_tall_skinny(M, N, K, a_t, b_t):
    """Few output tiles and a long K loop: the K range is split over CTAs and
    the partial sums reduced in a fixed order (conv weight gradients, dense wgrads)."""
    got, ref, tc = _gemm_case(M, N, K, a_t, b_t, kernels.DT_F32, seed=M + K)
    assert tc
    assert_close(got, ref, 2e-3, f"split-k {M}x{N}x{K}")
    got2, _, _ = _gemm_case(M, N, K, a_t, b_t, kernels.DT_F32, seed=M + K)
    np.testing.assert_array_equal(got, got2)  # deterministic


def test_gemm_simt_split_k_small_n():
    got, ref, tc = _gemm_case(1024, 10, 4096, False, False, kernels.DT_F32, seed=12)
    assert not tc
    assert_close(got, ref, 1e-5, "simt split-k")


def test_gemm_simt_fallback_for_unaligned_rows():
    got, ref, tc = _gemm_case(1024, 10, 1024, False, False, kernels.DT_F32, seed=9)
    assert not tc
    assert_close(got, ref, 1e-5, "simt N=10")
    got, ref, tc = _gemm_case(33, 17, 9, True, False, kernels.DT_F32, seed=10)
    assert not tc
    assert_close(got, ref, 1e-5, "simt odd")


# bf16 operands take the persistent kernel (two TMEM accumulators, TMA-store
# epilogue); these cover its tile edges, MN-major operands, f32 and bf16
# outputs, epilogues, batching and split-K.
@pytest.mark.parametrize("M,N,K,a_t,b_t,out_f32", [
    (1024, 2048, 512, False, False, False),    # FFN up
    (520, 776, 264, False, True, True),        # ragged edges, B transposed, f32 out
    (256, 512, 4096, True, False, False),      # weight-gradient form, split-K
    (300, 96, 192, True, True, True),          # BN 128, both transposed
    (4096, 64, 256, False, False, False),      # BN 64
])
def test_gemm_bf16_persistent(M, N, K, a_t, b_t, out_f32):
    if a_t and M % 8:
        M += 8 - M % 8  # an MN-major bf16 A needs 16-byte rows
    out = kernels.DT_F32 if out_f32 else kernels.DT_BF16
    got, ref, tc = _gemm_case(M, N, K, a_t, b_t, kernels.DT_BF16, seed=M + N, out_dt=out)
    assert tc
    assert_close(got, ref, 1e-2, f"bf16 gemm {M}x{N}x{K}")


def test_gemm_bf16_persistent_batched_epilogues():
    for epi in (1, 2, 3):
        got, ref, tc = _gemm_case(256, 256, 64, False, True, kernels.DT_BF16, batch=12, epi=epi,
                                  seed=40 + epi, out_dt=kernels.DT_F32)
        assert tc
        assert_close(got, ref, 1e-2, f"bf16 batched epi {epi}")
