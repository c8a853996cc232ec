"""CPU: pin the oracle (numpy StableHLO interpreter + closed forms) against the
reference's known-answer cases and against each other.  No GPU, no plugin."""
import numpy as np
import pytest

from cases import cases
from helpers import assert_close
from jax_b200 import programs
from oracle import hlo_interp, restate


@pytest.mark.parametrize("case", cases(), ids=lambda c: c[0])
def test_interpreter_matches_golden(case):
    name, prog, inputs, expected = case
    got = hlo_interp.run(prog, [inputs])[0][0]
    np.testing.assert_allclose(got, expected, rtol=1e-6, atol=1e-6, err_msg=name)


def test_sdpa_program_matches_closed_form():
    rng = np.random.default_rng(1)
    B, T, N, H = 2, 40, 3, 64
    q, k, v = (rng.standard_normal((B, T, N, H)).astype(np.float32) for _ in range(3))
    for causal in (True, False):
        got = hlo_interp.run(programs.sdpa(B, T, N, H, causal=causal), [[q, k, v]])[0][0]
        np.testing.assert_allclose(got, restate.sdpa_ref(q, k, v, causal=causal), rtol=1e-12, atol=1e-12)


def test_layer_norm_program_matches_closed_form():
    rng = np.random.default_rng(2)
    x, r = (rng.standard_normal((16, 128)).astype(np.float32) for _ in range(2))
    g = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    b = (0.1 * rng.standard_normal(128)).astype(np.float32)
    got = hlo_interp.run(programs.layer_norm(16, 128), [[x, r, g, b]])[0][0]
    np.testing.assert_allclose(got, restate.layer_norm_ref(x, r, g, b), rtol=1e-12, atol=1e-12)


def _mlp_inputs(rng, dims, batch):
    params = []
    for i in range(len(dims) - 1):
        params.append((rng.standard_normal((dims[i], dims[i + 1])) * 0.3).astype(np.float32))
        params.append((rng.standard_normal(dims[i + 1]) * 0.1).astype(np.float32))
    x = rng.random((batch, dims[0])).astype(np.float32)
    lab = rng.integers(0, dims[-1], batch).astype(np.int32)
    return params, x, lab


def test_mlp_step_program_matches_hand_backprop():
    rng = np.random.default_rng(3)
    dims, batch = (20, 16, 16, 5), 8
    params, x, lab = _mlp_inputs(rng, dims, batch)
    outs = hlo_interp.run(programs.mlp_step(batch=batch, dims=dims), [params + [x, lab]])[0]
    loss, new = restate.mlp_step_ref(params, x, lab)
    assert abs(outs[0] - loss) < 1e-12
    for a, b in zip(outs[1:], new):
        np.testing.assert_allclose(a, b, rtol=1e-12, atol=1e-12)


def test_data_parallel_program_equals_full_batch():
    """pmean over 2 replicas of half batches == one replica on the full batch."""
    rng = np.random.default_rng(4)
    dims, batch = (20, 16, 16, 5), 8
    params, x, lab = _mlp_inputs(rng, dims, batch)
    full = hlo_interp.run(programs.mlp_step(batch=batch, dims=dims), [params + [x, lab]])[0]
    dp = hlo_interp.run(programs.mlp_step(batch=batch // 2, dims=dims, num_replicas=2),
                        [params + [x[:4], lab[:4]], params + [x[4:], lab[4:]]])
    for rep in dp:
        for a, b in zip(rep, full):
            np.testing.assert_allclose(a, b, rtol=1e-12, atol=1e-13)


def test_cnn_gradients_match_finite_differences():
    rng = np.random.default_rng(5)
    shapes = [(3, 3, 1, 32), (32,), (3, 3, 32, 64), (64,), (3136, 256), (256,), (256, 10), (10,)]
    ps = [(rng.standard_normal(s) * 0.1).astype(np.float64) for s in shapes]
    x = rng.random((2, 28, 28, 1))
    lab = np.array([1, 7], dtype=np.int32)
    prog = programs.cnn_step(batch=2)
    interp = hlo_interp.Interp(prog)
    out = interp.run([ps + [x, lab]])[0]
    lr, eps = 1e-2, 1e-6
    for pi, idx in [(0, (1, 1, 0, 3)), (2, (0, 2, 5, 7)), (4, (100, 3)), (7, (4,))]:
        g_prog = (ps[pi][idx] - out[1 + pi][idx]) / lr
        pp = [p.copy() for p in ps]
        pp[pi][idx] += eps
        pm = [p.copy() for p in ps]
        pm[pi][idx] -= eps
        fd = (interp.run([pp + [x, lab]])[0][0] - interp.run([pm + [x, lab]])[0][0]) / (2 * eps)
        assert abs(g_prog - fd) <= 1e-6 + 1e-4 * abs(fd), (pi, idx, g_prog, fd)


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.0e-40, 3.0e38], np.float32)
    r = hlo_interp.bf16_round(x)
    assert r[0] == 1.0
    assert r[1] == 1.0                 # halfway, even mantissa stays
    assert r[2] == np.float32(1.0078125)
    assert np.isfinite(r[3])
    bits = hlo_interp.f32_to_bf16_bits(x)
    np.testing.assert_array_equal(hlo_interp.bf16_bits_to_f32(bits), r)


def test_reductions_over_empty_extents_give_init():
    """StableHLO reduce folds the operand into the init value: over an empty
    dimension each output is the init value itself (0 for sum, -inf for a
    max with JAX's init); with no outputs the result is empty."""
    from jax_b200.hlo import Builder
    b = Builder("empty_reduce")
    x, y = b.param((3, 0)), b.param((0, 5))
    text = b.module([b.sum(x, [1]), b.max(x, [1]), b.max(y, [1])])
    out = hlo_interp.run(text, [[np.zeros((3, 0), np.float32), np.zeros((0, 5), np.float32)]])[0]
    assert out[0].tolist() == [0.0] * 3 and out[1].tolist() == [-np.inf] * 3
    assert np.shape(out[2]) == (0,)


def test_bf16_chain_rounding_modes():
    """x * y + z in bf16 with x = y = 1 + 2^-7, z = -(1 + 2^-6).  Rounding each
    op (the default) drops the 2^-14 term of the product, so the sum is 0;
    excess precision keeps the chain unrounded until the bf16 output, which
    holds 2^-14 exactly.  A convert to bf16 inside the chain rounds in both
    modes."""
    from jax_b200.hlo import Builder
    b = Builder("bf16_chain")
    x, y, z = (b.param((4,), "bf16") for _ in range(3))
    prod = x * y
    held = b.convert(b.convert(prod, "f32"), "bf16")
    text = b.module([prod + z, held + z])
    one = np.float32(1 + 2.0 ** -7)
    args = [np.full(4, one), np.full(4, one), np.full(4, np.float32(-(1 + 2.0 ** -6)))]
    per_op = hlo_interp.run(text, [args])[0]
    excess = hlo_interp.run(text, [args], excess_bf16=True)[0]
    np.testing.assert_array_equal(per_op[0], 0.0)
    np.testing.assert_array_equal(excess[0], 2.0 ** -14)
    # the explicit f32 -> bf16 convert rounds the product in both modes
    np.testing.assert_array_equal(per_op[1], 0.0)
    np.testing.assert_array_equal(excess[1], 0.0)


def test_sdpa_bwd_restatement_matches_autodiff():
    """restate.sdpa_bwd_ref (reference sdpa.py:65-87) equals reverse-mode autodiff
    of the attention forward, both evaluated by the interpreter in f64."""
    from jax_b200.hlo import Builder
    from jax_b200.programs import softmax
    rng = np.random.default_rng(5)
    shp = (1, 16, 2, 8)
    q, k, v, g = (rng.standard_normal(shp) for _ in range(4))
    b = Builder()
    Q, K, Vv, G = (b.param(shp) for _ in range(4))
    logits = b.dot_general(Q, K, ([3], [3]), ([0, 2], [0, 2])) * 0.3
    o = b.transpose(b.dot_general(softmax(b, logits), Vv, ([3], [1]), ([0, 1], [0, 2])), [0, 2, 1, 3])
    loss = b.sum(o * G, [0, 1, 2, 3])
    grads = b.grad(loss, [Q, K, Vv])
    got = hlo_interp.run(b.module(grads), [[q, k, v, g]])[0]
    for gg, r in zip(got, restate.sdpa_bwd_ref(q, k, v, g, 0.3)):
        np.testing.assert_allclose(gg, r, rtol=1e-9, atol=1e-12)


@pytest.mark.parametrize("form,causal", [("autodiff", True), ("custom_jvp", True), ("custom_jvp", False)])
def test_attention_vjp_programs_match_closed_form(form, causal):
    """Both written forms of attention's vjp (programs.attention_vjp: the
    quotient-rule gradient and jax.nn.softmax's custom-JVP backward) evaluate,
    in f64, to restate.sdpa_bwd_ref -- the math the fused backward kernel runs."""
    from jax_b200 import programs
    rng = np.random.default_rng(17)
    shp = (1, 24, 2, 64)
    q, k, v, g = (rng.standard_normal(shp) for _ in range(4))
    text = programs.attention_vjp(B=1, T=24, N=2, H=64, causal=causal, dt="f32", form=form)
    o, dq, dk, dv = hlo_interp.run(text, [[q, k, v, g]])[0]
    np.testing.assert_allclose(o, restate.sdpa_ref(q, k, v, 0.125, causal), rtol=1e-9, atol=1e-12)
    for got, ref in zip((dq, dk, dv), restate.sdpa_bwd_ref(q, k, v, g, 0.125, causal)):
        np.testing.assert_allclose(got, ref, rtol=1e-9, atol=1e-12)


def test_layer_norm_bwd_restatement_matches_autodiff():
    from jax_b200.hlo import Builder
    rng = np.random.default_rng(6)
    x, dy = rng.standard_normal((5, 12)), rng.standard_normal((5, 12))
    w, bb = 1 + 0.1 * rng.standard_normal(12), 0.1 * rng.standard_normal(12)
    b = Builder()
    X, W, Bb, DY = b.param((5, 12)), b.param((12,)), b.param((12,)), b.param((5, 12))
    mean = b.sum(X, [1], keepdims=True) / 12.0
    d = X - mean
    var = b.sum(d * d, [1], keepdims=True) / 12.0
    y = d * b.rsqrt(var + 1e-5) * W + Bb
    grads = b.grad(b.sum(y * DY, [0, 1]), [X, W, Bb])
    got = hlo_interp.run(b.module(grads), [[x, w, bb, dy]])[0]
    for gg, r in zip(got, restate.layer_norm_bwd_ref(x, w, dy, 1e-5)):
        np.testing.assert_allclose(gg, r, rtol=1e-9, atol=1e-12)


# ------------------------------------------------ torch-CPU port (baseline) --
def _t(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(dtype) if dtype is not None else t


def test_torch_port_mlp_and_cnn_match_interpreter():
    """oracle/torch_port.py (timed as the CPU baseline, and the full-size
    oracle of the CNN step) restates the same programs: in float64 it agrees
    with the interpreter to 1e-10."""
    import torch
    from oracle import torch_port as tp
    rng = np.random.default_rng(61)
    dims, batch = (20, 16, 16, 5), 8
    params, x, lab = _mlp_inputs(rng, dims, batch)
    ref = hlo_interp.run(programs.mlp_step(batch=batch, dims=dims), [params + [x, lab]])[0]
    loss, new = tp.mlp_step([_t(p, torch.float64) for p in params], _t(x, torch.float64), _t(lab))
    assert abs(float(loss) - ref[0]) < 1e-10
    for a, b in zip(new, ref[1:]):
        np.testing.assert_allclose(a.numpy(), b, rtol=1e-10, atol=1e-12)
    shapes = [(3, 3, 1, 32), (32,), (3, 3, 32, 64), (64,), (3136, 256), (256,), (256, 10), (10,)]
    ps = [(rng.standard_normal(s) * (0.3 if len(s) > 1 else 0.05)).astype(np.float32) for s in shapes]
    xc = rng.random((3, 28, 28, 1)).astype(np.float32)
    lc = rng.integers(0, 10, 3).astype(np.int32)
    ref = hlo_interp.run(programs.cnn_step(batch=3, emit="grads"), [ps + [xc, lc]])[0]
    loss, new = tp.cnn_step([_t(p, torch.float64) for p in ps], _t(xc, torch.float64), _t(lc), lr=1.0)
    assert abs(float(loss) - ref[0]) < 1e-10
    for p, a, g in zip(ps, new, ref[1:]):
        np.testing.assert_allclose(p - a.numpy(), g, rtol=1e-9, atol=1e-11)


def test_torch_port_transformer_matches_interpreter():
    """The transformer port in float64 (every op in f64, no bf16 rounding)
    against the interpreter run with bf16 parameters widened to f64 the same
    way: loss to 1e-9 and every gradient to 1e-7 normwise."""
    import torch
    from oracle import torch_port as tp
    cfg = dict(batch=2, seq=32, layers=2, d=64, heads=2, ffn=128, vocab=97)
    shapes = programs.transformer_param_shapes(cfg["layers"], cfg["d"], cfg["heads"], cfg["ffn"],
                                               cfg["vocab"], cfg["seq"])
    rng = np.random.default_rng(62)
    params = [hlo_interp.bf16_round((rng.standard_normal(s) * (0.3 if len(s) > 1 else 0.1))
                                    .astype(np.float32)) for _, s in shapes]
    tok = rng.integers(0, cfg["vocab"], (cfg["batch"], cfg["seq"])).astype(np.int32)
    tgt = np.roll(tok, -1, axis=1)
    # the same program with f32 parameters: the interpreter evaluates it in f64
    text = programs.transformer_step(**cfg, emit="grads").replace("bf16", "f32")
    zeros = [np.zeros(s, np.float32) for _, s in shapes]
    ref = hlo_interp.run(text, [params + zeros + zeros + [np.array(0, np.int32), tok, tgt]])[0]
    names = [n for n, _ in shapes]
    loss, grads = tp.transformer_grads(names, [_t(p, torch.float64) for p in params], _t(tok), _t(tgt),
                                       layers=cfg["layers"], f32=torch.float64)
    assert abs(float(loss) - ref[0]) < 1e-9 * abs(ref[0])
    gd = {n: (g.numpy(), np.asarray(r, np.float64)) for n, g, r in zip(names, grads, ref[1:])}
    for n, (g, r) in gd.items():
        if n.endswith(".bk"):  # zero in exact arithmetic: both sides hold rounding noise
            scale = np.linalg.norm(gd[n[:-2] + "bq"][1])
            assert np.linalg.norm(g) < 1e-9 * scale and np.linalg.norm(r) < 1e-9 * scale
            continue
        rel = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-300)
        assert rel < 1e-7, f"{n}: {rel:.3e}"
