"""The reference's fused-op primitives, defined here for the "b200" platform.

The reference plugin exposes attention and LayerNorm as JAX primitives whose
lowerings on its platform are custom calls the plugin executes:

=====================  ==========================  ===========================
primitive              operands -> results         ``backend_config``
=====================  ==========================  ===========================
``mlx_sdpa``           q, k, v -> o                ``{"scale": s}``
``mlx_sdpa_bwd``       q, k, v, do -> dq, dk, dv   ``{"scale": s}``
``mlx_layer_norm``     x, w, b -> y                ``{"eps": e}``
``mlx_layer_norm_bwd`` x, w, b, dy -> dx, dw, db   ``{"eps": e}``
=====================  ==========================  ===========================

(reference ``src/jax_mlx/sdpa.py:35-151``, ``src/jax_mlx/layer_norm.py:29-138``;
q, k, v, o are [B, T, N, H]).  This module defines the same four primitives,
with the same names, operands, results, call targets and ``backend_config``
JSON, lowers them to those custom calls on platform "b200" (the plugin runs
``mlx_sdpa`` on its tcgen05 attention kernel and ``mlx_layer_norm`` on its
LayerNorm kernel, and expands the two backward calls at compile time), and
to plain JAX math everywhere else, as the reference does.  ``dot_product_attention``
and ``layer_norm`` wrap them with a custom VJP (forward primitive, backward
primitive), like the reference's ``mlx_dot_product_attention`` /
``_mlx_layer_norm_with_grad``.

Nothing here runs without JAX: the primitives are created on first use
(``primitives()``), so importing the package on a machine without JAX is
harmless.
"""
from __future__ import annotations

from typing import Dict

PLATFORM = "b200"
TARGETS = ("mlx_sdpa", "mlx_sdpa_bwd", "mlx_layer_norm", "mlx_layer_norm_bwd")

_PRIMS: Dict[str, object] = {}


# ---------------------------------------------------------------- math -----
def _sdpa_math(q, k, v, scale):
    """softmax(q k^T * scale) v over [B, T, N, H] (reference sdpa.py:19-31)."""
    import jax
    import jax.numpy as jnp
    qt, kt, vt = (jnp.transpose(a, (0, 2, 1, 3)) for a in (q, k, v))
    s = jnp.matmul(qt, jnp.swapaxes(kt, -2, -1)) * jnp.asarray(scale, dtype=qt.dtype)
    p = jax.nn.softmax(s, axis=-1)
    return jnp.transpose(jnp.matmul(p, vt), (0, 2, 1, 3))


def _sdpa_bwd_math(q, k, v, g, scale):
    """(dq, dk, dv) of _sdpa_math for output cotangent g (reference sdpa.py:65-87)."""
    import jax
    import jax.numpy as jnp
    qt, kt, vt, gt = (jnp.transpose(a, (0, 2, 1, 3)) for a in (q, k, v, g))
    p = jax.nn.softmax(jnp.matmul(qt, jnp.swapaxes(kt, -2, -1)) * scale, axis=-1)
    dv = jnp.matmul(jnp.swapaxes(p, -2, -1), gt)
    dp = jnp.matmul(gt, jnp.swapaxes(vt, -2, -1))
    ds = p * (dp - jnp.sum(dp * p, axis=-1, keepdims=True)) * scale
    dq = jnp.matmul(ds, kt)
    dk = jnp.matmul(jnp.swapaxes(ds, -2, -1), qt)
    return tuple(jnp.transpose(a, (0, 2, 1, 3)) for a in (dq, dk, dv))


def _ln_math(x, w, b, eps):
    """(x - mean) / sqrt(var + eps) * w + b over the last axis (layer_norm.py:20-25)."""
    import jax.numpy as jnp
    mean = jnp.mean(x, axis=-1, keepdims=True)
    var = jnp.var(x, axis=-1, keepdims=True)
    return (x - mean) / jnp.sqrt(var + eps) * w + b


def _ln_bwd_math(x, w, b, g, eps):
    """(dx, dw, db) of _ln_math for output cotangent g (layer_norm.py:59-76)."""
    import jax.numpy as jnp
    mean = jnp.mean(x, axis=-1, keepdims=True)
    std = jnp.sqrt(jnp.var(x, axis=-1, keepdims=True) + eps)
    xhat = (x - mean) / std
    lead = tuple(range(g.ndim - 1))
    db = jnp.sum(g, axis=lead)
    dw = jnp.sum(g * xhat, axis=lead)
    gw = g * w
    dx = (gw - jnp.mean(gw, axis=-1, keepdims=True)
          - xhat * jnp.mean(gw * xhat, axis=-1, keepdims=True)) / std
    return dx, dw, db


# ---------------------------------------------------------- primitives -----
def primitives() -> Dict[str, object]:
    """The four primitives (created once), with abstract evaluation and a
    plain-JAX implementation for eager use off the plugin."""
    if _PRIMS:
        return _PRIMS
    from jax._src import core
    sdpa = core.Primitive("mlx_sdpa")
    sdpa_bwd = core.Primitive("mlx_sdpa_bwd")
    sdpa_bwd.multiple_results = True
    ln = core.Primitive("mlx_layer_norm")
    ln_bwd = core.Primitive("mlx_layer_norm_bwd")
    ln_bwd.multiple_results = True

    sdpa.def_abstract_eval(lambda q, k, v, *, scale: core.ShapedArray(q.shape, q.dtype))
    sdpa.def_impl(lambda q, k, v, *, scale: _sdpa_math(q, k, v, scale))
    sdpa_bwd.def_abstract_eval(lambda q, k, v, g, *, scale: (core.ShapedArray(q.shape, q.dtype),
                                                              core.ShapedArray(k.shape, k.dtype),
                                                              core.ShapedArray(v.shape, v.dtype)))
    sdpa_bwd.def_impl(lambda q, k, v, g, *, scale: _sdpa_bwd_math(q, k, v, g, scale))
    ln.def_abstract_eval(lambda x, w, b, *, eps: core.ShapedArray(x.shape, x.dtype))
    ln.def_impl(lambda x, w, b, *, eps: _ln_math(x, w, b, eps))
    ln_bwd.def_abstract_eval(lambda x, w, b, g, *, eps: (core.ShapedArray(x.shape, x.dtype),
                                                          core.ShapedArray(w.shape, w.dtype),
                                                          core.ShapedArray(b.shape, b.dtype)))
    ln_bwd.def_impl(lambda x, w, b, g, *, eps: _ln_bwd_math(x, w, b, g, eps))
    _PRIMS.update({"mlx_sdpa": sdpa, "mlx_sdpa_bwd": sdpa_bwd, "mlx_layer_norm": ln,
                   "mlx_layer_norm_bwd": ln_bwd})
    return _PRIMS


def _custom_call_lowering(target: str, key: str):
    """A lowering that emits stablehlo.custom_call @target with the primitive's
    operands, its result types and backend_config {"<key>": value}."""
    def lower(ctx, *operands, **params):
        from jax._src.interpreters import mlir
        result_types = [mlir.aval_to_ir_type(a) for a in ctx.avals_out]
        out = mlir.custom_call(call_target_name=target, result_types=result_types,
                               operands=list(operands),
                               backend_config='{"%s": %s}' % (key, repr(float(params[key]))))
        return out.results
    lower.__name__ = f"{target}_lowering"
    return lower


def register_lowerings(platform: str = PLATFORM, prims: Dict[str, object] = None) -> Dict[str, object]:
    """Register the custom-call lowerings of the four primitives for
    `platform` (and plain-JAX lowerings for every other platform).  `prims`
    defaults to this module's primitives; the reference package's own
    primitive objects can be passed too, so that programs written against
    it lower to the same custom calls here."""
    from jax._src.interpreters import mlir
    prims = prims or primitives()
    keys = {"mlx_sdpa": "scale", "mlx_sdpa_bwd": "scale", "mlx_layer_norm": "eps",
            "mlx_layer_norm_bwd": "eps"}
    fallback = {
        "mlx_sdpa": (lambda q, k, v, scale=1.0: _sdpa_math(q, k, v, scale), False),
        "mlx_sdpa_bwd": (lambda q, k, v, g, scale=1.0: _sdpa_bwd_math(q, k, v, g, scale), True),
        "mlx_layer_norm": (lambda x, w, b, eps=1e-5: _ln_math(x, w, b, eps), False),
        "mlx_layer_norm_bwd": (lambda x, w, b, g, eps=1e-5: _ln_bwd_math(x, w, b, g, eps), True),
    }
    for name in TARGETS:
        p = prims[name]
        mlir.register_lowering(p, _custom_call_lowering(name, keys[name]), platform=platform)
        fn, multi = fallback[name]
        mlir.register_lowering(p, mlir.lower_fun(fn, multiple_results=multi))
    return prims


# ------------------------------------------------------ custom-VJP wrappers --
def dot_product_attention(query, key, value, scale: float):
    """Attention over [B, T, N, H] through mlx_sdpa, with mlx_sdpa_bwd as its
    VJP (reference sdpa.py:154-190, mlx_dot_product_attention)."""
    import jax
    P = primitives()
    scale = float(scale)

    @jax.custom_vjp
    def f(q, k, v):
        return P["mlx_sdpa"].bind(q, k, v, scale=scale)

    def fwd(q, k, v):
        return f(q, k, v), (q, k, v)

    def bwd(res, g):
        return tuple(P["mlx_sdpa_bwd"].bind(*res, g, scale=scale))

    f.defvjp(fwd, bwd)
    return f(query, key, value)


def layer_norm(x, weight, bias, eps: float = 1e-5):
    """LayerNorm over the last axis through mlx_layer_norm, with
    mlx_layer_norm_bwd as its VJP (reference layer_norm.py:141-171)."""
    import jax
    P = primitives()
    eps = float(eps)

    @jax.custom_vjp
    def f(a, w, b):
        return P["mlx_layer_norm"].bind(a, w, b, eps=eps)

    def fwd(a, w, b):
        return f(a, w, b), (a, w, b)

    def bwd(res, g):
        return tuple(P["mlx_layer_norm_bwd"].bind(*res, g, eps=eps))

    f.defvjp(fwd, bwd)
    return f(x, weight, bias)
