"""JAX plugin entry point for the B200 PJRT plugin.

Mirrors reference ``src/jax_mlx/plugin.py:24-47``: JAX discovers this module
through the ``jax_plugins`` entry point (``b200 = "jax_b200.plugin"`` in
``pyproject.toml``, as the reference declares ``mlx_plugin =
"jax_mlx.plugin"``) and calls ``initialize()``, which registers
``libb200_pjrt.so`` under the platform name "b200" and then registers the
lowerings of the reference's fused-op primitives (``mlx_sdpa``,
``mlx_sdpa_bwd``, ``mlx_layer_norm``, ``mlx_layer_norm_bwd``) for that
platform: this package's own primitives (``jax_b200.custom_calls``) and, when
the reference's ``jax_mlx`` package is importable too, the reference's
primitive objects, so that programs written against either lower to the same
custom calls.

Unlike the reference, ``initialize()`` does not replace
``jax.nn.dot_product_attention`` or flax's LayerNorm: the plugin's compiler
matches the plain lowering of both (including the causal mask, which the
reference's replacement leaves unfused) and runs them on the same kernels.

Without JAX installed, importing this module is harmless and
``initialize()`` raises ImportError.
"""
from __future__ import annotations

import os

from .pjrt import PJRT_LIB

PLATFORM = "b200"


def library_path() -> str:
    if not os.path.exists(PJRT_LIB):
        raise RuntimeError(f"B200 PJRT library not built: {PJRT_LIB}")
    return PJRT_LIB


def initialize():
    """Called by JAX (entry point ``jax_plugins: b200 = jax_b200.plugin``)."""
    from jax._src import xla_bridge
    xla_bridge.register_plugin(PLATFORM, library_path=library_path())
    _register_custom_call_lowerings()


def _register_custom_call_lowerings():
    """Lower the four fused-op primitives to the custom calls the plugin
    executes (call targets mlx_sdpa, mlx_sdpa_bwd, mlx_layer_norm,
    mlx_layer_norm_bwd; backend_config {"scale": s} / {"eps": e})."""
    from . import custom_calls
    custom_calls.register_lowerings(PLATFORM)
    try:  # the reference's own primitives, if that package is installed as well
        from jax_mlx import layer_norm as ref_ln
        from jax_mlx import sdpa as ref_sdpa
    except ImportError:
        return
    custom_calls.register_lowerings(PLATFORM, {
        "mlx_sdpa": ref_sdpa.mlx_sdpa_p, "mlx_sdpa_bwd": ref_sdpa.mlx_sdpa_bwd_p,
        "mlx_layer_norm": ref_ln.mlx_layer_norm_p, "mlx_layer_norm_bwd": ref_ln.mlx_layer_norm_bwd_p})
