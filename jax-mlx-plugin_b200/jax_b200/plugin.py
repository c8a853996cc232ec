"""JAX plugin entry point for the B200 PJRT plugin.

Mirrors reference ``src/jax_mlx/plugin.py:24-47``: JAX discovers this module
through the ``jax_plugins`` entry point and calls ``initialize()``, which
registers ``libb200_pjrt.so`` under the platform name "b200".  The
``mlx_sdpa`` / ``mlx_layer_norm`` custom-call primitives of the reference
(``src/jax_mlx/sdpa.py:35-151``, ``src/jax_mlx/layer_norm.py:29-138``) are
lowered for the "b200" platform with the same call targets, operands and
``backend_config`` JSON, so programs written against the reference's primitives
compile unchanged.  Without JAX installed, importing this module is harmless and
``initialize()`` raises.
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
    from jax._src import xla_bridge  # noqa: requires jax
    xla_bridge.register_plugin(PLATFORM, library_path=library_path())
    _register_custom_call_lowerings()


def _register_custom_call_lowerings():
    """Lower the reference's SDPA / LayerNorm primitives to custom calls the
    plugin executes (targets mlx_sdpa, mlx_layer_norm)."""
    try:
        from jax._src.interpreters import mlir
        from jax_mlx import layer_norm as ref_ln  # the reference's primitives, if installed
        from jax_mlx import sdpa as ref_sdpa
    except ImportError:
        return

    def sdpa_lowering(ctx, q, k, v, *, scale):
        out = mlir.custom_call(call_target_name="mlx_sdpa",
                               result_types=[mlir.aval_to_ir_type(ctx.avals_out[0])],
                               operands=[q, k, v], backend_config=f'{{"scale": {scale}}}')
        return out.results

    def ln_lowering(ctx, x, w, b, *, eps):
        out = mlir.custom_call(call_target_name="mlx_layer_norm",
                               result_types=[mlir.aval_to_ir_type(ctx.avals_out[0])],
                               operands=[x, w, b], backend_config=f'{{"eps": {eps}}}')
        return out.results

    mlir.register_lowering(ref_sdpa.mlx_sdpa_p, sdpa_lowering, platform=PLATFORM)
    mlir.register_lowering(ref_ln.mlx_layer_norm_p, ln_lowering, platform=PLATFORM)
