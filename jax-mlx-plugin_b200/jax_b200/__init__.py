"""B200 PJRT plugin: Python side.

pjrt      ctypes PJRT client over libb200_pjrt.so (what jaxlib binds)
kernels   ctypes binding of the sm_100a kernels' C ABI (libb200_kernels.so)
hlo       StableHLO emitter with autodiff (JAX's lowering, for environments without JAX)
programs  the benchmark programs
plugin    jax_plugins entry point: registers the platform with JAX when JAX is present
"""
__version__ = "0.1.0"
