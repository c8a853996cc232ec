"""GPU: host-side fault injection (B200_FAULT) through the PJRT C API.

An injected failure is raised on the host, where the real one would surface,
before any kernel of the failing call is launched: nothing on the GPU fails.
The process reads B200_FAULT once, so each case runs in a fresh interpreter."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_PROBE = """
import sys
sys.path[:0] = [{root!r}, {pkg!r}]
import numpy as np
from jax_b200 import pjrt, programs
stage = "client"
try:
    c = pjrt.Client()
    stage = "compile"
    exe = c.compile(programs.layer_norm(8, 256))
    stage = "buffers"
    rng = np.random.default_rng(0)
    args = [c.buffer_from_numpy(rng.standard_normal(s).astype(np.float32))
            for s in ((8, 256), (8, 256), (256,), (256,))]
    stage = "execute"
    exe.execute([args])[0][0].to_numpy()
    print("ok")
except pjrt.PjrtError as e:
    print(stage, e.code, e)
"""


@pytest.mark.parametrize("spec, stages, code", [
    ("execute", ("execute",), 13),
    ("alloc", ("client", "compile", "buffers"), 8),
])
def test_injected_fault_surfaces_as_pjrt_error(spec, stages, code):
    env = dict(os.environ, B200_FAULT=spec)
    src = _PROBE.format(root=ROOT, pkg=os.path.join(ROOT, "jax-mlx-plugin_b200"))
    r = subprocess.run([sys.executable, "-c", src], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-1500:]
    out = r.stdout.strip().split(" ", 2)
    assert out[0] in stages and int(out[1]) == code, r.stdout
    assert f"injected fault at {spec} (B200_FAULT)" in out[2]
