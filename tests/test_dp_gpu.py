"""GPU, two devices: data-parallel training steps (configs[2-4]) against the
full-batch oracle.

The global batch is split in two; each replica runs the `num_replicas=2`
program (the pmap / lax.pmean form: gradients and loss all-reduced through the
plugin's NCCL all_reduce, then divided by 2) on its half, and every replica
must end with the full-batch step.  Two launch forms:

* one process, two devices (ncclCommInitAll; PJRT Execute over two argument
  lists);
* one process per GPU, as `bench.py` runs under torchrun (ncclCommInitRank
  with the unique id published by rank 0 through the client's key-value
  callbacks over the gloo process group's store; tests/dp_rank_worker.py
  under torchrun).  The `nccl_init` fault point
  (B200_FAULT) is exercised here: both ranks get the injected UNAVAILABLE
  error from Execute, raised on the host before any collective starts.

Tolerances: contractions 2e-3 relative (elementwise on kink-safe inputs,
normwise on the configuration's own Glorot / U(0,1) inputs); bf16 transformer
gradients 3e-2 normwise against the excess-precision interpreter, as in the
one-device tests.  Skipped with fewer than two GPUs."""
import os
import socket
import sys

import numpy as np
import pytest

from helpers import assert_close
from jax_b200 import kernels, pjrt, programs
from oracle import hlo_interp, restate

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TR_SMALL = dict(batch=4, seq=64, layers=2, d=128, heads=2, ffn=256, vocab=512)


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


needs2 = pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")


@pytest.fixture(scope="module")
def client():
    c = pjrt.Client()
    yield c


def _glorot_mlp(rng, dims, batch):
    params = []
    for i in range(len(dims) - 1):
        lim = np.sqrt(6.0 / (dims[i] + dims[i + 1]))
        params.append(rng.uniform(-lim, lim, (dims[i], dims[i + 1])).astype(np.float32))
        params.append(np.zeros(dims[i + 1], np.float32))
    x = rng.random((batch, dims[0])).astype(np.float32)
    lab = rng.integers(0, dims[-1], batch).astype(np.int32)
    return params, x, lab


def _kink_safe_mlp(rng, dims, batch):
    """Weights k/64, inputs k/4: every pre-activation exact in f32 on both sides."""
    params = []
    for i in range(len(dims) - 1):
        params.append((rng.integers(-3, 4, (dims[i], dims[i + 1])) / 64.0).astype(np.float32))
        params.append((rng.integers(-2, 3, dims[i + 1]) / 64.0).astype(np.float32))
    x = (rng.integers(0, 5, (batch, dims[0])) / 4.0).astype(np.float32)
    lab = rng.integers(0, dims[-1], batch).astype(np.int32)
    return params, x, lab


def _cnn_inputs(rng, batch):
    shapes = [(3, 3, 1, 32), (32,), (3, 3, 32, 64), (64,), (3136, 256), (256,), (256, 10), (10,)]
    ps = []
    for s in shapes:
        fan_in = int(np.prod(s[:-1])) if len(s) > 1 else 1
        ps.append((rng.standard_normal(s) * np.sqrt(2.0 / fan_in)).astype(np.float32) if len(s) > 1
                  else (0.01 * rng.standard_normal(s)).astype(np.float32))
    x = rng.random((batch, 28, 28, 1)).astype(np.float32)
    lab = rng.integers(0, 10, batch).astype(np.int32)
    return ps, x, lab


def _tr_inputs(cfg, seed):
    rng = np.random.default_rng(seed)
    shapes = programs.transformer_param_shapes(cfg["layers"], cfg["d"], cfg["heads"], cfg["ffn"],
                                               cfg["vocab"], cfg["seq"])

    def init(name, s):
        leaf = name.split(".")[-1]
        if leaf.endswith("_g"):
            return 1 + 0.1 * rng.standard_normal(s)
        if leaf in ("wq", "wk"):
            return 0.1 * rng.standard_normal(s)
        return 0.02 * rng.standard_normal(s)
    params = [hlo_interp.bf16_round(init(n, s).astype(np.float32)) for n, s in shapes]
    zeros = [np.zeros(s, np.float32) for _, s in shapes]
    tok = rng.integers(0, cfg["vocab"], (cfg["batch"], cfg["seq"])).astype(np.int32)
    return [n for n, _ in shapes], params, zeros, np.array(0, np.int32), tok, np.roll(tok, -1, axis=1)


def _normwise(got, ref, tol, what):
    g, r = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    assert np.isfinite(g).all(), f"{what}: non-finite values"
    rel = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
    assert rel <= tol, f"{what}: normwise difference {rel:.3e} > {tol}"


def _to_np(o):
    a = o.to_numpy()
    return pjrt.from_bf16_bits(a) if o.dtype == pjrt.BF16 else a


def _execute_dp(client, text, shared, per_device, bf16_shared=0):
    """Execute `text` on the first two devices: `shared` arguments replicated
    (the first bf16_shared of them bf16), then each device's own batch slice."""
    exe = client.compile(text)
    devs = client.addressable_devices[:2]
    args = []
    for d, own in zip(devs, per_device):
        row = [client.buffer_from_numpy(pjrt.to_bf16_bits(a), device=d, bf16=True)
               if i < bf16_shared else client.buffer_from_numpy(a, device=d)
               for i, a in enumerate(shared)]
        args.append(row + [client.buffer_from_numpy(a, device=d) for a in own])
    outs = exe.execute(args)
    return [[_to_np(o) for o in outs[d]] for d in range(2)]


# ------------------------------------------------------ one process, 2 GPUs --
@needs2
def test_dp2_mlp_full_config_kink_safe(client):
    """configs[2] at full size, batch 1024 split 512 + 512: loss and every
    gradient elementwise against hand backprop of the full batch (f64)."""
    dims = (784, 1024, 1024, 1024, 10)
    params, x, lab = _kink_safe_mlp(np.random.default_rng(50), dims, 1024)
    text = programs.mlp_step(batch=512, dims=dims, num_replicas=2, emit="grads")
    got = _execute_dp(client, text, params, [[x[:512], lab[:512]], [x[512:], lab[512:]]])
    loss, new = restate.mlp_step_ref(params, x, lab, lr=1.0)
    for d in range(2):
        assert_close(got[d][0], loss, 2e-3, f"dp2 loss (device {d})")
        for i, (p, g, r) in enumerate(zip(params, got[d][1:], new)):
            assert_close(g, p.astype(np.float64) - r, 2e-3, f"dp2 grad {i} (device {d})")
    np.testing.assert_array_equal(got[0][1], got[1][1])  # replicas agree bit for bit


@needs2
def test_dp2_mlp_glorot_inputs_step(client):
    """configs[2] on its own Glorot-uniform weights and U(0,1) inputs: the SGD
    step's loss at 2e-3 and each applied update normwise at 2e-3."""
    dims = (784, 1024, 1024, 1024, 10)
    params, x, lab = _glorot_mlp(np.random.default_rng(8), dims, 1024)
    text = programs.mlp_step(batch=512, dims=dims, num_replicas=2)
    got = _execute_dp(client, text, params, [[x[:512], lab[:512]], [x[512:], lab[512:]]])
    loss, new = restate.mlp_step_ref(params, x, lab, lr=1e-2)
    for d in range(2):
        assert_close(got[d][0], loss, 2e-3, f"dp2 loss (device {d})")
        for i, (p, g, r) in enumerate(zip(params, got[d][1:], new)):
            _normwise(p.astype(np.float64) - g, p.astype(np.float64) - r, 2e-3, f"update {i}")


@needs2
def test_dp2_cnn_step_matches_interpreter(client):
    """configs[4] network, batch 8 split 4 + 4, against the interpreter's
    full-batch gradients."""
    ps, x, lab = _cnn_inputs(np.random.default_rng(51), 8)
    text = programs.cnn_step(batch=4, num_replicas=2, emit="grads")
    got = _execute_dp(client, text, ps, [[x[:4], lab[:4]], [x[4:], lab[4:]]])
    full = programs.cnn_step(batch=8, emit="grads")
    ref = hlo_interp.run(full, [ps + [x, lab]])[0]
    for d in range(2):
        for i, (g, r) in enumerate(zip(got[d], ref)):
            assert_close(g, r, 2e-3, f"dp2 cnn output {i} (device {d})")


@needs2
def test_dp2_transformer_grads_match_full_batch(client):
    """configs[3] architecture at reduced size, batch 4 split 2 + 2: loss at
    2e-3 and every bf16 gradient 3e-2 normwise against the excess-precision
    interpreter on the full batch (bf16 gradients all-reduced in bf16, as the
    program says)."""
    names, params, zeros, count, tok, tgt = _tr_inputs(TR_SMALL, 52)
    half = dict(TR_SMALL, batch=2)
    text = programs.transformer_step(**half, num_replicas=2, emit="grads")
    shared = params + zeros + zeros + [count]
    got = _execute_dp(client, text, shared, [[tok[:2], tgt[:2]], [tok[2:], tgt[2:]]],
                      bf16_shared=len(params))
    full = programs.transformer_step(**TR_SMALL, emit="grads")
    ref = hlo_interp.run(full, [params + zeros + zeros + [count, tok, tgt]], excess_bf16=True)[0]
    for d in range(2):
        assert_close(got[d][0], ref[0], 2e-3, f"dp2 transformer loss (device {d})")
        for n, g, r in zip(names, got[d][1:], ref[1:]):
            if n.endswith(".bk"):  # zero in exact arithmetic (softmax shift invariance)
                continue
            _normwise(g, r, 3e-2, f"dp2 grad {n} (device {d})")
    assert kernels.device_error(clear=True) == 0


# ------------------------------------------------- one process per GPU ----
def _run_ranks(tmp_path, kind, fault="", extra_env=None):
    """torchrun, two ranks, each running tests/dp_rank_worker.py as bench.py
    runs its ranks.  Each rank records the stage it reached, so that a rank
    that does not finish in time says where it stopped."""
    import subprocess
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", B200_KV_TIMEOUT_MS="60000")
    env.pop("B200_FAULT", None)
    if fault:
        env["B200_FAULT"] = fault
    env.update(extra_env or {})
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "dp_rank_worker.py"), str(tmp_path), kind]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    stages = {rk: (tmp_path / f"rank{rk}.stage").read_text() if (tmp_path / f"rank{rk}.stage").exists()
              else "not started" for rk in range(2)}
    faults = {rk: (tmp_path / f"rank{rk}.fault").read_text()[-2500:] for rk in range(2)
              if (tmp_path / f"rank{rk}.fault").exists()}
    assert r.returncode == 0, (f"ranks failed (rc {r.returncode}), stages {stages}, faults {faults}: "
                               f"{r.stderr[-2000:]}")


@needs2
def test_dp2_mlp_one_process_per_gpu(tmp_path):
    """configs[2] full step (SGD) as bench.py runs it under torchrun."""
    _run_ranks(tmp_path, "mlp")
    dims = (784, 1024, 1024, 1024, 10)
    params, x, lab = _kink_safe_mlp(np.random.default_rng(53), dims, 1024)
    loss, new = restate.mlp_step_ref(params, x, lab, lr=1e-2)
    res = []
    for r in range(2):
        z = np.load(tmp_path / f"rank{r}.npz")
        got = [z[f"arr_{i}"] for i in range(len(z.files))]
        res.append(got)
        assert_close(got[0], loss, 2e-3, f"loss (rank {r})")
        for i, (p, g, rr) in enumerate(zip(params, got[1:], new)):
            assert_close(p.astype(np.float64) - g, p.astype(np.float64) - rr, 2e-3, f"update {i} (rank {r})")
    for a, b in zip(res[0], res[1]):
        np.testing.assert_array_equal(a, b)


@needs2
def test_dp2_transformer_one_process_per_gpu(tmp_path):
    """configs[3] architecture at reduced size across two processes: the
    gradient all-reduce of bf16 gradients through NCCL, against the
    full-batch interpreter."""
    _run_ranks(tmp_path, "transformer")
    names, params, zeros, count, tok, tgt = _tr_inputs(TR_SMALL, 54)
    full = programs.transformer_step(**TR_SMALL, emit="grads")
    ref = hlo_interp.run(full, [params + zeros + zeros + [count, tok, tgt]], excess_bf16=True)[0]
    for r in range(2):
        z = np.load(tmp_path / f"rank{r}.npz")
        got = [z[f"arr_{i}"] for i in range(len(z.files))]
        assert_close(got[0], ref[0], 2e-3, f"loss (rank {r})")
        for n, g, rr in zip(names, got[1:], ref[1:]):
            if not n.endswith(".bk"):
                _normwise(g, rr, 3e-2, f"grad {n} (rank {r})")


@needs2
def test_dp2_nccl_init_fault_point(tmp_path):
    """B200_FAULT=nccl_init on both ranks: the first Execute that needs the
    communicator fails with UNAVAILABLE (14) on each rank, on the host, before
    any NCCL call; both processes exit cleanly."""
    _run_ranks(tmp_path, "mlp", fault="nccl_init")
    for r in range(2):
        assert not (tmp_path / f"rank{r}.npz").exists()
        msg = (tmp_path / f"rank{r}.err").read_text()
        assert msg.startswith("14 ") and "injected fault at nccl_init" in msg, msg


@needs2
def test_dp2_peer_leaves_watchdog_aborts(tmp_path):
    """A rank that leaves between steps: the surviving rank's next all-reduce
    cannot complete.  With B200_NCCL_TIMEOUT_MS=3000 the plugin's NCCL
    watchdog aborts the communicator, the step's result reports the error
    (DEADLINE_EXCEEDED, or INTERNAL when NCCL itself reports the lost peer
    first) within seconds instead of hanging, and the next step is refused with
    ABORTED before anything is launched.  NVLS is off (NCCL_NVLS_ENABLE=0), so
    no multicast object spans the ranks."""
    _run_ranks(tmp_path, "leave", extra_env={"B200_NCCL_TIMEOUT_MS": "3000"})
    lines = (tmp_path / "leave.txt").read_text().splitlines()
    assert lines[0].startswith("step1 ")
    code2 = int(lines[1].split()[1])
    assert code2 in (4, 13), lines[1]
    assert float(lines[1].split()[2].rstrip("s")) < 60, lines[1]
    assert "aborted" in lines[1] or "NCCL" in lines[1], lines[1]
    assert lines[2].startswith("step3 10 ") and "aborted" in lines[2], lines[2]
