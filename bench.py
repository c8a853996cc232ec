"""Benchmark of the B200 PJRT plugin on BASELINE.json's configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload transformer|ln|sdpa|mlp|cnn|gemm] [--no-extra]

Default workload: configs[3], the jitted transformer training step
(value_and_grad + Adam, bf16, 64 x 256 tokens global), whose metric is
samples/s.  Under torchrun (one process per GPU) the global batch is split N
ways and the gradients are all-reduced by the plugin's NCCL all_reduce inside
the step (strong scaling: the global batch stays 64).  One step = one PJRT
Execute of the compiled step; steps run back to back with the updated
parameters and Adam moments feeding the next step, as a training loop does
(the working set, 104 MB of bf16 parameters plus 415 MB of f32 moments, is
larger than the 126 MB L2).  Each step is timed with CUDA events on the
plugin's own stream; the reported time is the max over ranks.

``e2e`` repeats the measurement through the calls a jax.jit user triggers,
every step copying its token and target slices from pinned host memory
(BufferFromHostBuffer) and reading the loss back (ToHostBuffer) inside the
timed region.  ``roofline`` relates the step's algorithmic FLOPs to the
measured sustained bf16 peak and names the dominant kernel, timed live.  At
N=1 the line also carries the other configurations under ``extra``
(residual+LayerNorm HBM GB/s, causal SDPA TFLOP/s, MLP and CNN training-step
samples/s), each with its own roofline, e2e and CPU baseline.

--impl reference times the reference's CPU path for the same workload.  The
reference plugin needs macOS + Metal (MLX) and JAX, neither of which exists on
this pool, so the arithmetic is timed through the torch-CPU restatement in
oracle/torch_port.py (the "port") on all host cores.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
# per-Execute device timing inside the plugin (events around the launch sequence)
os.environ.setdefault("B200_TIMING", "1")
for p in (ROOT, os.path.join(ROOT, "jax-mlx-plugin_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

LN_ROWS, LN_COLS = 4096, 1024
LN_BYTES = 3 * LN_ROWS * LN_COLS * 4 + 2 * LN_COLS * 4          # 50,339,840 B
SDPA_SHAPE = (8, 512, 8, 64)
SDPA_FLOPS = 4 * 8 * 8 * 64 * (512 * 513 // 2)                  # 2,151,677,952 (causal, incl. diagonal)
SDPA_MIN_BYTES = 4 * 8 * 512 * 8 * 64 * 4                       # q, k, v read + o written (f32)
MLP_DIMS = (784, 1024, 1024, 1024, 10)
MLP_FLOPS = 16_236_150_784
CNN_FLOPS = 7_017_332_736
LN_TRAFFIC = 33_600_000  # bytes, ncu dram read + write of one ln_fwd_reg<float,8> launch
# 6 * (matmul params 6*3,145,728 + head 16,384,000) * 16,384 tokens
# + attention 3 (fwd + 2x bwd) * 6 layers * 4 * 64 * 256^2 * 512
TR_CFG = dict(batch=64, seq=256, layers=6, d=512, heads=8, ffn=2048, vocab=32000)
TR_FLOPS = 6 * (6 * 3_145_728 + 16_384_000) * 64 * 256 + 3 * 6 * 4 * 64 * 256 * 256 * 512
TR_CPU_SAMPLE_SEQS = 8  # sequences per value_and_grad sample in the CPU baseline
GLOBAL_BATCH = {"mlp": 1024, "cnn": 256, "transformer": TR_CFG["batch"]}
STEP_FLOPS = {"mlp": MLP_FLOPS, "cnn": CNN_FLOPS, "transformer": TR_FLOPS}


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return FALLBACK_PEAKS, "fallback"


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ------------------------------------------------- metric / config names --
def describe(workload: str, world: int, args) -> dict:
    """metric, unit, dtype, scaling and config of a workload: one definition
    shared by both arms so that their lines name the same measurement."""
    dp = workload in ("mlp", "cnn", "transformer")
    par = f"dp{world}" if dp else f"replicas x{world}"
    if workload == "transformer":
        return dict(metric="transformer training step samples/s (jitted value_and_grad + Adam, configs[3])",
                    unit="samples/s", dtype="bf16", scaling="strong",
                    config={"workload": "transformer_train_step", "model": "pre-LN causal encoder",
                            "layers": 6, "d_model": 512, "heads": 8, "ffn": 2048, "vocab": 32000,
                            "global_batch": TR_CFG["batch"], "seq_len": TR_CFG["seq"],
                            "optimizer": "Adam lr 3e-4 (f32 moments)", "parallelism": par,
                            "l2": "working set larger than L2 (bf16 params 104 MB + f32 Adam "
                                  "moments 415 MB); steps back to back"})
    if workload == "mlp":
        return dict(metric="MLP training step samples/s (jitted value_and_grad + SGD, configs[2])",
                    unit="samples/s", dtype="f32", scaling="strong",
                    config={"workload": "mlp_train_step", "dims": list(MLP_DIMS),
                            "global_batch": 1024, "optimizer": "SGD lr 1e-2", "parallelism": par,
                            "l2": "not flushed (47 MB of parameters and activations); steps back to back"})
    if workload == "cnn":
        return dict(metric="CNN training step samples/s (jitted value_and_grad + SGD, configs[4])",
                    unit="samples/s", dtype="f32", scaling="strong",
                    config={"workload": "cnn_train_step", "input": [256, 28, 28, 1],
                            "global_batch": 256, "optimizer": "SGD lr 1e-2", "parallelism": par,
                            "l2": "not flushed; steps back to back"})
    if workload == "ln":
        return dict(metric="residual+LayerNorm fwd HBM throughput (jitted, configs[1])",
                    unit="GB/s", dtype="f32", scaling="weak",
                    config={"workload": "residual_layernorm_fwd", "shape": [LN_ROWS, LN_COLS],
                            "eps": 1e-5, "parallelism": par,
                            "l2": "evicted between timed steps (2 GB read on the same stream)",
                            "algorithmic_bytes_per_step": LN_BYTES})
    if workload == "sdpa":
        return dict(metric="causal SDPA fwd f32 TFLOP/s (jitted, configs[0])", unit="TFLOP/s",
                    dtype="f32", scaling="weak",
                    config={"workload": "causal_sdpa_fwd", "shape_btnh": list(SDPA_SHAPE),
                            "scale": 0.125, "parallelism": par,
                            "l2": "evicted between timed steps (2 GB read on the same stream)",
                            "algorithmic_flops_per_step": SDPA_FLOPS})
    shape = args.gemm_shape if args is not None else "8192,8192,8192"
    return dict(metric=f"GEMM {shape} TFLOP/s", unit="TFLOP/s",
                dtype=args.gemm_dtype if args is not None else "bf16", scaling="weak",
                config={"workload": "gemm", "shape": shape,
                        "trans": args.gemm_trans if args is not None else "", "parallelism": par,
                        "l2": "flushed between steps"})


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)  # the first sample lands before the timed work starts
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[4 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ------------------------------------------------------------- our plugin --
class Rig:
    """Plugin client + timing helpers on the plugin's stream."""

    def __init__(self, local_rank: int, kv=None, world: int = 1, rank: int = 0, dp: bool = False):
        import torch
        from jax_b200 import pjrt
        self.torch, self.pjrt = torch, pjrt
        opts = {"visible_devices": [local_rank]}
        if dp and world > 1:
            opts.update({"node_id": rank, "num_nodes": world})
        self.client = pjrt.Client(opts, kv=kv if dp else None)
        self.dev = self.client.addressable_devices[0]
        torch.cuda.set_device(local_rank)
        self.local_rank = local_rank
        self.stream = torch.cuda.ExternalStream(self.client.device_stream(self.dev))
        self.flush = torch.ones(2 * 1024 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
        self.sink = None
        self.world = world

    def barrier(self):
        """All ranks enter (and leave) a timed region together."""
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def time_steps(self, fn, steps: int, warmup: int, flush: bool = True):
        torch = self.torch
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        # no Python garbage-collection pauses inside the timed region (with torch
        # loaded a full collection stalls the launching thread for tens of ms)
        gc.collect()
        gc.disable()
        self.barrier()
        try:
            ts = self._timed(fn, steps, flush)
        finally:
            gc.enable()
        self.barrier()
        return ts

    def _timed(self, fn, steps: int, flush: bool):
        from jax_b200.pjrt import kernel_launches
        torch = self.torch
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        n0 = kernel_launches()
        for i in range(steps):
            if flush:
                # evict L2 by reading 2 GB (a read leaves clean lines: no write-back
                # traffic lands in the timed kernel, unlike a flushing write).  The
                # read takes ~0.3 ms, so the host enqueues the step before the GPU
                # gets to it and no launch latency falls inside the timed region.
                with torch.cuda.stream(self.stream):
                    self.sink = self.flush.sum()
            ev[i][0].record(self.stream)
            fn()
            ev[i][1].record(self.stream)
        # this package's kernels launched by the timed steps (library counters)
        self.timed_launches = kernel_launches() - n0
        torch.cuda.synchronize()
        return [a.elapsed_time(b) * 1e-3 for a, b in ev]  # seconds

    def bufs(self, arrays):
        return [self.client.buffer_from_numpy(a, device=self.dev) for a in arrays]

    def host_inputs(self, arrays):
        """Pinned host copies of `arrays` (the per-step inputs of an e2e step)."""
        return [self.torch.from_numpy(np.ascontiguousarray(a)).pin_memory() for a in arrays]

    def upload(self, pinned):
        """BufferFromHostBuffer of pinned host tensors: (buffers, done events)."""
        from jax_b200.pjrt import _NP2PJRT
        bs, evs = [], []
        for h in pinned:
            t = _NP2PJRT[np.dtype(str(h.dtype).replace("torch.", ""))]
            b, ev = self.client.buffer_from_host_ptr(h.data_ptr(), t, tuple(h.shape), self.dev,
                                                     semantics=1)
            bs.append(b)
            evs.append(ev)
        return bs, evs


def _await_all(evs):
    from jax_b200.pjrt import api
    for ev in evs:
        api().await_event(ev)


def ln_inputs(seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((LN_ROWS, LN_COLS)).astype(np.float32)
    r = rng.standard_normal((LN_ROWS, LN_COLS)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(LN_COLS)).astype(np.float32)
    b = (0.1 * rng.standard_normal(LN_COLS)).astype(np.float32)
    return [x, r, g, b]


def _device_mean(exe, steps, ts):
    dev_ms = exe.device_times_ms()[-steps:]
    return float(np.mean(dev_ms)) * 1e-3 if len(dev_ms) == steps else float(np.mean(ts))


def bench_ln(rig: Rig, steps, warmup):
    from jax_b200 import programs
    from jax_b200.pjrt import api
    text = programs.layer_norm()
    exe = rig.client.compile(text)
    args = rig.bufs(ln_inputs())
    holder = []

    def step():
        holder[:] = exe.execute([args])
    with ClockSampler(rig.local_rank) as clk:
        ts = rig.time_steps(step, steps, warmup)
    launches = rig.timed_launches / steps
    t = _device_mean(exe, steps, ts)
    # end to end: pinned host inputs -> device -> execute -> host, per step
    host_in = rig.host_inputs(ln_inputs())
    out_np = rig.torch.empty((LN_ROWS, LN_COLS), dtype=rig.torch.float32).pin_memory().numpy()

    def e2e_step():
        bs, evs = rig.upload(host_in)
        o = exe.execute([bs])[0][0]
        api().await_event(o.to_host_async(out_np))
        _await_all(evs)
    e2e_t = float(np.mean(rig.time_steps(e2e_step, steps, warmup, flush=True)))
    exe.device_times_ms()
    kt, kcfg = ln_kernel_time(rig, steps)
    return {"value": LN_BYTES / t / 1e9, "t": t, "outer_event_ms_per_step": float(np.mean(ts)) * 1e3,
            "e2e_t": e2e_t, "h2d": sum(h.numel() * 4 for h in host_in), "d2h": LN_ROWS * LN_COLS * 4,
            "launches_per_step": launches, "clocks": clk.summary(), "kernel_time_s": kt,
            "kernel_timing": kcfg}


def ln_kernel_time(rig: Rig, launches: int):
    """Average duration of the LayerNorm kernel itself: `launches` launches
    through the C ABI, rotating over 4 input / output sets (201 MB, more than the
    126 MB L2, so each launch reads cold data), captured once into a CUDA graph
    and replayed between one pair of CUDA events on the replay stream.  Replayed
    back to back the GPU never waits for the (Python) host, and no per-launch
    event overhead is counted."""
    from jax_b200 import kernels
    torch = rig.torch
    sets = []
    for i in range(4):
        x, r, g, b = (torch.from_numpy(a).cuda() for a in ln_inputs(i))
        sets.append((x, r, g, b, torch.empty_like(x)))

    def launch(i, st):
        x, r, g, b, y = sets[i % 4]
        kernels.ln_residual_fwd(x.data_ptr(), r.data_ptr(), g.data_ptr(), b.data_ptr(), y.data_ptr(),
                                0, 0, 0, LN_ROWS, LN_COLS, 1e-5, kernels.DT_F32, 0, st)
    n = max(launches, 20)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        for i in range(8):
            launch(i, side.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(n):
            launch(i, side.cuda_stream)
    torch.cuda.synchronize()
    graph.replay()  # warm
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(side):
        e0.record(side)
        graph.replay()
        e1.record(side)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) * 1e-3 / n
    del graph
    return t, {"launches": n, "l2": "4 rotating input/output sets (201 MB > 126 MB L2)",
               "stream": "CUDA-graph replay of the C-ABI launches", "per_launch_us": t * 1e6}


def bench_sdpa(rig: Rig, steps, warmup):
    from jax_b200 import programs
    from jax_b200.pjrt import api
    text = programs.sdpa(*SDPA_SHAPE, causal=True)
    exe = rig.client.compile(text)
    rng = np.random.default_rng(1)
    arrays = [rng.standard_normal(SDPA_SHAPE).astype(np.float32) for _ in range(3)]
    args = rig.bufs(arrays)
    holder = []
    with ClockSampler(rig.local_rank) as clk:
        ts = rig.time_steps(lambda: holder.__setitem__(slice(None), exe.execute([args])), steps, warmup)
    launches = rig.timed_launches / steps
    t = _device_mean(exe, steps, ts)
    host_in = rig.host_inputs(arrays)
    out_np = rig.torch.empty(SDPA_SHAPE, dtype=rig.torch.float32).pin_memory().numpy()

    def e2e_step():
        bs, evs = rig.upload(host_in)
        o = exe.execute([bs])[0][0]
        api().await_event(o.to_host_async(out_np))
        _await_all(evs)
    e2e_t = float(np.mean(rig.time_steps(e2e_step, steps, warmup, flush=True)))
    exe.device_times_ms()
    return {"value": SDPA_FLOPS / t / 1e12, "t": t, "e2e_t": e2e_t,
            "h2d": 3 * int(np.prod(SDPA_SHAPE)) * 4, "d2h": int(np.prod(SDPA_SHAPE)) * 4,
            "launches_per_step": launches, "clocks": clk.summary(),
            "tensor_path": "tcgen05 kind::f16 (f32 inputs as bf16 hi+lo, 3 products)"}


def bench_gemm(rig: Rig, steps, warmup, shape, dtype="bf16", trans=""):
    """The dot_general GEMM kernel alone through the C ABI (b200_gemm): C[M,N] =
    A[M,K] B[K,N] with A stored [K,M] when trans contains 'a' and B stored [N,K]
    when it contains 'b'.  Inputs larger than L2 are not guaranteed, so L2 is
    flushed between steps."""
    from jax_b200 import kernels
    torch = rig.torch
    M, N, K = shape
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    code = kernels.DT_BF16 if dtype == "bf16" else kernels.DT_F32
    a_t, b_t = "a" in trans, "b" in trans
    A = torch.randn((K, M) if a_t else (M, K), device="cuda", dtype=tdt)
    B = torch.randn((N, K) if b_t else (K, N), device="cuda", dtype=tdt)
    C = torch.empty((M, N), device="cuda", dtype=tdt)
    st = rig.client.device_stream(rig.dev)
    sAm, sAk = (1, M) if a_t else (K, 1)
    sBk, sBn = (1, K) if b_t else (N, 1)

    def step():
        kernels.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), 0, 1, M, N, K, 0, sAm, sAk, 0, sBk, sBn,
                     N, 1.0, code, code, 0, st)
    with ClockSampler(rig.local_rank) as clk:
        ts = rig.time_steps(step, steps, warmup)
    t = float(np.mean(ts))
    fl = 2.0 * M * N * K
    return {"value": fl / t / 1e12, "t": t, "launches_per_step": rig.timed_launches / steps,
            "clocks": clk.summary(),
            "flops_per_step": fl}


def dominant_gemm_time(rig: Rig, launches: int = 20):
    """The transformer step's largest single kernel, the LM-head GEMM
    (logits [16384, 32000] = y [16384, 512] . W [512, 32000], bf16, f32
    accumulation), timed live through the C ABI: `launches` launches over two
    rotating operand / output sets (2 x 1.1 GB, far above L2) between one event
    pair on the plugin's stream."""
    from jax_b200 import kernels
    torch = rig.torch
    M, N, K = TR_CFG["batch"] * TR_CFG["seq"], TR_CFG["vocab"], TR_CFG["d"]
    sets = [(torch.randn(M, K, device="cuda", dtype=torch.bfloat16),
             torch.randn(K, N, device="cuda", dtype=torch.bfloat16),
             torch.empty(M, N, device="cuda", dtype=torch.bfloat16)) for _ in range(2)]
    st = rig.client.device_stream(rig.dev)

    def launch(i):
        A, B, C = sets[i % 2]
        kernels.gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), 0, 1, M, N, K, 0, K, 1, 0, N, 1, N, 1.0,
                     kernels.DT_BF16, kernels.DT_BF16, 0, st)
    for i in range(4):
        launch(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(rig.stream)
    for i in range(launches):
        launch(i)
    e1.record(rig.stream)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) * 1e-3 / launches
    del sets
    torch.cuda.empty_cache()
    return t, 2.0 * M * N * K


def attention_kernel_times(rig: Rig, batch: int, launches: int = 20):
    """The transformer's fused attention kernels at the step's per-GPU shape
    ([batch, 256, 8, 64] bf16, causal, scale 1/8), timed live through the C ABI:
    the forward with row statistics (b200_sdpa_fwd_lse) and the backward
    (b200_sdpa_bwd), each `launches` launches over three rotating input /
    output sets (each above 100 MB at batch 64) between one event pair on the
    plugin's stream.  Algorithmic FLOPs count the causal half of each product:
    forward 2 products (Q K^T, P V), backward 5 (S, dP, dV, dK, dQ)."""
    from jax_b200 import kernels
    torch = rig.torch
    B, T, N, H = batch, TR_CFG["seq"], TR_CFG["heads"], TR_CFG["d"] // TR_CFG["heads"]
    st = rig.client.device_stream(rig.dev)
    dense = [T * N * H, N * H, H]

    def mk():
        q, k, v, g = (torch.randn(B, T, N, H, device="cuda", dtype=torch.bfloat16) for _ in range(4))
        o = torch.empty_like(q)
        lse = torch.empty(B, N, T, device="cuda")
        return q, k, v, g, o, lse, torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
    sets = [mk() for _ in range(3)]

    def fwd(i):
        q, k, v, g, o, lse, dq, dk, dv = sets[i % 3]
        kernels.sdpa_fwd_lse(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, T,
                             T, N, H, dense * 4, 0.125, True, kernels.DT_BF16, st)

    def bwd(i):
        q, k, v, g, o, lse, dq, dk, dv = sets[i % 3]
        kernels.sdpa_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), g.data_ptr(), lse.data_ptr(),
                         dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, T, N, H, dense * 8, 0.125, True,
                         kernels.DT_BF16, st)
    out = {}
    for name, fn, nprod in (("fwd", fwd, 2), ("bwd", bwd, 5)):
        for i in range(6):
            fwd(i)
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(rig.stream)
        for i in range(launches):
            fn(i)
        e1.record(rig.stream)
        torch.cuda.synchronize()
        out[name] = (e0.elapsed_time(e1) * 1e-3 / launches, nprod * 2.0 * B * N * T * T * H / 2)
    del sets
    torch.cuda.empty_cache()
    return out


def _mlp_args(rng, batch):
    params = []
    for i in range(len(MLP_DIMS) - 1):
        lim = np.sqrt(6.0 / (MLP_DIMS[i] + MLP_DIMS[i + 1]))
        params.append(rng.uniform(-lim, lim, (MLP_DIMS[i], MLP_DIMS[i + 1])).astype(np.float32))
        params.append(np.zeros(MLP_DIMS[i + 1], np.float32))
    x = rng.random((batch, MLP_DIMS[0])).astype(np.float32)
    lab = rng.integers(0, 10, batch).astype(np.int32)
    return params + [x, lab]


def _cnn_args(rng, batch):
    shapes = [(3, 3, 1, 32), (32,), (3, 3, 32, 64), (64,), (3136, 256), (256,), (256, 10), (10,)]
    ps = []
    for s in shapes:
        if len(s) > 1:
            fan_in = int(np.prod(s[:-1]))
            ps.append((rng.standard_normal(s) * np.sqrt(2.0 / fan_in)).astype(np.float32))
        else:
            ps.append(np.zeros(s, np.float32))
    x = rng.random((batch, 28, 28, 1)).astype(np.float32)
    lab = rng.integers(0, 10, batch).astype(np.int32)
    return ps + [x, lab]


def _tokens(rng):
    c = TR_CFG
    tok = rng.integers(0, c["vocab"], (c["batch"], c["seq"])).astype(np.int32)
    return tok, np.roll(tok, -1, axis=1)


def _transformer_state(rig: Rig, rng):
    """configs[3] state: N(0, 0.02) bf16 params, zero f32 Adam moments, count 0."""
    from jax_b200 import pjrt, programs
    c = TR_CFG
    shapes = programs.transformer_param_shapes(c["layers"], c["d"], c["heads"], c["ffn"], c["vocab"],
                                               c["seq"])
    bufs = [rig.client.buffer_from_numpy(pjrt.to_bf16_bits(rng.standard_normal(s).astype(np.float32)
                                                           * np.float32(0.02)), rig.dev, bf16=True)
            for _, s in shapes]
    zeros = [np.zeros(s, np.float32) for _, s in shapes]
    return bufs + rig.bufs(zeros + zeros + [np.array(0, np.int32)])


def bench_train(rig: Rig, kind, steps, warmup, world=1, rank=0, with_e2e=True):
    """One training configuration: device-resident step time, and (with_e2e)
    the same step with this rank's batch slice uploaded from pinned host
    memory and the loss read back every step."""
    from jax_b200 import programs
    from jax_b200.pjrt import api
    gb = GLOBAL_BATCH[kind]
    per = gb // world
    if kind == "mlp":
        text = programs.mlp_step(batch=per, num_replicas=world)
    elif kind == "cnn":
        text = programs.cnn_step(batch=per, num_replicas=world)
    else:
        text = programs.transformer_step(**dict(TR_CFG, batch=per), num_replicas=world)
    exe = rig.client.compile(text)
    rng = np.random.default_rng({"mlp": 8, "cnn": 13, "transformer": 11}[kind])
    sl = slice(rank * per, (rank + 1) * per)
    if kind == "transformer":
        state = _transformer_state(rig, rng)
        tok, tgt = _tokens(rng)
        batch_arrays = [tok[sl], tgt[sl]]
    else:
        full = _mlp_args(rng, gb) if kind == "mlp" else _cnn_args(rng, gb)
        state = rig.bufs(full[:-2])
        batch_arrays = [full[-2][sl], full[-1][sl]]
    n_state = len(state)
    args = state + rig.bufs(batch_arrays)
    holder = []

    def step():
        # the updated state feeds the next step, as a training loop does
        outs = exe.execute([args])[0]
        holder[:] = outs
        args[:n_state] = outs[1:1 + n_state]
    with ClockSampler(rig.local_rank) as clk:
        ts = rig.time_steps(step, steps, warmup, flush=False)
    launches = rig.timed_launches / steps
    exe.device_times_ms()
    t = float(np.mean(ts))  # back-to-back steps: host launch overhead is part of a training step
    res = {"value": gb / t, "t": t, "launches_per_step": launches, "clocks": clk.summary(),
           "flops_per_step": STEP_FLOPS[kind], "tflops": STEP_FLOPS[kind] / t / 1e12, "global_batch": gb}
    if with_e2e:
        host_in = rig.host_inputs(batch_arrays)
        loss_np = np.empty((), np.float32)

        def e2e_step():
            bs, evs = rig.upload(host_in)
            outs = exe.execute([args[:n_state] + bs])[0]
            api().await_event(outs[0].to_host_async(loss_np))
            args[:n_state] = outs[1:1 + n_state]
            holder[:] = outs
            _await_all(evs)
        e2e_ts = rig.time_steps(e2e_step, steps, warmup, flush=False)
        exe.device_times_ms()
        res.update(e2e_t=float(np.mean(e2e_ts)), h2d=sum(h.numel() * h.element_size() for h in host_in),
                   d2h=4, last_loss=float(loss_np))
    return res


# -------------------------------------------------------- CPU baseline ---
def _torch_threads(threads):
    import torch
    torch.set_num_threads(threads)
    return torch


def _bounded(fn, budget_s: float, max_reps: int, min_reps: int = 2, warm: bool = True):
    """Run fn() (after one untimed warm-up unless warm is False) until
    budget_s has passed or max_reps runs are done; returns the per-run times."""
    if warm:
        fn()
    ts = []
    t_end = time.perf_counter() + budget_s
    while len(ts) < max_reps and (len(ts) < min_reps or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return ts


_CPU_INPUTS = {}


def _cpu_inputs(workload: str):
    """Host inputs of the torch-CPU port, built once per process."""
    if workload in _CPU_INPUTS:
        return _CPU_INPUTS[workload]
    import torch
    from oracle import torch_port as tp
    if workload == "ln":
        v = [torch.from_numpy(a) for a in ln_inputs()]
    elif workload == "sdpa":
        rng = np.random.default_rng(1)
        v = [torch.from_numpy(rng.standard_normal(SDPA_SHAPE).astype(np.float32)) for _ in range(3)]
    elif workload in ("mlp", "cnn"):
        gb = GLOBAL_BATCH[workload]
        rng = np.random.default_rng(8 if workload == "mlp" else 13)
        full = _mlp_args(rng, gb) if workload == "mlp" else _cnn_args(rng, gb)
        v = ([torch.from_numpy(a) for a in full[:-2]], torch.from_numpy(full[-2]), torch.from_numpy(full[-1]))
    else:
        from jax_b200 import programs
        shapes = programs.transformer_param_shapes()
        params, ms, vs = tp.transformer_state(shapes)
        tok, tgt = _tokens(np.random.default_rng(11))
        S = TR_CPU_SAMPLE_SEQS
        v = ([n for n, _ in shapes], params, ms, vs, torch.from_numpy(tok[:S]), torch.from_numpy(tgt[:S]))
    _CPU_INPUTS[workload] = v
    return v


def cpu_sample(workload: str, threads: int, budget_s: float = 10.0, max_reps: int = 50,
               warm: bool = True):
    """Time the torch-CPU port (oracle/torch_port.py) of `workload` on
    `threads` host threads.  Returns (value in the workload's unit, seconds
    per sample, description of the sample)."""
    _torch_threads(threads)
    from oracle import torch_port as tp
    inp = _cpu_inputs(workload)
    if workload == "ln":
        x, r, g, b = inp
        ts = _bounded(lambda: tp.residual_layer_norm(x, r, g, b), budget_s, max_reps, warm=warm)
        t = float(np.median(ts))
        return LN_BYTES / t / 1e9, t, (f"{len(ts)} full [4096,1024] f32 residual+LayerNorm passes "
                                       f"(torch CPU), median {t * 1e3:.2f} ms")
    if workload == "sdpa":
        q, k, v = inp
        ts = _bounded(lambda: tp.sdpa(q, k, v, causal=True), budget_s, max_reps, warm=warm)
        t = float(np.median(ts))
        return SDPA_FLOPS / t / 1e12, t, (f"{len(ts)} full [8,512,8,64] f32 causal attention calls "
                                          f"(torch CPU), median {t * 1e3:.1f} ms")
    if workload in ("mlp", "cnn"):
        gb = GLOBAL_BATCH[workload]
        ps, x, lab = inp
        fn = tp.mlp_step if workload == "mlp" else tp.cnn_step
        ts = _bounded(lambda: fn(ps, x, lab), budget_s, max_reps, warm=warm)
        t = float(np.median(ts))
        return gb / t, t, (f"{len(ts)} full batch-{gb} f32 {workload.upper()} steps (value_and_grad + "
                           f"SGD, torch CPU), median {t * 1e3:.1f} ms")
    if workload == "transformer":
        names, params, ms, vs, tt, tg = inp
        S = TR_CPU_SAMPLE_SEQS
        holder = {}

        def grads():
            holder["g"] = tp.transformer_grads(names, params, tt, tg)[1]

        def adam():
            tp.adam_update(params, ms, vs, holder["g"], 0)
        half = budget_s / 2
        tg_s = float(np.median(_bounded(grads, half, max(1, max_reps // 2), 1, warm=warm)))
        ta_s = float(np.median(_bounded(adam, half, max(1, max_reps // 2), 1, warm=warm)))
        gb = TR_CFG["batch"]
        t_step = tg_s * gb / S + ta_s
        return gb / t_step, t_step, (
            f"value_and_grad of {S} of the 64 sequences ({tg_s * 1e3:.0f} ms) scaled to 64, plus one "
            f"full Adam update of all 52.2 M parameters ({ta_s * 1e3:.0f} ms): {t_step:.2f} s per "
            f"64-sequence step (torch CPU, bf16 parameters and activations, f32 loss)")
    raise ValueError(workload)


def cpu_baseline(workload: str, threads: int, budget_s: float = 10.0) -> dict:
    unit = describe(workload, 1, None)["unit"]
    v, _, sample = cpu_sample(workload, threads, budget_s)
    return {"value": v, "unit": unit, "cores": threads, "kind": "port", "sample": sample,
            "what": "torch-CPU restatement (oracle/torch_port.py); JAX-CPU and the reference's "
                    "MLX plugin are unavailable on this pool"}


def reference_arm(a, world, rank):
    """--impl reference: the port on all host cores, rank 0 only."""
    if rank != 0:
        return
    if a.workload == "gemm":
        print(json.dumps({"impl": "reference", "unavailable":
                          "the GEMM micro-benchmark has no reference counterpart"}))
        return
    threads = host_cores()
    d = describe(a.workload, world, a)
    vals, ts, sample = [], [], ""
    _cpu_inputs(a.workload)  # inputs are built before the first step, as the GPU arm's are
    for i in range(a.warmup + a.steps):
        # one step = one bounded sample of the workload (no inner warm-up)
        v, t, sample = cpu_sample(a.workload, threads, budget_s=0.0, max_reps=1 if a.workload ==
                                  "transformer" else 3, warm=False)
        if i >= a.warmup:
            vals.append(v)
            ts.append(t)
    value = float(np.mean(vals))
    line = {"impl": "reference", "metric": d["metric"], "value": value, "unit": d["unit"],
            "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": float(np.mean(ts)) * 1e3,
            "higher_is_better": True, "scaling": d["scaling"], "vs_baseline": None, "dtype": d["dtype"],
            "data": "synthetic (seeded)", "config": d["config"],
            "cpu_baseline": {"value": value, "unit": d["unit"], "cores": threads, "kind": "port",
                             "sample": "per step: " + sample},
            "e2e": {"value": value, "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference plugin needs macOS/Metal (MLX) and JAX; its arithmetic is timed "
                    "through the torch-CPU port oracle/torch_port.py on all host cores"}
    print(json.dumps(line))


# ------------------------------------------------------------- rooflines --
def roofline_for(workload: str, res: dict, world: int, pk: dict, pk_kind: str, t_max: float) -> dict:
    if workload == "ln":
        ach = LN_BYTES / res["kernel_time_s"] / 1e9
        return {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": ach / pk["hbm_gbs"], "peak_kind": pk_kind,
                # dram__bytes_read.sum + dram__bytes_write.sum of one launch (ncu
                # capture summarised in profiles/): y is still in L2 when the kernel ends
                "traffic": LN_TRAFFIC, "kernel": "ln_fwd_reg<float,8>", "timing": res["kernel_timing"],
                "per_launch_bytes": LN_BYTES,
                "jitted_step": {"achieved": res["value"], "frac": res["value"] / pk["hbm_gbs"]}}
    if workload == "sdpa":
        ach = SDPA_FLOPS / res["t"] / 1e12
        floor_us = SDPA_MIN_BYTES / (pk["hbm_gbs"] * 1e9) * 1e6
        return {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": ach / pk["bf16_tflops"], "peak_kind": pk_kind + " bf16 dense (burst)",
                "traffic": None, "kernel": "sdpa_fwd_ws (one launch per step)",
                "per_launch_flops": SDPA_FLOPS,
                "memory_floor_us": floor_us, "frac_of_memory_floor": floor_us / (res["t"] * 1e6)}
    if workload == "gemm":
        return {"bound": "tensor", "achieved": res["value"], "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": res["value"] / pk["bf16_tflops"], "peak_kind": pk_kind, "traffic": None,
                "kernel": "b200_gemm: gemm_tc_pair (two-SM 256 x 256 tiles, K splits when tiles are few) "
                          "or gemm_tc_pers (one-SM tiles) by shape"}
    # training steps: the whole step on one GPU's share of the FLOPs
    peak = pk["bf16_tflops_sustained"]
    ach = STEP_FLOPS[workload] / world / t_max / 1e12
    out = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
           "peak_kind": pk_kind + " bf16 dense (sustained)", "traffic": None,
           "kernel": f"whole jitted step ({res['launches_per_step']:g} launches), per GPU",
           "per_step_flops": STEP_FLOPS[workload] // world}
    if "dominant" in res:
        dt, dfl = res["dominant"]
        out["dominant_kernel"] = {"kernel": "gemm_tc_pair<bf16> LM head 16384x32000x512",
                                  "achieved": dfl / dt / 1e12, "peak": pk["bf16_tflops"],
                                  "frac": dfl / dt / 1e12 / pk["bf16_tflops"],
                                  "peak_kind": pk_kind + " bf16 dense (burst)",
                                  "per_launch_us": dt * 1e6, "per_launch_flops": dfl,
                                  "timing": "20 C-ABI launches over 2 rotating 1.1 GB operand sets, "
                                            "one event pair on the plugin's stream"}
    if "attention" in res:
        att = {}
        for name, (t, fl) in res["attention"].items():
            att[name] = {"kernel": "sdpa_fwd_ws<bf16> + row statistics" if name == "fwd" else "sdpa_bwd_tc",
                         "per_launch_us": t * 1e6, "per_launch_flops": fl, "achieved": fl / t / 1e12,
                         "peak": pk["bf16_tflops"], "frac": fl / t / 1e12 / pk["bf16_tflops"],
                         "peak_kind": pk_kind + " bf16 dense (burst)"}
        att["shape_btnh"] = [TR_CFG["batch"] // world, TR_CFG["seq"], TR_CFG["heads"],
                             TR_CFG["d"] // TR_CFG["heads"]]
        att["flops"] = "causal half of each product: forward 2, backward 5"
        att["timing"] = "20 C-ABI launches over 3 rotating input / output sets, one event pair"
        out["attention_kernels"] = att
    return out


def run_ours(rig: Rig, workload: str, a, world: int, rank: int) -> dict:
    if workload == "ln":
        return bench_ln(rig, a.steps, a.warmup)
    if workload == "sdpa":
        return bench_sdpa(rig, a.steps, a.warmup)
    if workload == "gemm":
        return bench_gemm(rig, a.steps, a.warmup, tuple(int(v) for v in a.gemm_shape.split(",")),
                          a.gemm_dtype, a.gemm_trans)
    res = bench_train(rig, workload, a.steps, a.warmup, world, rank)
    if workload == "transformer":
        res["dominant"] = dominant_gemm_time(rig)
        res["attention"] = attention_kernel_times(rig, TR_CFG["batch"] // world)
    return res


def line_for(workload, res, a, world, t_max, e2e_max, pk, pk_kind, with_cpu: bool) -> dict:
    d = describe(workload, world, a)
    kernel_only = workload in ("ln", "sdpa", "gemm")
    if kernel_only:
        # independent replicas: each GPU's throughput at the slowest rank's time
        per_gpu = res["value"] * res["t"] / t_max
        value = per_gpu * world
    else:
        value = res["global_batch"] / t_max
    line = {"metric": d["metric"], "value": value, "unit": d["unit"], "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": t_max * 1e3, "higher_is_better": True,
            "scaling": d["scaling"], "vs_baseline": None, "dtype": d["dtype"],
            "data": "synthetic (seeded; BASELINE.json shapes and distributions)", "config": d["config"]}
    if e2e_max is not None and "h2d" in res:
        if kernel_only:
            e2e_v = res["value"] * res["t"] / e2e_max * world
        else:
            e2e_v = res["global_batch"] / e2e_max
        line["e2e"] = {"value": e2e_v, "unit": d["unit"], "ms_per_step": e2e_max * 1e3,
                       # whole job: every rank copies its own inputs and reads its result
                       "h2d_bytes_per_step": res["h2d"] * world, "d2h_bytes_per_step": res["d2h"] * world,
                       "path": "PJRT BufferFromHostBuffer (pinned) -> Execute -> ToHostBuffer, every step"}
    line["roofline"] = roofline_for(workload, res, world, pk, pk_kind, t_max)
    line["clocks"] = res.get("clocks")
    line["gpu_launches"] = int(round(res["launches_per_step"] * a.steps))
    if "tflops" in res:
        line["tflops_per_step_whole_job"] = STEP_FLOPS[workload] / t_max / 1e12
    if "last_loss" in res:
        line["loss_after_timed_steps"] = res["last_loss"]
    if with_cpu and workload != "gemm":
        try:
            line["cpu_baseline"] = cpu_baseline(workload, host_cores())
        except Exception as e:  # report, do not hide
            line["cpu_baseline"] = {"error": str(e)[:300]}
    return line


# ------------------------------------------------------------------ main --
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="transformer",
                    choices=["transformer", "ln", "sdpa", "mlp", "cnn", "gemm"])
    ap.add_argument("--gemm-shape", default="8192,8192,8192", help="M,N,K for --workload gemm")
    ap.add_argument("--gemm-dtype", default="bf16", choices=["bf16", "f32"])
    ap.add_argument("--gemm-trans", default="", help="'a', 'b' or 'ab': operands stored transposed")
    ap.add_argument("--no-extra", action="store_true")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if a.impl == "reference":
        reference_arm(a, world, rank)
        return

    import torch
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    dp = a.workload in ("mlp", "cnn", "transformer") and world > 1
    kv = None
    if dp:
        store = dist.distributed_c10d._get_default_store()

        class KV:
            def set(self, k, v):
                store.set(k, v)

            def get(self, k):
                return bytes(store.get(k))
        kv = KV()
    rig = Rig(local_rank, kv=kv, world=world, rank=rank, dp=dp)
    res = run_ours(rig, a.workload, a, world, rank)
    t_local = res["t"]
    e2e_local = res.get("e2e_t")
    if dist is not None:
        tt = torch.tensor([t_local, e2e_local if e2e_local is not None else 0.0], dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max, e2e_max = float(tt[0]), (float(tt[1]) if e2e_local is not None else None)
        dist.barrier()
    else:
        t_max, e2e_max = t_local, e2e_local
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
    pk, pk_kind = peaks()
    line = line_for(a.workload, res, a, world, t_max, e2e_max, pk, pk_kind, with_cpu=(world == 1))
    if world == 1 and not a.no_extra and a.workload == "transformer":
        extra = {}
        for kind in ("ln", "sdpa", "mlp", "cnn"):
            try:
                r = run_ours(rig, kind, argparse.Namespace(**dict(vars(a), steps=20, warmup=3)), 1, 0)
                ex = line_for(kind, r, argparse.Namespace(**dict(vars(a), steps=20, warmup=3)), 1,
                              r["t"], r.get("e2e_t"), pk, pk_kind, with_cpu=True)
                extra[kind] = ex
            except Exception as e:  # report, do not hide
                extra[kind] = {"error": str(e)[:300]}
        line["extra"] = extra
    print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
