"""Benchmark of the B200 PJRT plugin on BASELINE.json's configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload ln|sdpa|mlp|cnn|transformer|gemm] [--no-extra]

Default workload: configs[1], the jitted residual-add + LayerNorm forward
(x, r [4096,1024] f32), whose metric is HBM GB/s.  One step = one PJRT
Execute of the compiled program on inputs resident in HBM; the L2 (126 MB) is
flushed between timed steps by reading a 2 GB buffer, and each step is timed
with CUDA events on the plugin's own stream.  ``e2e`` repeats the measurement through the
same PJRT calls a jax.jit user triggers, with the inputs copied from pinned host
memory (BufferFromHostBuffer) and the output read back (ToHostBuffer) inside
the timed region.  At N=1 the line also carries the other configurations
(causal SDPA TFLOP/s, MLP, CNN and transformer training-step samples/s) under
"extra".

Multi-GPU (torchrun, one process per GPU): LayerNorm and SDPA are independent
replicas (no collective); the MLP/CNN/transformer steps shard the global batch
and all-reduce gradients through the plugin's NCCL all_reduce.

--impl reference times the reference's CPU path for the same workload.  The
reference plugin needs macOS + Metal (MLX) and cannot be built here, so its
arithmetic is timed through the CPU restatement in oracle/ (the "port") on all
host cores.
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
MLP_DIMS = (784, 1024, 1024, 1024, 10)
MLP_FLOPS = 16_236_150_784
CNN_FLOPS = 7_017_332_736
LN_TRAFFIC = 33_600_000  # bytes, ncu dram read + write of one ln_fwd_reg<float,8> launch
# 6 * (matmul params 6*3,145,728 + head 16,384,000) * 16,384 tokens
# + attention 3 (fwd + 2x bwd) * 6 layers * 4 * 64 * 256^2 * 512
TR_CFG = dict(batch=64, seq=256, layers=6, d=512, heads=8, ffn=2048, vocab=32000)
TR_FLOPS = 6 * (6 * 3_145_728 + 16_384_000) * 64 * 256 + 3 * 6 * 4 * 64 * 256 * 256 * 512


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
        torch = self.torch
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
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
        torch.cuda.synchronize()
        return [a.elapsed_time(b) * 1e-3 for a, b in ev]  # seconds

    def bufs(self, arrays):
        return [self.client.buffer_from_numpy(a, device=self.dev) for a in arrays]


def plan_launches(text: str) -> int:
    from jax_b200 import pjrt
    plan = pjrt.inspect(text, 1)
    steps = plan.split("steps:")[1].strip().splitlines()
    return sum(1 for s in steps if not s.strip().startswith(("copy", "all_reduce")))


def ln_inputs(seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((LN_ROWS, LN_COLS)).astype(np.float32)
    r = rng.standard_normal((LN_ROWS, LN_COLS)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(LN_COLS)).astype(np.float32)
    b = (0.1 * rng.standard_normal(LN_COLS)).astype(np.float32)
    return [x, r, g, b]


def bench_ln(rig: Rig, steps, warmup):
    from jax_b200 import programs
    text = programs.layer_norm()
    exe = rig.client.compile(text)
    args = rig.bufs(ln_inputs())
    launches = plan_launches(text)
    holder = []

    def step():
        holder[:] = exe.execute([args])
    with ClockSampler(rig.torch.cuda.current_device()) as clk:
        ts = rig.time_steps(step, steps, warmup)
    dev_ms = exe.device_times_ms()[-steps:]
    t = float(np.mean(dev_ms)) * 1e-3 if len(dev_ms) == steps else float(np.mean(ts))
    value = LN_BYTES / t / 1e9
    # end to end: pinned host inputs -> device -> execute -> host, per step
    torch = rig.torch
    host_in = [torch.from_numpy(a).pin_memory() for a in ln_inputs()]
    host_out = torch.empty((LN_ROWS, LN_COLS), dtype=torch.float32).pin_memory()
    out_np = host_out.numpy()
    from jax_b200.pjrt import F32, api

    def e2e_step():
        bs, evs = [], []
        for h in host_in:
            b, ev = rig.client.buffer_from_host_ptr(h.data_ptr(), F32, tuple(h.shape), rig.dev, semantics=1)
            bs.append(b)
            evs.append(ev)
        o = exe.execute([bs])[0][0]
        api().await_event(o.to_host_async(out_np))
        for ev in evs:
            api().await_event(ev)
    e2e_ts = rig.time_steps(e2e_step, steps, warmup, flush=True)
    exe.device_times_ms()
    e2e_t = float(np.mean(e2e_ts))
    kt, kcfg = ln_kernel_time(rig, steps)
    h2d = sum(h.numel() * 4 for h in host_in)
    return {
        "metric": "residual+LayerNorm fwd HBM throughput (jitted, configs[1])", "unit": "GB/s",
        "value": value, "ms_per_step": t * 1e3, "dtype": "f32",
        "outer_event_ms_per_step": float(np.mean(ts)) * 1e3,
        "config": {"workload": "residual_layernorm_fwd", "shape": [LN_ROWS, LN_COLS], "eps": 1e-5,
                   "l2": "evicted between timed steps (2 GB read on the same stream)",
                   "algorithmic_bytes_per_step": LN_BYTES},
        "e2e": {"value": LN_BYTES / e2e_t / 1e9, "unit": "GB/s", "ms_per_step": e2e_t * 1e3,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": LN_ROWS * LN_COLS * 4},
        "launches_per_step": launches, "clocks": clk.summary(),
        "kernel_time_s": kt, "kernel_timing": kcfg, "algorithmic": LN_BYTES, "bound": "hbm",
    }


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
    text = programs.sdpa(*SDPA_SHAPE, causal=True)
    exe = rig.client.compile(text)
    rng = np.random.default_rng(1)
    args = rig.bufs([rng.standard_normal(SDPA_SHAPE).astype(np.float32) for _ in range(3)])
    holder = []
    ts = rig.time_steps(lambda: holder.__setitem__(slice(None), exe.execute([args])), steps, warmup)
    dev_ms = exe.device_times_ms()[-steps:]
    t = float(np.mean(dev_ms)) * 1e-3 if len(dev_ms) == steps else float(np.mean(ts))
    return {"metric": "causal SDPA fwd f32 (jitted, configs[0])", "unit": "TFLOP/s",
            "value": SDPA_FLOPS / t / 1e12, "ms_per_step": t * 1e3, "flops_per_step": SDPA_FLOPS,
            "tensor_path": "tcgen05 kind::f16 (f32 inputs as bf16 hi+lo, 3 products)",
            "launches_per_step": plan_launches(text),
            "l2": "flushed between steps"}


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
    ts = rig.time_steps(step, steps, warmup)
    t = float(np.mean(ts))
    fl = 2.0 * M * N * K
    return {"metric": f"GEMM {M}x{N}x{K} {dtype} ({'A^T' if a_t else 'A'}, {'B^T' if b_t else 'B'})",
            "unit": "TFLOP/s", "value": fl / t / 1e12, "ms_per_step": t * 1e3, "flops_per_step": fl,
            "launches_per_step": 1, "dtype": dtype}


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


def _transformer_bufs(rig: Rig, rng, per, rank):
    """configs[3] arguments: N(0, 0.02) bf16 params, zero f32 Adam moments,
    count 0, this rank's slice of the [64, 256] tokens and next-token targets."""
    from jax_b200 import pjrt, programs
    c = TR_CFG
    shapes = programs.transformer_param_shapes(c["layers"], c["d"], c["heads"], c["ffn"], c["vocab"],
                                               c["seq"])
    bufs = [rig.client.buffer_from_numpy(pjrt.to_bf16_bits(rng.standard_normal(s).astype(np.float32)
                                                           * np.float32(0.02)), rig.dev, bf16=True)
            for _, s in shapes]
    zeros = [np.zeros(s, np.float32) for _, s in shapes]
    tok = rng.integers(0, c["vocab"], (c["batch"], c["seq"])).astype(np.int32)
    tgt = np.roll(tok, -1, axis=1)
    sl = slice(rank * per, (rank + 1) * per)
    return bufs + rig.bufs(zeros + zeros + [np.array(0, np.int32), tok[sl], tgt[sl]])


def bench_train(rig: Rig, kind, steps, warmup, world=1, rank=0):
    from jax_b200 import programs
    gb = {"mlp": 1024, "cnn": 256, "transformer": TR_CFG["batch"]}[kind]
    per = gb // world
    if kind == "mlp":
        text = programs.mlp_step(batch=per, num_replicas=world)
    elif kind == "cnn":
        text = programs.cnn_step(batch=per, num_replicas=world)
    else:
        text = programs.transformer_step(**dict(TR_CFG, batch=per), num_replicas=world)
    exe = rig.client.compile(text)
    rng = np.random.default_rng({"mlp": 8, "cnn": 13, "transformer": 11}[kind])
    if kind == "transformer":
        args = _transformer_bufs(rig, rng, per, rank)
        n_state = len(args) - 2  # params, moments and count feed the next step
    else:
        full = _mlp_args(rng, gb) if kind == "mlp" else _cnn_args(rng, gb)
        arrays = full[:-2] + [full[-2][rank * per:(rank + 1) * per],
                              full[-1][rank * per:(rank + 1) * per]]
        args = rig.bufs(arrays)
        n_state = len(args) - 2
    holder = []

    def step():
        # the updated state feeds the next step, as a training loop does
        outs = exe.execute([args])[0]
        holder[:] = outs
        args[:n_state] = outs[1:1 + n_state]
    ts = rig.time_steps(step, steps, warmup, flush=False)
    exe.device_times_ms()
    t = float(np.mean(ts))  # back-to-back steps: host launch overhead is part of a training step
    flops = {"mlp": MLP_FLOPS, "cnn": CNN_FLOPS, "transformer": TR_FLOPS}[kind]
    opt = "Adam" if kind == "transformer" else "SGD"
    return {"metric": f"{kind.upper()} training step (jitted value_and_grad + {opt})",
            "unit": "samples/s", "value": gb / t, "ms_per_step": t * 1e3, "global_batch": gb,
            "flops_per_step": flops, "tflops": flops / t / 1e12,
            "launches_per_step": plan_launches(text),
            "dtype": "bf16" if kind == "transformer" else "f32"}


# -------------------------------------------------------- CPU baseline ---
def cpu_ln_baseline(threads: int, budget_s: float = 10.0):
    """oracle/restate.layer_norm_ref on row chunks, `threads` host threads."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import restate
    x, r, g, b = ln_inputs()
    chunks = np.array_split(np.arange(LN_ROWS), threads)

    def one(ix):
        restate.layer_norm_ref(x[ix], r[ix], g, b)
    done, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(threads) as pool:
        while time.perf_counter() - t0 < budget_s and done < 50:
            list(pool.map(one, chunks))
            done += 1
    t = (time.perf_counter() - t0) / done
    return {"value": LN_BYTES / t / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{done} full [4096,1024] residual+LayerNorm passes of oracle/restate.py "
                      f"(numpy f64) over {threads} threads, {t * 1e3:.1f} ms each"}


# ------------------------------------------------------------------ main --
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="ln", choices=["ln", "sdpa", "mlp", "cnn", "transformer", "gemm"])
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
        if rank != 0:
            return
        threads = host_cores()
        if a.workload != "ln":
            print(json.dumps({"impl": "reference", "unavailable":
                              "only the LayerNorm workload has a CPU port timed here"}))
            return
        cb = cpu_ln_baseline(threads, budget_s=min(60.0, 2.0 * max(a.steps, 1)))
        print(json.dumps({
            "impl": "reference", "metric": "residual+LayerNorm fwd HBM throughput (jitted, configs[1])",
            "value": cb["value"], "unit": "GB/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1))",
            "config": {"workload": "residual_layernorm_fwd", "shape": [LN_ROWS, LN_COLS]},
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                                         "d2h_bytes_per_step": 0},
            "note": "reference plugin needs macOS/Metal (MLX); its arithmetic is timed via the oracle port"}))
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
    if a.workload == "ln":
        res = bench_ln(rig, a.steps, a.warmup)
    elif a.workload == "sdpa":
        res = bench_sdpa(rig, a.steps, a.warmup)
        res.update(bound="tensor", kernel_time_s=res["ms_per_step"] * 1e-3, algorithmic=SDPA_FLOPS)
    elif a.workload == "gemm":
        res = bench_gemm(rig, a.steps, a.warmup, tuple(int(v) for v in a.gemm_shape.split(",")),
                         a.gemm_dtype, a.gemm_trans)
    else:
        res = bench_train(rig, a.workload, a.steps, a.warmup, world, rank)
    t_local = res["ms_per_step"]
    if dist is not None:
        tt = torch.tensor([t_local], dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max = float(tt.item())
        dist.barrier()
    else:
        t_max = t_local
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
    pk, pk_kind = peaks()
    line = {
        "metric": res["metric"], "unit": res["unit"], "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "higher_is_better": True, "vs_baseline": None, "data": "synthetic (seeded)",
        "dtype": res.get("dtype", "f32"),
    }
    if a.workload == "ln":
        per_gpu = res["value"] * res["ms_per_step"] / t_max
        line.update(value=per_gpu * world, ms_per_step=t_max, scaling="weak",
                    config=dict(res["config"], parallelism=f"replicas x{world}"))
        line["e2e"] = dict(res["e2e"], value=res["e2e"]["value"] * world)
        ach = LN_BYTES / res["kernel_time_s"] / 1e9
        line["roofline"] = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                            "frac": ach / pk["hbm_gbs"], "peak_kind": pk_kind,
                            # dram__bytes_read.sum + dram__bytes_write.sum of one launch
                            # (ncu capture summarised in profiles/): the 16.8 MB of y is
                            # still in L2 when the kernel ends
                            "traffic": LN_TRAFFIC,
                            "kernel": "ln_fwd_reg<float,8>", "timing": res["kernel_timing"],
                            "per_launch_bytes": LN_BYTES}
        line["clocks"] = res["clocks"]
        line["gpu_launches"] = res["launches_per_step"] * a.steps
        if world == 1:
            line["cpu_baseline"] = cpu_ln_baseline(host_cores(), budget_s=10.0)
    else:
        kernel_only = a.workload in ("sdpa", "gemm")
        line.update(value=res["value"] * (world if kernel_only else 1) if kernel_only
                    else res["global_batch"] / (t_max * 1e-3),
                    ms_per_step=t_max, scaling="weak" if kernel_only else "strong",
                    config={"workload": a.workload, "parallelism": f"dp{world}" if dp else f"replicas x{world}"})
        if a.workload == "gemm":
            line["config"].update(shape=a.gemm_shape, trans=a.gemm_trans, l2="flushed between steps")
        line["gpu_launches"] = res["launches_per_step"] * a.steps
    if world == 1 and not a.no_extra and a.workload == "ln":
        extra = {}
        try:
            extra["sdpa"] = bench_sdpa(rig, 20, 3)
            s = extra["sdpa"]
            s["roofline"] = {"bound": "tensor", "achieved": s["value"], "peak": pk["bf16_tflops"],
                             "unit": "TFLOP/s", "frac_of_bf16_peak": s["value"] / pk["bf16_tflops"],
                             "peak_kind": pk_kind}
        except Exception as e:  # report, do not hide
            extra["sdpa"] = {"error": str(e)[:300]}
        for kind in ("mlp", "cnn", "transformer"):
            try:
                extra[f"{kind}_step"] = bench_train(rig, kind, 20, 3)
            except Exception as e:
                extra[f"{kind}_step"] = {"error": str(e)[:300]}
        line["extra"] = extra
    print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
