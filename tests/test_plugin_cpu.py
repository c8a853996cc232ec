"""CPU: the C-ABI libraries load and export what include/*.h declares; the PJRT
table layout matches the header; the compile pipeline (parse -> SDPA/LN match ->
plan -> NVRTC) works without a device.  No kernel is launched."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from cases import cases
from jax_b200 import kernels, pjrt, programs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")


def _declared(header):
    text = open(os.path.join(INC, header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b((?:b200|GetPjrt)\w*)\s*\(", text))
    return {n for n in names if not n.startswith("B200_")}


def test_kernel_library_exports_every_declared_symbol():
    lib = C.CDLL(kernels.KERNELS_LIB)
    declared = _declared("b200_kernels.h")
    assert {"b200_ln_residual_fwd", "b200_sdpa_fwd", "b200_gemm"} <= declared
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.b200_kernels_version and kernels.lib().b200_kernels_version().startswith(b"b200-kernels")


def test_pjrt_library_exports_every_declared_symbol():
    lib = C.CDLL(pjrt.PJRT_LIB)
    declared = _declared("b200_pjrt.h") | _declared("b200_pjrt_inspect.h")
    assert "GetPjrtApi" in declared
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing


def test_api_table_matches_header():
    text = open(os.path.join(INC, "b200_pjrt.h")).read()
    block = text[text.index("#define B200_PJRT_API_SLOTS(X)"):text.index("#define B200_PJRT_SLOT_FIELD")]
    slots = re.findall(r"X\((\w+)\)", block)
    assert slots == pjrt.API_SLOTS
    assert len(slots) == 128
    api = pjrt.api()
    assert api.version == (0, 90)
    assert api.struct_size == 40 + 8 * 128
    # every slot is filled (unimplemented ones return an error, never NULL)
    assert all(api._fn[n] is not None for n in pjrt.API_SLOTS)


def test_unimplemented_slot_returns_error_not_crash():
    api = pjrt.api()

    class Args(C.Structure):
        _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p), ("pad", C.c_void_p * 8)]
    err = api.raw("CopyToDeviceStream_Destroy", Args())
    with pytest.raises(pjrt.PjrtError) as e:
        api.check(err)
    assert e.value.code == 12


def test_client_create_without_device_fails_cleanly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.Client()
    assert e.value.code in (13, 14)


def test_config_programs_fuse_and_compile():
    g = pjrt.inspect(programs.sdpa(), 0)
    assert "fused_sdpa" in g and "causal=1" in g and "scale=0.125" in g
    assert "dot_general" not in g and "exponential" not in g
    g = pjrt.inspect(programs.layer_norm(), 0)
    assert "fused_layer_norm" in g and "flags=14" in g
    assert pjrt.inspect(programs.layer_norm(), 1).count("layer_norm in=") == 1
    for text in (programs.mlp_step(), programs.cnn_step(), programs.mlp_step(batch=512, num_replicas=2)):
        assert pjrt.inspect(text, 3).startswith("ok ")
    # the loss and all 8 gradient means go out as one bucketed collective
    plan = pjrt.inspect(programs.mlp_step(batch=512, num_replicas=2), 1)
    steps = plan.split("steps:")[1]
    assert steps.count("all_reduce_bucket in=") == 1 and steps.count("all_reduce in=") == 0
    bucket = [l for l in steps.splitlines() if "all_reduce_bucket" in l][0]
    assert bucket.split(" out=")[0].count(",") == 9  # 9 inputs, comma-terminated
    # each gradient is computed in its piece of the bucket and read back from
    # there: 9 inputs and 9 reduced values are views of the bucket slot
    bslot = bucket.split(" out=")[1].split(" ip=")[0].rstrip(",").split(",")[-1]
    assert plan.split("steps:")[0].count(f"view={bslot}+") == 18


def test_row_wise_kernels_share_one_pass():
    """Row reductions and loops over the same rows run as one row-group kernel
    (one HBM pass per row); a reduction reading an earlier phase's output at
    transposed positions starts a kernel of its own."""
    steps = pjrt.inspect(programs.logits_cross_entropy(2400, 5000), 1).split("steps:")[1]
    names = [l.split()[0] for l in steps.strip().splitlines()]
    # forward statistics (max, sum of exponentials, target logit) in one kernel,
    # the logits gradient (with its row sums) in another, then the bias column sum
    assert names[0].endswith("_rows") and sum(n.endswith("_rows") for n in names) == 2
    assert not any(n.endswith("_loop") and "in=s0," in n for n in names)
    steps = pjrt.inspect(programs.softmax_then_transposed_sum(), 1).split("steps:")[1]
    names = [l.split()[0] for l in steps.strip().splitlines()]
    assert names == ["k0_rows", "k1_reduce"]
    # transformer step: every layer norm and the loss
    steps = pjrt.inspect(programs.transformer_step(), 1).split("steps:")[1]
    assert steps.count("_rows in=") >= 6 * 3 + 2


def test_kernels_with_one_body_run_as_one_launch():
    """Generated loop and reduction kernels that compile to the same code run
    as one launch (a pointer table, blockIdx.z picking the member) where they
    can all meet: the optimizer's per-parameter updates (one body per
    parameter shape), the bias / norm-gain gradient reductions that feed them,
    and each block's q / k / v bias additions."""
    steps = pjrt.inspect(programs.transformer_step(), 1).split("steps:")[1].strip().splitlines()
    names = [l.split()[0] for l in steps]
    batched = [n for n in names if re.match(r"k\d+_(loop|reduce|reduce_parts)_x\d+_\d+$", n)]
    loops = sorted(int(re.search(r"_x(\d+)_", n).group(1)) for n in batched if "_loop_x" in n)
    # the five update bodies repeat across the blocks (the embeddings and the
    # head have shapes of their own); the bias additions come in threes
    for size in (6, 12, 24, 26, 30):
        assert size in loops, loops
    assert any("_reduce_x" in n for n in batched) and any("_reduce_parts_x" in n for n in batched)
    assert len(steps) < 230
    kernels = pjrt.inspect(programs.transformer_step(), 2)
    assert kernels.count("const __grid_constant__") >= len(batched)


def _step_names(text):
    steps = pjrt.inspect(text, 1).split("steps:")[1]
    return [l.split()[0] for l in steps.strip().splitlines()]


def test_attention_with_its_backward_fuses():
    """Attention whose probabilities also feed its backward (dV = P^T dO,
    dP = dO V^T, the softmax vjp, dQ = dS K, dK = dS^T Q) becomes one forward
    kernel that keeps the row statistics plus one backward kernel: no GEMM,
    softmax row group or transpose is left.  The softmax vjp is recognized by
    its value (a symbolic form in P, the row sum and dP), so the quotient-rule
    form of generic autodiff and the form of jax.nn.softmax's custom JVP both
    match."""
    for form, causal in (("autodiff", True), ("custom_jvp", True), ("custom_jvp", False)):
        names = _step_names(programs.attention_vjp(form=form, causal=causal))
        assert names.count("sdpa") == 1 and names.count("sdpa_bwd") == 1, (form, names)
        assert "gemm" not in names and not any(n.endswith("_rows") for n in names), (form, names)
    # outside the backward kernel's limits (T > 256; f32) the chain stays unfused
    for kw in (dict(T=384), dict(dt="f32")):
        names = _step_names(programs.attention_vjp(form="custom_jvp", **kw))
        assert "sdpa_bwd" not in names and "gemm" in names, (kw, names)
    names = _step_names(programs.transformer_step())
    assert names.count("sdpa") == 6 and names.count("sdpa_bwd") == 6
    # the reference's mlx_sdpa_bwd custom call: bf16 runs the forward with row
    # statistics and the fused backward; f32 keeps the compile-time expansion
    names = _step_names(programs.sdpa_custom_calls(2, 128, 2, 64, 0.125, "bf16"))
    assert names == ["sdpa", "sdpa", "sdpa_bwd"], names
    names = _step_names(programs.sdpa_custom_calls(2, 128, 2, 64, 0.125, "f32"))
    assert "sdpa_bwd" not in names and "gemm" in names, names


def test_attention_backward_with_another_value_is_not_fused():
    """A backward whose dS is not the softmax vjp (wrong sign of the row-sum
    term, or a scale other than the forward's) keeps its unfused plan."""
    from jax_b200.hlo import Builder
    from jax_b200.programs import softmax
    B, T, N, H = 1, 128, 2, 64
    for sign, sc in ((+1.0, 0.125), (-1.0, 0.25)):
        b = Builder("jit_attention_vjp_altered")
        q, k, v, g = (b.param((B, T, N, H), "bf16") for _ in range(4))
        qt, kt, vt, gt = (b.transpose(x, [0, 2, 1, 3]) for x in (q, k, v, g))
        logits = b.dot_general(qt, kt, ([3], [3]), ([0, 1], [0, 1]), out_dt="f32") * 0.125
        y = softmax(b, logits)
        yb = b.convert(y, "bf16")
        o = b.dot_general(yb, vt, ([3], [2]), ([0, 1], [0, 1]))
        dv = b.dot_general(yb, gt, ([2], [2]), ([0, 1], [0, 1]))
        dy = b.convert(b.dot_general(gt, vt, ([3], [3]), ([0, 1], [0, 1])), "f32")
        yg = y * dy
        dx = yg + y * b.broadcast_in_dim(b.sum(yg, [3]), yg.shape, [0, 1, 2]) * sign
        ds = dx * sc
        dq = b.convert(b.dot_general(ds, kt, ([3], [2]), ([0, 1], [0, 1])), "bf16")
        dk = b.convert(b.dot_general(ds, qt, ([2], [2]), ([0, 1], [0, 1])), "bf16")
        names = _step_names(b.module([o, dq, dk, dv]))
        assert "sdpa_bwd" not in names, (sign, sc, names)


def test_identical_kernels_compile_once_and_cache_on_disk(tmp_path, monkeypatch):
    """Every block's layer norm, softmax and update kernels are the same code:
    each distinct body is compiled once (the others alias it), in parallel
    units; with B200_CACHE_DIR the cubins of a new program are written there
    and a later compile of the same units reads them back."""
    text = programs.transformer_step(batch=2, seq=32, layers=3, d=64, heads=2, ffn=128, vocab=96)
    steps = pjrt.inspect(text, 1).split("steps:")[1].strip().splitlines()
    rows = [l.split()[0] for l in steps if re.match(r"k\d+_rows$", l.split()[0])]
    source = pjrt.inspect(text, 2)
    row_bodies = len(re.findall(r"__global__ void __launch_bounds__\(\d+\) k\d+_rows\(", source))
    # (the first and last blocks' kernels differ a little from the middle one's)
    assert row_bodies <= len(rows) * 0.7, (row_bodies, len(rows))
    # batched launches leave their members' own kernels uncompiled
    launched = {l.split()[0] for l in steps}
    compiled = re.findall(r"__global__ void __launch_bounds__\(\d+\) (k\w+)\(", source)
    assert set(compiled) <= launched, set(compiled) - launched
    # a program no earlier test compiled (its constant is unique to this test)
    from jax_b200.hlo import Builder
    b = Builder("cache_probe")
    x = b.param((3, 1000))
    prog = b.module([b.exp(x * 0.123456789) + b.sum(x, [1], keepdims=True)])
    monkeypatch.setenv("B200_CACHE_DIR", str(tmp_path))
    first = pjrt.inspect(prog, 3)
    files = sorted(tmp_path.glob("b200-nvrtc*.cubin"))
    assert first.startswith("ok ") and files
    assert sum(f.stat().st_size for f in files) == int(first.split()[1])
    assert not list(tmp_path.glob("*.tmp*"))


def _plan_tables(text):
    plan = pjrt.inspect(text, 1)
    head, steps = plan.split("steps:")
    slots = {}
    for m in re.finditer(r"^\s+s(\d+) (\w+)\[-?\d+\] (\S+) (.*)$", head, flags=re.M):
        slots[int(m.group(1))] = (m.group(2), m.group(3), m.group(4))
    rows = []
    for line in steps.strip().splitlines():
        ins = line.split(" in=")[1].split(" out=")[0].rstrip(",")
        rows.append((line.split()[0], [int(s[1:]) for s in ins.split(",") if s]))
    return slots, rows


def test_gemm_operands_arrive_as_planes():
    """An f32 value read only by GEMMs is stored by the kernel that computes it
    as two bf16 planes (hi and lo = the rounding remainder), which the GEMM
    reads as its split operand: attention's dS in the transformer step, and
    every im2col patch matrix of the CNN step (K a multiple of 8).  No f32
    copy of such a value is stored."""
    slots, rows = _plan_tables(programs.transformer_step(batch=2, seq=32, layers=1, d=64, heads=2,
                                                         ffn=128, vocab=96))
    planed = [ins for name, ins in rows if name == "gemm" and len(ins) == 3]
    assert len(planed) >= 2
    for ins in planed:
        lo = slots[ins[2]]
        assert lo[1].endswith("xbf16>") and lo[2].endswith(".lo")
        hi = [slots[s] for s in ins[:2] if slots[s][2] == lo[2][:-3] + ".hi"]
        assert len(hi) == 1 and hi[0][1] == lo[1]
        # the f32 value itself is not a slot of the plan
        assert not any(s[2] == lo[2][:-3] for s in slots.values())

    slots, rows = _plan_tables(programs.cnn_step())
    im2col_out = {s: slots[s][2] for s, v in slots.items() if v[2].startswith("im2col")}
    # the first conv's patches have K = 3*3*1 = 9 columns: stored in f32
    f32 = [s for s, n in im2col_out.items() if n == "im2col"]
    assert [slots[s][1] for s in f32] == ["tensor<200704x9xf32>"]
    for s in f32:
        del im2col_out[s]
    # the weight gradient of the second conv stores its patches transposed
    # ([K, M], eight channels of one pixel per thread); the rest as [M, K]
    assert len(im2col_out) == 8 and all(n in ("im2col_hi", "im2col_lo", "im2col_t_hi", "im2col_t_lo")
                                        for n in im2col_out.values())
    assert sorted(slots[s][1] for s, n in im2col_out.items() if n.startswith("im2col_t")) == \
        ["tensor<50176x288xbf16>"] * 2
    assert all(slots[s][1].endswith("xbf16>") for s in im2col_out)
    gemms = [ins for name, ins in rows if name == "gemm"]
    for s, n in im2col_out.items():
        readers = [ins for ins in gemms if s in ins]
        assert len(readers) == 1 and len(readers[0]) == 3
        # hi is the A operand, lo the trailing plane input
        assert readers[0].index(s) == (0 if n.endswith("_hi") else 2)


def test_attention_operands_are_written_in_gemm_order():
    """Attention over [B, T, N, H] contracts with batch dims (B, N) that are not
    one strided group.  The q / k / v and dS values are written in the GEMMs'
    batch order by the kernels that compute them, so the transformer step
    has no standalone transpose (permute) kernel and every GEMM reads its
    operands as they are stored."""
    layers = 2
    slots, rows = _plan_tables(programs.transformer_step(batch=2, seq=32, layers=layers, d=64,
                                                         heads=2, ffn=128, vocab=96))
    kinds = {name.split("_", 1)[-1] for name, _ in rows}
    assert "permute" not in kinds and "gemm" in kinds
    # the batched attention GEMMs ([B*N] x [T, T] and [T, H] products)
    batched = [ins for name, ins in rows if name == "gemm"
               and slots[ins[0]][1].startswith("tensor<2x2x32x")]
    assert len(batched) == layers * 6  # QK^T and PV forward; 4 in the backward


def test_non_causal_and_bnth_attention_also_match():
    g = pjrt.inspect(programs.sdpa(2, 256, 4, 64, causal=False), 0)
    assert "fused_sdpa" in g and "causal=0" in g


def test_external_consumer_blocks_fusion():
    """An intermediate of the softmax chain that is also a program output must
    stay materialized: no fused_sdpa (reference src/jax_mlx_pjrt.cpp:1843-1855)."""
    from jax_b200.hlo import Builder
    b = Builder()
    q, k, v = (b.param((1, 128, 2, 64)) for _ in range(3))
    logits = b.dot_general(q, k, ([3], [3]), ([0, 2], [0, 2])) * 0.125
    m = b.max(logits, [3], keepdims=True)
    e = b.exp(logits - m)
    p = e / b.sum(e, [3], keepdims=True)
    o = b.dot_general(p, v, ([3], [1]), ([0, 1], [0, 2]))
    g = pjrt.inspect(b.module([o, p]), 0)
    assert "fused_sdpa" not in g


@pytest.mark.parametrize("case", cases(), ids=lambda c: c[0])
def test_golden_case_programs_compile(case):
    assert pjrt.inspect(case[1], 3).startswith("ok")


def test_parse_errors_are_invalid_argument():
    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.inspect("module { func.func @main(%a: tensor<4xf32>) -> tensor<4xf32> { %0 = stablehlo.add %a, : tensor<4xf32> return %0 : tensor<4xf32> } }", 0)
    assert e.value.code == 3


_FAULT_PROBE = """
import sys
sys.path[:0] = [{root!r}, {pkg!r}]
from jax_b200 import pjrt, programs
try:
    pjrt.inspect(programs.layer_norm(), 0)
    print("ok")
except pjrt.PjrtError as e:
    print(e.code, e)
"""


@pytest.mark.parametrize("spec, expect", [
    ("compile", "13 INTERNAL: injected fault at compile (B200_FAULT)"),
    ("alloc, execute,nccl_init", "ok"),
    ("", "ok"),
])
def test_fault_injection_is_host_side_and_named(spec, expect):
    """B200_FAULT lists host-side failure points; the compile point fails the
    compile pipeline with the error a real compile failure raises, and points
    of later stages leave compilation alone.  (The process reads the variable
    once, so each case runs in a fresh interpreter.)"""
    import subprocess
    import sys
    env = dict(os.environ, B200_FAULT=spec)
    code = _FAULT_PROBE.format(root=ROOT, pkg=os.path.join(ROOT, "jax-mlx-plugin_b200"))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-1500:]
    assert r.stdout.strip() == expect


def test_portable_artifact_without_mlir_c_api_is_unimplemented():
    """A program given as MLIR bytecode (what jax hands a plugin) is converted
    through the StableHLO C API that jaxlib loads; in a process without it the
    compile fails with UNIMPLEMENTED and says to pass text instead."""
    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.inspect(b"ML\xefR\x00\x01\x02stablehlo", 0)
    assert e.value.code == 12 and "StableHLO C API" in str(e.value)
    # text still goes straight to the parser
    assert "fused_layer_norm" in pjrt.inspect(programs.layer_norm().encode(), 0)


_RW = ('module @m {{ func.func public @main(%arg0: tensor<2x4x4x3xf32>) -> tensor<2x2x2x3xf32> {{\n'
       '  %0 = stablehlo.constant dense<0xFF800000> : tensor<f32>\n'
       '  %1 = "stablehlo.reduce_window"(%arg0, %0) <{{padding = dense<0> : tensor<4x2xi64>, '
       'window_dimensions = array<i64: {win}>, window_strides = array<i64: 1, 2, 2, 1>}}> ({{\n'
       '  ^bb0(%a: tensor<f32>, %b: tensor<f32>):\n'
       '    %m = stablehlo.maximum %a, %b : tensor<f32>\n'
       '    stablehlo.return {ret}\n'
       '  }}) : (tensor<2x4x4x3xf32>, tensor<f32>) -> tensor<2x2x2x3xf32>\n'
       '  return %1 : tensor<2x2x2x3xf32>\n}} }}\n')
_PAD = ('module @m {{ func.func public @main(%arg0: tensor<2x2xf32>) -> tensor<3x3xf32> {{\n'
        '  %0 = stablehlo.constant dense<0.0> : tensor<f32>\n'
        '  %1 = stablehlo.pad %arg0, %0, {low}, high = [0, 0], interior = [1, 1] : '
        '(tensor<2x2xf32>, tensor<f32>) -> tensor<3x3xf32>\n'
        '  return %1 : tensor<3x3xf32>\n}} }}\n')
_NEG = ('module @m {{ func.func public @main(%arg0: tensor<4xf32>) -> tensor<4xf32> {{\n'
        '  %0 = stablehlo.negate {arg}: tensor<4xf32>\n'
        '  return %0 : tensor<4xf32>\n}} }}\n')


_SLICE = ('module @m {{ func.func public @main(%arg0: tensor<8xf32>) -> tensor<{n}xf32> {{\n'
          '  %0 = stablehlo.slice %arg0 [0:4] : (tensor<8xf32>) -> tensor<{n}xf32>\n'
          '  return %0 : tensor<{n}xf32>\n}} }}\n')

_GATHER = ('module @m {{ func.func public @main(%arg0: tensor<12x8xf32>, %arg1: tensor<2x4x1xi32>) -> '
           'tensor<2x4x{od}xf32> {{\n'
           '  %0 = "stablehlo.gather"(%arg0, %arg1) <{{dimension_numbers = #stablehlo.gather<offset_dims = [2], '
           'collapsed_slice_dims = [0], start_index_map = [0], index_vector_dim = 2>, indices_are_sorted = false, '
           'slice_sizes = array<i64: 1, {ss}>}}> : (tensor<12x8xf32>, tensor<2x4x1xi32>) -> tensor<2x4x{od}xf32>\n'
           '  return %0 : tensor<2x4x{od}xf32>\n}} }}\n')


def _conv(out):
    """The reference's conv case (1x8x8x3 * 3x3x3x16, SAME) with the output's
    spatial size given as `out`."""
    t = [c for c in cases() if c[0] == "conv_same_ones"][0][1]
    return t.replace("1x8x8x16xf32", f"1x{out}x{out}x16xf32")


@pytest.mark.parametrize("good, bad, what", [
    (_RW.format(win="1, 2, 2, 1", ret="%m : tensor<f32>"), _RW.format(win="2, 1", ret="%m : tensor<f32>"),
     "window attributes"),
    (_RW.format(win="1, 2, 2, 1", ret="%m : tensor<f32>"), _RW.format(win="1, 2, 2, 1", ret=""),
     "body returns 0 values"),
    (_PAD.format(low="low = [0, 0]"), _PAD.format(low="lo = [0, 0]"), "padding"),
    (_NEG.format(arg="%arg0 "), _NEG.format(arg=""), "needs 1 operands"),
    (_RW.format(win="1, 2, 2, 1", ret="%m : tensor<f32>"),
     _RW.format(win="1, 2, 2, 1", ret="%m : tensor<f32>").replace("-> tensor<2x2x2x3xf32>\n", "-> tensor<22x3xf32>\n"),
     "result rank differs"),
    (_SLICE.format(n=4), _SLICE.format(n=6), "result shape does not match the slice"),
    (_GATHER.format(ss=8, od=8), _GATHER.format(ss=9, od=9), "slice size out of range"),
    (_GATHER.format(ss=8, od=8), _GATHER.format(ss=4, od=8), "result shape does not match the gather"),
    (_conv(8), _conv(9), "result spatial size does not match the window"),
    # splat padding dense<1> pads both edges of every dimension by 1: windows
    # [1, 2, 2, 1] at strides [1, 2, 2, 1] over 2x4x4x3 give 4x3x3x5, not 2x2x2x3
    (_RW.format(win="1, 2, 2, 1", ret="%m : tensor<f32>").replace("dense<0> : tensor<4x2xi64>", "dense<1> : tensor<4x2xi64>")
     .replace("tensor<2x2x2x3xf32>", "tensor<4x3x3x5xf32>"),
     _RW.format(win="1, 2, 2, 1", ret="%m : tensor<f32>").replace("dense<0> : tensor<4x2xi64>", "dense<1> : tensor<4x2xi64>"),
     "result shape does not match the windows"),
])
def test_malformed_attributes_are_invalid_argument(good, bad, what):
    """Programs whose attribute lists or bodies do not fit their operands (each
    once drove the code generator out of range under a fuzzer) are rejected
    right after parsing; the well-formed versions compile."""
    assert pjrt.inspect(good, 1).startswith("slots")
    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.inspect(bad, 1)
    assert e.value.code == 3 and what in str(e.value), str(e.value)


def test_unsupported_op_is_unimplemented():
    text = ('module @m { func.func public @main(%arg0: tensor<8xf32>) -> tensor<8xf32> {\n'
            '  %0 = "stablehlo.sort"(%arg0) <{dimension = 0 : i64}> ({\n'
            '  ^bb0(%a: tensor<f32>, %b: tensor<f32>):\n'
            '    %c = stablehlo.compare  LT, %a, %b,  FLOAT : (tensor<f32>, tensor<f32>) -> tensor<i1>\n'
            '    stablehlo.return %c : tensor<i1>\n  }) : (tensor<8xf32>) -> tensor<8xf32>\n'
            '  return %0 : tensor<8xf32>\n} }\n')
    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.inspect(text, 1)
    assert e.value.code == 12


def test_generic_printing_and_func_call_inlining():
    text = '''module @jit_f attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func public @main(%arg0: tensor<4x8xf32> {mhlo.layout_mode = "default"}) -> (tensor<4x8xf32> {jax.result_info = ""}) {
    %0 = call @relu(%arg0) : (tensor<4x8xf32>) -> tensor<4x8xf32>
    %1 = "stablehlo.add"(%0, %0) : (tensor<4x8xf32>, tensor<4x8xf32>) -> tensor<4x8xf32>
    return %1 : tensor<4x8xf32>
  }
  func.func private @relu(%arg0: tensor<4x8xf32>) -> tensor<4x8xf32> {
    %cst = stablehlo.constant dense<0.000000e+00> : tensor<f32>
    %0 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<4x8xf32>
    %1 = stablehlo.maximum %arg0, %0 : tensor<4x8xf32>
    return %1 : tensor<4x8xf32>
  }
}
'''
    g = pjrt.inspect(text, 0)
    assert "call" not in g and "maximum" in g
    plan = pjrt.inspect(text, 1)
    assert plan.count("_loop") == 1  # relu and add fuse into one kernel


def test_backward_custom_calls_expand_to_kernels():
    """mlx_sdpa_bwd / mlx_layer_norm_bwd (reference custom_vjp backward targets)
    compile: expanded into StableHLO, lowered to GEMMs and fused kernels."""
    from jax_b200 import programs
    plan = pjrt.inspect(programs.sdpa_custom_calls(), 1)
    steps = plan.split("steps:")[1]
    assert steps.count("gemm ") == 5 and "sdpa " in steps
    plan = pjrt.inspect(programs.layer_norm_custom_calls(), 1)
    steps = plan.split("steps:")[1]
    assert "layer_norm " in steps and "_reduce" in steps


def test_portable_artifact_through_jaxlib_python_bindings(monkeypatch):
    """In a Python process with jaxlib (the `jax.jit` case) the plugin turns a
    portable artifact into text through jaxlib's own bindings, under the GIL:
    jax._src.interpreters.mlir.make_ir_context() and
    jaxlib.mlir._mlir_libs._stablehlo.deserialize_portable_artifact(ctx, code).
    Stub modules stand in for jaxlib here: the stub deserializer hands back the
    StableHLO text of the LayerNorm program for one artifact and raises for
    another, which the plugin reports as INVALID_ARGUMENT with the message."""
    import sys
    import types
    text = programs.layer_norm(64, 256)
    artifact = b"ML\xefR\x00vhlo-portable-artifact-1"
    seen = {}

    class Module:
        def __init__(self, s):
            self.s = s

        def __str__(self):
            return self.s

    def make_ir_context():
        seen["ctx"] = seen.get("ctx", 0) + 1
        return object()

    def deserialize_portable_artifact(ctx, code):
        seen["code"] = bytes(code)
        if code == artifact:
            return Module(text)
        raise ValueError("unsupported VHLO version")

    mods = {}
    for name in ("jax", "jax._src", "jax._src.interpreters", "jaxlib", "jaxlib.mlir",
                 "jaxlib.mlir._mlir_libs"):
        mods[name] = types.ModuleType(name)
    mods["jax._src.interpreters.mlir"] = types.ModuleType("jax._src.interpreters.mlir")
    mods["jax._src.interpreters.mlir"].make_ir_context = make_ir_context
    mods["jaxlib.mlir._mlir_libs._stablehlo"] = types.ModuleType("jaxlib.mlir._mlir_libs._stablehlo")
    mods["jaxlib.mlir._mlir_libs._stablehlo"].deserialize_portable_artifact = deserialize_portable_artifact
    for name, m in mods.items():
        monkeypatch.setitem(sys.modules, name, m)
    graph = pjrt.inspect(artifact, 0)
    assert "fused_layer_norm" in graph and seen["code"] == artifact and seen["ctx"] == 1
    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.inspect(b"ML\xefR\x00other", 0)
    assert e.value.code == 3 and "unsupported VHLO version" in str(e.value)


def _stub_jax(monkeypatch):
    """Stand-ins for the parts of jax that plugin.initialize() touches, which
    record what the plugin registers."""
    import sys
    import types
    rec = {"plugins": [], "lowerings": [], "calls": []}

    class Primitive:
        def __init__(self, name):
            self.name, self.multiple_results = name, False

        def def_abstract_eval(self, f):
            self.abstract = f

        def def_impl(self, f):
            self.impl = f

    class ShapedArray:
        def __init__(self, shape, dtype):
            self.shape, self.dtype = shape, dtype

    class Result:
        def __init__(self, n):
            self.results = [f"r{i}" for i in range(n)]

    def custom_call(call_target_name, result_types, operands, backend_config):
        rec["calls"].append((call_target_name, list(result_types), list(operands), backend_config))
        return Result(len(result_types))

    mods = {n: types.ModuleType(n) for n in ("jax", "jax._src", "jax._src.interpreters")}
    core = mods["jax._src.core"] = types.ModuleType("jax._src.core")
    core.Primitive, core.ShapedArray = Primitive, ShapedArray
    xb = mods["jax._src.xla_bridge"] = types.ModuleType("jax._src.xla_bridge")
    xb.register_plugin = lambda name, library_path=None: rec["plugins"].append((name, library_path))
    mlir = mods["jax._src.interpreters.mlir"] = types.ModuleType("jax._src.interpreters.mlir")
    mlir.register_lowering = lambda prim, fn, platform=None: rec["lowerings"].append((prim, fn, platform))
    mlir.aval_to_ir_type = lambda aval: f"type{tuple(aval.shape)}"
    mlir.custom_call = custom_call
    mlir.lower_fun = lambda fn, multiple_results: ("lower_fun", fn, multiple_results)
    mods["jax"]._src = mods["jax._src"]
    mods["jax._src"].core, mods["jax._src"].xla_bridge = core, xb
    mods["jax._src"].interpreters = mods["jax._src.interpreters"]
    mods["jax._src.interpreters"].mlir = mlir
    for n, m in mods.items():
        monkeypatch.setitem(sys.modules, n, m)
    monkeypatch.delitem(sys.modules, "jax_mlx", raising=False)
    return rec


def test_plugin_initialize_registers_platform_and_four_lowerings(monkeypatch):
    """initialize() against stub jax modules: the library is registered as
    platform "b200", and the four fused-op primitives get custom-call
    lowerings for "b200" (plus plain-JAX lowerings elsewhere) whose call
    targets, operands, result types and backend_config JSON are the
    reference's (src/jax_mlx/sdpa.py:97-135, layer_norm.py:86-122)."""
    from jax_b200 import custom_calls, plugin
    rec = _stub_jax(monkeypatch)
    monkeypatch.setattr(custom_calls, "_PRIMS", {})
    plugin.initialize()
    assert rec["plugins"] == [("b200", pjrt.PJRT_LIB)]
    b200 = {p.name: fn for p, fn, plat in rec["lowerings"] if plat == "b200"}
    other = {p.name: fn for p, fn, plat in rec["lowerings"] if plat is None}
    assert sorted(b200) == sorted(other) == sorted(custom_calls.TARGETS)
    assert other["mlx_sdpa_bwd"][2] is True and other["mlx_sdpa"][2] is False

    class Aval:
        def __init__(self, *shape):
            self.shape, self.dtype = shape, "float32"

    class Ctx:
        def __init__(self, n, shape):
            self.avals_out = [Aval(*shape)] * n

    qkv = (2, 128, 2, 64)
    assert b200["mlx_sdpa"](Ctx(1, qkv), "q", "k", "v", scale=0.125) == ["r0"]
    assert b200["mlx_sdpa_bwd"](Ctx(3, qkv), "q", "k", "v", "g", scale=0.125) == ["r0", "r1", "r2"]
    assert b200["mlx_layer_norm"](Ctx(1, (8, 512)), "x", "w", "b", eps=1e-05) == ["r0"]
    b200["mlx_layer_norm_bwd"](Ctx(3, (8, 512)), "x", "w", "b", "dy", eps=1e-05)
    assert rec["calls"] == [
        ("mlx_sdpa", ["type(2, 128, 2, 64)"], ["q", "k", "v"], '{"scale": 0.125}'),
        ("mlx_sdpa_bwd", ["type(2, 128, 2, 64)"] * 3, ["q", "k", "v", "g"], '{"scale": 0.125}'),
        ("mlx_layer_norm", ["type(8, 512)"], ["x", "w", "b"], '{"eps": 1e-05}'),
        ("mlx_layer_norm_bwd", ["type(8, 512)"] * 3, ["x", "w", "b", "dy"], '{"eps": 1e-05}'),
    ]
    prims = custom_calls.primitives()
    assert prims["mlx_sdpa_bwd"].multiple_results and not prims["mlx_sdpa"].multiple_results
    out = prims["mlx_sdpa"].abstract(Aval(*qkv), Aval(*qkv), Aval(*qkv), scale=0.125)
    assert out.shape == qkv


def test_package_declares_jax_plugins_entry_point():
    """pyproject.toml declares the entry point JAX scans (jax_plugins), and it
    names a module with initialize()."""
    import importlib
    import tomllib
    with open(os.path.join(ROOT, "jax-mlx-plugin_b200", "pyproject.toml"), "rb") as f:
        meta = tomllib.load(f)
    eps = meta["project"]["entry-points"]["jax_plugins"]
    assert eps == {"b200": "jax_b200.plugin"}
    mod = importlib.import_module(eps["b200"])
    assert callable(mod.initialize) and mod.PLATFORM == "b200"


def test_row_reduction_through_a_reshape_loads_each_vector_once():
    """A row reduction over a reshape that keeps the innermost dim ([4, 8, 64]
    bf16 logits seen as [32, 64] rows) plus a broadcast bias: each vector group
    of the logits is one 16-byte load, and the bias column is the row position
    itself, with no integer division or remainder inside the row loop."""
    from jax_b200.hlo import Builder
    b = Builder("row_reduce_through_reshape")
    x = b.param((4, 8, 64), "bf16")
    bias = b.param((64,), "bf16")
    y = b.reshape(x + b.broadcast_in_dim(bias, (4, 8, 64), [2]), (32, 64))
    m = b.max(b.convert(y, "f32"), [1])
    source = pjrt.inspect(b.module([m]), 2)
    body = source[source.index("for (int r = "):source.index("for (int off = 16")]
    # one vector load of the logits and one of the bias per group of 8
    assert body.count("__ldg(reinterpret_cast<const uint4*>(") == 2, body
    assert "% 64" not in body and "/ 64" not in body, body


def test_gemm_k_splits_on_sm_pairs():
    """The split-K plan of the two-SM GEMM, read through the workspace query
    (host logic only: no kernel runs).  With fewer 256 x 256 tiles than the 74
    SM pairs of a B200, K is split so that about one unit lands on each pair
    (two when one would leave more than a tenth of the pairs idle), and the
    workspace holds splits x M x N f32 partials; with enough tiles nothing is
    split."""
    lib = kernels.lib()
    f = lib.b200_gemm_workspace_bytes
    f.restype = C.c_int64
    f.argtypes = [C.c_void_p] * 4 + [C.c_int64] * 11 + [C.c_float, C.c_int, C.c_int, C.c_int,
                                                        C.c_void_p]
    fake = 1 << 20  # 16-byte aligned stand-in addresses: the query dereferences nothing

    def splits(M, N, K, a_t):
        sAm, sAk = (1, M) if a_t else (K, 1)
        ws = f(fake, fake, fake, None, 1, M, N, K, M * K, sAm, sAk, K * N, N, 1, N, 1.0,
               kernels.DT_BF16, kernels.DT_BF16, 0, None)
        assert ws >= 0 and ws % (4 * M * N) == 0, ws
        return ws // (4 * M * N)
    # the transformer's weight gradients (activations transposed, K = 16384 tokens)
    assert splits(512, 512, 16384, True) == 18    # 4 tiles x 18 = 72 units
    assert splits(2048, 512, 16384, True) == 9    # 16 tiles: 64 units idle 14%, so 144
    assert splits(512, 2048, 16384, True) == 9
    assert splits(1024, 1024, 1024, False) == 4   # K = 16 blocks: at least 4 per unit
    # 128 and 1024 tiles: whole tiles, no partials
    assert splits(16384, 512, 512, False) == 0
    assert splits(8192, 8192, 8192, False) == 0
