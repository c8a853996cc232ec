"""CPU: the host compile pipeline (parser, passes, planner, code generator and
the parallel NVRTC compile) under AddressSanitizer and UBSan.

`make sanitize` builds the host library with both sanitizers into
jax-mlx-plugin_b200/_build_san (never into lib/); a fresh interpreter with the
sanitizer runtimes preloaded runs b200_pjrt_inspect over every program the
tests use -- the golden cases, the five configurations' programs, the
backward custom calls, and inputs that fail (a parse error, a bytecode
artifact with no MLIR C API) -- at each inspection level.  Any heap error,
use after free or undefined behaviour aborts that process."""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "jax-mlx-plugin_b200")
SAN_LIB = os.path.join(PKG, "_build_san", "libb200_pjrt_san.so")

_PROBE = r"""
import ctypes as C, sys
sys.path[:0] = [{root!r}, {pkg!r}, {tests!r}]
lib = C.CDLL({lib!r})
lib.b200_pjrt_inspect.argtypes = [C.c_char_p, C.c_size_t, C.c_int, C.POINTER(C.c_void_p)]
lib.b200_pjrt_free.argtypes = [C.c_void_p]
from cases import cases
from jax_b200 import programs
tr = programs.transformer_step(batch=2, seq=32, layers=2, d=64, heads=2, ffn=128, vocab=96)
progs = [(t, (0, 1, 2)) for _, t, *_ in cases()]
progs += [(t, (0, 1, 2)) for t in (
    programs.sdpa(), programs.sdpa(2, 256, 4, 64, causal=False), programs.layer_norm(),
    programs.mlp_step(), programs.cnn_step(), programs.mlp_step(batch=512, num_replicas=2),
    programs.logits_cross_entropy(240, 500), programs.softmax_then_transposed_sum(),
    programs.sdpa_custom_calls(), programs.layer_norm_custom_calls(),
    "module {{ func.func @main(%a: tensor<4xf32>) -> tensor<4xf32> {{ %0 = stablehlo.add %a, : "
    "tensor<4xf32> return %0 : tensor<4xf32> }} }}",
    b"ML\xefR\x00\x01")]
progs.append((tr, (0, 1, 2, 3)))
calls = failed = 0
for t, levels in progs:
    b = t if isinstance(t, bytes) else t.encode()
    for what in levels:
        out = C.c_void_p()
        rc = lib.b200_pjrt_inspect(b, len(b), what, C.byref(out))
        lib.b200_pjrt_free(out)
        calls += 1
        failed += rc != 0
print("calls", calls, "errors", failed)
"""


def _runtime(name):
    cxx = os.environ.get("SAN_CXX", "g++")
    if not shutil.which(cxx):
        return None
    p = subprocess.run([cxx, f"-print-file-name={name}"], capture_output=True, text=True).stdout.strip()
    return p if os.path.isabs(p) and os.path.exists(p) else None


def test_compile_pipeline_is_clean_under_asan_and_ubsan():
    asan, ubsan = _runtime("libasan.so"), _runtime("libubsan.so")
    if not (asan and ubsan):
        pytest.skip("no AddressSanitizer / UBSan runtime for the host compiler")
    r = subprocess.run(["make", "-j8", "sanitize"], cwd=os.path.join(PKG, "csrc"), capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    env = dict(os.environ, LD_PRELOAD=f"{asan}:{ubsan}", ASAN_OPTIONS="detect_leaks=0",
               UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1")
    code = _PROBE.format(root=ROOT, pkg=PKG, tests=os.path.join(ROOT, "tests"), lib=SAN_LIB)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout[-1000:], r.stderr[-4000:])
    assert "runtime error" not in r.stderr and "AddressSanitizer" not in r.stderr, r.stderr[-4000:]
    n_calls, n_err = int(r.stdout.split()[1]), int(r.stdout.split()[3])
    # every golden case and config program compiles; the parse error and the
    # bytecode artifact fail at each of their 3 levels
    assert n_calls >= 90 and n_err == 6, r.stdout


_FUZZ = r"""
import ctypes as C, random, re, sys
sys.path[:0] = [{root!r}, {pkg!r}, {tests!r}]
lib = C.CDLL({lib!r})
lib.b200_pjrt_inspect.argtypes = [C.c_char_p, C.c_size_t, C.c_int, C.POINTER(C.c_void_p)]
lib.b200_pjrt_free.argtypes = [C.c_void_p]
from cases import cases
from jax_b200 import programs
seeds = [t for _, t, *_ in cases()] + [programs.mlp_step(), programs.sdpa(), programs.layer_norm(),
                                        programs.cnn_step()]
pieces = list("{{}}()[]<>%:,=x0123456789-.\"@ \n") + ["tensor<", "stablehlo.", "dense<", "f32", "i32",
                                                       "bf16", "0x", "1e40"]
number = re.compile(r"(?<![%\w.#])\d+(?![\w.])")
runs = accepted = 0
for seed in {seeds!r}:
    rng = random.Random(seed)
    for _ in range({iters}):
        t = rng.choice(seeds)
        k = rng.randrange(5)
        if k == 4:  # an integer literal (a dimension, an attribute value) replaced
            spans = [m.span() for m in number.finditer(t)]
            a, e = rng.choice(spans)
            t = t[:a] + str(rng.choice([0, 1, 2, 3, 5, 8, 16, 100])) + t[e:]
        elif k == 0:
            t = t[:rng.randrange(len(t))]
        elif k == 1:
            for _ in range(rng.randint(1, 5)):
                i = rng.randrange(len(t))
                t = t[:i] + rng.choice(pieces) + t[i + 1:]
        elif k == 2:
            i = rng.randrange(len(t))
            t = t[:i] + t[min(len(t), i + rng.randint(1, 40)):]
        else:
            i, j = rng.randrange(len(t)), rng.randrange(len(t))
            t = t[:i] + t[j:j + rng.randint(1, 60)] + t[i:]
        b = t.encode()
        out = C.c_void_p()
        rc = lib.b200_pjrt_inspect(b, len(b), rng.choice((0, 1, 2)), C.byref(out))
        lib.b200_pjrt_free(out)
        runs += 1
        accepted += rc == 0
print("runs", runs, "accepted", accepted)
"""


def test_mutated_programs_fail_cleanly_under_asan_and_ubsan():
    """Seeded mutations of valid programs (truncations, replaced characters,
    cut and duplicated spans, replaced integer literals, i.e. wrong shapes and
    attribute values in valid syntax) through the whole compile pipeline: each
    is either compiled or rejected with an error, never read out of range."""
    asan, ubsan = _runtime("libasan.so"), _runtime("libubsan.so")
    if not (asan and ubsan):
        pytest.skip("no AddressSanitizer / UBSan runtime for the host compiler")
    r = subprocess.run(["make", "-j8", "sanitize"], cwd=os.path.join(PKG, "csrc"), capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    env = dict(os.environ, LD_PRELOAD=f"{asan}:{ubsan}", ASAN_OPTIONS="detect_leaks=0",
               UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1")
    code = _FUZZ.format(root=ROOT, pkg=PKG, tests=os.path.join(ROOT, "tests"), lib=SAN_LIB,
                        seeds=[2, 4], iters=800)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.stdout[-1000:], r.stderr[-4000:])
    assert "runtime error" not in r.stderr and "AddressSanitizer" not in r.stderr, r.stderr[-4000:]
    assert r.stdout.split()[:2] == ["runs", "1600"], r.stdout
