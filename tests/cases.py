"""Known-answer StableHLO programs for the golden fixtures (tests/golden).

Each case: (name, program text, inputs, expected output).  The programs are
the ops the reference's parity script exercises on these inputs
(tests/test_exhaustive.py:463-768 in the reference); the expected outputs come
from tests/golden/reference_cases.npz.
"""
import math
import os

import numpy as np

from jax_b200.hlo import Builder

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.npz")


def golden():
    return dict(np.load(GOLDEN))


def _prog(build):
    b = Builder("jit_case")
    outs = build(b)
    return b.module(outs if isinstance(outs, (list, tuple)) else [outs])


def cases():
    d = golden()
    out = []

    def add(name, build, inputs, expected):
        out.append((name, _prog(build), inputs, expected))

    add("conv_same_ones", lambda b: b.conv(b.param((1, 8, 8, 3)), b.param((3, 3, 3, 16)),
                                            padding=((1, 1), (1, 1))),
        [d["conv_in"], d["conv_w"]], d["conv_out"])
    for kind in ("max", "min", "sum"):
        k = {"sum": "add"}.get(kind, kind)
        add(f"pool_{kind}", lambda b, k=k: b.reduce_window(b.param((2, 4, 4, 3)), k, (1, 2, 2, 1), (1, 2, 2, 1)),
            [d["pool_in"]], d[f"pool_{kind}"])
    add("pool_overlap_max", lambda b: b.reduce_window(b.param((2, 4, 4, 3)), "max", (1, 3, 3, 1), (1, 1, 1, 1)),
        [d["pool_in"]], d["pool_overlap_max"])
    add("pool_avg", lambda b: b.reduce_window(b.param((2, 4, 4, 3)), "add", (1, 2, 2, 1), (1, 2, 2, 1)) / 4.0,
        [d["pool_in"]], d["pool_avg"])

    def pool_grad(b):
        x = b.param((2, 4, 4, 3))
        y = b.max_pool(x, (1, 2, 2, 1), (1, 2, 2, 1))
        loss = b.sum(y, [0, 1, 2, 3])
        return b.grad(loss, [x])[0]
    add("pool_max_grad", pool_grad, [d["pool_in"]], d["pool_max_grad"])
    add("matmul", lambda b: b.matmul(b.param((2, 2)), b.param((2, 2))), [d["mat"], d["mat"]], d["matmul"])
    add("dot_general_ones", lambda b: b.dot_general(b.param((2, 3)), b.param((3, 4)), ([1], [0])),
        [np.ones((2, 3), np.float32), np.ones((3, 4), np.float32)], d["dot_general_ones"])
    add("relu", lambda b: b.maximum(b.param((4,)), 0.0), [d["nn_in"]], d["relu"])
    add("sigmoid", lambda b: b.logistic(b.param((4,))), [d["nn_in"]], d["sigmoid"])

    def softmax(b):
        x = b.param((5,))
        e = b.exp(x - b.max(x, [0], keepdims=True))
        return e / b.sum(e, [0], keepdims=True)
    add("softmax_ones5", softmax, [np.ones(5, np.float32)], d["softmax_ones5"])

    def log_softmax(b):
        x = b.param((5,))
        s = x - b.max(x, [0], keepdims=True)
        return s - b.log(b.sum(b.exp(s), [0], keepdims=True))
    add("log_softmax_ones5", log_softmax, [np.ones(5, np.float32)], d["log_softmax_ones5"])

    def gelu(b):
        x = b.param((4,))
        inner = (x + x * x * x * 0.044715) * math.sqrt(2.0 / math.pi)
        return x * 0.5 * (b.tanh(inner) + 1.0)
    add("gelu_tanh", gelu, [d["nn_in"]], d["gelu_tanh"])

    def grad_sq(b):
        x = b.param((3,))
        return b.grad(b.sum(x * x, [0]), [x])[0]
    add("grad_sum_sq", grad_sq, [d["grad_in"]], d["grad_sum_sq"])
    add("pad_edge", lambda b: b.pad(b.param((3, 3)), 0.0, (1, 1), (1, 1), (0, 0)),
        [np.ones((3, 3), np.float32)], d["pad_edge"])
    add("pad_interior", lambda b: b.pad(b.param((2, 2)), 0.0, (0, 0), (0, 0), (1, 1)),
        [d["mat"]], d["pad_interior"])
    return out
