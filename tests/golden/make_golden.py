"""Generate tests/golden/reference_cases.npz: known-answer fixtures for the hot path.

The reference keeps no stored outputs; its parity script compares live JAX-CPU
against the plugin on fixed inputs (reference tests/test_exhaustive.py).  This
script takes those exact inputs -- the same constructors and seeds -- and
computes each expected output by an independent closed form (counting, numpy
reshape-max, the analytic derivative), not by the oracle interpreter or the
plugin, so the fixtures can check both.

  conv      test_exhaustive.py:578-580  ones(1,8,8,3) * ones(3,3,3,16), SAME, NHWC/HWIO
  pool      test_exhaustive.py:597-607  RandomState(42).randn(2,4,4,3) f32, 2x2/2 max/min/sum,
                                        3x3/1 max, grad of sum(maxpool), avg pool
  dot       test_exhaustive.py:463-469  [[1,2],[3,4]] matmul / einsum / dot
  dot_gen   test_exhaustive.py:631      ones(2,3) . ones(3,4)
  nn        test_exhaustive.py:747-753  relu / sigmoid / softmax(ones 5) / log_softmax / gelu(tanh)
  grad      test_exhaustive.py:765-766  grad(sum(x**2)) at a = [1, 2, 3]
  pad       test_exhaustive.py:612-613  pad ones(3,3) by 1; interior pad of [[1,2],[3,4]]

Run:  python tests/golden/make_golden.py
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    out = {}
    # conv of ones: each output = C_in * (# valid taps of the 3x3 window)
    rows = np.array([2, 3, 3, 3, 3, 3, 3, 2], dtype=np.float64)
    taps = np.outer(rows, rows)
    out["conv_in"] = np.ones((1, 8, 8, 3), np.float32)
    out["conv_w"] = np.ones((3, 3, 3, 16), np.float32)
    out["conv_out"] = np.broadcast_to((3 * taps)[None, :, :, None], (1, 8, 8, 16)).astype(np.float32)

    x = np.random.RandomState(42).randn(2, 4, 4, 3).astype(np.float32)
    out["pool_in"] = x
    w = x.reshape(2, 2, 2, 2, 2, 3)
    out["pool_max"] = w.max(axis=(2, 4))
    out["pool_min"] = w.min(axis=(2, 4))
    out["pool_sum"] = w.astype(np.float64).sum(axis=(2, 4)).astype(np.float32)
    out["pool_avg"] = (w.astype(np.float64).sum(axis=(2, 4)) / 4.0).astype(np.float32)
    ov = np.full((2, 2, 2, 3), -np.inf, np.float32)
    for i in range(2):
        for j in range(2):
            ov[:, i, j, :] = x[:, i:i + 3, j:j + 3, :].max(axis=(1, 2))
    out["pool_overlap_max"] = ov
    # grad of sum(maxpool): 1 at the first (row-major) maximum of each window
    g = np.zeros_like(x)
    for n in range(2):
        for i in range(2):
            for j in range(2):
                for c in range(3):
                    win = x[n, 2 * i:2 * i + 2, 2 * j:2 * j + 2, c]
                    k = int(np.argmax(win.reshape(-1)))
                    g[n, 2 * i + k // 2, 2 * j + k % 2, c] = 1.0
    out["pool_max_grad"] = g

    mat = np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)
    out["mat"] = mat
    out["matmul"] = np.array([[7.0, 10.0], [15.0, 22.0]], np.float32)
    out["dot_general_ones"] = np.full((2, 4), 3.0, np.float32)

    nn_in = np.array([-1.0, 0.0, 1.0, 2.0], np.float32)
    out["nn_in"] = nn_in
    out["relu"] = np.array([0.0, 0.0, 1.0, 2.0], np.float32)
    xd = nn_in.astype(np.float64)
    out["sigmoid"] = (1.0 / (1.0 + np.exp(-xd))).astype(np.float32)
    out["softmax_ones5"] = np.full(5, 0.2, np.float32)
    out["log_softmax_ones5"] = np.full(5, -np.log(5.0), np.float32)
    out["gelu_tanh"] = (0.5 * xd * (1 + np.tanh(np.sqrt(2 / np.pi) * (xd + 0.044715 * xd ** 3)))).astype(np.float32)

    a = np.array([1.0, 2.0, 3.0], np.float32)
    out["grad_in"] = a
    out["grad_sum_sq"] = 2 * a
    out["pad_edge"] = np.pad(np.ones((3, 3), np.float32), 1)
    pi = np.zeros((3, 3), np.float32)
    pi[::2, ::2] = [[1.0, 2.0], [3.0, 4.0]]
    out["pad_interior"] = pi
    np.savez_compressed(os.path.join(HERE, "reference_cases.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
