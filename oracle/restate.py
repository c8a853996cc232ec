"""Test infrastructure -- closed-form CPU restatements of the reference's math.

float64 numpy, used to pin the StableHLO programs (and the interpreter in
hlo_interp.py) and as the timed CPU baseline's core.  Each function names the
reference code whose arithmetic it restates.  Not imported by the product.
"""
from __future__ import annotations

import numpy as np

NEG_FILL_F32 = -0.7 * float(np.finfo(np.float32).max)


def sdpa_ref(q, k, v, scale=None, causal=False):
    """softmax(Q K^T * scale [+ causal fill]) V in layout (B, T, N, H).

    Follows reference src/jax_mlx/sdpa.py:19-31 (_mlx_sdpa_impl: transpose to
    BNTH, matmul, * scale, softmax over keys, matmul, transpose back).  The
    causal branch applies the fill JAX's dot_product_attention uses for masked
    logits (-0.7 * finfo(f32).max where key > query), which that reference
    function does not have (its monkey patch falls back to stock JAX for
    is_causal, src/jax_mlx/sdpa.py:214-225)."""
    q, k, v = (np.asarray(a, dtype=np.float64) for a in (q, k, v))
    H = q.shape[-1]
    if scale is None:
        scale = 1.0 / np.sqrt(H)
    qb, kb, vb = (np.transpose(a, (0, 2, 1, 3)) for a in (q, k, v))
    logits = qb @ np.swapaxes(kb, -1, -2) * scale
    if causal:
        T, S = logits.shape[-2:]
        mask = np.tril(np.ones((T, S), dtype=bool))
        logits = np.where(mask, logits, NEG_FILL_F32)
    logits = logits - logits.max(-1, keepdims=True)
    w = np.exp(logits)
    w /= w.sum(-1, keepdims=True)
    return np.transpose(w @ vb, (0, 2, 1, 3))


def sdpa_bwd_ref(q, k, v, g, scale, causal=False, probs_bf16=False, o=None):
    """dQ, dK, dV of softmax(Q K^T scale [+ causal fill]) V, layout (B, T, N, H).

    Follows reference src/jax_mlx/sdpa.py:65-87 (_mlx_sdpa_bwd_impl): weights =
    softmax(logits), dv = weights^T g, d_weights = g v^T, d_scores = weights *
    (d_weights - sum(d_weights * weights, -1)) * scale, dq = d_scores k,
    dk = d_scores^T q.  `causal` fills logits of keys after the query with
    -0.7 * finfo(f32).max first, as sdpa_ref does (their weights are 0).
    `probs_bf16` rounds the weights to bf16 where jax.nn.dot_product_attention
    on bf16 operands does (``probs.astype(value.dtype)``), i.e. in dv; the
    softmax backward keeps them exact.  `o` (B, T, N, H), when given, replaces
    the row term sum(d_weights * weights) by sum(g * o) -- the same value
    when o is the exact output -- as flash-style backward kernels compute it
    from the forward's stored (rounded) output."""
    q, k, v, g = (np.transpose(np.asarray(a, dtype=np.float64), (0, 2, 1, 3)) for a in (q, k, v, g))
    logits = q @ np.swapaxes(k, -1, -2) * scale
    if causal:
        T, S = logits.shape[-2:]
        logits = np.where(np.tril(np.ones((T, S), bool)), logits, -0.7 * np.finfo(np.float32).max)
    w = np.exp(logits - logits.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    wv = w
    if probs_bf16:
        from .hlo_interp import bf16_round
        wv = bf16_round(w.astype(np.float32)).astype(np.float64)
    dv = np.swapaxes(wv, -1, -2) @ g
    dw = g @ np.swapaxes(v, -1, -2)
    if o is None:
        rowterm = (dw * w).sum(-1, keepdims=True)
    else:
        rowterm = (g * np.transpose(np.asarray(o, dtype=np.float64), (0, 2, 1, 3))).sum(-1)[..., None]
    ds = w * (dw - rowterm) * scale
    dq = ds @ k
    dk = np.swapaxes(ds, -1, -2) @ q
    t = lambda a: np.transpose(a, (0, 2, 1, 3))
    return t(dq), t(dk), t(dv)


def layer_norm_ref(x, residual, gamma, beta, eps=1e-5):
    """LayerNorm over the last axis of (x + residual), then * gamma + beta.

    Follows reference src/jax_mlx/layer_norm.py:20-25 (_mlx_layer_norm_impl:
    mean, var = mean((x-mean)^2), (x - mean) * rsqrt(var + eps) * w + b); the
    residual add is the config's (the reference fuses none)."""
    h = np.asarray(x, dtype=np.float64)
    if residual is not None:
        h = h + np.asarray(residual, dtype=np.float64)
    mean = h.mean(-1, keepdims=True)
    var = ((h - mean) ** 2).mean(-1, keepdims=True)
    y = (h - mean) / np.sqrt(var + eps)
    if gamma is not None:
        y = y * np.asarray(gamma, dtype=np.float64)
    if beta is not None:
        y = y + np.asarray(beta, dtype=np.float64)
    return y


def layer_norm_bwd_ref(x, gamma, dy, eps=1e-5):
    """dx, dgamma, dbeta of LayerNorm; reference src/jax_mlx/layer_norm.py:59-76."""
    x = np.asarray(x, dtype=np.float64)
    dy = np.asarray(dy, dtype=np.float64)
    g = np.ones(x.shape[-1]) if gamma is None else np.asarray(gamma, dtype=np.float64)
    n = x.shape[-1]
    mean = x.mean(-1, keepdims=True)
    var = ((x - mean) ** 2).mean(-1, keepdims=True)
    rstd = 1.0 / np.sqrt(var + eps)
    xhat = (x - mean) * rstd
    gdy = dy * g
    dx = rstd * (gdy - gdy.mean(-1, keepdims=True) - xhat * (gdy * xhat).mean(-1, keepdims=True))
    dgamma = (dy * xhat).reshape(-1, n).sum(0)
    dbeta = dy.reshape(-1, n).sum(0)
    return dx, dgamma, dbeta


def mlp_step_ref(params, x, labels, lr=1e-2):
    """One SGD step of a ReLU MLP with mean softmax cross-entropy (config 3).

    params: [W1, b1, ..., WL, bL].  Returns (loss, new_params).  Backprop by
    hand in float64: the value jax.value_and_grad of the jitted step computes."""
    x = np.asarray(x, dtype=np.float64)
    Ws = [np.asarray(p, dtype=np.float64) for p in params[0::2]]
    bs = [np.asarray(p, dtype=np.float64) for p in params[1::2]]
    acts, pre = [x], []
    h = x
    for i, (W, b) in enumerate(zip(Ws, bs)):
        z = h @ W + b
        pre.append(z)
        h = np.maximum(z, 0.0) if i < len(Ws) - 1 else z
        acts.append(h)
    logits = h
    n, c = logits.shape
    m = logits.max(1, keepdims=True)
    lse = np.log(np.exp(logits - m).sum(1, keepdims=True)) + m
    logp = logits - lse
    onehot = np.eye(c)[np.asarray(labels)]
    loss = -(onehot * logp).sum() / n
    g = (np.exp(logp) - onehot) / n
    new = [None] * len(params)
    for i in reversed(range(len(Ws))):
        if i < len(Ws) - 1:
            g = g * (pre[i] > 0)
        gW = acts[i].T @ g
        gb = g.sum(0)
        new[2 * i] = Ws[i] - lr * gW
        new[2 * i + 1] = bs[i] - lr * gb
        g = g @ Ws[i].T
    return loss, new


def maxpool2x2_ref(x):
    """2x2 / stride 2 max pooling of an NHWC array (reference tests/test_exhaustive.py:599)."""
    n, h, w, c = x.shape
    return np.asarray(x).reshape(n, h // 2, 2, w // 2, 2, c).max(axis=(2, 4))


def maxpool2x2_grad_ref(x):
    """Gradient of sum(maxpool2x2(x)) (reference tests/test_exhaustive.py:603): 1 at
    the first maximum of each window in row-major window order, else 0."""
    x = np.asarray(x)
    n, h, w, c = x.shape
    win = x.reshape(n, h // 2, 2, w // 2, 2, c).transpose(0, 1, 3, 5, 2, 4).reshape(n, h // 2, w // 2, c, 4)
    first = win.argmax(-1)
    g = np.zeros((n, h // 2, w // 2, c, 4))
    np.put_along_axis(g, first[..., None], 1.0, axis=-1)
    return g.reshape(n, h // 2, w // 2, c, 2, 2).transpose(0, 1, 4, 2, 5, 3).reshape(n, h, w, c)
