"""CPU stand-in for "the same jitted program on JAX's CPU backend": the five
BASELINE configurations restated in torch on the host cores.

TEST / MEASUREMENT INFRASTRUCTURE ONLY.  Nothing in the product imports this
file.  It serves `bench.py` (the `cpu_baseline` leg and `--impl reference`,
timed on the host's cores) and CPU tests that check it against the numpy
interpreter (`oracle/hlo_interp.py`).  JAX/jaxlib are not installed on this
pool, and the reference plugin (MLX/Metal, macOS only) cannot run here, so the
reference arm times this restatement of the reference's arithmetic instead.

Each function follows the program `jax_b200/programs.py` emits for the same
configuration, op for op and in the same dtypes, which in turn follows what
`jax.jit` lowers for the reference's workloads:

* sdpa: reference `src/jax_mlx/sdpa.py:19-31` (the fallback math) with JAX's
  causal fill `where(tril, s, -0.7 * f32max)` before an f32 softmax;
* residual + LayerNorm: `src/jax_mlx/layer_norm.py:20-25` after `h = x + r`;
* MLP / CNN / transformer training steps: the BASELINE configurations
  (value_and_grad of mean softmax cross-entropy; SGD, or optax-style Adam with
  f32 moments for the transformer; bf16 parameters and activations with f32
  statistics, logits, softmax and loss, as flax/jax.nn do).
"""
from __future__ import annotations

import math
from typing import List, Sequence

import numpy as np
import torch
import torch.nn.functional as F

F32_MAX = 3.4028234663852886e38


def sdpa(q, k, v, causal=True, scale=None):
    """q, k, v [B, T, N, H] -> [B, T, N, H] (reference sdpa.py:19-31)."""
    B, T, N, H = q.shape
    scale = 1.0 / math.sqrt(H) if scale is None else scale
    s = torch.einsum("btnh,bsnh->bnts", q, k) * scale
    if causal:
        S = k.shape[1]
        tri = torch.ones(T, S, dtype=torch.bool).tril()
        s = torch.where(tri, s, torch.tensor(-0.7 * F32_MAX, dtype=s.dtype))
    p = torch.softmax(s.float(), dim=-1).to(v.dtype)
    return torch.einsum("bnts,bsnh->btnh", p, v)


def residual_layer_norm(x, r, g, b, eps=1e-5):
    """h = x + r; (h - mean) * rsqrt(var + eps) * g + b (layer_norm.py:20-25)."""
    h = x + r
    mean = h.mean(-1, keepdim=True)
    d = h - mean
    var = (d * d).mean(-1, keepdim=True)
    return d * torch.rsqrt(var + eps) * g + b


def _cross_entropy(logits, labels):
    return -(torch.log_softmax(logits, -1).gather(1, labels.long()[:, None])).mean()


def mlp_step(params: Sequence[torch.Tensor], x, labels, lr=1e-2):
    """One SGD step of the ReLU MLP (programs.mlp_step): (loss, new params)."""
    ps = [p.detach().clone().requires_grad_() for p in params]
    h = x
    nl = len(ps) // 2
    for i in range(nl):
        h = h @ ps[2 * i] + ps[2 * i + 1]
        if i < nl - 1:
            h = torch.relu(h)
    loss = _cross_entropy(h, labels)
    grads = torch.autograd.grad(loss, ps)
    with torch.no_grad():
        return loss.detach(), [p - lr * g for p, g in zip(ps, grads)]


def cnn_step(params: Sequence[torch.Tensor], x, labels, lr=1e-2):
    """One SGD step of the NHWC CNN (programs.cnn_step): (loss, new params).
    Kernels are HWIO as in flax; torch's NCHW convolution is fed permuted
    views (the arithmetic is the same convolution)."""
    ps = [p.detach().clone().requires_grad_() for p in params]
    w1, b1, w2, b2, w3, b3, w4, b4 = ps
    h = x.permute(0, 3, 1, 2)
    h = torch.relu(F.conv2d(h, w1.permute(3, 2, 0, 1), b1, padding=1))
    h = F.max_pool2d(h, 2)
    h = torch.relu(F.conv2d(h, w2.permute(3, 2, 0, 1), b2, padding=1))
    h = F.max_pool2d(h, 2)
    h = h.permute(0, 2, 3, 1).reshape(x.shape[0], -1)  # NHWC flatten order
    h = torch.relu(h @ w3 + b3)
    logits = h @ w4 + b4
    loss = _cross_entropy(logits, labels)
    grads = torch.autograd.grad(loss, ps)
    with torch.no_grad():
        return loss.detach(), [p - lr * g for p, g in zip(ps, grads)]


PER_LAYER = ("ln1_g", "ln1_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo",
             "ln2_g", "ln2_b", "w1", "b1", "w2", "b2")


def _ln_bf16(x, g, b, eps=1e-6, f32=torch.float32):
    """flax LayerNorm on bf16 activations: f32 statistics and affine, bf16 out."""
    h = x.to(f32)
    mean = h.mean(-1, keepdim=True)
    d = h - mean
    var = (d * d).mean(-1, keepdim=True)
    return (d * torch.rsqrt(var + eps) * g.to(f32) + b.to(f32)).to(x.dtype)


def _gelu_tanh(x):
    inner = (x + x * x * x * 0.044715) * math.sqrt(2.0 / math.pi)
    return x * ((torch.tanh(inner) + 1.0) * 0.5)


def _attention(q, k, v, f32=torch.float32):
    B, T, N, H = q.shape
    s = torch.einsum("btnh,bsnh->bnts", q.to(f32), k.to(f32)) * (1.0 / math.sqrt(H))
    tri = torch.ones(T, T, dtype=torch.bool).tril()
    s = torch.where(tri, s, torch.tensor(-0.7 * F32_MAX, dtype=f32))
    p = torch.softmax(s, -1).to(v.dtype)
    return torch.einsum("bnts,bsnh->btnh", p, v)


def transformer_loss(P: dict, tokens, targets, layers: int, f32=torch.float32):
    """Mean next-token cross-entropy (f32) of the pre-LN causal encoder.  `f32`
    is the type of the program's f32 values (float64 to evaluate the program
    with no rounding at all, given float64 parameters)."""
    B, T = tokens.shape
    x = P["tok_emb"][tokens.long()] + P["pos_emb"][None]
    for i in range(layers):
        L = lambda n: P[f"l{i}.{n}"]
        y = _ln_bf16(x, L("ln1_g"), L("ln1_b"), f32=f32)
        q, k, v = (torch.einsum("btd,dnh->btnh", y, L(w)) + L(bb)
                   for w, bb in (("wq", "bq"), ("wk", "bk"), ("wv", "bv")))
        att = _attention(q, k, v, f32)
        x = x + (torch.einsum("btnh,nhd->btd", att, L("wo")) + L("bo"))
        y = _ln_bf16(x, L("ln2_g"), L("ln2_b"), f32=f32)
        f = _gelu_tanh(y @ L("w1") + L("b1"))
        x = x + (f @ L("w2") + L("b2"))
    y = _ln_bf16(x, P["lnf_g"], P["lnf_b"], f32=f32)
    logits = (y @ P["w_head"] + P["b_head"]).reshape(B * T, -1).to(f32)
    return _cross_entropy(logits, targets.reshape(-1))


def transformer_grads(names: List[str], params, tokens, targets, layers=6, f32=torch.float32):
    """value_and_grad of transformer_loss: (loss, gradients in the parameters' type)."""
    ps = [p.detach().requires_grad_() for p in params]
    loss = transformer_loss(dict(zip(names, ps)), tokens, targets, layers, f32)
    grads = torch.autograd.grad(loss, ps)
    return loss.detach(), grads


def adam_update(params, ms, vs, grads, count: int, lr=3e-4, b1=0.9, b2=0.999, eps=1e-8):
    """optax-style Adam with f32 moments on bf16 parameters (programs.transformer_step):
    returns (new params, new m, new v, count + 1)."""
    cnt = count + 1
    bc1, bc2 = 1.0 - b1 ** cnt, 1.0 - b2 ** cnt
    new_p, new_m, new_v = [], [], []
    with torch.no_grad():
        for p, m, v, g in zip(params, ms, vs, grads):
            g32 = g.float()
            m2 = m * b1 + g32 * (1.0 - b1)
            v2 = v * b2 + g32 * g32 * (1.0 - b2)
            upd = (m2 / bc1) / (torch.sqrt(v2 / bc2) + eps)
            new_p.append((p.float() - upd * lr).to(torch.bfloat16))
            new_m.append(m2)
            new_v.append(v2)
    return new_p, new_m, new_v, cnt


def transformer_step(names: List[str], params, ms, vs, count: int, tokens, targets, layers=6,
                     lr=3e-4, b1=0.9, b2=0.999, eps=1e-8):
    """One Adam step (programs.transformer_step): bf16 params, f32 moments.
    Returns (loss, new params, new m, new v, count + 1)."""
    loss, grads = transformer_grads(names, params, tokens, targets, layers)
    return (loss,) + adam_update(params, ms, vs, grads, count, lr, b1, b2, eps)


def transformer_state(shapes, seed=12):
    """N(0, 0.02) bf16 parameters and zero f32 moments for `shapes`
    ([(name, shape)] in argument order)."""
    rng = np.random.default_rng(seed)
    params = [torch.from_numpy((rng.standard_normal(s).astype(np.float32) * np.float32(0.02)))
              .to(torch.bfloat16) for _, s in shapes]
    zeros = [torch.zeros(s, dtype=torch.float32) for _, s in shapes]
    return params, zeros, [z.clone() for z in zeros]
