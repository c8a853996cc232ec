"""The five benchmark programs, as ``jax.jit`` would lower them to StableHLO.

Each builder mirrors the JAX source of its configuration:

* ``sdpa``: ``jax.nn.dot_product_attention(q, k, v, is_causal=True)`` on the
  XLA path -- einsum logits, ``* scale``, ``jnp.where(tril_mask, logits,
  -0.7*finfo.max)``, ``jax.nn.softmax`` in f32, einsum with V.
* ``layer_norm``: ``h = x + r; (h - mean) * rsqrt(var + eps) * gamma + beta``
  with ``jnp.mean`` / ``jnp.square`` (two-pass variance).
* ``mlp_step`` / ``cnn_step``: ``jax.value_and_grad`` of softmax cross-entropy,
  SGD update; with ``num_replicas > 1`` the pmap form whose gradients and loss
  are ``lax.pmean``-ed (``all_reduce`` + divide).
* ``transformer_step``: a pre-LN causal encoder in bf16 (flax-style
  ``DenseGeneral`` q/k/v/out projections, ``jax.nn.dot_product_attention``
  with f32 logits and softmax, tanh GELU, learned positions, untied head),
  f32 next-token cross-entropy, and an Adam update with f32 moments.
"""
from __future__ import annotations

import math
from typing import List, Sequence, Tuple

from .hlo import Builder, V

F32_MAX = 3.4028234663852886e38


def softmax(b: Builder, x: V, axis: int = -1) -> V:
    ax = axis % len(x.shape)
    m = b.stop_gradient(b.max(x, [ax], keepdims=True))
    e = b.exp(x - m)
    return e / b.sum(e, [ax], keepdims=True)


def log_softmax(b: Builder, x: V, axis: int = -1) -> V:
    ax = axis % len(x.shape)
    shifted = x - b.stop_gradient(b.max(x, [ax], keepdims=True))
    lse = b.log(b.sum(b.exp(shifted), [ax], keepdims=True))
    return shifted - lse


def cross_entropy(b: Builder, logits: V, labels: V) -> V:
    """mean over the batch of -sum(one_hot(labels) * log_softmax(logits))."""
    n, c = logits.shape
    logp = log_softmax(b, logits)
    classes = b.iota((n, c), 1, labels.dtype)
    lab = b.broadcast_in_dim(labels, (n, c), [0])
    onehot = b.convert(b.compare(lab, classes, "EQ"), logits.dtype)
    per = b.neg(b.sum(onehot * logp, [1]))
    return b.sum(per, [0]) / float(n)


def logits_cross_entropy(rows=64, cols=5000, dt="f32") -> str:
    """value_and_grad of the mean softmax cross-entropy of logits + bias (the
    language-model head's loss) with respect to both.  Inputs: logits
    [rows, cols], bias [cols] (both `dt`), labels [rows] i32.  Outputs: loss
    (f32), d logits, d bias.  Exercises row-wise reductions and loops over long
    rows."""
    b = Builder("jit_logits_cross_entropy")
    logits, bias = b.param((rows, cols), dt), b.param((cols,), dt)
    labels = b.param((rows,), "i32")
    z = logits + bias
    if dt != "f32":
        z = b.convert(z, "f32")
    loss = cross_entropy(b, z, labels)
    grads = b.grad(loss, [logits, bias])
    return b.module([loss] + grads)


def row_softmax(rows=2400, cols=300) -> str:
    """jax.nn.softmax over the last axis of f32 x [rows, cols] and the row
    log-sum-exp (max + log of the shifted sum)."""
    b = Builder("jit_row_softmax")
    x = b.param((rows, cols))
    m = b.stop_gradient(b.max(x, [1], keepdims=True))
    e = b.exp(x - m)
    s = b.sum(e, [1], keepdims=True)
    return b.module([e / s, b.reshape(m + b.log(s), (rows,))])


def softmax_then_transposed_sum(n=96) -> str:
    """p = softmax(x) over rows; out = sum over the last axis of p^T * x.  The
    second reduction reads p at transposed positions, so it cannot run in the
    same row pass as the softmax."""
    b = Builder("jit_softmax_transposed")
    x = b.param((n, n))
    p = softmax(b, x)
    return b.module([p, b.sum(b.transpose(p, [1, 0]) * x, [1])])


def sdpa(B=8, T=512, N=8, H=64, causal=True, dt="f32") -> str:
    b = Builder("jit_dot_product_attention")
    q, k, v = b.param((B, T, N, H), dt), b.param((B, T, N, H), dt), b.param((B, T, N, H), dt)
    logits = b.dot_general(q, k, ([3], [3]), ([0, 2], [0, 2]))  # [B, N, T, S]
    logits = logits * (1.0 / math.sqrt(H))
    if causal:
        row = b.iota((T, T), 0)
        col = b.iota((T, T), 1)
        tri = b.compare(row + b.constant(0, "i32", (T, T)), col, "GE", "SIGNED")
        ones = b.constant(True, "i1", (T, T))
        zeros = b.constant(False, "i1", (T, T))
        mask = b.select(tri, ones, zeros)
        mask = b.reshape(mask, (1, 1, T, T))
        big_neg = b.constant(-0.7 * F32_MAX, dt, logits.shape)
        logits = b.select(b.broadcast_to(mask, logits.shape), logits, big_neg)
    probs = softmax(b, b.convert(logits, "f32"))
    probs = b.convert(probs, dt)
    enc = b.dot_general(probs, v, ([3], [1]), ([0, 1], [0, 2]))  # [B, N, T, H]
    out = b.transpose(enc, [0, 2, 1, 3])
    return b.module([out])


def layer_norm(rows=4096, cols=1024, eps=1e-5, dt="f32") -> str:
    b = Builder("jit_residual_layer_norm")
    x, r = b.param((rows, cols), dt), b.param((rows, cols), dt)
    gamma, beta = b.param((cols,), dt), b.param((cols,), dt)
    h = x + r
    mean = b.sum(h, [1], keepdims=True) / float(cols)
    d = h - mean
    var = b.sum(d * d, [1], keepdims=True) / float(cols)
    y = d * b.rsqrt(var + eps) * gamma + beta
    return b.module([y])


def _dp_mean(b: Builder, xs: List[V], num_replicas: int) -> List[V]:
    if num_replicas == 1:
        return xs
    groups = [list(range(num_replicas))]
    return [b.all_reduce_sum(x, groups) / float(num_replicas) for x in xs]


def mlp_step(batch=1024, dims=(784, 1024, 1024, 1024, 10), lr=1e-2, num_replicas=1, emit="params") -> str:
    """One SGD step of the 784-1024-1024-1024-10 ReLU MLP.  Inputs: W1,b1,...,W4,b4,
    x [batch, 784] f32, labels [batch] i32.  Outputs: loss, updated params (or the
    gradients themselves with emit="grads")."""
    b = Builder("jit_train_step", num_replicas)
    params = []
    for i in range(len(dims) - 1):
        params.append(b.param((dims[i], dims[i + 1])))
        params.append(b.param((dims[i + 1],)))
    x = b.param((batch, dims[0]))
    labels = b.param((batch,), "i32")
    h = x
    nl = len(dims) - 1
    for i in range(nl):
        h = b.matmul(h, params[2 * i]) + params[2 * i + 1]
        if i < nl - 1:
            h = b.maximum(h, 0.0)
    loss = cross_entropy(b, h, labels)
    grads = b.grad(loss, params)
    both = _dp_mean(b, [loss] + grads, num_replicas)
    loss, grads = both[0], both[1:]
    if emit == "grads":
        return b.module([loss] + grads)
    new = [p - g * lr for p, g in zip(params, grads)]
    return b.module([loss] + new)


def cnn_step(batch=256, lr=1e-2, num_replicas=1, emit="params") -> str:
    """conv3x3(32)+ReLU -> maxpool2 -> conv3x3(64)+ReLU -> maxpool2 -> flatten ->
    Dense 256 ReLU -> Dense 10, softmax CE, SGD.  Inputs: w1,b1,w2,b2,w3,b3,w4,b4,
    x [batch,28,28,1] f32, labels [batch] i32.  Outputs: loss, updated params."""
    b = Builder("jit_cnn_train_step", num_replicas)
    w1, b1 = b.param((3, 3, 1, 32)), b.param((32,))
    w2, b2 = b.param((3, 3, 32, 64)), b.param((64,))
    w3, b3 = b.param((7 * 7 * 64, 256)), b.param((256,))
    w4, b4 = b.param((256, 10)), b.param((10,))
    params = [w1, b1, w2, b2, w3, b3, w4, b4]
    x = b.param((batch, 28, 28, 1))
    labels = b.param((batch,), "i32")
    h = b.maximum(b.conv(x, w1, padding=((1, 1), (1, 1))) + b1, 0.0)
    h = b.max_pool(h, (1, 2, 2, 1), (1, 2, 2, 1))
    h = b.maximum(b.conv(h, w2, padding=((1, 1), (1, 1))) + b2, 0.0)
    h = b.max_pool(h, (1, 2, 2, 1), (1, 2, 2, 1))
    h = b.reshape(h, (batch, 7 * 7 * 64))
    h = b.maximum(b.matmul(h, w3) + b3, 0.0)
    logits = b.matmul(h, w4) + b4
    loss = cross_entropy(b, logits, labels)
    grads = b.grad(loss, params)
    both = _dp_mean(b, [loss] + grads, num_replicas)
    loss, grads = both[0], both[1:]
    if emit == "grads":
        return b.module([loss] + grads)
    new = [p - g * lr for p, g in zip(params, grads)]
    return b.module([loss] + new)


def _layer_norm_bf16(b: Builder, x: V, g: V, beta: V, eps: float = 1e-6) -> V:
    """flax LayerNorm on bf16 activations: statistics and affine in f32, result bf16."""
    ax = len(x.shape) - 1
    n = float(x.shape[ax])
    h = b.convert(x, "f32")
    mean = b.sum(h, [ax], keepdims=True) / n
    d = h - mean
    var = b.sum(d * d, [ax], keepdims=True) / n
    y = d * b.rsqrt(var + eps) * b.convert(g, "f32") + b.convert(beta, "f32")
    return b.convert(y, x.dtype)


def _gelu_tanh(b: Builder, x: V) -> V:
    """jax.nn.gelu(approximate=True), in the activation dtype."""
    inner = (x + x * x * x * 0.044715) * math.sqrt(2.0 / math.pi)
    return x * ((b.tanh(inner) + 1.0) * 0.5)


def _causal_attention(b: Builder, q: V, k: V, v: V) -> V:
    """jax.nn.dot_product_attention(q, k, v, is_causal=True) for bf16 [B,T,N,H]:
    f32 logits, f32 softmax, bf16 probabilities."""
    B, T, N, H = q.shape
    logits = b.dot_general(q, k, ([3], [3]), ([0, 2], [0, 2]), out_dt="f32")  # [B,N,T,S]
    logits = logits * (1.0 / math.sqrt(H))
    row, col = b.iota((T, T), 0), b.iota((T, T), 1)
    mask = b.reshape(b.compare(row, col, "GE", "SIGNED"), (1, 1, T, T))
    big_neg = b.constant(-0.7 * F32_MAX, "f32", logits.shape)
    logits = b.select(b.broadcast_to(mask, logits.shape), logits, big_neg)
    probs = b.convert(softmax(b, logits), v.dtype)
    enc = b.dot_general(probs, v, ([3], [1]), ([0, 1], [0, 2]))  # [B,N,T,H]
    return b.transpose(enc, [0, 2, 1, 3])


def attention_vjp(B=2, T=256, N=2, H=64, causal=True, dt="bf16", form="autodiff") -> str:
    """O and the vjp (dQ, dK, dV) of jax.nn.dot_product_attention for the
    output cotangent dO; inputs Q, K, V, dO [B, T, N, H].

    form="autodiff": the gradient as ``grad`` of sum(O * dO) derives it
    (quotient rule through the softmax, as the transformer step has it);
    form="custom_jvp": the backward of ``jax.nn.softmax``'s custom JVP
    rule transposed, dx = y * g - y * sum(y * g), written out by hand."""
    b = Builder("jit_attention_vjp")
    q, k, v, g = (b.param((B, T, N, H), dt) for _ in range(4))
    if form == "autodiff":
        o = _causal_attention(b, q, k, v) if causal else None
        if o is None:
            raise ValueError("form='autodiff' builds the causal attention of the transformer")
        loss = b.sum(b.convert(o, "f32") * b.convert(g, "f32"), [0, 1, 2, 3])
        dq, dk, dv = b.grad(loss, [q, k, v])
        return b.module([o, dq, dk, dv])
    scale = 1.0 / math.sqrt(H)
    qt, kt, vt, gt = (b.transpose(x, [0, 2, 1, 3]) for x in (q, k, v, g))  # [B,N,T,H]
    logits = b.dot_general(qt, kt, ([3], [3]), ([0, 1], [0, 1]), out_dt="f32") * scale
    if causal:
        row, col = b.iota((T, T), 0), b.iota((T, T), 1)
        mask = b.broadcast_to(b.reshape(b.compare(row, col, "GE", "SIGNED"), (1, 1, T, T)),
                              logits.shape)
        logits = b.select(mask, logits, b.constant(-0.7 * F32_MAX, "f32", logits.shape))
    y = softmax(b, logits)
    yb = b.convert(y, dt)
    o = b.transpose(b.dot_general(yb, vt, ([3], [2]), ([0, 1], [0, 1])), [0, 2, 1, 3])
    dv = b.transpose(b.dot_general(yb, gt, ([2], [2]), ([0, 1], [0, 1])), [0, 2, 1, 3])
    dy = b.convert(b.dot_general(gt, vt, ([3], [3]), ([0, 1], [0, 1])), "f32")
    yg = y * dy
    dx = yg - y * b.broadcast_in_dim(b.sum(yg, [3]), yg.shape, [0, 1, 2])
    if causal:
        dx = b.select(mask, dx, b.constant(0.0, "f32", dx.shape))
    ds = dx * scale
    dq = b.dot_general(ds, kt, ([3], [2]), ([0, 1], [0, 1]))
    dk = b.dot_general(ds, qt, ([2], [2]), ([0, 1], [0, 1]))
    dq, dk = (b.transpose(b.convert(x, dt), [0, 2, 1, 3]) for x in (dq, dk))
    return b.module([o, dq, dk, dv])


TRANSFORMER_PARAMS_PER_LAYER = ("ln1_g", "ln1_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo",
                                "ln2_g", "ln2_b", "w1", "b1", "w2", "b2")


def transformer_param_shapes(layers=6, d=512, heads=8, ffn=2048, vocab=32000, seq=256):
    """[(name, shape)] in argument order: embeddings, blocks, final LN, head."""
    hd = d // heads
    per = {"ln1_g": (d,), "ln1_b": (d,), "wq": (d, heads, hd), "bq": (heads, hd),
           "wk": (d, heads, hd), "bk": (heads, hd), "wv": (d, heads, hd), "bv": (heads, hd),
           "wo": (heads, hd, d), "bo": (d,), "ln2_g": (d,), "ln2_b": (d,), "w1": (d, ffn),
           "b1": (ffn,), "w2": (ffn, d), "b2": (d,)}
    out = [("tok_emb", (vocab, d)), ("pos_emb", (seq, d))]
    for i in range(layers):
        out += [(f"l{i}.{n}", per[n]) for n in TRANSFORMER_PARAMS_PER_LAYER]
    out += [("lnf_g", (d,)), ("lnf_b", (d,)), ("w_head", (d, vocab)), ("b_head", (vocab,))]
    return out


def transformer_step(batch=64, seq=256, layers=6, d=512, heads=8, ffn=2048, vocab=32000,
                     lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, num_replicas=1, emit="state") -> str:
    """One Adam step of the pre-LN causal transformer.

    Arguments: the bf16 parameters in ``transformer_param_shapes`` order, then the
    f32 first and second Adam moments in the same order, the i32 step count,
    tokens [batch, seq] i32 and next-token targets [batch, seq] i32.
    Outputs: f32 loss, new parameters, new moments (m then v), new count
    (optax.adam: count += 1; mu_hat = mu / (1 - b1^count); p -= lr * mu_hat /
    (sqrt(nu_hat) + eps)); with emit="grads", the loss and the bf16 gradients."""
    b = Builder("jit_transformer_train_step", num_replicas)
    shapes = transformer_param_shapes(layers, d, heads, ffn, vocab, seq)
    params = [b.param(s, "bf16") for _, s in shapes]
    ms = [b.param(s, "f32") for _, s in shapes]
    vs = [b.param(s, "f32") for _, s in shapes]
    count = b.param((), "i32")
    tokens = b.param((batch, seq), "i32")
    targets = b.param((batch, seq), "i32")
    P = dict(zip([n for n, _ in shapes], params))
    x = b.take_rows(P["tok_emb"], tokens) + b.broadcast_in_dim(P["pos_emb"], (batch, seq, d), [1, 2])
    for i in range(layers):
        L = lambda n: P[f"l{i}.{n}"]
        y = _layer_norm_bf16(b, x, L("ln1_g"), L("ln1_b"))
        qkv = [b.dot_general(y, L(w), ([2], [0])) + L(bb) for w, bb in (("wq", "bq"), ("wk", "bk"),
                                                                     ("wv", "bv"))]
        att = _causal_attention(b, *qkv)
        x = x + (b.dot_general(att, L("wo"), ([2, 3], [0, 1])) + L("bo"))
        y = _layer_norm_bf16(b, x, L("ln2_g"), L("ln2_b"))
        f = _gelu_tanh(b, b.dot_general(y, L("w1"), ([2], [0])) + L("b1"))
        x = x + (b.dot_general(f, L("w2"), ([2], [0])) + L("b2"))
    y = _layer_norm_bf16(b, x, P["lnf_g"], P["lnf_b"])
    logits = b.dot_general(y, P["w_head"], ([2], [0])) + P["b_head"]
    logits = b.convert(b.reshape(logits, (batch * seq, vocab)), "f32")
    loss = cross_entropy(b, logits, b.reshape(targets, (batch * seq,)))
    grads = b.grad(loss, params)
    both = _dp_mean(b, [loss] + grads, num_replicas)
    loss, grads = both[0], both[1:]
    if emit == "grads":
        return b.module([loss] + grads)
    cnt = count + b.constant(1, "i32")
    cf = b.convert(cnt, "f32")
    bc1 = 1.0 - b.power(b.constant(b1, "f32"), cf)
    bc2 = 1.0 - b.power(b.constant(b2, "f32"), cf)
    new_p, new_m, new_v = [], [], []
    for p, m, v, g in zip(params, ms, vs, grads):
        g32 = b.convert(g, "f32")
        m2 = m * b1 + g32 * (1.0 - b1)
        v2 = v * b2 + g32 * g32 * (1.0 - b2)
        upd = (m2 / b.broadcast_to(bc1, m2.shape)) / (b.sqrt(v2 / b.broadcast_to(bc2, v2.shape)) + eps)
        new_p.append(b.convert(b.convert(p, "f32") - upd * lr, "bf16"))
        new_m.append(m2)
        new_v.append(v2)
    return b.module([loss] + new_p + new_m + new_v + [cnt])


def sdpa_custom_calls(B=2, T=128, N=2, H=64, scale=0.125, dt="f32") -> str:
    """The reference's custom_vjp attention (src/jax_mlx/sdpa.py:154-190) under
    jax.vjp: forward mlx_sdpa(Q, K, V) and backward mlx_sdpa_bwd(Q, K, V, dO).
    Inputs Q, K, V, dO [B, T, N, H]; outputs O, dQ, dK, dV."""
    b = Builder("jit_sdpa_vjp")
    q, k, v, g = (b.param((B, T, N, H), dt) for _ in range(4))
    cfg = '{"scale": %s}' % repr(float(scale))
    o = b.custom_call("mlx_sdpa", [q, k, v], [((B, T, N, H), dt)], cfg)
    dq, dk, dv = b.custom_call("mlx_sdpa_bwd", [q, k, v, g], [((B, T, N, H), dt)] * 3, cfg)
    return b.module([o, dq, dk, dv])


def layer_norm_custom_calls(rows=64, cols=256, eps=1e-5, dt="f32") -> str:
    """The reference's custom_vjp LayerNorm (src/jax_mlx/layer_norm.py:141-171)
    under jax.vjp: mlx_layer_norm(x, w, b) and mlx_layer_norm_bwd(x, w, b, dy).
    Outputs y, dx, dw, db."""
    b = Builder("jit_layer_norm_vjp")
    x, w, bb, dy = b.param((rows, cols), dt), b.param((cols,), dt), b.param((cols,), dt), b.param((rows, cols), dt)
    cfg = '{"eps": %s}' % repr(float(eps))
    y = b.custom_call("mlx_layer_norm", [x, w, bb], [((rows, cols), dt)], cfg)
    dx, dw, db = b.custom_call("mlx_layer_norm_bwd", [x, w, bb, dy],
                               [((rows, cols), dt), ((cols,), dt), ((cols,), dt)], cfg)
    return b.module([y, dx, dw, db])
