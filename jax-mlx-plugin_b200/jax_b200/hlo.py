"""StableHLO text emitter with reverse-mode autodiff.

JAX is not available in this build's environment, so the programs that
``jax.jit(f).lower(...)`` would hand the plugin are produced here: a builder
records primitive ops (one StableHLO op each, in the pretty printing JAX uses:
scalar constants broadcast with ``broadcast_in_dim``, ``dot_general`` with
batching/contracting dims, ``reduce ... applies``), and ``grad`` appends the
backward pass the way ``jax.value_and_grad`` does -- transposed
``dot_general``s, ``broadcast_in_dim`` <-> ``reduce`` duals,
``select_and_scatter`` for max-pooling, ``scatter`` for embedding lookups,
lhs-dilated / batch-feature-swapped convolutions for conv gradients.
The same text is executed by the plugin and by the numpy interpreter in
``oracle/``.
"""
from __future__ import annotations

import math
import struct
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


def ttype(shape: Sequence[int], dt: str) -> str:
    return "tensor<" + "".join(f"{d}x" for d in shape) + dt + ">"


def _fmt_float(v: float, dt: str) -> str:
    if math.isinf(v) or math.isnan(v):
        if dt == "bf16":
            bits = struct.unpack("<I", struct.pack("<f", v))[0] >> 16
            return f"0x{bits:04X}"
        if dt == "f64":
            return "0x%016X" % struct.unpack("<Q", struct.pack("<d", v))[0]
        return "0x%08X" % struct.unpack("<I", struct.pack("<f", v))[0]
    return "%.9e" % v


class V:
    __slots__ = ("b", "name", "shape", "dtype", "stopped")

    def __init__(self, b, name, shape, dtype, stopped=False):
        self.b, self.name, self.shape, self.dtype = b, name, tuple(shape), dtype
        self.stopped = stopped  # lax.stop_gradient: same SSA value, no gradient through it

    @property
    def ty(self):
        return ttype(self.shape, self.dtype)

    # arithmetic sugar with numpy-style broadcasting
    def __add__(self, o): return self.b.add(self, o)
    def __radd__(self, o): return self.b.add(o, self)
    def __sub__(self, o): return self.b.sub(self, o)
    def __rsub__(self, o): return self.b.sub(o, self)
    def __mul__(self, o): return self.b.mul(self, o)
    def __rmul__(self, o): return self.b.mul(o, self)
    def __truediv__(self, o): return self.b.div(self, o)
    def __neg__(self): return self.b.neg(self)


class Builder:
    def __init__(self, name: str = "jit_f", num_replicas: int = 1):
        self.name, self.num_replicas = name, num_replicas
        self.params: List[V] = []
        self.stmts: List[str] = []
        self.n = 0
        self.tape: List[tuple] = []
        self.recording = True

    # ------------------------------------------------------------ basics --
    def _fresh(self) -> str:
        self.n += 1
        return f"%{self.n - 1}"

    def param(self, shape, dt="f32") -> V:
        v = V(self, f"%arg{len(self.params)}", shape, dt)
        self.params.append(v)
        return v

    def _emit(self, rhs: str, shape, dt) -> V:
        name = self._fresh()
        self.stmts.append(f"{name} = {rhs}")
        return V(self, name, shape, dt)

    def _rec(self, kind, out, ins, **kw):
        if self.recording:
            self.tape.append((kind, out, list(ins), kw))
        return out

    def constant(self, value, dt="f32", shape=()) -> V:
        if dt in ("f32", "bf16", "f64"):
            lit = _fmt_float(float(value), dt)
        elif dt == "i1":
            lit = "true" if value else "false"
        else:
            lit = str(int(value))
        c = self._emit(f"stablehlo.constant dense<{lit}> : {ttype((), dt)}", (), dt)
        if tuple(shape) != ():
            c = self.broadcast_in_dim(c, shape, [])
        return c

    def dense_constant(self, arr: np.ndarray, dt: str) -> V:
        flat = ", ".join(str(int(x)) if dt.startswith("i") or dt.startswith("ui") else _fmt_float(float(x), dt)
                         for x in arr.reshape(-1))
        return self._emit(f"stablehlo.constant dense<[{flat}]> : {ttype(arr.shape, dt)}", arr.shape, dt)

    def _lift(self, x, like: V) -> V:
        if isinstance(x, V):
            return x
        return self.constant(x, like.dtype, like.shape)

    def _bcast_pair(self, a, b) -> Tuple[V, V]:
        if not isinstance(a, V):
            a = self._lift(a, b)
        if not isinstance(b, V):
            b = self._lift(b, a)
        if a.shape == b.shape:
            return a, b
        shape = np.broadcast_shapes(a.shape, b.shape)
        return self.broadcast_to(a, shape), self.broadcast_to(b, shape)

    def broadcast_to(self, x: V, shape) -> V:
        shape = tuple(shape)
        if x.shape == shape:
            return x
        # numpy rule: align on the right; size-1 dims expand (JAX drops them with reshape first)
        off = len(shape) - len(x.shape)
        keep = [i for i, d in enumerate(x.shape) if d == shape[off + i]]
        if len(keep) != len(x.shape):
            x = self.reshape(x, [x.shape[i] for i in keep])
        return self.broadcast_in_dim(x, shape, [off + i for i in keep])

    # ------------------------------------------------------- elementwise --
    def _binary(self, op, a, b, kind):
        a, b = self._bcast_pair(a, b)
        out = self._emit(f"stablehlo.{op} {a.name}, {b.name} : {a.ty}", a.shape, a.dtype)
        return self._rec(kind, out, [a, b])

    def add(self, a, b): return self._binary("add", a, b, "add")
    def sub(self, a, b): return self._binary("subtract", a, b, "sub")
    def mul(self, a, b): return self._binary("multiply", a, b, "mul")
    def div(self, a, b): return self._binary("divide", a, b, "div")
    def maximum(self, a, b): return self._binary("maximum", a, b, "max")
    def minimum(self, a, b): return self._binary("minimum", a, b, "min")
    def power(self, a, b): return self._binary("power", a, b, "pow")

    def _unary(self, op, x, kind):
        out = self._emit(f"stablehlo.{op} {x.name} : {x.ty}", x.shape, x.dtype)
        return self._rec(kind, out, [x])

    def neg(self, x): return self._unary("negate", x, "neg")
    def exp(self, x): return self._unary("exponential", x, "exp")
    def log(self, x): return self._unary("log", x, "log")
    def tanh(self, x): return self._unary("tanh", x, "tanh")
    def rsqrt(self, x): return self._unary("rsqrt", x, "rsqrt")
    def sqrt(self, x): return self._unary("sqrt", x, "sqrt")
    def logistic(self, x): return self._unary("logistic", x, "logistic")

    def compare(self, a, b, direction: str, ctype: Optional[str] = None) -> V:
        a, b = self._bcast_pair(a, b)
        if ctype is None:
            ctype = "FLOAT" if a.dtype in ("f32", "bf16", "f64") else ("UNSIGNED" if a.dtype.startswith("ui") else "SIGNED")
        return self._emit(f"stablehlo.compare  {direction}, {a.name}, {b.name},  {ctype} : "
                          f"({a.ty}, {b.ty}) -> {ttype(a.shape, 'i1')}", a.shape, "i1")

    def select(self, p: V, a, b) -> V:
        if not isinstance(a, V):
            a = self._lift(a, b)
        if not isinstance(b, V):
            b = self._lift(b, a)
        p = self.broadcast_to(p, a.shape)
        out = self._emit(f"stablehlo.select {p.name}, {a.name}, {b.name} : {p.ty}, {a.ty}", a.shape, a.dtype)
        return self._rec("select", out, [p, a, b])

    def convert(self, x: V, dt: str) -> V:
        if x.dtype == dt:
            return x
        out = self._emit(f"stablehlo.convert {x.name} : ({x.ty}) -> {ttype(x.shape, dt)}", x.shape, dt)
        return self._rec("convert", out, [x])

    def iota(self, shape, dim: int, dt="i32") -> V:
        return self._emit(f"stablehlo.iota dim = {dim} : {ttype(shape, dt)}", shape, dt)

    def stop_gradient(self, x: V) -> V:
        """lax.stop_gradient: emits nothing (as jax.jit does); the returned handle
        names the same value but gradients reaching it are dropped."""
        return V(self, x.name, x.shape, x.dtype, stopped=True)

    # ------------------------------------------------------------ layout --
    def broadcast_in_dim(self, x: V, shape, dims) -> V:
        out = self._emit(f"stablehlo.broadcast_in_dim {x.name}, dims = [{', '.join(map(str, dims))}] : "
                         f"({x.ty}) -> {ttype(shape, x.dtype)}", shape, x.dtype)
        return self._rec("bcast", out, [x], dims=list(dims))

    def reshape(self, x: V, shape) -> V:
        shape = tuple(shape)
        if shape == x.shape:
            return x
        out = self._emit(f"stablehlo.reshape {x.name} : ({x.ty}) -> {ttype(shape, x.dtype)}", shape, x.dtype)
        return self._rec("reshape", out, [x])

    def transpose(self, x: V, perm) -> V:
        shape = [x.shape[p] for p in perm]
        out = self._emit(f"stablehlo.transpose {x.name}, dims = [{', '.join(map(str, perm))}] : "
                         f"({x.ty}) -> {ttype(shape, x.dtype)}", shape, x.dtype)
        return self._rec("transpose", out, [x], perm=list(perm))

    # -------------------------------------------------------- reductions --
    def reduce(self, x: V, dims, kind: str = "add", keepdims: bool = False) -> V:
        dims = sorted(d % len(x.shape) for d in dims)
        init = {"add": 0.0, "max": -math.inf, "min": math.inf}[kind]
        c = self.constant(init, x.dtype)
        shape = [d for i, d in enumerate(x.shape) if i not in dims]
        op = {"add": "add", "max": "maximum", "min": "minimum"}[kind]
        out = self._emit(f"stablehlo.reduce({x.name} init: {c.name}) applies stablehlo.{op} across "
                         f"dimensions = [{', '.join(map(str, dims))}] : ({x.ty}, {c.ty}) -> "
                         f"{ttype(shape, x.dtype)}", shape, x.dtype)
        out = self._rec("reduce_" + kind, out, [x], dims=dims)
        if keepdims:
            out = self.reshape(out, [1 if i in dims else d for i, d in enumerate(x.shape)])
        return out

    def sum(self, x, dims, keepdims=False): return self.reduce(x, dims, "add", keepdims)

    def max(self, x, dims, keepdims=False): return self.reduce(x, dims, "max", keepdims)

    # ------------------------------------------------------------- dot --
    def dot_general(self, a: V, b: V, contract: Tuple[Sequence[int], Sequence[int]],
                    batch: Tuple[Sequence[int], Sequence[int]] = ((), ()), out_dt: Optional[str] = None) -> V:
        lc, rc = list(contract[0]), list(contract[1])
        lb, rb = list(batch[0]), list(batch[1])
        lf = [i for i in range(len(a.shape)) if i not in lc and i not in lb]
        rf = [i for i in range(len(b.shape)) if i not in rc and i not in rb]
        shape = [a.shape[i] for i in lb] + [a.shape[i] for i in lf] + [b.shape[i] for i in rf]
        dt = out_dt or a.dtype
        j = lambda v: ", ".join(map(str, v))
        bd = f"batching_dims = [{j(lb)}] x [{j(rb)}], " if lb else ""
        out = self._emit(f"stablehlo.dot_general {a.name}, {b.name}, {bd}contracting_dims = [{j(lc)}] x [{j(rc)}], "
                         f"precision = [DEFAULT, DEFAULT] : ({a.ty}, {b.ty}) -> {ttype(shape, dt)}", shape, dt)
        return self._rec("dot", out, [a, b], lc=lc, rc=rc, lb=lb, rb=rb)

    def matmul(self, a: V, b: V) -> V:
        return self.dot_general(a, b, ([len(a.shape) - 1], [0]))

    # ----------------------------------------------------- conv / windows --
    def conv(self, x: V, w: V, strides=(1, 1), padding=((0, 0), (0, 0)), lhs_dil=(1, 1), rhs_dil=(1, 1),
             dn=("b01f", "01io", "b01f")) -> V:
        """NHWC x HWIO -> NHWC by default; dn strings name each dim (b,f / i,o / 0,1 spatial)."""
        lhs, rhs, out = dn

        def spec(s):
            return "[" + ", ".join(s) + "]"
        ls, rs_ = list(lhs), list(rhs)
        osz = [0] * len(out)
        for k, ch in enumerate(out):
            if ch == "b":
                osz[k] = x.shape[ls.index("b")]
            elif ch == "f":
                osz[k] = w.shape[rs_.index("o")]
            else:
                s = int(ch)
                n_in = x.shape[ls.index(ch)]
                kk = w.shape[rs_.index(ch)]
                n_in_d = (n_in - 1) * lhs_dil[s] + 1
                k_d = (kk - 1) * rhs_dil[s] + 1
                osz[k] = (n_in_d + padding[s][0] + padding[s][1] - k_d) // strides[s] + 1
        j = lambda v: ", ".join(map(str, v))
        pad = ", ".join(f"[{lo}, {hi}]" for lo, hi in padding)
        o = self._emit(
            f"stablehlo.convolution({x.name}, {w.name}) dim_numbers = {spec(ls)}x{spec(rs_)}->{spec(out)}, "
            f"window = {{stride = [{j(strides)}], pad = [{pad}], lhs_dilate = [{j(lhs_dil)}], "
            f"rhs_dilate = [{j(rhs_dil)}]}} {{batch_group_count = 1 : i64, feature_group_count = 1 : i64}} : "
            f"({x.ty}, {w.ty}) -> {ttype(osz, x.dtype)}", osz, x.dtype)
        return self._rec("conv", o, [x, w], strides=tuple(strides), padding=tuple(map(tuple, padding)),
                         lhs_dil=tuple(lhs_dil), rhs_dil=tuple(rhs_dil), dn=dn)

    def reverse(self, x: V, dims) -> V:
        o = self._emit(f"stablehlo.reverse {x.name}, dims = [{', '.join(map(str, dims))}] : {x.ty}", x.shape, x.dtype)
        return self._rec("reverse", o, [x], dims=list(dims))

    def reduce_window(self, x: V, kind: str, window, strides) -> V:
        """VALID-padded window reduction (lax.reduce_window); kind max / min / add."""
        init = self.constant({"max": -math.inf, "min": math.inf, "add": 0.0}[kind], x.dtype)
        op = {"max": "maximum", "min": "minimum", "add": "add"}[kind]
        shape = [(d - w) // s + 1 for d, w, s in zip(x.shape, window, strides)]
        j = lambda v: ", ".join(map(str, v))
        o = self._emit(
            f'"stablehlo.reduce_window"({x.name}, {init.name}) <{{padding = dense<0> : tensor<{len(x.shape)}x2xi64>, '
            f"window_dilations = array<i64: {j([1] * len(x.shape))}>, window_dimensions = array<i64: {j(window)}>, "
            f"window_strides = array<i64: {j(strides)}>}}> ({{\n    ^bb0(%a: tensor<{x.dtype}>, %b: tensor<{x.dtype}>):\n"
            f"      %m = stablehlo.{op} %a, %b : tensor<{x.dtype}>\n      stablehlo.return %m : tensor<{x.dtype}>\n"
            f"    }}) : ({x.ty}, {init.ty}) -> {ttype(shape, x.dtype)}", shape, x.dtype)
        return self._rec("maxpool" if kind == "max" else "rwin_" + kind, o, [x], window=list(window),
                         strides=list(strides))

    def max_pool(self, x: V, window, strides) -> V:
        return self.reduce_window(x, "max", window, strides)

    def pad(self, x: V, value: float, low, high, interior) -> V:
        pv = self.constant(value, x.dtype)
        shape = [l + h + d + max(d - 1, 0) * i for d, l, h, i in zip(x.shape, low, high, interior)]
        j = lambda v: ", ".join(map(str, v))
        return self._emit(f"stablehlo.pad {x.name}, {pv.name}, low = [{j(low)}], high = [{j(high)}], "
                          f"interior = [{j(interior)}] : ({x.ty}, {pv.ty}) -> {ttype(shape, x.dtype)}", shape, x.dtype)

    def select_and_scatter_add(self, operand: V, source: V, window, strides) -> V:
        init = self.constant(0.0, operand.dtype)
        j = lambda v: ", ".join(map(str, v))
        dt = operand.dtype
        return self._emit(
            f'"stablehlo.select_and_scatter"({operand.name}, {source.name}, {init.name}) <{{padding = dense<0> : '
            f"tensor<{len(operand.shape)}x2xi64>, window_dimensions = array<i64: {j(window)}>, "
            f"window_strides = array<i64: {j(strides)}>}}> ({{\n    ^bb0(%a: tensor<{dt}>, %b: tensor<{dt}>):\n"
            f"      %c = stablehlo.compare  GE, %a, %b,  FLOAT : (tensor<{dt}>, tensor<{dt}>) -> tensor<i1>\n"
            f"      stablehlo.return %c : tensor<i1>\n    }}, {{\n    ^bb0(%a: tensor<{dt}>, %b: tensor<{dt}>):\n"
            f"      %s = stablehlo.add %a, %b : tensor<{dt}>\n      stablehlo.return %s : tensor<{dt}>\n"
            f"    }}) : ({operand.ty}, {source.ty}, {init.ty}) -> {operand.ty}", operand.shape, dt)

    # ----------------------------------------------------- gather/scatter --
    def take_rows(self, table: V, ids: V) -> V:
        """table[ids] for a 2-D table and integer ids of any rank (embedding lookup)."""
        ids2 = self.reshape(ids, list(ids.shape) + [1])
        shape = list(ids.shape) + [table.shape[1]]
        nb = len(ids.shape)
        o = self._emit(
            f'"stablehlo.gather"({table.name}, {ids2.name}) <{{dimension_numbers = #stablehlo.gather<offset_dims = [{nb}], '
            f"collapsed_slice_dims = [0], start_index_map = [0], index_vector_dim = {nb}>, indices_are_sorted = false, "
            f"slice_sizes = array<i64: 1, {table.shape[1]}>}}> : ({table.ty}, {ids2.ty}) -> {ttype(shape, table.dtype)}",
            shape, table.dtype)
        return self._rec("take_rows", o, [table], ids=ids2)

    def scatter_add_rows(self, zeros: V, ids2: V, upd: V) -> V:
        nb = len(ids2.shape) - 1
        dt = zeros.dtype
        return self._emit(
            f'"stablehlo.scatter"({zeros.name}, {ids2.name}, {upd.name}) <{{indices_are_sorted = false, '
            f"scatter_dimension_numbers = #stablehlo.scatter<update_window_dims = [{nb}], inserted_window_dims = [0], "
            f"scatter_dims_to_operand_dims = [0], index_vector_dim = {nb}>, unique_indices = false}}> ({{\n"
            f"    ^bb0(%a: tensor<{dt}>, %b: tensor<{dt}>):\n      %s = stablehlo.add %a, %b : tensor<{dt}>\n"
            f"      stablehlo.return %s : tensor<{dt}>\n    }}) : ({zeros.ty}, {ids2.ty}, {upd.ty}) -> {zeros.ty}",
            zeros.shape, dt)

    # --------------------------------------------------------- custom call --
    def custom_call(self, target: str, operands: Sequence[V], results: Sequence[Tuple[Sequence[int], str]],
                    backend_config: str = ""):
        """stablehlo.custom_call as jax's mlir.custom_call prints it; one V per result."""
        rt = [ttype(sh, dt) for sh, dt in results]
        cfg = backend_config.replace('"', "\\22")
        ins = ", ".join(o.name for o in operands)
        sig = f"({', '.join(o.ty for o in operands)}) -> " + (rt[0] if len(rt) == 1 else f"({', '.join(rt)})")
        name = self._fresh()
        head = name if len(rt) == 1 else f"{name}:{len(rt)}"
        self.stmts.append(f'{head} = stablehlo.custom_call @{target}({ins}) {{backend_config = "{cfg}"}} : {sig}')
        if len(rt) == 1:
            return V(self, name, tuple(results[0][0]), results[0][1])
        return [V(self, f"{name}#{i}", tuple(sh), dt) for i, (sh, dt) in enumerate(results)]

    # -------------------------------------------------------- collectives --
    def all_reduce_sum(self, x: V, groups: Sequence[Sequence[int]]) -> V:
        g = "[" + ", ".join("[" + ", ".join(map(str, r)) + "]" for r in groups) + "]"
        dt = x.dtype
        return self._emit(
            f'"stablehlo.all_reduce"({x.name}) <{{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, '
            f"replica_groups = dense<{g}> : tensor<{len(groups)}x{len(groups[0])}xi64>, use_global_device_ids}}> ({{\n"
            f"    ^bb0(%a: tensor<{dt}>, %b: tensor<{dt}>):\n      %s = stablehlo.add %a, %b : tensor<{dt}>\n"
            f"      stablehlo.return %s : tensor<{dt}>\n    }}) : ({x.ty}) -> {x.ty}", x.shape, dt)

    # ---------------------------------------------------------- autodiff --
    def grad(self, loss: V, wrt: Sequence[V]) -> List[V]:
        """Reverse-mode gradient of scalar `loss` w.r.t. `wrt` (emits the backward ops)."""
        was, self.recording = self.recording, False
        ct: Dict[str, V] = {loss.name: self.constant(1.0, loss.dtype)}

        def acc(v: V, g: V):
            if g is None or v.stopped:
                return
            if g.shape != v.shape:
                g = self.reshape(g, v.shape)
            ct[v.name] = self.add(ct[v.name], g) if v.name in ct else g

        for kind, out, ins, kw in reversed(self.tape):
            g = ct.get(out.name)
            if g is None:
                continue
            if kind == "add":
                acc(ins[0], g); acc(ins[1], g)
            elif kind == "sub":
                acc(ins[0], g); acc(ins[1], self.neg(g))
            elif kind == "mul":
                acc(ins[0], self.mul(g, ins[1])); acc(ins[1], self.mul(ins[0], g))
            elif kind == "div":
                a, b = ins
                acc(a, self.div(g, b))
                acc(b, self.neg(self.div(self.mul(g, out), b)))
            elif kind == "max":
                a, b = ins
                mask = self.compare(a, b, "GT")
                zero = self.constant(0.0, g.dtype, g.shape)
                acc(a, self.select(mask, g, zero))
                acc(b, self.select(mask, zero, g))
            elif kind == "neg":
                acc(ins[0], self.neg(g))
            elif kind == "exp":
                acc(ins[0], self.mul(g, out))
            elif kind == "log":
                acc(ins[0], self.div(g, ins[0]))
            elif kind == "tanh":
                acc(ins[0], self.mul(g, self.sub(1.0, self.mul(out, out))))
            elif kind == "rsqrt":
                acc(ins[0], self.mul(self.mul(g, self.div(out, ins[0])), -0.5))
            elif kind == "sqrt":
                acc(ins[0], self.div(g, self.mul(out, 2.0)))
            elif kind == "logistic":
                acc(ins[0], self.mul(g, self.mul(out, self.sub(1.0, out))))
            elif kind == "select":
                p, a, b = ins
                zero = self.constant(0.0, g.dtype, g.shape)
                acc(a, self.select(p, g, zero))
                acc(b, self.select(p, zero, g))
            elif kind == "convert":
                acc(ins[0], self.convert(g, ins[0].dtype))
            elif kind == "bcast":
                x = ins[0]
                dims = kw["dims"]
                red = [i for i in range(len(out.shape)) if i not in dims]
                red += [dims[j] for j, d in enumerate(x.shape) if d == 1 and out.shape[dims[j]] != 1]
                s = self.sum(g, sorted(red)) if red else g
                acc(x, self.reshape(s, x.shape))
            elif kind == "reshape":
                acc(ins[0], self.reshape(g, ins[0].shape))
            elif kind == "transpose":
                perm = kw["perm"]
                inv = [0] * len(perm)
                for i, p in enumerate(perm):
                    inv[p] = i
                acc(ins[0], self.transpose(g, inv))
            elif kind == "reduce_add":
                x = ins[0]
                keep = [i for i in range(len(x.shape)) if i not in kw["dims"]]
                acc(x, self.broadcast_in_dim(g, x.shape, keep))
            elif kind == "reduce_max":
                x = ins[0]
                keep = [i for i in range(len(x.shape)) if i not in kw["dims"]]
                ob = self.broadcast_in_dim(out, x.shape, keep)
                gb = self.broadcast_in_dim(g, x.shape, keep)
                eq = self.compare(x, ob, "EQ")
                acc(x, self.select(eq, gb, self.constant(0.0, g.dtype, x.shape)))
            elif kind == "dot":
                self._dot_vjp(g, out, ins, kw, acc)
            elif kind == "conv":
                self._conv_vjp(g, ins, kw, acc)
            elif kind == "maxpool":
                acc(ins[0], self.select_and_scatter_add(ins[0], g, kw["window"], kw["strides"]))
            elif kind == "take_rows":
                table = ins[0]
                ids2 = kw["ids"]
                z = self.constant(0.0, table.dtype, table.shape)
                acc(table, self.scatter_add_rows(z, ids2, g))
            elif kind == "reverse":
                acc(ins[0], self.reverse(g, kw["dims"]))
            else:
                raise NotImplementedError(f"no VJP for {kind}")
        self.recording = was
        outs = []
        for w in wrt:
            outs.append(ct[w.name] if w.name in ct else self.constant(0.0, w.dtype, w.shape))
        return outs

    def _dot_vjp(self, g: V, out: V, ins, kw, acc):
        a, b = ins
        lc, rc, lb, rb = kw["lc"], kw["rc"], kw["lb"], kw["rb"]
        nb = len(lb)
        lf = [i for i in range(len(a.shape)) if i not in lc and i not in lb]
        rf = [i for i in range(len(b.shape)) if i not in rc and i not in rb]
        # g dims: [batch..., lf..., rf...]
        g_b = list(range(nb))
        g_lf = list(range(nb, nb + len(lf)))
        g_rf = list(range(nb + len(lf), nb + len(lf) + len(rf)))
        # dA = g . B over rf (and batch): result [batch, lf, rc-dims of B in order]
        # JAX's transpose rule keeps the forward's preferred_element_type (the
        # operands may then be mixed, e.g. f32 cotangent x bf16 operand) and
        # converts the product to the primal's dtype afterwards.
        pref = out.dtype
        da = self.convert(self.dot_general(g, b, (g_rf, rf), (g_b, rb), out_dt=pref), a.dtype)
        # da dims: [batch (a's lb order), lf..., b's remaining dims = rc order]
        src_order = lb + lf + [lc[rc.index(d)] for d in sorted(rc)] if rc else lb + lf
        # map each a-dim to its position in da
        perm = [src_order.index(d) for d in range(len(a.shape))]
        acc(a, self.transpose(da, perm) if perm != list(range(len(perm))) else da)
        # dB = A . g over lf (and batch): result [batch, a's remaining = lc order, rf...]
        db = self.convert(self.dot_general(a, g, (lf, g_lf), (lb, g_b), out_dt=pref), b.dtype)
        src_b = rb + [rc[lc.index(d)] for d in sorted(lc)] + rf
        perm_b = [src_b.index(d) for d in range(len(b.shape))]
        acc(b, self.transpose(db, perm_b) if perm_b != list(range(len(perm_b))) else db)

    def _conv_vjp(self, g: V, ins, kw, acc):
        x, w = ins
        lhs, rhs, out = kw["dn"]
        if kw["lhs_dil"] != (1, 1) or kw["rhs_dil"] != (1, 1):
            raise NotImplementedError("conv VJP with dilation")
        strides, padding = kw["strides"], kw["padding"]
        ns = 2
        # ---- input gradient: conv(g, reverse(w)) with lhs dilation = strides
        sp = [rhs.index(str(s)) for s in range(ns)]
        w_rev = self.reverse(w, sp)
        k = [w.shape[rhs.index(str(s))] for s in range(ns)]
        in_sz = [x.shape[lhs.index(str(s))] for s in range(ns)]
        out_sz = [g.shape[out.index(str(s))] for s in range(ns)]
        pads = []
        for s in range(ns):
            lo = k[s] - 1 - padding[s][0]
            dil_out = (out_sz[s] - 1) * strides[s] + 1
            hi = in_sz[s] + k[s] - 1 - dil_out - lo
            pads.append((lo, hi))
        # kernel with in/out swapped: rhs spec swaps 'i' and 'o'
        rhs_t = rhs.replace("i", "X").replace("o", "i").replace("X", "o")
        dx = self.conv(g, w_rev, strides=(1, 1), padding=pads, lhs_dil=tuple(strides), dn=(out, rhs_t, lhs))
        acc(x, dx)
        # ---- kernel gradient: conv(x, g) with batch<->feature roles swapped
        lhs_t = lhs.replace("b", "X").replace("f", "b").replace("X", "f")
        g_as_k = out.replace("b", "i").replace("f", "o")
        out_t = rhs.replace("i", "b").replace("o", "f")
        pads_w = []
        for s in range(ns):
            lo = padding[s][0]
            dil_g = (out_sz[s] - 1) * strides[s] + 1
            hi = k[s] - 1 + dil_g - in_sz[s] - lo
            pads_w.append((lo, hi))
        dw = self.conv(x, g, strides=(1, 1), padding=pads_w, rhs_dil=tuple(strides), dn=(lhs_t, g_as_k, out_t))
        acc(w, dw)

    # --------------------------------------------------------------- text --
    def module(self, outputs: Sequence[V]) -> str:
        args = ", ".join(f"{p.name}: {p.ty}" for p in self.params)
        res = ", ".join(f"{o.ty}" for o in outputs)
        body = "\n".join("    " + s.replace("\n", "\n    ") for s in self.stmts)
        ret = ", ".join(o.name for o in outputs)
        rtys = ", ".join(o.ty for o in outputs)
        return (f"module @{self.name} attributes {{mhlo.num_partitions = 1 : i32, "
                f"mhlo.num_replicas = {self.num_replicas} : i32}} {{\n"
                f"  func.func public @main({args}) -> ({res}) {{\n{body}\n    return {ret} : {rtys}\n  }}\n}}\n")
