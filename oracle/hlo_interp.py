"""Test infrastructure -- the CPU oracle.  NOT part of the product path.

A numpy interpreter for StableHLO text: the semantics the reference's parity
tests compare against (reference ``tests/test_exhaustive.py:112-155`` runs each
jitted lambda on JAX's CPU backend and on the plugin).  JAX is not installed
here, so this module stands in for "the same jitted program on JAX's CPU
backend": it evaluates the identical StableHLO text op by op in float64 (f32
programs) and with per-op bf16 rounding (bf16 values), on the host -- or, with
``excess_bf16=True``, keeping bf16 elementwise chains unrounded until a convert,
a non-elementwise op or a program output (XLA's default excess precision).

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module.  It has its own small parser, independent of the plugin's
C++ parser, so a parsing bug does not cancel out in the comparison.

Replicated programs (``all_reduce``) are evaluated for all replicas in lockstep:
``run(text, [args_replica0, args_replica1, ...])``; or one replica per process,
``run(text, [args], process_sum=f)`` with ``f`` summing over the processes.
"""
from __future__ import annotations

import math
import re
import struct
from typing import Dict, List, Sequence

import numpy as np

_DT = {"f32": np.float32, "f64": np.float64, "bf16": np.float32, "i32": np.int32, "i64": np.int64,
       "i1": np.bool_, "ui32": np.uint32, "i8": np.int8, "ui8": np.uint8}


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round f32 values to the nearest bf16 (ties to even), returned as f32."""
    a = np.asarray(x, dtype=np.float32).copy()
    u = a.view(np.uint32)
    nan = np.isnan(a)
    u += np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    u &= np.uint32(0xFFFF0000)
    out = u.view(np.float32)
    out[nan] = np.nan
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


class TT:
    """Tensor type."""

    def __init__(self, shape, dt):
        self.shape, self.dt = tuple(shape), dt


_TT_RE = re.compile(r"tensor<((?:\d+x)*)([a-z0-9]+)>")


def parse_type(s: str) -> TT:
    m = _TT_RE.search(s)
    if not m:
        raise ValueError(f"no tensor type in {s!r}")
    dims = [int(d) for d in m.group(1).split("x") if d]
    return TT(dims, m.group(2))


def all_types(s: str) -> List[TT]:
    return [TT([int(d) for d in m.group(1).split("x") if d], m.group(2)) for m in _TT_RE.finditer(s)]


def _ints(s: str) -> List[int]:
    return [int(x) for x in re.findall(r"-?\d+", s)]


def _cast(x, dt: str):
    if dt == "bf16":
        return bf16_round(np.asarray(x, dtype=np.float64).astype(np.float32)).astype(np.float64)
    if dt in ("f32",):
        return np.asarray(x, dtype=np.float64)  # f32 programs are evaluated in f64
    if dt == "f64":
        return np.asarray(x, dtype=np.float64)
    if dt == "i1":
        return np.asarray(x).astype(np.bool_)
    return np.asarray(x).astype(_DT[dt])


def _const(body: str, t: TT):
    body = body.strip()
    if body.startswith('"0x'):
        raw = bytes.fromhex(body[3:-1])
        npdt = {"f32": np.float32, "bf16": np.uint16, "i32": np.int32, "i1": np.uint8, "i64": np.int64,
                "f64": np.float64, "ui32": np.uint32}[t.dt]
        arr = np.frombuffer(raw, dtype=npdt)
        if t.dt == "bf16":
            arr = bf16_bits_to_f32(arr)
        n = int(np.prod(t.shape)) if t.shape else 1
        arr = np.broadcast_to(arr, (n,)) if arr.size == 1 else arr
        return _cast(arr.reshape(t.shape), t.dt)
    toks = re.findall(r"0x[0-9A-Fa-f]+|true|false|[-+]?(?:\d+\.?\d*(?:[eE][-+]?\d+)?|inf|nan)", body)

    def one(tok):
        if tok.startswith("0x"):
            bits = int(tok, 16)
            if t.dt == "f32":
                return struct.unpack("<f", struct.pack("<I", bits))[0]
            if t.dt == "bf16":
                return struct.unpack("<f", struct.pack("<I", bits << 16))[0]
            if t.dt == "f64":
                return struct.unpack("<d", struct.pack("<Q", bits))[0]
            return bits
        if tok == "true":
            return 1
        if tok == "false":
            return 0
        return float(tok)
    vals = [one(x) for x in toks]
    if len(vals) == 1:
        return _cast(np.full(t.shape, vals[0]), t.dt)
    return _cast(np.array(vals).reshape(t.shape), t.dt)


# Elementwise ops whose bf16 results stay unrounded in excess-precision mode.
_EXCESS_OPS = {"negate", "exponential", "log", "tanh", "sqrt", "abs", "rsqrt", "logistic",
               "exponential_minus_one", "log_plus_one", "sine", "cosine", "add", "subtract",
               "multiply", "maximum", "minimum", "power", "divide", "select", "clamp"}


class Interp:
    """excess_bf16: bf16 elementwise results are not rounded (only explicit
    converts, non-elementwise ops such as reduce / dot_general and the
    program's outputs round to bf16) -- XLA's default excess-precision
    treatment of bf16 chains, which a fusing compiler follows.  Default: every
    bf16 op's result is rounded.

    process_sum: for a replicated program run with one replica per process,
    a callable that sums an array over the processes (e.g. a torch.distributed
    all_reduce); ``all_reduce`` results are then that sum of this process's
    replicas."""

    def __init__(self, text: str, excess_bf16: bool = False, process_sum=None):
        self.text = re.sub(r"\s*loc\([^)]*\)", "", text)
        self.funcs = self._split_funcs(self.text)
        self.excess_bf16 = excess_bf16
        self.process_sum = process_sum

    # ------------------------------------------------------------ parsing --
    @staticmethod
    def _split_funcs(text: str) -> Dict[str, tuple]:
        funcs = {}
        for m in re.finditer(r"func\.func\s+(?:public|private)?\s*@(\w+)\((.*?)\)\s*->\s*(.*?)\{\n", text):
            name = m.group(1)
            params = re.findall(r"(%[\w#]+)\s*:\s*(tensor<[^>]*>)", m.group(2))
            start = m.end()
            depth, i = 1, start
            while depth:
                c = text[i]
                if c == "{":
                    depth += 1
                elif c == "}":
                    depth -= 1
                i += 1
            funcs[name] = ([p[0] for p in params], [parse_type(p[1]) for p in params], text[start:i - 1])
        return funcs

    @staticmethod
    def _statements(body: str) -> List[str]:
        """Split a function body into statements; an op with regions spans several
        lines until its brackets balance (quoted strings are skipped)."""
        out, cur, depth = [], [], 0
        for line in body.split("\n"):
            s = line.strip()
            if not s:
                continue
            cur.append(s)
            unq = re.sub(r'"(?:[^"\\]|\\.)*"', '""', s)
            depth += sum(unq.count(ch) for ch in "({[") - sum(unq.count(ch) for ch in ")}]")
            if depth <= 0:
                out.append("\n".join(cur))
                cur, depth = [], 0
        return out

    # --------------------------------------------------------- evaluation --
    def run(self, replica_args: Sequence[Sequence[np.ndarray]], func: str = "main") -> List[List[np.ndarray]]:
        """Evaluate `func` for each replica; returns outputs[replica][i] as float64/int arrays."""
        names, types, body = self.funcs[func]
        R = len(replica_args)
        env: Dict[str, list] = {}
        for i, (n, t) in enumerate(zip(names, types)):
            env[n] = [_cast(replica_args[r][i] if t.dt != "bf16" else replica_args[r][i], t.dt) for r in range(R)]
        for st in self._statements(body):
            if st.startswith("return") or st.startswith("func.return"):
                rets = re.findall(r"%[\w#]+", st.split(":")[0])
                outs = [[self._get(env, x)[r] for x in rets] for r in range(R)]
                if self.excess_bf16 and func == "main" and ":" in st:
                    rt = all_types(st.split(":", 1)[1])
                    outs = [[_cast(v, t.dt) if t.dt == "bf16" else v for v, t in zip(o, rt)]
                            for o in outs]
                return outs
            self._exec(st, env, R)
        raise ValueError("function has no return")

    @staticmethod
    def _get(env, name):
        if "#" in name:
            base, k = name.split("#")
            return [v[int(k)] for v in env[base]]
        return env[name]

    def _exec(self, st: str, env, R):
        m = re.match(r"(%[\w]+)(?::(\d+))?\s*=\s*(.*)", st, re.S)
        res, nres, rhs = m.group(1), m.group(2), m.group(3)
        generic = rhs.startswith('"')
        op = re.match(r'"?([\w.]+)"?', rhs).group(1).replace("stablehlo.", "")
        sig = rhs[rhs.rfind("})") + 2:] if generic and "})" in rhs else rhs
        tys = all_types(sig.split(" : ", 1)[1] if " : " in sig else sig)
        out_t = tys[-1]
        head = rhs.split(" : ")[0] if not generic else rhs[:rhs.find(")")]
        operands = re.findall(r"%[\w#]+", head if not generic else rhs[rhs.find("(") + 1:rhs.find(")")])
        if op == "reduce":
            operands = re.findall(r"%[\w#]+", rhs.split(" applies")[0].split(" across")[0])
        args = [self._get(env, o) for o in operands]
        out = []
        for r in range(R):
            a = [x[r] for x in args]
            out.append(self._op(op, rhs, a, out_t, tys, env, r, args))
        if op == "all_reduce":
            s = sum(o for o in out)
            if self.process_sum is not None:
                s = self.process_sum(np.asarray(s, np.float64))
            out = [_cast(s, out_t.dt) for _ in range(R)]
        env[res] = out

    def _op(self, op, rhs, a, t: TT, tys, env, r, all_args):
        dt = t.dt
        c = lambda x: _cast(x, dt)
        if self.excess_bf16 and dt == "bf16" and op in _EXCESS_OPS:
            c = lambda x: np.asarray(x, dtype=np.float64)
        if op == "constant":
            body = re.search(r"dense<(.*)>\s*:", rhs).group(1)
            return _const(body, t)
        if op == "iota":
            d = int(re.search(r"dim = (\d+)", rhs).group(1))
            shape = [1] * len(t.shape)
            shape[d] = t.shape[d]
            return c(np.broadcast_to(np.arange(t.shape[d]).reshape(shape), t.shape))
        un = {"negate": np.negative, "exponential": np.exp, "log": np.log, "tanh": np.tanh,
              "sqrt": np.sqrt, "abs": np.abs, "floor": np.floor, "ceil": np.ceil,
              "rsqrt": lambda x: 1.0 / np.sqrt(x), "logistic": lambda x: 1.0 / (1.0 + np.exp(-x)),
              "not": lambda x: np.logical_not(x) if x.dtype == np.bool_ else ~x,
              "exponential_minus_one": np.expm1, "log_plus_one": np.log1p, "sine": np.sin,
              "cosine": np.cos, "sign": np.sign}
        if op in un:
            with np.errstate(all="ignore"):
                return c(un[op](a[0]))
        bi = {"add": np.add, "subtract": np.subtract, "multiply": np.multiply, "maximum": np.maximum,
              "minimum": np.minimum, "power": np.power, "and": np.logical_and, "or": np.logical_or}
        if op in bi:
            with np.errstate(all="ignore"):
                return c(bi[op](a[0], a[1]))
        if op == "divide":
            with np.errstate(all="ignore"):
                if dt.startswith("i") and dt != "i1":
                    return c(np.trunc(a[0] / a[1]))
                return c(a[0] / a[1])
        if op == "compare":
            d = re.search(r"compare\s+(\w+)", rhs).group(1)
            f = {"EQ": np.equal, "NE": np.not_equal, "LT": np.less, "LE": np.less_equal,
                 "GT": np.greater, "GE": np.greater_equal}[d]
            return f(a[0], a[1])
        if op == "select":
            return c(np.where(a[0], a[1], a[2]))
        if op == "clamp":
            return c(np.minimum(np.maximum(a[1], a[0]), a[2]))
        if op == "convert":
            x = a[0]
            if np.issubdtype(np.asarray(x).dtype, np.floating) and (dt.startswith("i") or dt.startswith("ui")) and dt != "i1":
                x = np.trunc(x)
            return c(x)
        if op == "broadcast_in_dim":
            dims = _ints(re.search(r"dims = \[([^\]]*)\]", rhs).group(1))
            x = np.asarray(a[0])
            shape = [1] * len(t.shape)
            for j, d in enumerate(dims):
                shape[d] = x.shape[j]
            return np.broadcast_to(x.reshape(shape), t.shape).copy()
        if op == "reshape":
            return np.asarray(a[0]).reshape(t.shape)
        if op == "transpose":
            perm = _ints(re.search(r"dims = \[([^\]]*)\]", rhs).group(1))
            return np.transpose(a[0], perm).copy()
        if op == "reverse":
            dims = _ints(re.search(r"dims = \[([^\]]*)\]", rhs).group(1))
            return np.flip(a[0], dims).copy()
        if op == "reduce":
            dims = tuple(_ints(re.search(r"dimensions = \[([^\]]*)\]", rhs).group(1)))
            kind = re.search(r"applies stablehlo\.(\w+)", rhs).group(1)
            f = {"add": np.sum, "maximum": np.max, "minimum": np.min, "multiply": np.prod}[kind]
            init = a[1]
            g = {"add": np.add, "maximum": np.maximum, "minimum": np.minimum, "multiply": np.multiply}[kind]
            if np.size(a[0]) == 0:  # nothing to fold: every output is the init value
                return c(np.broadcast_to(init, t.shape).copy())
            return c(g(f(a[0], axis=dims), init))
        if op == "dot_general":
            bd = re.search(r"batching_dims = \[([^\]]*)\] x \[([^\]]*)\]", rhs)
            cd = re.search(r"contracting_dims = \[([^\]]*)\] x \[([^\]]*)\]", rhs)
            lb, rb = (_ints(bd.group(1)), _ints(bd.group(2))) if bd else ([], [])
            lc, rc = _ints(cd.group(1)), _ints(cd.group(2))
            return c(dot_general(a[0], a[1], lb, rb, lc, rc))
        if op == "convolution":
            return c(self._conv(rhs, a[0], a[1]))
        if op == "reduce_window":
            return c(self._reduce_window(rhs, a[0], a[1]))
        if op == "select_and_scatter":
            return c(self._select_and_scatter(rhs, a[0], a[1], a[2]))
        if op == "gather":
            return c(self._gather(rhs, a[0], a[1], t))
        if op == "scatter":
            return c(self._scatter(rhs, a[0], a[1], a[2]))
        if op == "all_reduce":
            return a[0]
        if op == "pad":
            lo = _ints(re.search(r"low = \[([^\]]*)\]", rhs).group(1))
            hi = _ints(re.search(r"high = \[([^\]]*)\]", rhs).group(1))
            it = _ints(re.search(r"interior = \[([^\]]*)\]", rhs).group(1))
            x = np.asarray(a[0])
            shp = [d + max(d - 1, 0) * i for d, i in zip(x.shape, it)]
            full = np.full(shp, a[1], dtype=np.float64 if x.dtype.kind == "f" else x.dtype)
            full[tuple(slice(None, None, i + 1) for i in it)] = x
            pw = [(max(l, 0), max(h, 0)) for l, h in zip(lo, hi)]
            full = np.pad(full, pw, constant_values=a[1])
            crop = tuple(slice(-min(l, 0) or None, full.shape[k] + min(h, 0)) for k, (l, h) in enumerate(zip(lo, hi)))
            return c(full[crop])
        if op == "custom_call":
            r = self._custom(rhs, a, t)
            if isinstance(r, tuple):  # multi-result: one type per result, last in the signature
                return tuple(_cast(x, tt.dt) for x, tt in zip(r, tys[-len(r):]))
            return c(r)
        raise NotImplementedError(f"oracle: op {op}")

    # ---------------------------------------------------------------- ops --
    def _conv(self, rhs, x, w):
        m = re.search(r"dim_numbers = \[([^\]]*)\]x\[([^\]]*)\]->\[([^\]]*)\]", rhs)
        ls, ks, os_ = [s.strip() for s in m.group(1).split(",")], [s.strip() for s in m.group(2).split(",")], \
            [s.strip() for s in m.group(3).split(",")]
        ns = len(ls) - 2
        get = lambda key, default: _ints(re.search(key + r" = \[([^\]]*)\]", rhs).group(1)) if re.search(key + r" = \[", rhs) else default
        stride = get("stride", [1] * ns)
        lhs_dil = get("lhs_dilate", [1] * ns)
        rhs_dil = get("rhs_dilate", [1] * ns)
        pm = re.search(r"pad = \[(.*?)\]\]", rhs)
        pads = _ints(pm.group(1)) if pm else [0] * (2 * ns)
        rev = re.search(r"reverse = \[([^\]]*)\]", rhs)
        reverse = [s.strip() == "true" for s in rev.group(1).split(",")] if rev else [False] * ns
        # canonical: x [N, s0, s1, C], w [k0, k1, I, O]
        xp = np.transpose(x, [ls.index("b")] + [ls.index(str(i)) for i in range(ns)] + [ls.index("f")])
        wp = np.transpose(w, [ks.index(str(i)) for i in range(ns)] + [ks.index("i"), ks.index("o")])
        for i in range(ns):
            if reverse[i]:
                wp = np.flip(wp, i)
        # lhs dilation
        if any(d != 1 for d in lhs_dil):
            shp = list(xp.shape)
            for i in range(ns):
                shp[1 + i] = (xp.shape[1 + i] - 1) * lhs_dil[i] + 1
            xd = np.zeros(shp, dtype=xp.dtype)
            xd[(slice(None),) + tuple(slice(None, None, lhs_dil[i]) for i in range(ns)) + (slice(None),)] = xp
            xp = xd
        # padding (negative = crop)
        pw = [(0, 0)] + [(max(pads[2 * i], 0), max(pads[2 * i + 1], 0)) for i in range(ns)] + [(0, 0)]
        xp = np.pad(xp, pw)
        crop = [slice(None)] + [slice(-min(pads[2 * i], 0) or None, (xp.shape[1 + i] + min(pads[2 * i + 1], 0))) for i in range(ns)] + [slice(None)]
        xp = xp[tuple(crop)]
        K = wp.shape[:ns]
        kd = [(K[i] - 1) * rhs_dil[i] + 1 for i in range(ns)]
        osz = [(xp.shape[1 + i] - kd[i]) // stride[i] + 1 for i in range(ns)]
        out = np.zeros([xp.shape[0]] + osz + [wp.shape[-1]], dtype=np.float64)
        for k0 in range(K[0]):
            for k1 in range(K[1]):
                o0, o1 = k0 * rhs_dil[0], k1 * rhs_dil[1]
                patch = xp[:, o0:o0 + (osz[0] - 1) * stride[0] + 1:stride[0],
                           o1:o1 + (osz[1] - 1) * stride[1] + 1:stride[1], :]
                out += patch @ wp[k0, k1]
        perm = [0] * (ns + 2)
        # out currently [b, s0, s1, f]; place into os_ order
        src = ["b"] + [str(i) for i in range(ns)] + ["f"]
        return np.transpose(out, [src.index(ch) for ch in os_])

    @staticmethod
    def _window_attrs(rhs, rank):
        wd = _ints(re.search(r"window_dimensions = array<i64: ([^>]*)>", rhs).group(1))
        ws = re.search(r"window_strides = array<i64: ([^>]*)>", rhs)
        ws = _ints(ws.group(1)) if ws else [1] * rank
        pad = re.search(r"padding = dense<(.*?)> : tensor", rhs)
        p = _ints(pad.group(1)) if pad else [0]
        if len(p) == 1:
            p = p * (2 * rank)
        return wd, ws, p

    def _reduce_window(self, rhs, x, init):
        wd, ws, p = self._window_attrs(rhs, x.ndim)
        body = rhs[rhs.find("({"):]
        kind = "max" if "maximum" in body else ("min" if "minimum" in body else "add")
        fill = float(init)
        xp = np.pad(x, [(p[2 * i], p[2 * i + 1]) for i in range(x.ndim)], constant_values=fill)
        osz = [(xp.shape[i] - wd[i]) // ws[i] + 1 for i in range(x.ndim)]
        out = np.full(osz, fill, dtype=np.float64)
        f = {"max": np.maximum, "min": np.minimum, "add": np.add}[kind]
        for off in np.ndindex(*wd):
            sl = tuple(slice(off[i], off[i] + (osz[i] - 1) * ws[i] + 1, ws[i]) for i in range(x.ndim))
            out = f(out, xp[sl])
        return out

    def _select_and_scatter(self, rhs, x, src, init):
        wd, ws, p = self._window_attrs(rhs, x.ndim)
        sel_body = rhs[rhs.find("({"):rhs.find("}, {")]
        ge = "GE" in sel_body
        le = "LE" in sel_body
        out = np.full(x.shape, float(init), dtype=np.float64)
        for w in np.ndindex(*src.shape):
            best, bpos = None, None
            for off in np.ndindex(*wd):
                pos = tuple(w[i] * ws[i] + off[i] - p[2 * i] for i in range(x.ndim))
                if any(q < 0 or q >= x.shape[i] for i, q in enumerate(pos)):
                    continue
                v = x[pos]
                keep = best is not None and ((best >= v) if ge else (best <= v) if le else (best > v))
                if best is None or not keep:
                    best, bpos = v, pos
            if bpos is not None:
                out[bpos] += src[w]
        return out

    @staticmethod
    def _gather(rhs, table, idx, t: TT):
        od = _ints(re.search(r"offset_dims = \[([^\]]*)\]", rhs).group(1))
        cd = _ints(re.search(r"collapsed_slice_dims = \[([^\]]*)\]", rhs).group(1))
        sm = _ints(re.search(r"start_index_map = \[([^\]]*)\]", rhs).group(1))
        if not (cd == [0] and sm == [0] and table.ndim == 2):
            raise NotImplementedError("oracle gather: only row lookups")
        ids = np.clip(np.asarray(idx)[..., 0].astype(np.int64), 0, table.shape[0] - 1)
        return table[ids]

    @staticmethod
    def _scatter(rhs, base, idx, upd):
        iw = _ints(re.search(r"inserted_window_dims = \[([^\]]*)\]", rhs).group(1))
        if iw != [0] or base.ndim != 2:
            raise NotImplementedError("oracle scatter: only row scatter-add")
        out = np.array(base, dtype=np.float64)
        ids = np.asarray(idx)[..., 0].astype(np.int64).reshape(-1)
        u = np.asarray(upd, dtype=np.float64).reshape(-1, base.shape[1])
        ok = (ids >= 0) & (ids < base.shape[0])
        np.add.at(out, ids[ok], u[ok])
        return out

    @staticmethod
    def _custom(rhs, a, t):
        target = re.search(r"custom_call @(\w+)", rhs).group(1)
        if target == "mlx_sdpa":
            m = re.search(r"scale\\?\"?\\?\"?:\s*([-\d.eE+]+)", rhs.replace("\\22", '"'))
            scale = float(m.group(1)) if m else 1.0 / math.sqrt(a[0].shape[-1])
            from .restate import sdpa_ref
            return sdpa_ref(a[0], a[1], a[2], scale=scale, causal=False)
        if target == "mlx_layer_norm":
            m = re.search(r"eps\\?\"?\\?\"?:\s*([-\d.eE+]+)", rhs.replace("\\22", '"'))
            eps = float(m.group(1)) if m else 1e-5
            from .restate import layer_norm_ref
            return layer_norm_ref(a[0], None, a[1], a[2], eps)
        if target == "mlx_sdpa_bwd":
            m = re.search(r"scale\\?\"?\\?\"?:\s*([-\d.eE+]+)", rhs.replace("\\22", '"'))
            from .restate import sdpa_bwd_ref
            return tuple(sdpa_bwd_ref(a[0], a[1], a[2], a[3], float(m.group(1)) if m else 1.0))
        if target == "mlx_layer_norm_bwd":
            m = re.search(r"eps\\?\"?\\?\"?:\s*([-\d.eE+]+)", rhs.replace("\\22", '"'))
            from .restate import layer_norm_bwd_ref
            return tuple(layer_norm_bwd_ref(a[0], a[1], a[3], float(m.group(1)) if m else 1e-5))
        raise NotImplementedError(f"oracle custom_call @{target}")


def dot_general(x, y, lb, rb, lc, rc):
    """StableHLO dot_general: result dims [batch..., lhs free..., rhs free...]."""
    letters = iter("abcdefghijklmnopqrstuvwxyz")
    xs = [None] * x.ndim
    ys = [None] * y.ndim
    for i, j in zip(lb, rb):
        xs[i] = ys[j] = next(letters)
    for i, j in zip(lc, rc):
        xs[i] = ys[j] = next(letters)
    for i in range(x.ndim):
        if xs[i] is None:
            xs[i] = next(letters)
    for j in range(y.ndim):
        if ys[j] is None:
            ys[j] = next(letters)
    out = [xs[i] for i in lb] + [xs[i] for i in range(x.ndim) if i not in lb and i not in lc] + \
          [ys[j] for j in range(y.ndim) if j not in rb and j not in rc]
    return np.einsum("".join(xs) + "," + "".join(ys) + "->" + "".join(out), x, y)


def run(text: str, replica_args, func: str = "main", excess_bf16: bool = False, process_sum=None):
    """Evaluate StableHLO `text`.  replica_args: list (one per replica) of arg lists."""
    return Interp(text, excess_bf16, process_sum).run(replica_args, func)
