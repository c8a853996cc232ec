// Compile-time graph passes: call inlining, identity forwarding, DCE, host
// evaluation of constant subgraphs, and the SDPA / LayerNorm pattern matchers.
// The matchers play the role of reference src/jax_mlx_pjrt.cpp:1816-2769
// (RecognizePatterns) but match on dataflow (uses, shapes, constants) instead
// of op order, and also recognise the causal select(iota >= iota, s, -big)
// mask that JAX emits for is_causal=True.
#include "passes.h"

#include <cstdlib>

#include "custom_calls.h"

#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <set>
#include <sstream>

namespace b200 {

// ------------------------------------------------------------- inlining ---
namespace {
void inline_into(const Module& m, const Graph& src, const std::vector<ValueRef>& args,
                 Graph& dst, std::vector<ValueRef>& outs, int depth) {
  if (depth > 64) throw PjrtErr(3, "call nesting too deep (recursive func.call?)");
  std::vector<std::vector<ValueRef>> map(src.nodes.size());
  for (size_t i = 0; i < src.nodes.size(); ++i) {
    const Node& n = src.nodes[i];
    if (n.op == Op::Parameter) {
      map[i] = {args.at(n.param_index)};
      continue;
    }
    std::vector<ValueRef> ops;
    for (auto& o : n.operands) ops.push_back(map.at(o.node).at(o.idx));
    if (n.op == Op::Call) {
      auto it = m.funcs.find(n.target);
      if (it == m.funcs.end()) throw PjrtErr(3, "call to undefined function @" + n.target);
      std::vector<ValueRef> r;
      inline_into(m, *it->second, ops, dst, r, depth + 1);
      map[i] = r;
      continue;
    }
    if (n.op == Op::CustomCall && expands_custom_call(n.target)) {
      std::vector<ValueRef> r;
      if (fused_sdpa_bwd_call(n, ops, dst, r)) {  // the fused attention kernels
        map[i] = r;
        continue;
      }
      // backward custom calls become ordinary StableHLO (custom_calls.cc)
      std::vector<TensorType> types;
      for (auto& o : ops) types.push_back(dst.type(o));
      Module sub = parse_module(custom_call_expansion(n, types));
      inline_into(sub, *sub.main(), ops, dst, r, depth + 1);
      if (r.size() != n.results.size()) throw PjrtErr(13, "custom call expansion result count");
      for (size_t k = 0; k < r.size(); ++k)
        if (dst.type(r[k]) != n.results[k])
          throw PjrtErr(3, "custom_call @" + n.target + " result " + std::to_string(k) + " has type " +
                               n.results[k].str() + ", expected " + dst.type(r[k]).str());
      map[i] = r;
      continue;
    }
    Node c = n;
    c.operands = ops;
    int id = dst.add(std::move(c));
    for (size_t k = 0; k < n.results.size(); ++k) map[i].push_back(ValueRef{id, (int)k});
  }
  for (auto& o : src.outputs) outs.push_back(map.at(o.node).at(o.idx));
}
}  // namespace

Graph inline_calls(const Module& m) {
  auto main = m.main();
  Graph g;
  g.name = main->name;
  g.param_types = main->param_types;
  std::vector<ValueRef> args;
  for (size_t i = 0; i < main->param_types.size(); ++i) {
    Node p;
    p.op = Op::Parameter;
    p.param_index = (int64_t)i;
    p.results = {main->param_types[i]};
    p.name = "%arg" + std::to_string(i);
    args.push_back(ValueRef{g.add(std::move(p)), 0});
  }
  // Parameters of `main` appear first in `g`; skip main's own parameter nodes.
  inline_into(m, *main, args, g, g.outputs, 0);
  return g;
}

// ------------------------------------------------------------- simplify ---
static bool is_identity_perm(const std::vector<int64_t>& p) {
  for (size_t i = 0; i < p.size(); ++i)
    if (p[i] != (int64_t)i) return false;
  return true;
}

void simplify(Graph& g) {
  std::map<ValueRef, ValueRef> fwd;
  auto res = [&](ValueRef v) {
    for (int k = 0; k < 64; ++k) {
      auto it = fwd.find(v);
      if (it == fwd.end()) break;
      v = it->second;
    }
    return v;
  };
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    Node& n = g.nodes[i];
    if (n.dead) continue;
    for (auto& o : n.operands) o = res(o);
    const int id = (int)i;
    switch (n.op) {
      case Op::OptimizationBarrier:
        for (size_t k = 0; k < n.results.size(); ++k) fwd[{id, (int)k}] = n.operands.at(k);
        n.dead = true;
        break;
      case Op::Convert: case Op::Reshape: case Op::BitcastConvert:
        if (g.type(n.operands[0]) == n.results[0]) { fwd[{id, 0}] = n.operands[0]; n.dead = true; }
        break;
      case Op::Transpose:
        if (is_identity_perm(n.dims)) { fwd[{id, 0}] = n.operands[0]; n.dead = true; }
        break;
      case Op::BroadcastInDim:
        if (g.type(n.operands[0]) == n.results[0] && is_identity_perm(n.dims)) {
          fwd[{id, 0}] = n.operands[0];
          n.dead = true;
        }
        break;
      case Op::CustomCall:
        if ((n.target == "Sharding" || n.target == "SPMDFullToShardShape" ||
             n.target == "SPMDShardToFullShape" || n.target == "annotate_device_placement" ||
             n.target == "mhlo.sharding") &&
            n.operands.size() == 1 && n.results.size() == 1 &&
            g.type(n.operands[0]) == n.results[0]) {
          fwd[{id, 0}] = n.operands[0];
          n.dead = true;
        }
        break;
      default: break;
    }
  }
  for (auto& o : g.outputs) o = res(o);
}

// ----------------------------------------------------------------- DCE ---
void dce(Graph& g) {
  std::vector<char> live(g.nodes.size(), 0);
  std::vector<int> stack;
  for (auto& o : g.outputs) stack.push_back(o.node);
  while (!stack.empty()) {
    int n = stack.back();
    stack.pop_back();
    if (live[n]) continue;
    live[n] = 1;
    for (auto& o : g.nodes[n].operands) stack.push_back(o.node);
  }
  for (size_t i = 0; i < g.nodes.size(); ++i)
    if (!live[i] && g.nodes[i].op != Op::Parameter) g.nodes[i].dead = true;
}

Uses compute_uses(const Graph& g) {
  Uses u;
  u.users.assign(g.nodes.size(), {});
  u.output_refs.assign(g.nodes.size(), 0);
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (g.nodes[i].dead) continue;
    for (auto& o : g.nodes[i].operands) {
      auto& us = u.users[o.node];
      if (us.empty() || us.back() != (int)i) us.push_back((int)i);  // one entry per consumer
    }
  }
  for (auto& o : g.outputs) u.output_refs[o.node]++;
  return u;
}

// ------------------------------------------------------------ host eval ---
namespace {
std::vector<int64_t> strides_of(const std::vector<int64_t>& d) {
  std::vector<int64_t> s(d.size(), 1);
  for (int i = (int)d.size() - 2; i >= 0; --i) s[i] = s[i + 1] * d[i + 1];
  return s;
}
double read_elem(const uint8_t* p, DType t) {
  switch (t) {
    case DType::PRED: return *p ? 1 : 0;
    case DType::S8: return (int8_t)*p;
    case DType::U8: return *p;
    case DType::S16: { int16_t v; std::memcpy(&v, p, 2); return v; }
    case DType::U16: { uint16_t v; std::memcpy(&v, p, 2); return v; }
    case DType::S32: { int32_t v; std::memcpy(&v, p, 4); return v; }
    case DType::U32: { uint32_t v; std::memcpy(&v, p, 4); return v; }
    case DType::S64: { int64_t v; std::memcpy(&v, p, 8); return (double)v; }
    case DType::U64: { uint64_t v; std::memcpy(&v, p, 8); return (double)v; }
    case DType::F32: { float v; std::memcpy(&v, p, 4); return v; }
    case DType::F64: { double v; std::memcpy(&v, p, 8); return v; }
    case DType::BF16: { uint16_t b; std::memcpy(&b, p, 2); uint32_t u = (uint32_t)b << 16; float f; std::memcpy(&f, &u, 4); return f; }
    default: return 0;
  }
}
double cast_to(double v, DType t) {
  if (t == DType::PRED) return v != 0 ? 1 : 0;
  if (dtype_is_int(t)) return std::trunc(v);
  if (t == DType::F32 || t == DType::BF16) return (double)(float)v;
  return v;
}
}  // namespace

std::optional<HostTensor> host_eval(const Graph& g, ValueRef root, int64_t max_elems) {
  std::map<ValueRef, HostTensor> memo;
  std::function<std::optional<HostTensor>(ValueRef)> ev = [&](ValueRef v) -> std::optional<HostTensor> {
    auto it = memo.find(v);
    if (it != memo.end()) return it->second;
    const Node& n = g.nodes.at(v.node);
    const TensorType& t = n.results.at(v.idx);
    if (t.numel() > max_elems) return std::nullopt;
    HostTensor out;
    out.type = t;
    const int64_t N = t.numel();
    out.v.resize(N);
    auto in = [&](int k) { return ev(n.operands.at(k)); };
    switch (n.op) {
      case Op::Constant: {
        const int es = dtype_size(t.dtype);
        for (int64_t i = 0; i < N; ++i)
          out.v[i] = read_elem(n.cdata.bytes.data() + (n.cdata.splat ? 0 : i * es), t.dtype);
        break;
      }
      case Op::Iota: {
        auto st = strides_of(t.dims);
        for (int64_t i = 0; i < N; ++i) out.v[i] = (double)((i / st[n.iota_dim]) % t.dims[n.iota_dim]);
        break;
      }
      case Op::BroadcastInDim: case Op::Transpose: case Op::Reshape: case Op::Convert: {
        auto a = in(0);
        if (!a) return std::nullopt;
        if (n.op == Op::Reshape) { out.v = a->v; break; }
        if (n.op == Op::Convert) {
          for (int64_t i = 0; i < N; ++i) out.v[i] = cast_to(a->v[i], t.dtype);
          break;
        }
        auto so = strides_of(t.dims), si = strides_of(a->type.dims);
        for (int64_t i = 0; i < N; ++i) {
          int64_t src = 0;
          for (int d = 0; d < t.rank(); ++d) {
            int64_t idx = (i / so[d]) % t.dims[d];
            if (n.op == Op::BroadcastInDim) {
              // output dim d receives input dim j where dims[j] == d
              for (size_t j = 0; j < n.dims.size(); ++j)
                if (n.dims[j] == d && a->type.dims[j] != 1) src += idx * si[j];
            } else {  // transpose: out dim d = in dim perm[d]
              src += idx * si[n.dims[d]];
            }
          }
          out.v[i] = a->v[src];
        }
        break;
      }
      case Op::Compare: {
        auto a = in(0), b = in(1);
        if (!a || !b) return std::nullopt;
        for (int64_t i = 0; i < N; ++i) {
          double x = a->v[i], y = b->v[i];
          bool r = false;
          switch (n.cmp_dir) {
            case CmpDir::EQ: r = x == y; break; case CmpDir::NE: r = x != y; break;
            case CmpDir::LT: r = x < y; break; case CmpDir::LE: r = x <= y; break;
            case CmpDir::GT: r = x > y; break; case CmpDir::GE: r = x >= y; break;
          }
          out.v[i] = r;
        }
        break;
      }
      case Op::Select: {
        auto p = in(0), a = in(1), b = in(2);
        if (!p || !a || !b) return std::nullopt;
        const bool ps = p->type.numel() == 1 && N != 1;
        for (int64_t i = 0; i < N; ++i) out.v[i] = (ps ? p->v[0] : p->v[i]) != 0 ? a->v[i] : b->v[i];
        break;
      }
      case Op::Not: {
        auto a = in(0);
        if (!a) return std::nullopt;
        for (int64_t i = 0; i < N; ++i)
          out.v[i] = t.dtype == DType::PRED ? (a->v[i] == 0) : (double)(~(int64_t)a->v[i]);
        break;
      }
      case Op::Neg: case Op::Abs: {
        auto a = in(0);
        if (!a) return std::nullopt;
        for (int64_t i = 0; i < N; ++i) out.v[i] = n.op == Op::Neg ? -a->v[i] : std::fabs(a->v[i]);
        break;
      }
      case Op::Add: case Op::Sub: case Op::Mul: case Op::Div: case Op::Max: case Op::Min:
      case Op::And: case Op::Or: case Op::Xor: {
        auto a = in(0), b = in(1);
        if (!a || !b) return std::nullopt;
        for (int64_t i = 0; i < N; ++i) {
          double x = a->v[i], y = b->v[i], r = 0;
          switch (n.op) {
            case Op::Add: r = x + y; break; case Op::Sub: r = x - y; break;
            case Op::Mul: r = x * y; break;
            case Op::Div: r = dtype_is_int(t.dtype) ? (y != 0 ? std::trunc(x / y) : 0) : x / y; break;
            case Op::Max: r = std::max(x, y); break; case Op::Min: r = std::min(x, y); break;
            case Op::And: r = (double)((int64_t)x & (int64_t)y); break;
            case Op::Or: r = (double)((int64_t)x | (int64_t)y); break;
            case Op::Xor: r = (double)((int64_t)x ^ (int64_t)y); break;
            default: break;
          }
          out.v[i] = cast_to(r, t.dtype);
        }
        break;
      }
      default: return std::nullopt;
    }
    memo[v] = out;
    return out;
  };
  return ev(root);
}

// ------------------------------------------------------------- matching ---
namespace {

struct Matcher {
  Graph& g;
  Uses u;
  explicit Matcher(Graph& gr) : g(gr), u(compute_uses(gr)) {}

  const Node& N(ValueRef v) const { return g.nodes.at(v.node); }
  const Node& N(int v) const { return g.nodes.at(v); }

  // Scalar value of a (broadcast of a) splat/scalar constant.
  std::optional<double> scalar_const(ValueRef v) const {
    for (int k = 0; k < 8; ++k) {
      const Node& n = N(v);
      if (n.op == Op::BroadcastInDim || n.op == Op::Reshape || n.op == Op::Convert) {
        v = n.operands[0];
        continue;
      }
      if (n.op == Op::Constant) {
        if (!n.cdata.splat && n.results[0].numel() != 1) return std::nullopt;
        return read_elem(n.cdata.bytes.data(), n.results[0].dtype);
      }
      return std::nullopt;
    }
    return std::nullopt;
  }
  // Follow broadcast_in_dim / reshape chains back to their source.
  ValueRef strip_bcast(ValueRef v, std::vector<int>* chain = nullptr) const {
    for (int k = 0; k < 16; ++k) {
      const Node& n = N(v);
      if (n.op != Op::BroadcastInDim && n.op != Op::Reshape) break;
      if (chain) chain->push_back(v.node);
      v = n.operands[0];
    }
    return v;
  }
  // Kind of a single-output reduction body: Add/Max/Min/Mul, or Parameter if complex.
  static Op reduce_kind(const Node& n) {
    if (n.regions.empty()) return Op::Parameter;
    const Graph& r = *n.regions[0];
    if (r.outputs.size() != 1) return Op::Parameter;
    const Node& b = r.nodes.at(r.outputs[0].node);
    if (b.operands.size() != 2) return Op::Parameter;
    if (r.nodes.at(b.operands[0].node).op != Op::Parameter ||
        r.nodes.at(b.operands[1].node).op != Op::Parameter)
      return Op::Parameter;
    return b.op;
  }
  // v = reduce_<kind>(x, dims={axis}) (+ optional max(., -inf)), through reshapes.
  bool is_reduce(ValueRef v, Op kind, int axis, ValueRef* x, std::vector<int>* chain) const {
    v = strip_bcast(v, chain);
    const Node* n = &N(v);
    if (kind == Op::Max && n->op == Op::Max) {  // max(reduce, -inf) from jnp.max(initial=-inf)
      for (int s = 0; s < 2; ++s) {
        auto c = scalar_const(n->operands[1 - s]);
        if (c && std::isinf(*c) && *c < 0) {
          if (chain) chain->push_back(v.node);
          v = strip_bcast(n->operands[s], chain);
          n = &N(v);
          break;
        }
      }
    }
    if (n->op != Op::Reduce || n->operands.size() != 2) return false;
    if (reduce_kind(*n) != kind) return false;
    const TensorType& in = g.type(n->operands[0]);
    if (n->dims.size() != 1 || n->dims[0] != (axis < 0 ? in.rank() + axis : axis)) return false;
    if (chain) chain->push_back(v.node);
    *x = n->operands[0];
    return true;
  }
  // True when every consumer of the nodes in `inner` is in `inner` or `outer`,
  // and none of them is a graph output.
  bool closed(const std::set<int>& inner, const std::set<int>& outer) const {
    for (int n : inner) {
      if (u.output_refs[n]) return false;
      for (int c : u.users[n])
        if (!inner.count(c) && !outer.count(c)) return false;
    }
    return true;
  }
  void replace_uses(ValueRef from, ValueRef to) {
    for (auto& n : g.nodes) {
      if (n.dead) continue;
      for (auto& o : n.operands)
        if (o == from) o = to;
    }
    for (auto& o : g.outputs)
      if (o == from) o = to;
  }

  // ---------------------------------------------------------------- SDPA --
  // softmax(x) along the last axis: div(exp(sub(x, bcast(max(x)))), bcast(sum(.)))
  bool softmax(ValueRef p, ValueRef* x, std::set<int>& nodes) const {
    const Node& d = N(p);
    if (d.op != Op::Div) return false;
    const int rank = g.type(p).rank();
    std::vector<int> ch;
    ValueRef e_from_sum;
    if (!is_reduce(d.operands[1], Op::Add, rank - 1, &e_from_sum, &ch)) return false;
    ValueRef e = d.operands[0];
    if (!(e == e_from_sum)) return false;
    const Node& ex = N(e);
    if (ex.op != Op::Exp) return false;
    const Node& sb = N(ex.operands[0]);
    if (sb.op != Op::Sub) return false;
    ValueRef xin = sb.operands[0], xm;
    if (!is_reduce(sb.operands[1], Op::Max, rank - 1, &xm, &ch)) return false;
    if (!(xm == xin)) return false;
    nodes.insert(p.node);
    nodes.insert(e.node);
    nodes.insert(ex.operands[0].node);
    for (int c : ch) nodes.insert(c);
    *x = xin;
    return true;
  }

  // Positions of (B, T|S, N, D) in a 4-D dot operand, given its batch and
  // contracting dims, when batch = {B, N} and contracting = {D}.
  static bool roles(const std::vector<int64_t>& batch, const std::vector<int64_t>& contract,
                    int rank, int64_t* b, int64_t* n, int64_t* t, int64_t* d) {
    if (rank != 4 || batch.size() != 2 || contract.size() != 1) return false;
    *b = batch[0];
    *n = batch[1];
    *d = contract[0];
    for (int64_t i = 0; i < 4; ++i)
      if (i != *b && i != *n && i != *d) *t = i;
    return true;
  }

  // The forward chain ending at dot_general node `i`:
  //   d1 = dot_general(Q, K) -> [* scale] -> [select(mask, ., -big)] ->
  //   softmax -> [convert] -> d2 = dot_general(P, V)
  // with batch {B, N}, Q / K contracted over the head dim and P over keys.
  struct AttnFwd {
    std::set<int> nodes;  // d1 .. d2, without the mask chain
    int d1 = -1, d2 = -1;
    ValueRef p, pb, e, sum;  // softmax quotient, its convert (== p if none), exp, row-sum reduce
    ValueRef mask{-1, 0};    // select predicate (through broadcasts), if masked
    int keep = 0;            // select operand that carries the logits (1 or 2)
    double scale = 1.0;
    int causal = 0;
    int64_t qb = 0, qn = 0, qt = 0, qd = 0, kb = 0, kn = 0, ks = 0, kd = 0;
    int64_t vb = 0, vn = 0, vs = 0, vd = 0;
    int64_t B = 0, T = 0, S = 0, H = 0, D = 0;
  };

  bool attn_forward(int i, AttnFwd& f) const {
    const Node& d2 = g.nodes[i];
    if (d2.dead || d2.op != Op::DotGeneral) return false;
    f.d2 = i;
    f.nodes.insert(i);
    // lhs of the second dot: softmax output, maybe converted
    ValueRef pv = d2.operands[0];
    f.pb = pv;
    if (N(pv).op == Op::Convert) { f.nodes.insert(pv.node); pv = N(pv).operands[0]; }
    f.p = pv;
    ValueRef logits;
    if (!softmax(pv, &logits, f.nodes)) return false;
    f.e = N(pv).operands[0];
    f.sum = strip_bcast(N(pv).operands[1]);
    if (N(logits).op == Op::Convert) { f.nodes.insert(logits.node); logits = N(logits).operands[0]; }
    // optional causal select
    if (N(logits).op == Op::Select) {
      const Node& s = N(logits);
      int keep = -1;
      for (int side = 1; side <= 2; ++side) {
        auto c = scalar_const(s.operands[side]);
        if (c && *c < -1e30) keep = 3 - side;
      }
      if (keep < 0) return false;
      std::vector<int> mch;
      ValueRef msrc = strip_bcast(s.operands[0], &mch);
      auto mask = host_eval(g, msrc, 1 << 24);
      if (!mask) return false;
      // mask source dims must end with (T, S); leading dims are 1
      const auto& md = mask->type.dims;
      if (md.size() < 2) return false;
      const int64_t T = md[md.size() - 2], S = md[md.size() - 1];
      bool lead1 = true;
      for (size_t k = 0; k + 2 < md.size(); ++k) lead1 &= md[k] == 1;
      if (!lead1) return false;
      bool is_tril = true, all_true = true;
      for (int64_t t = 0; t < T && (is_tril || all_true); ++t)
        for (int64_t sidx = 0; sidx < S; ++sidx) {
          bool m = mask->v[t * S + sidx] != 0;
          if (keep == 2) m = !m;  // select(pred, -big, x): pred marks masked-out
          if (m != (sidx <= t)) is_tril = false;
          if (!m) all_true = false;
        }
      if (!is_tril && !all_true) return false;
      f.causal = is_tril && !all_true;
      f.keep = keep;
      f.mask = msrc;
      f.nodes.insert(logits.node);
      for (int c : mch)
        if (u.count(c) == 1) f.nodes.insert(c);
      logits = s.operands[keep];
    }
    // optional scale
    {
      const Node& m = N(logits);
      if (m.op == Op::Mul || m.op == Op::Div) {
        for (int side = 0; side < 2; ++side) {
          if (m.op == Op::Div && side == 0) continue;
          auto c = scalar_const(m.operands[side]);
          if (c) {
            f.scale = m.op == Op::Mul ? *c : 1.0 / *c;
            f.nodes.insert(logits.node);
            logits = m.operands[1 - side];
            break;
          }
        }
      }
    }
    const Node& d1 = N(logits);
    if (d1.op != Op::DotGeneral) return false;
    f.d1 = logits.node;
    f.nodes.insert(logits.node);
    // roles of Q, K in d1 and of P, V in d2
    const TensorType &qt = g.type(d1.operands[0]), &kt = g.type(d1.operands[1]);
    const TensorType& vt = g.type(d2.operands[1]);
    if (!roles(d1.lhs_batch, d1.lhs_contract, qt.rank(), &f.qb, &f.qn, &f.qt, &f.qd)) return false;
    if (!roles(d1.rhs_batch, d1.rhs_contract, kt.rank(), &f.kb, &f.kn, &f.ks, &f.kd)) return false;
    // d1 result is [B, N, T, S]; d2 lhs is that, batch {0,1}, contract {3}
    if (d2.lhs_batch != std::vector<int64_t>{0, 1} || d2.lhs_contract != std::vector<int64_t>{3})
      return false;
    if (vt.rank() != 4 || d2.rhs_batch.size() != 2 || d2.rhs_contract.size() != 1) return false;
    f.vb = d2.rhs_batch[0], f.vn = d2.rhs_batch[1], f.vs = d2.rhs_contract[0], f.vd = -1;
    for (int64_t k = 0; k < 4; ++k)
      if (k != f.vb && k != f.vn && k != f.vs) f.vd = k;
    f.B = qt.dims[f.qb], f.T = qt.dims[f.qt], f.H = qt.dims[f.qn], f.D = qt.dims[f.qd];
    f.S = kt.dims[f.ks];
    if (kt.dims[f.kb] != f.B || kt.dims[f.kn] != f.H || kt.dims[f.kd] != f.D) return false;
    if (vt.dims[f.vb] != f.B || vt.dims[f.vn] != f.H || vt.dims[f.vs] != f.S) return false;
    if (qt.dtype != kt.dtype || qt.dtype != vt.dtype) return false;
    if (qt.dtype != DType::F32 && qt.dtype != DType::BF16) return false;
    if (f.D != 64) return false;
    return true;
  }

  static std::vector<int64_t> dense_strides(const TensorType& t) {
    std::vector<int64_t> s(t.rank(), 1);
    for (int k = t.rank() - 2; k >= 0; --k) s[k] = s[k + 1] * t.dims[k + 1];
    return s;
  }

  int match_sdpa() {
    int count = 0;
    for (size_t i = 0; i < g.nodes.size(); ++i) {
      AttnFwd f;
      if (!attn_forward((int)i, f)) continue;
      const Node& d1 = N(f.d1);
      const Node& d2 = N(f.d2);
      if (f.qd != 3 || f.kd != 3 || f.vd != 3) continue;  // head dim must be contiguous
      // output: d2 gives [B, N, T, D]; an exclusive transpose to BTND is folded in
      ValueRef outv{(int)i, 0};
      std::vector<int64_t> out_perm = {0, 1, 2, 3};  // out tensor dim k holds role out_perm[k]
      if (u.count((int)i) == 1 && u.output_refs[i] == 0) {
        const Node& tr = N(u.users[i][0]);
        if (tr.op == Op::Transpose) {
          outv = ValueRef{u.users[i][0], 0};
          out_perm = tr.dims;
          f.nodes.insert(outv.node);
        }
      }
      std::set<int> inner = f.nodes;
      inner.erase(outv.node);
      if (!closed(inner, {outv.node})) continue;
      // strides (elements) of role b,t,n in Q/K/V/O; role order of d2 output: B,N,T,D
      auto qs = dense_strides(g.type(d1.operands[0])), ks_ = dense_strides(g.type(d1.operands[1]));
      auto vs_ = dense_strides(g.type(d2.operands[1]));
      const TensorType& ot = g.type(outv);
      auto os = dense_strides(ot);
      // role r (0=B,1=N,2=T,3=D) sits at output position p where out_perm[p] == r
      int64_t o_pos[4];
      for (int p = 0; p < 4; ++p) o_pos[out_perm[p]] = p;
      if (o_pos[3] != 3) continue;
      Node fn;
      fn.op = Op::FusedSdpa;
      fn.operands = {d1.operands[0], d1.operands[1], d2.operands[1]};
      fn.results = {ot};
      fn.name = g.nodes[outv.node].name;
      fn.f_scale = (float)f.scale;
      fn.i_flags = f.causal;
      // dims: B T S N D ; strides: q(b,t,n) k(b,s,n) v(b,s,n) o(b,t,n)
      fn.dims = {f.B, f.T, f.S, f.H, f.D};
      fn.strides = {qs[f.qb], qs[f.qt], qs[f.qn], ks_[f.kb], ks_[f.ks], ks_[f.kn],
                    vs_[f.vb], vs_[f.vs], vs_[f.vn], os[o_pos[0]], os[o_pos[2]], os[o_pos[1]]};
      int fid = g.add(std::move(fn));
      replace_uses(outv, ValueRef{fid, 0});
      for (int n : f.nodes) g.nodes[n].dead = true;
      u = compute_uses(g);
      ++count;
    }
    return count;
  }

  // ------------------------------------------- attention with its backward --
  // Role letters of a tensor's dims: b batch, n head, t query, s key, h head dim.
  using Roles = std::string;
  // A value seen through its transposes: the source and each role's element
  // stride in the (dense, row-major) source.
  struct View {
    ValueRef src;
    std::map<char, int64_t> st;
    bool operator==(const View& o) const { return src == o.src && st == o.st; }
  };
  View view_of(ValueRef v, Roles r) const {
    for (int k = 0; k < 8 && N(v).op == Op::Transpose; ++k) {
      const Node& t = N(v);
      Roles rs(r.size(), '?');
      for (size_t d = 0; d < t.dims.size(); ++d) rs[t.dims[d]] = r[d];
      r = rs;
      v = t.operands[0];
    }
    View w;
    w.src = v;
    auto st = dense_strides(g.type(v));
    for (size_t d = 0; d < r.size(); ++d) w.st[r[d]] = st[d];
    return w;
  }
  static bool has(const std::vector<int64_t>& v, int64_t x) {
    return std::find(v.begin(), v.end(), x) != v.end();
  }
  // Roles of the other operand of dot `d`, given one operand's: paired batch
  // and contracting dims share a role, the single free dim gets `free_role`.
  static std::optional<Roles> other_roles(const Node& d, bool known_lhs, const Roles& known,
                                          int other_rank, char free_role) {
    const auto& kb = known_lhs ? d.lhs_batch : d.rhs_batch;
    const auto& kc = known_lhs ? d.lhs_contract : d.rhs_contract;
    const auto& ob = known_lhs ? d.rhs_batch : d.lhs_batch;
    const auto& oc = known_lhs ? d.rhs_contract : d.lhs_contract;
    if (kb.size() != ob.size() || kc.size() != oc.size()) return std::nullopt;
    Roles r(other_rank, '?');
    for (size_t k = 0; k < kb.size(); ++k) r[ob[k]] = known[kb[k]];
    for (size_t k = 0; k < kc.size(); ++k) r[oc[k]] = known[kc[k]];
    int free = 0;
    for (auto& c : r)
      if (c == '?') { c = free_role; ++free; }
    if (free != 1) return std::nullopt;
    return r;
  }
  // Roles of a dot_general result: batch dims, then lhs free, then rhs free.
  static Roles dot_out_roles(const Node& d, const Roles& lr, const Roles& rr) {
    Roles o;
    for (auto b : d.lhs_batch) o += lr[b];
    for (int k = 0; k < (int)lr.size(); ++k)
      if (!has(d.lhs_batch, k) && !has(d.lhs_contract, k)) o += lr[k];
    for (int k = 0; k < (int)rr.size(); ++k)
      if (!has(d.rhs_batch, k) && !has(d.rhs_contract, k)) o += rr[k];
    return o;
  }
  // The contracted role of a dot whose operands carry roles lr / rr (all
  // pairs must agree), or 0.
  static char contracted(const Node& d, const Roles& lr, const Roles& rr) {
    for (size_t k = 0; k < d.lhs_batch.size(); ++k)
      if (lr[d.lhs_batch[k]] != rr[d.rhs_batch[k]]) return 0;
    if (d.lhs_contract.size() != 1 || d.rhs_contract.size() != 1) return 0;
    const char c = lr[d.lhs_contract[0]];
    return c == rr[d.rhs_contract[0]] ? c : 0;
  }
  // Follow v through exclusive convert / transpose consumers; returns the last
  // value and its roles.
  ValueRef follow_out(ValueRef v, Roles& r) const {
    for (int k = 0; k < 4; ++k) {
      if (u.count(v.node) != 1 || u.output_refs[v.node]) break;
      const Node& c = N(u.users[v.node][0]);
      if (c.op == Op::Convert) {
        v = ValueRef{u.users[v.node][0], 0};
        continue;
      }
      if (c.op == Op::Transpose) {
        Roles rs;
        for (auto d : c.dims) rs += r[d];
        r = rs;
        v = ValueRef{u.users[v.node][0], 0};
        continue;
      }
      break;
    }
    return v;
  }

  // Symbolic form of the softmax backward: every value of the region between
  // dP and dS is a monomial factor c * P^p * sum^s * mask^m (no dP), or a sum
  // of terms, each a monomial times dP or times the row sum of (monomial * dP).
  // exp(x - max) is P * sum.
  struct Mono {
    int p = 0, s = 0, m = 0;
    double c = 1.0;
  };
  struct Term {
    Mono out, in;
    bool rowsum = false;
  };
  struct Sym {
    bool lin = false;  // terms (linear in dP) or a factor
    Mono f;
    std::vector<Term> t;
  };
  static Mono mono_mul(Mono a, const Mono& b, int sign = 1) {
    a.p += sign * b.p;
    a.s += sign * b.s;
    a.m = std::max(a.m, b.m);
    a.c = sign > 0 ? a.c * b.c : a.c / b.c;
    return a;
  }
  std::optional<Sym> sym_eval(ValueRef v, const AttnFwd& f, ValueRef dp, int64_t S,
                              std::map<ValueRef, std::optional<Sym>>& memo, int depth) const {
    auto it = memo.find(v);
    if (it != memo.end()) return it->second;
    auto done = [&](std::optional<Sym> r) { memo[v] = r; return r; };
    if (depth > 64) return done(std::nullopt);
    Sym r;
    if (v == dp) {
      r.lin = true;
      r.t.push_back(Term{});
      return done(r);
    }
    if (v == f.p) { r.f.p = 1; return done(r); }
    if (v == f.e) { r.f.p = 1; r.f.s = 1; return done(r); }
    if (strip_bcast(v) == f.sum) { r.f.s = 1; return done(r); }
    if (auto c = scalar_const(v)) { r.f.c = *c; return done(r); }
    const Node& n = N(v);
    auto ev = [&](int k) { return sym_eval(n.operands[k], f, dp, S, memo, depth + 1); };
    switch (n.op) {
      case Op::Mul: {
        auto a = ev(0), b = ev(1);
        if (!a || !b || (a->lin && b->lin)) return done(std::nullopt);
        if (!a->lin && !b->lin) { r.f = mono_mul(a->f, b->f); return done(r); }
        if (b->lin) std::swap(a, b);  // terms * factor
        r = *a;
        for (auto& t : r.t) t.out = mono_mul(t.out, b->f);
        return done(r);
      }
      case Op::Div: {
        auto a = ev(0), b = ev(1);
        if (!a || !b || b->lin || b->f.m || b->f.c == 0.0) return done(std::nullopt);
        if (!a->lin) { r.f = mono_mul(a->f, b->f, -1); return done(r); }
        r = *a;
        for (auto& t : r.t) t.out = mono_mul(t.out, b->f, -1);
        return done(r);
      }
      case Op::Add: case Op::Sub: {
        auto a = ev(0), b = ev(1);
        if (!a || !b || !a->lin || !b->lin) return done(std::nullopt);
        r = *a;
        for (Term t : b->t) {
          if (n.op == Op::Sub) t.out.c = -t.out.c;
          r.t.push_back(t);
        }
        return done(r);
      }
      case Op::Neg: {
        auto a = ev(0);
        if (!a) return done(std::nullopt);
        r = *a;
        if (r.lin) for (auto& t : r.t) t.out.c = -t.out.c;
        else r.f.c = -r.f.c;
        return done(r);
      }
      case Op::Select: {
        // select(mask, terms, 0) with the forward's mask and kept side
        if (f.mask.node < 0 || !(strip_bcast(n.operands[0]) == f.mask)) return done(std::nullopt);
        auto z = scalar_const(n.operands[3 - f.keep]);
        if (!z || *z != 0.0) return done(std::nullopt);
        auto a = ev(f.keep);
        if (!a || !a->lin) return done(std::nullopt);
        r = *a;
        for (auto& t : r.t) t.out.m = 1;
        return done(r);
      }
      case Op::Reduce: {
        // sum over the key axis of terms without row sums
        const TensorType& in = g.type(n.operands[0]);
        if (reduce_kind(n) != Op::Add || n.operands.size() != 2 || in.rank() != 4 ||
            n.dims != std::vector<int64_t>{3} || in.dims[3] != S)
          return done(std::nullopt);
        auto init = scalar_const(n.operands[1]);
        auto a = ev(0);
        if (!init || *init != 0.0 || !a || !a->lin) return done(std::nullopt);
        r = *a;
        for (auto& t : r.t) {
          if (t.rowsum) return done(std::nullopt);
          t.rowsum = true;
          t.in = t.out;  // the non-row-constant part stays inside the sum
          t.in.s = 0;
          t.in.c = 1.0;
          t.out.p = 0;
          t.out.m = 0;
        }
        return done(r);
      }
      case Op::Reshape: case Op::BroadcastInDim: case Op::Convert: {
        // layout ops between the row shape [B,N,T](,1) and [B,N,T,S]
        const TensorType &it = g.type(n.operands[0]), &ot = n.results[0];
        if (n.op == Op::Convert && (it.dtype != DType::F32 || ot.dtype != DType::F32))
          return done(std::nullopt);
        if (n.op != Op::Convert) {
          auto lead = [](const TensorType& t) {
            return std::vector<int64_t>(t.dims.begin(), t.dims.begin() + std::min(3, t.rank()));
          };
          if (it.rank() < 3 || ot.rank() < 3 || lead(it) != lead(ot)) return done(std::nullopt);
          if (n.op == Op::BroadcastInDim)
            for (int d = 0; d < std::min(3, it.rank()); ++d)
              if (n.dims[d] != d) return done(std::nullopt);
        }
        return done(ev(0));
      }
      default:
        return done(std::nullopt);
    }
  }
  // Merge equal terms; true when the form is scale * (P dP - P rowsum(P dP))
  // (mask factors allowed anywhere: P is zero where the mask is).
  static bool is_softmax_bwd(std::vector<Term> t, double scale) {
    std::vector<Term> m;
    for (auto& x : t) {
      bool merged = false;
      for (auto& y : m)
        if (y.rowsum == x.rowsum && y.out.p == x.out.p && y.out.s == x.out.s && y.out.m == x.out.m &&
            (!x.rowsum || (y.in.p == x.in.p && y.in.s == x.in.s && y.in.m == x.in.m))) {
          y.out.c += x.out.c;
          merged = true;
          break;
        }
      if (!merged) m.push_back(x);
    }
    double big = 0;
    for (auto& x : m) big = std::max(big, std::fabs(x.out.c));
    std::vector<Term> nz;
    for (auto& x : m)
      if (std::fabs(x.out.c) > 1e-9 * big) nz.push_back(x);
    if (nz.size() != 2) return false;
    const Term* d = nz[0].rowsum ? &nz[1] : &nz[0];
    const Term* r = nz[0].rowsum ? &nz[0] : &nz[1];
    if (d->rowsum || !r->rowsum) return false;
    auto near = [](double a, double b) { return std::fabs(a - b) <= 1e-6 * std::fabs(b); };
    return d->out.p == 1 && d->out.s == 0 && near(d->out.c, scale) && r->out.p == 1 && r->out.s == 0 &&
           r->in.p == 1 && r->in.s == 0 && near(r->out.c, -scale);
  }

  // Causal or full attention whose probabilities also feed its backward (a
  // jax.grad / value_and_grad program): the forward chain plus
  //   dV = P^T dO, dP = dO V^T, dS = softmax-bwd(P, dP) * scale,
  //   dQ = dS K, dK = dS^T Q
  // becomes FusedSdpa (O and the row statistic) + FusedSdpaBwd (dQ, dK, dV).
  // bf16 operands, head dim 64, T == S <= 256 (the backward kernel's limits).
  int match_sdpa_train() {
    int count = 0;
    for (size_t i = 0; i < g.nodes.size(); ++i) {
      AttnFwd f;
      if (!attn_forward((int)i, f)) continue;
      if (N(f.pb).op != Op::Convert) continue;  // bf16 probabilities
      if (g.type(f.pb).dtype != DType::BF16 || f.T != f.S || f.T > 256) continue;
      const Node& d1 = N(f.d1);
      const Node& d2 = N(f.d2);
      Roles qr(4, '?'), kr(4, '?'), vr(4, '?');
      qr[f.qb] = 'b', qr[f.qn] = 'n', qr[f.qt] = 't', qr[f.qd] = 'h';
      kr[f.kb] = 'b', kr[f.kn] = 'n', kr[f.ks] = 's', kr[f.kd] = 'h';
      vr[f.vb] = 'b', vr[f.vn] = 'n', vr[f.vs] = 's', vr[f.vd] = 'h';
      const View qv = view_of(d1.operands[0], qr), kv = view_of(d1.operands[1], kr);
      const View vv = view_of(d2.operands[1], vr);
      // dV = dot(P, dO): P's only consumer besides d2
      const auto& pbu = u.users[f.pb.node];
      if (pbu.size() != 2 || u.output_refs[f.pb.node]) continue;
      const int dvi = pbu[0] == f.d2 ? pbu[1] : pbu[0];
      const Node& dvn = N(dvi);
      if (dvn.op != Op::DotGeneral || dvn.operands[0] == dvn.operands[1]) continue;
      const bool p_lhs = dvn.operands[0] == f.pb;
      const ValueRef gx = dvn.operands[p_lhs ? 1 : 0];
      auto gr = other_roles(dvn, p_lhs, "bnts", g.type(gx).rank(), 'h');
      if (!gr || contracted(dvn, p_lhs ? "bnts" : *gr, p_lhs ? *gr : "bnts") != 't') continue;
      const View gv = view_of(gx, *gr);
      Roles dvr = p_lhs ? dot_out_roles(dvn, "bnts", *gr) : dot_out_roles(dvn, *gr, "bnts");
      // dP = dot(dO, V) with result roles b n t s, and its f32 value
      int dpi = -1;
      for (size_t k = 0; k < g.nodes.size() && dpi < 0; ++k) {
        const Node& c = g.nodes[k];
        if (c.dead || c.op != Op::DotGeneral || (int)k == dvi) continue;
        if (g.type(c.operands[0]).rank() != 4 || g.type(c.operands[1]).rank() != 4) continue;
        Roles lr(4, '?'), rr(4, '?');
        // lhs: dO (roles from its batch / contract dims), rhs: V
        auto try_roles = [&](const std::vector<int64_t>& bd, const std::vector<int64_t>& cd, char fr,
                             Roles& out) {
          if (bd.size() != 2 || cd.size() != 1) return false;
          out[bd[0]] = 'b', out[bd[1]] = 'n', out[cd[0]] = 'h';
          for (auto& ch : out)
            if (ch == '?') ch = fr;
          return true;
        };
        if (!try_roles(c.lhs_batch, c.lhs_contract, 't', lr) || !try_roles(c.rhs_batch, c.rhs_contract, 's', rr))
          continue;
        if (!(view_of(c.operands[0], lr) == gv) || !(view_of(c.operands[1], rr) == vv)) continue;
        if (dot_out_roles(c, lr, rr) != "bnts") continue;
        dpi = (int)k;
      }
      if (dpi < 0) continue;
      ValueRef dp{dpi, 0};
      if (g.type(dp).dtype != DType::F32) {
        if (u.count(dpi) != 1 || u.output_refs[dpi] || N(u.users[dpi][0]).op != Op::Convert) continue;
        dp = ValueRef{u.users[dpi][0], 0};
        if (g.type(dp).dtype != DType::F32) continue;
      }
      // dS: the value both remaining products read; search forward from dP
      std::set<int> region;
      std::vector<int> stack = {dp.node};
      std::set<int> dots;
      bool bad = false;
      while (!stack.empty() && !bad) {
        const int x = stack.back();
        stack.pop_back();
        if (!region.insert(x).second) continue;
        if (region.size() > 64) bad = true;
        for (int c : u.users[x]) {
          const Op op = g.nodes[c].op;
          if (op == Op::DotGeneral) dots.insert(c);
          else if (op == Op::Add || op == Op::Sub || op == Op::Mul || op == Op::Div || op == Op::Neg ||
                   op == Op::Select || op == Op::Reduce || op == Op::Reshape ||
                   op == Op::BroadcastInDim || op == Op::Convert)
            stack.push_back(c);
          else bad = true;
        }
      }
      if (bad || dots.size() != 2) continue;
      const int da = *dots.begin(), db = *dots.rbegin();
      ValueRef ds{-1, 0};
      for (const auto& o : N(da).operands)
        for (const auto& o2 : N(db).operands)
          if (o == o2 && region.count(o.node)) ds = o;
      if (ds.node < 0 || g.type(ds).dtype != DType::F32) continue;
      std::map<ValueRef, std::optional<Sym>> memo;
      auto sym = sym_eval(ds, f, dp, f.S, memo, 0);
      if (!sym || !sym->lin || !is_softmax_bwd(sym->t, f.scale)) continue;
      // dQ = dot(dS, K) over keys, dK = dot(dS, Q) over queries
      ValueRef dqf{-1, 0}, dkf{-1, 0};
      Roles dqr, dkr;
      bool ok = true;
      for (int di : {da, db}) {
        const Node& dn = N(di);
        const bool s_lhs = dn.operands[0] == ds;
        const ValueRef other = dn.operands[s_lhs ? 1 : 0];
        if (dn.operands[0] == dn.operands[1]) { ok = false; break; }
        auto orl = other_roles(dn, s_lhs, "bnts", g.type(other).rank(), 'h');
        if (!orl) { ok = false; break; }
        const char c = contracted(dn, s_lhs ? "bnts" : *orl, s_lhs ? *orl : "bnts");
        Roles outr = s_lhs ? dot_out_roles(dn, "bnts", *orl) : dot_out_roles(dn, *orl, "bnts");
        if (c == 's') {  // dQ: the other operand is K (its query role is 's' there)
          Roles kk = *orl;
          if (!(view_of(other, kk) == kv)) { ok = false; break; }
          dqr = outr;
          dqf = follow_out(ValueRef{di, 0}, dqr);
        } else if (c == 't') {  // dK: the other operand is Q (roles t for its rows)
          Roles qq = *orl;
          if (!(view_of(other, qq) == qv)) { ok = false; break; }
          dkr = outr;
          dkf = follow_out(ValueRef{di, 0}, dkr);
        } else {
          ok = false;
          break;
        }
      }
      if (!ok || dqf.node < 0 || dkf.node < 0) continue;
      ValueRef dvf = follow_out(ValueRef{dvi, 0}, dvr);
      // O: d2's result [B, N, T, D], through an exclusive transpose
      Roles orr = "bnth";
      ValueRef of{f.d2, 0};
      if (u.count(f.d2) == 1 && !u.output_refs[f.d2] && N(u.users[f.d2][0]).op == Op::Transpose)
        of = follow_out(of, orr);
      for (ValueRef x : {dqf, dkf, dvf, of})
        if (g.type(x).dtype != DType::BF16) ok = false;
      for (ValueRef x : {qv.src, kv.src, vv.src, gv.src})
        if (g.type(x).dtype != DType::BF16) ok = false;
      if (!ok) continue;
      // strides by role; the head dim must be contiguous and every stride a
      // multiple of 8 elements (16 bytes)
      auto rs = [&](ValueRef x, const Roles& r) {
        std::map<char, int64_t> m;
        auto st = dense_strides(g.type(x));
        for (size_t d = 0; d < r.size(); ++d) m[r[d]] = st[d];
        return m;
      };
      auto oS = rs(of, orr), dqS = rs(dqf, dqr), dkS = rs(dkf, dkr), dvS = rs(dvf, dvr);
      // dK's and dV's row role is the key 's'
      std::vector<std::map<char, int64_t>> all = {qv.st, kv.st, vv.st, oS, gv.st, dqS, dkS, dvS};
      const char row[8] = {'t', 's', 's', 't', 't', 't', 's', 's'};
      std::vector<int64_t> strides;
      for (int k = 0; k < 8 && ok; ++k) {
        auto& m = all[k];
        if (!m.count('b') || !m.count('n') || !m.count(row[k]) || !m.count('h') || m['h'] != 1) ok = false;
        else strides.insert(strides.end(), {m['b'], m[row[k]], m['n']});
      }
      for (auto x : strides) ok = ok && x % 8 == 0;
      if (!ok) continue;
      Node fw;
      fw.op = Op::FusedSdpa;
      fw.operands = {qv.src, kv.src, vv.src};
      TensorType lt;
      lt.dtype = DType::F32;
      lt.dims = {f.B, f.H, f.T};
      fw.results = {g.type(of), lt};
      fw.name = g.nodes[of.node].name;
      fw.f_scale = (float)f.scale;
      fw.i_flags = f.causal | 2;
      fw.dims = {f.B, f.T, f.S, f.H, f.D};
      fw.strides = std::vector<int64_t>(strides.begin(), strides.begin() + 12);
      const int fid = g.add(std::move(fw));
      Node bw;
      bw.op = Op::FusedSdpaBwd;
      bw.operands = {qv.src, kv.src, vv.src, ValueRef{fid, 0}, gv.src, ValueRef{fid, 1}};
      bw.results = {g.type(dqf), g.type(dkf), g.type(dvf)};
      bw.name = g.nodes[dqf.node].name;
      bw.f_scale = (float)f.scale;
      bw.i_flags = f.causal;
      bw.dims = {f.B, f.T, f.S, f.H, f.D};
      bw.strides = strides;
      const int bid = g.add(std::move(bw));
      replace_uses(of, ValueRef{fid, 0});
      replace_uses(dqf, ValueRef{bid, 0});
      replace_uses(dkf, ValueRef{bid, 1});
      replace_uses(dvf, ValueRef{bid, 2});
      dce(g);
      u = compute_uses(g);
      ++count;
    }
    return count;
  }

  // ----------------------------------------------------------- LayerNorm --
  // v == x * c or x / c' with c == 1/n (relative 1e-6): returns x
  bool mean_scale(ValueRef v, double n, ValueRef* x, std::set<int>& nodes) const {
    const Node& m = N(v);
    if (m.op == Op::Mul) {
      for (int s = 0; s < 2; ++s) {
        auto c = scalar_const(m.operands[s]);
        if (c && std::fabs(*c * n - 1.0) < 1e-6) { *x = m.operands[1 - s]; nodes.insert(v.node); return true; }
      }
    }
    if (m.op == Op::Div) {
      auto c = scalar_const(m.operands[1]);
      if (c && std::fabs(*c - n) < 1e-6 * n) { *x = m.operands[0]; nodes.insert(v.node); return true; }
    }
    return false;
  }
  // v = mean over last axis of `x`: returns x
  bool mean_of(ValueRef v, int64_t cols, ValueRef* x, std::set<int>& nodes) const {
    std::vector<int> ch;
    ValueRef s = strip_bcast(v, &ch);
    ValueRef r;
    std::set<int> tmp;
    if (!mean_scale(s, (double)cols, &r, tmp)) return false;
    ValueRef in;
    std::vector<int> ch2;
    if (!is_reduce(r, Op::Add, -1, &in, &ch2)) return false;
    for (int c : ch) nodes.insert(c);
    for (int c : ch2) nodes.insert(c);
    nodes.insert(tmp.begin(), tmp.end());
    *x = in;
    return true;
  }
  bool is_square_of(ValueRef v, ValueRef* x) const {
    const Node& m = N(v);
    if (m.op == Op::Mul && m.operands[0] == m.operands[1]) { *x = m.operands[0]; return true; }
    if (m.op == Op::Pow) {
      auto c = scalar_const(m.operands[1]);
      if (c && *c == 2.0) { *x = m.operands[0]; return true; }
    }
    return false;
  }

  int match_layer_norm() {
    int count = 0;
    for (size_t i = 0; i < g.nodes.size(); ++i) {
      Node& rs = g.nodes[i];
      if (rs.dead || rs.op != Op::Rsqrt) continue;
      std::set<int> nodes{(int)i};
      // rsqrt(var + eps)
      const Node& a = N(rs.operands[0]);
      if (a.op != Op::Add) continue;
      double eps = 0;
      ValueRef var;
      bool got = false;
      for (int s = 0; s < 2 && !got; ++s) {
        auto c = scalar_const(a.operands[s]);
        if (c) { eps = *c; var = a.operands[1 - s]; got = true; }
      }
      if (!got) continue;
      nodes.insert(rs.operands[0].node);
      // find the normalized product among users of bcast(rsqrt)
      // candidates: walk users through reshape/broadcast to a Mul
      std::vector<int> frontier{(int)i};
      std::vector<int> bchain;
      int mul_node = -1;
      for (int step = 0; step < 4 && mul_node < 0; ++step) {
        std::vector<int> next;
        for (int f : frontier)
          for (int c : u.users[f]) {
            const Node& cn = N(c);
            if (cn.op == Op::BroadcastInDim || cn.op == Op::Reshape) { next.push_back(c); bchain.push_back(c); }
            else if (cn.op == Op::Mul && mul_node < 0) mul_node = c;
          }
        frontier = next;
      }
      if (mul_node < 0) continue;
      const TensorType& yt = g.type(ValueRef{mul_node, 0});
      if (yt.rank() < 1) continue;
      const int64_t cols = yt.dims.back();
      const int64_t rows = yt.numel() / cols;
      if (yt.dtype != DType::F32 && yt.dtype != DType::BF16) continue;
      for (int c : bchain) nodes.insert(c);
      // Form B: mul_node = bcast(r) * bcast(gamma); the product with the
      // centered input is its consumer.  Form A: mul_node = centered * bcast(r).
      ValueRef gamma{-1, 0}, beta{-1, 0};
      int y0 = mul_node;
      ValueRef centered{-1, 0};
      {
        const Node& m = N(mul_node);
        int rside = -1;
        for (int s = 0; s < 2; ++s) {
          ValueRef src = strip_bcast(m.operands[s]);
          if (src.node == (int)i) rside = s;
        }
        if (rside < 0) continue;
        ValueRef other = m.operands[1 - rside];
        ValueRef osrc = strip_bcast(other);
        if (g.type(osrc).rank() == 1 && g.type(osrc).dims[0] == cols &&
            N(other).op == Op::BroadcastInDim) {
          // Form B
          gamma = osrc;
          nodes.insert(other.node);
          if (u.count(mul_node) != 1) continue;
          y0 = u.users[mul_node][0];
          const Node& m2 = N(y0);
          if (m2.op != Op::Mul) continue;
          centered = m2.operands[0].node == mul_node ? m2.operands[1] : m2.operands[0];
          nodes.insert(mul_node);
        } else {
          centered = other;
        }
      }
      // centered = h - bcast(mean(h))  (LayerNorm) or h (RMSNorm)
      int kind = 0;
      ValueRef h{-1, 0}, mean{-1, 0};
      {
        const Node& c = N(centered);
        ValueRef hh;
        std::set<int> mn;
        if (c.op == Op::Sub && mean_of(c.operands[1], cols, &hh, mn) && hh == c.operands[0]) {
          h = hh;
          mean = c.operands[1];
          nodes.insert(centered.node);
          nodes.insert(mn.begin(), mn.end());
        } else {
          h = centered;
          kind = 1;
        }
      }
      // variance forms
      {
        std::set<int> vn;
        ValueRef x, sq;
        bool ok = false;
        std::vector<int> vch;
        ValueRef vv = strip_bcast(var, &vch);
        if (kind == 0) {
          // two-pass: mean((h - mean)^2)
          if (mean_of(vv, cols, &sq, vn) && is_square_of(sq, &x)) {
            const Node& xc = N(x);
            ValueRef h2;
            std::set<int> mn2;
            if (xc.op == Op::Sub && xc.operands[0] == h && mean_of(xc.operands[1], cols, &h2, mn2) && h2 == h) {
              ok = true;
              vn.insert(sq.node);
              vn.insert(x.node);
              vn.insert(mn2.begin(), mn2.end());
            }
          }
          // fast variance: [max(0, ] mean(h*h) - mean(h)^2 [)]
          if (!ok) {
            ValueRef w = vv;
            const Node& mx = N(w);
            if (mx.op == Op::Max) {
              for (int s = 0; s < 2; ++s) {
                auto c = scalar_const(mx.operands[s]);
                if (c && *c == 0.0) { vn.insert(w.node); w = mx.operands[1 - s]; break; }
              }
            }
            const Node& sb = N(w);
            ValueRef m2in, msq, hm;
            std::set<int> t1, t2;
            if (sb.op == Op::Sub && mean_of(sb.operands[0], cols, &m2in, t1) &&
                is_square_of(m2in, &x) && x == h && is_square_of(sb.operands[1], &msq) &&
                mean_of(msq, cols, &hm, t2) && hm == h) {
              ok = true;
              vn.insert(w.node);
              vn.insert(m2in.node);
              vn.insert(sb.operands[1].node);
              vn.insert(t1.begin(), t1.end());
              vn.insert(t2.begin(), t2.end());
            }
          }
        } else {
          if (mean_of(vv, cols, &sq, vn) && is_square_of(sq, &x) && x == h) {
            ok = true;
            vn.insert(sq.node);
          }
        }
        if (!ok) continue;
        nodes.insert(vn.begin(), vn.end());
        for (int c : vch) nodes.insert(c);
        nodes.insert(var.node);
      }
      // optional * bcast(gamma) (form A) and + bcast(beta)
      int yend = y0;
      auto affine = [&](Op op, ValueRef* param) {
        if (u.count(yend) != 1 || u.output_refs[yend]) return;
        int c = u.users[yend][0];
        const Node& cn = N(c);
        if (cn.op != op) return;
        ValueRef other = cn.operands[0].node == yend ? cn.operands[1] : cn.operands[0];
        if (N(other).op != Op::BroadcastInDim) return;
        ValueRef src = strip_bcast(other);
        const TensorType& st = g.type(src);
        if (st.rank() != 1 || st.dims[0] != cols || st.dtype != yt.dtype) return;
        const Node& bn = N(other);
        if (bn.dims.size() != 1 || bn.dims[0] != yt.rank() - 1) return;
        *param = src;
        nodes.insert(yend);
        nodes.insert(other.node);
        yend = c;
      };
      if (gamma.node < 0) affine(Op::Mul, &gamma);
      affine(Op::Add, &beta);
      if (gamma.node >= 0 && g.type(gamma).dtype != yt.dtype) continue;
      // residual: h = x + r (same shape)
      ValueRef x = h, res{-1, 0};
      bool h_external = false;
      if (N(h).op == Op::Add && g.type(N(h).operands[0]) == g.type(N(h).operands[1]) &&
          g.type(h) == yt) {
        x = N(h).operands[0];
        res = N(h).operands[1];
      }
      if (g.type(x) != yt) continue;
      // guard: everything but the final node and h is internal
      std::set<int> inner = nodes;
      inner.erase(yend);
      inner.erase(h.node);
      if (!closed(inner, {yend})) continue;
      if (res.node >= 0) {
        for (int c : u.users[h.node])
          if (!inner.count(c) && c != yend) h_external = true;
        if (u.output_refs[h.node]) h_external = true;
      }
      (void)rows;
      Node f;
      f.op = Op::FusedLayerNorm;
      f.operands = {x};
      int flags = kind;
      if (res.node >= 0) { f.operands.push_back(res); flags |= 2; }
      if (gamma.node >= 0) { f.operands.push_back(gamma); flags |= 4; }
      if (beta.node >= 0) { f.operands.push_back(beta); flags |= 8; }
      if (h_external) flags |= 16;
      f.i_flags = flags;
      f.f_eps = (float)eps;
      f.results = {yt};
      if (h_external) f.results.push_back(yt);
      f.name = g.nodes[yend].name;
      (void)mean;
      int fid = g.add(std::move(f));
      replace_uses(ValueRef{yend, 0}, ValueRef{fid, 0});
      if (h_external) replace_uses(h, ValueRef{fid, 1});
      for (int n : nodes) g.nodes[n].dead = true;
      g.nodes[yend].dead = true;
      if (res.node >= 0) g.nodes[h.node].dead = true;
      u = compute_uses(g);
      ++count;
    }
    return count;
  }
};

}  // namespace

MatchStats match_patterns(Graph& g) {
  MatchStats st;
  Matcher m(g);
  st.sdpa = m.match_sdpa();
  // B200_BF16_ROUND_EACH_OP=1 compiles a program that rounds after every bf16
  // op (to be compared element by element with an interpreter that does the
  // same); the fused attention backward rounds only at its outputs, so that
  // mode keeps the attention backward as the program writes it.
  const char* each = getenv("B200_BF16_ROUND_EACH_OP");
  if (!(each && each[0] == '1')) st.sdpa_train = m.match_sdpa_train();
  st.layer_norm = m.match_layer_norm();
  if (st.sdpa || st.sdpa_train || st.layer_norm) dce(g);
  return st;
}

std::string dump_graph(const Graph& g) {
  std::ostringstream os;
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& n = g.nodes[i];
    if (n.dead) continue;
    os << "%" << i << " = " << op_name(n.op) << "(";
    for (size_t k = 0; k < n.operands.size(); ++k)
      os << (k ? ", " : "") << "%" << n.operands[k].node
         << (n.operands[k].idx ? "#" + std::to_string(n.operands[k].idx) : "");
    os << ")";
    if (n.op == Op::FusedSdpa || n.op == Op::FusedSdpaBwd)
      os << " {scale=" << n.f_scale << ", causal=" << (n.i_flags & 1) << "}";
    if (n.op == Op::FusedLayerNorm) os << " {eps=" << n.f_eps << ", flags=" << n.i_flags << "}";
    if (n.op == Op::CustomCall) os << " {target=" << n.target << "}";
    os << " :";
    for (auto& r : n.results) os << " " << r.str();
    os << "\n";
  }
  os << "return";
  for (auto& o : g.outputs) os << " %" << o.node << (o.idx ? "#" + std::to_string(o.idx) : "");
  os << "\n";
  return os.str();
}

}  // namespace b200
