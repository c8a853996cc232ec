// Backward custom calls of the reference's custom_vjp primitives, expanded into
// StableHLO at compile time so that the ordinary fusion planner lowers them
// (GEMMs on tcgen05, softmax / normalisation pieces as fused loop and reduce
// kernels):
//
//   mlx_sdpa_bwd(Q, K, V, dO) {"scale": s} -> (dQ, dK, dV), layout (B, T, N, H)
//     reference src/jax_mlx_pjrt.cpp:8152-8206 (mx::vjp of
//     fast::scaled_dot_product_attention); math of src/jax_mlx/sdpa.py:65-87:
//     W = softmax(Q K^T s), dV = W^T dO, dW = dO V^T,
//     dS = W (dW - rowsum(dW W)) s, dQ = dS K, dK = dS^T Q.
//   mlx_layer_norm_bwd(x, w, b, dy) {"eps": e} -> (dx, dw, db), last axis
//     reference src/jax_mlx_pjrt.cpp:8238-8281 (mx::vjp of fast::layer_norm);
//     math of src/jax_mlx/layer_norm.py:59-76:
//     xhat = (x - mean) rstd, g = dy w,
//     dx = rstd (g - mean(g) - xhat mean(g xhat)), dw = sum(dy xhat), db = sum(dy).
//
// Arithmetic runs in f32 whatever the operand type (bf16 operands are widened
// and the results rounded back), as MLX accumulates these in f32.  bf16
// attention with head dim 64 and at most 256 positions skips the expansion:
// fused_sdpa_bwd_call puts the tcgen05 forward (which keeps each row's
// softmax statistic) and the fused backward kernel in its place, with f32
// accumulation, P rounded to bf16 for dV and dS kept to about 16 bits.
#include "custom_calls.h"

#include <cstdio>
#include <sstream>

namespace b200 {
namespace {

// Minimal StableHLO text emitter (pretty printing, as the parser reads it).
struct Emit {
  std::ostringstream body;
  int next = 0;
  struct V {
    std::string name;
    std::vector<int64_t> dims;
    std::string dt;
  };
  static std::string ty(const std::vector<int64_t>& d, const std::string& dt) {
    std::string s = "tensor<";
    for (auto x : d) s += std::to_string(x) + "x";
    return s + dt + ">";
  }
  static std::string ty(const V& v) { return ty(v.dims, v.dt); }
  static std::string ints(const std::vector<int64_t>& v) {
    std::string s;
    for (size_t i = 0; i < v.size(); ++i) s += (i ? ", " : "") + std::to_string(v[i]);
    return s;
  }
  V fresh(const std::vector<int64_t>& d, const std::string& dt) {
    return V{"%v" + std::to_string(next++), d, dt};
  }
  V convert(const V& x, const std::string& dt) {
    if (x.dt == dt) return x;
    V o = fresh(x.dims, dt);
    body << "    " << o.name << " = stablehlo.convert " << x.name << " : (" << ty(x) << ") -> "
         << ty(o) << "\n";
    return o;
  }
  V scalar(double v, const std::vector<int64_t>& d) {
    V c = fresh({}, "f32");
    char buf[64];
    std::snprintf(buf, sizeof buf, "%.9e", v);
    body << "    " << c.name << " = stablehlo.constant dense<" << buf << "> : tensor<f32>\n";
    return bcast(c, d, {});
  }
  V bcast(const V& x, const std::vector<int64_t>& d, const std::vector<int64_t>& dims) {
    V o = fresh(d, x.dt);
    body << "    " << o.name << " = stablehlo.broadcast_in_dim " << x.name << ", dims = ["
         << ints(dims) << "] : (" << ty(x) << ") -> " << ty(o) << "\n";
    return o;
  }
  V bin(const char* op, const V& a, const V& b) {
    V o = fresh(a.dims, a.dt);
    body << "    " << o.name << " = stablehlo." << op << " " << a.name << ", " << b.name << " : "
         << ty(o) << "\n";
    return o;
  }
  V un(const char* op, const V& a) {
    V o = fresh(a.dims, a.dt);
    body << "    " << o.name << " = stablehlo." << op << " " << a.name << " : " << ty(o) << "\n";
    return o;
  }
  V reduce(const V& x, const std::vector<int64_t>& dims, bool max) {
    std::vector<int64_t> od;
    for (size_t i = 0; i < x.dims.size(); ++i) {
      bool r = false;
      for (auto d : dims) r |= d == (int64_t)i;
      if (!r) od.push_back(x.dims[i]);
    }
    V init = fresh({}, x.dt);
    body << "    " << init.name << " = stablehlo.constant dense<"
         << (max ? "0xFF800000" : "0.000000e+00") << "> : tensor<f32>\n";
    V o = fresh(od, x.dt);
    body << "    " << o.name << " = stablehlo.reduce(" << x.name << " init: " << init.name
         << ") applies stablehlo." << (max ? "maximum" : "add") << " across dimensions = ["
         << ints(dims) << "] : (" << ty(x) << ", tensor<f32>) -> " << ty(o) << "\n";
    return o;
  }
  V dot(const V& a, const V& b, const std::vector<int64_t>& lb, const std::vector<int64_t>& rb,
        const std::vector<int64_t>& lc, const std::vector<int64_t>& rc) {
    std::vector<int64_t> d;
    for (auto i : lb) d.push_back(a.dims[i]);
    auto has = [](const std::vector<int64_t>& v, int64_t x) {
      for (auto y : v)
        if (y == x) return true;
      return false;
    };
    for (int64_t i = 0; i < (int64_t)a.dims.size(); ++i)
      if (!has(lb, i) && !has(lc, i)) d.push_back(a.dims[i]);
    for (int64_t i = 0; i < (int64_t)b.dims.size(); ++i)
      if (!has(rb, i) && !has(rc, i)) d.push_back(b.dims[i]);
    V o = fresh(d, "f32");
    body << "    " << o.name << " = stablehlo.dot_general " << a.name << ", " << b.name
         << ", batching_dims = [" << ints(lb) << "] x [" << ints(rb) << "], contracting_dims = ["
         << ints(lc) << "] x [" << ints(rc) << "], precision = [DEFAULT, DEFAULT] : (" << ty(a)
         << ", " << ty(b) << ") -> " << ty(o) << "\n";
    return o;
  }
  V transpose(const V& x, const std::vector<int64_t>& perm) {
    std::vector<int64_t> d;
    for (auto p : perm) d.push_back(x.dims[p]);
    V o = fresh(d, x.dt);
    body << "    " << o.name << " = stablehlo.transpose " << x.name << ", dims = [" << ints(perm)
         << "] : (" << ty(x) << ") -> " << ty(o) << "\n";
    return o;
  }
};

std::string dt_str(DType t) {
  switch (t) {
    case DType::F32: return "f32";
    case DType::BF16: return "bf16";
    default: throw PjrtErr(12, std::string("custom call operand type ") + dtype_name(t) + " is not supported");
  }
}

float config_value(const std::string& cfg, const char* key, float dflt) {
  auto pos = cfg.find(key);
  if (pos == std::string::npos) return dflt;
  pos = cfg.find(':', pos);
  if (pos == std::string::npos) return dflt;
  return std::stof(cfg.substr(pos + 1));
}

std::string module_text(Emit& e, const std::vector<Emit::V>& params, const std::vector<Emit::V>& outs) {
  std::ostringstream m;
  m << "module @custom_call_expansion {\n  func.func public @main(";
  for (size_t i = 0; i < params.size(); ++i)
    m << (i ? ", " : "") << params[i].name << ": " << Emit::ty(params[i]);
  m << ") -> (";
  for (size_t i = 0; i < outs.size(); ++i) m << (i ? ", " : "") << Emit::ty(outs[i]);
  m << ") {\n" << e.body.str() << "    return ";
  for (size_t i = 0; i < outs.size(); ++i) m << (i ? ", " : "") << outs[i].name;
  m << " : ";
  for (size_t i = 0; i < outs.size(); ++i) m << (i ? ", " : "") << Emit::ty(outs[i]);
  m << "\n  }\n}\n";
  return m.str();
}

std::string sdpa_bwd(const Node& n, const std::vector<TensorType>& in) {
  if (in.size() != 4 || in[0].rank() != 4)
    throw PjrtErr(3, "mlx_sdpa_bwd expects (Q, K, V, dO) of rank 4 (B, T, N, H)");
  const float scale = config_value(n.backend_config, "scale", 1.0f);
  Emit e;
  std::vector<Emit::V> P;
  for (size_t i = 0; i < 4; ++i) P.push_back(Emit::V{"%p" + std::to_string(i), in[i].dims, dt_str(in[i].dtype)});
  auto q = e.convert(P[0], "f32"), k = e.convert(P[1], "f32"), v = e.convert(P[2], "f32"),
       g = e.convert(P[3], "f32");
  auto logits = e.bin("multiply", e.dot(q, k, {0, 2}, {0, 2}, {3}, {3}),
                      e.scalar(scale, {in[0].dims[0], in[0].dims[2], in[0].dims[1], in[1].dims[1]}));
  const std::vector<int64_t> row_dims = {0, 1, 2};
  auto m = e.bcast(e.reduce(logits, {3}, true), logits.dims, row_dims);
  auto ex = e.un("exponential", e.bin("subtract", logits, m));
  auto w = e.bin("divide", ex, e.bcast(e.reduce(ex, {3}, false), logits.dims, row_dims));
  auto dv = e.transpose(e.dot(w, g, {0, 1}, {0, 2}, {2}, {1}), {0, 2, 1, 3});
  auto dw = e.dot(g, v, {0, 2}, {0, 2}, {3}, {3});
  auto t = e.bcast(e.reduce(e.bin("multiply", dw, w), {3}, false), logits.dims, row_dims);
  auto ds = e.bin("multiply", e.bin("multiply", w, e.bin("subtract", dw, t)),
                  e.scalar(scale, logits.dims));
  auto dq = e.transpose(e.dot(ds, k, {0, 1}, {0, 2}, {3}, {1}), {0, 2, 1, 3});
  auto dk = e.transpose(e.dot(ds, q, {0, 1}, {0, 2}, {2}, {1}), {0, 2, 1, 3});
  std::vector<Emit::V> outs = {e.convert(dq, dt_str(n.results[0].dtype)),
                               e.convert(dk, dt_str(n.results[1].dtype)),
                               e.convert(dv, dt_str(n.results[2].dtype))};
  return module_text(e, P, outs);
}

std::string layer_norm_bwd(const Node& n, const std::vector<TensorType>& in) {
  if (in.size() != 4 || in[0].rank() < 1)
    throw PjrtErr(3, "mlx_layer_norm_bwd expects (x, w, b, dy)");
  const float eps = config_value(n.backend_config, "eps", 1e-5f);
  Emit e;
  std::vector<Emit::V> P;
  for (size_t i = 0; i < 4; ++i) P.push_back(Emit::V{"%p" + std::to_string(i), in[i].dims, dt_str(in[i].dtype)});
  const auto& xd = in[0].dims;
  const int64_t r = (int64_t)xd.size(), D = xd.back();
  std::vector<int64_t> rows;
  for (int64_t i = 0; i < r - 1; ++i) rows.push_back(i);
  auto x = e.convert(P[0], "f32"), wv = e.convert(P[1], "f32"), dy = e.convert(P[3], "f32");
  auto inv_d = e.scalar(1.0 / (double)D, std::vector<int64_t>(xd.begin(), xd.end() - 1));
  auto row = [&](const Emit::V& s) { return e.bcast(s, xd, rows); };
  auto mean = e.bin("multiply", e.reduce(x, {r - 1}, false), inv_d);
  auto xc = e.bin("subtract", x, row(mean));
  auto var = e.bin("multiply", e.reduce(e.bin("multiply", xc, xc), {r - 1}, false), inv_d);
  auto rstd = e.un("rsqrt", e.bin("add", var, e.scalar(eps, var.dims)));
  auto rb = row(rstd);
  auto xhat = e.bin("multiply", xc, rb);
  auto gw = e.bin("multiply", dy, e.bcast(wv, xd, {r - 1}));
  auto m1 = e.bin("multiply", e.reduce(gw, {r - 1}, false), inv_d);
  auto m2 = e.bin("multiply", e.reduce(e.bin("multiply", gw, xhat), {r - 1}, false), inv_d);
  auto dx = e.bin("multiply", rb,
                  e.bin("subtract", e.bin("subtract", gw, row(m1)), e.bin("multiply", xhat, row(m2))));
  Emit::V dw, db;
  if (rows.empty()) {
    dw = e.bin("multiply", dy, xhat);
    db = dy;
  } else {
    dw = e.reduce(e.bin("multiply", dy, xhat), rows, false);
    db = e.reduce(dy, rows, false);
  }
  std::vector<Emit::V> outs = {e.convert(dx, dt_str(n.results[0].dtype)),
                               e.convert(dw, dt_str(n.results[1].dtype)),
                               e.convert(db, dt_str(n.results[2].dtype))};
  return module_text(e, P, outs);
}

}  // namespace

bool fused_sdpa_bwd_call(const Node& n, const std::vector<ValueRef>& ops, Graph& dst,
                         std::vector<ValueRef>& outs) {
  if (n.target != "mlx_sdpa_bwd" || ops.size() != 4 || n.results.size() != 3) return false;
  const TensorType& t = dst.type(ops[0]);
  if (t.dtype != DType::BF16 || t.rank() != 4 || t.dims[3] != 64 || t.dims[1] > 256) return false;
  for (const auto& o : ops)
    if (dst.type(o) != t) return false;
  for (const auto& r : n.results)
    if (r != t) return false;
  const float scale = config_value(n.backend_config, "scale", 1.0f);
  if (!(scale > 0.f)) return false;
  const int64_t B = t.dims[0], T = t.dims[1], N = t.dims[2], D = t.dims[3];
  const std::vector<int64_t> st = {T * N * D, N * D, D};  // (b, t, n) of a dense BTNH tensor
  Node fw;
  fw.op = Op::FusedSdpa;
  fw.operands = {ops[0], ops[1], ops[2]};
  TensorType lt;
  lt.dtype = DType::F32;
  lt.dims = {B, N, T};
  fw.results = {t, lt};
  fw.name = n.name + ".fwd";
  fw.f_scale = scale;
  fw.i_flags = 2;  // no mask, row statistics
  fw.dims = {B, T, T, N, D};
  for (int k = 0; k < 4; ++k) fw.strides.insert(fw.strides.end(), st.begin(), st.end());
  const int fid = dst.add(std::move(fw));
  Node bw;
  bw.op = Op::FusedSdpaBwd;
  bw.operands = {ops[0], ops[1], ops[2], ValueRef{fid, 0}, ops[3], ValueRef{fid, 1}};
  bw.results = n.results;
  bw.name = n.name;
  bw.f_scale = scale;
  bw.dims = {B, T, T, N, D};
  for (int k = 0; k < 8; ++k) bw.strides.insert(bw.strides.end(), st.begin(), st.end());
  const int bid = dst.add(std::move(bw));
  outs = {ValueRef{bid, 0}, ValueRef{bid, 1}, ValueRef{bid, 2}};
  return true;
}

bool expands_custom_call(const std::string& target) {
  return target == "mlx_sdpa_bwd" || target == "mlx_layer_norm_bwd";
}

std::string custom_call_expansion(const Node& n, const std::vector<TensorType>& operand_types) {
  if (n.target == "mlx_sdpa_bwd") return sdpa_bwd(n, operand_types);
  if (n.target == "mlx_layer_norm_bwd") return layer_norm_bwd(n, operand_types);
  throw PjrtErr(12, "custom_call @" + n.target + " has no expansion");
}

}  // namespace b200
