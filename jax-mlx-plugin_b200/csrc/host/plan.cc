// Executable planner: IR -> slots + launch steps.
//
// Fusion policy (what the reference left to mx::compile, src/jax_mlx_pjrt.cpp
// :9056-9143): elementwise and layout ops are recomputed inside their
// consumers' kernels when they have a single consumer or are pure index
// arithmetic (broadcast, reshape, transpose, slice, convert, iota, constants);
// everything else is materialized once.  Reductions, windows, gathers and
// scatters read their operands through the same fused expressions.  dot_general
// and convolution lower to the tcgen05 GEMM (convolution through an im2col
// kernel), the matched SDPA / LayerNorm nodes to their hand-written kernels.
#include "plan.h"

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <functional>
#include <map>
#include <set>
#include <sstream>

#include "codegen.h"
#include "gemm_ws.h"
#include "passes.h"

namespace b200 {
namespace {

bool is_fusible(Op op) {
  switch (op) {
    case Op::Constant: case Op::Iota:
    case Op::Neg: case Op::Abs: case Op::Exp: case Op::Expm1: case Op::Log: case Op::Log1p:
    case Op::Sqrt: case Op::Rsqrt: case Op::Cbrt: case Op::Tanh: case Op::Logistic: case Op::Sin:
    case Op::Cos: case Op::Tan: case Op::Erf: case Op::Floor: case Op::Ceil: case Op::RoundAfz:
    case Op::RoundEven: case Op::Sign: case Op::Not: case Op::IsFinite:
    case Op::Add: case Op::Sub: case Op::Mul: case Op::Div: case Op::Rem: case Op::Max:
    case Op::Min: case Op::Pow: case Op::Atan2: case Op::And: case Op::Or: case Op::Xor:
    case Op::ShiftLeft: case Op::ShiftRightArith: case Op::ShiftRightLogical:
    case Op::Compare: case Op::Select: case Op::Clamp: case Op::Convert: case Op::BitcastConvert:
    case Op::BroadcastInDim: case Op::Reshape: case Op::Transpose: case Op::Slice:
    case Op::DynamicSlice: case Op::DynamicUpdateSlice: case Op::Pad: case Op::Concatenate:
    case Op::Reverse:
      return true;
    default:
      return false;
  }
}
// Ops whose recomputation costs only index arithmetic.
bool is_cheap(const Node& n) {
  switch (n.op) {
    case Op::Constant: case Op::Iota: case Op::BroadcastInDim: case Op::Reshape:
    case Op::Transpose: case Op::Slice: case Op::Reverse: case Op::Convert: case Op::Neg:
      return true;
    default:
      return false;
  }
}
// Consumers that read operands through generated expressions.
bool reads_expressions(Op op) {
  return is_fusible(op) || op == Op::Reduce || op == Op::ReduceWindow ||
         op == Op::SelectAndScatter || op == Op::Gather || op == Op::Scatter;
}

struct Builder {
  Plan& p;
  Graph& g;
  Uses u;
  std::map<ValueRef, int> slot;  // materialized values
  CodeGen cg;
  std::vector<GenKernel> kernels;
  // f32 values whose only readers are GEMMs are stored as the GEMMs' bf16
  // hi / lo planes (hi slot -> lo slot): no split pass in front of each GEMM
  std::map<int, int> plane_lo;

  Builder(Plan& pl, Graph& gr)
      : p(pl), g(gr), u(compute_uses(gr)),
        cg(gr, pl.slots, [this](ValueRef v) {
          auto it = slot.find(v);
          return it == slot.end() ? -1 : it->second;
        }) {
    cg.plane_lo = &plane_lo;
  }
  void maybe_planes(int n) {
    const Node& nd = g.nodes[n];
    if (nd.results.size() != 1 || nd.results[0].dtype != DType::F32 || u.output_refs[n] ||
        u.users[n].empty())
      return;
    for (int c : u.users[n])
      if (g.nodes[c].op != Op::DotGeneral) return;
    const int s = slot.at(ValueRef{n, 0});
    Slot& sl = p.slots[s];
    sl.type.dtype = DType::BF16;
    sl.bytes = sl.type.bytes();
    sl.what += ".hi";
    TensorType lt = sl.type;
    plane_lo[s] = new_slot(Slot::TEMP, lt, nd.name + ".lo");
  }

  int new_slot(Slot::Kind k, const TensorType& t, const std::string& what, int index = -1) {
    Slot s;
    s.kind = k;
    s.type = t;
    s.bytes = t.bytes();
    s.index = index;
    s.what = what;
    p.slots.push_back(s);
    return (int)p.slots.size() - 1;
  }
  int temp_for(ValueRef v) {
    auto it = slot.find(v);
    if (it != slot.end()) return it->second;
    const Node& n = g.nodes[v.node];
    int s = new_slot(Slot::TEMP, g.type(v), n.name.empty() ? op_name(n.op) : n.name);
    slot[v] = s;
    return s;
  }
  void add_kernel(GenKernel k) {
    Step st;
    st.kind = StepKind::Kernel;
    st.name = k.name;
    st.grid[0] = k.grid;
    st.grid[1] = std::max<int64_t>(k.grid_y, 1);
    if (k.block_y > 1) {  // column reduction: 2-D block (32, RY)
      st.block[0] = 32;
      st.block[1] = k.block_y;
    } else {
      st.block[0] = k.block;
    }
    for (size_t i = 0; i < k.ptr_slots.size(); ++i) {
      Arg a;
      a.kind = Arg::PTR;
      a.slot = k.ptr_slots[i];
      st.args.push_back(a);
      (k.ptr_written[i] ? st.out : st.in).push_back(k.ptr_slots[i]);
    }
    p.steps.push_back(st);
    p.kernel_names.push_back(k.name);
    kernels.push_back(std::move(k));
  }

  // ----------------------------------------------------------- ordering --
  std::vector<int> topo() {
    std::vector<int> order, state(g.nodes.size(), 0);
    std::function<void(int)> visit = [&](int n) {
      if (state[n] == 2) return;
      if (state[n] == 1) throw PjrtErr(13, "cycle in graph");
      state[n] = 1;
      for (auto& o : g.nodes[n].operands) visit(o.node);
      state[n] = 2;
      order.push_back(n);
    };
    for (auto& o : g.outputs) visit(o.node);
    return order;
  }

  bool must_materialize(int n) {
    const Node& nd = g.nodes[n];
    if (nd.op == Op::Parameter) return true;
    if (nd.op == Op::Constant && !nd.cdata.splat && nd.results[0].numel() > 1) return true;
    if (!is_fusible(nd.op)) return true;
    if (u.output_refs[n]) return true;
    for (int c : u.users[n])
      if (!reads_expressions(g.nodes[c].op)) {
        // convolution reads its lhs through the im2col expression
        if (g.nodes[c].op == Op::Convolution && g.nodes[c].operands[0].node == n &&
            g.nodes[c].operands[1].node != n)
          continue;
        return true;
      }
    if (u.count(n) <= 1) return false;
    // A value with a few consumers is recomputed inside each of them when its
    // fused expression is small: on HBM-bound kernels re-reading the inputs
    // (often narrower, e.g. bf16 logits) beats writing and re-reading an f32
    // intermediate.  Consumers that read each element several times (windows,
    // im2col, gathers, broadcasts) keep it materialized.  Layout ops and
    // converts are free to recompute.  In both cases the expression's memory
    // inputs, read once more by every extra consumer, must not cost more than
    // writing the value once and reading it back in each consumer: a long
    // residual chain (embedding + every block's output) is stored, not summed
    // again from a dozen tensors in each of its readers.
    if (!is_cheap(nd)) {
      if (u.count(n) > 8 || amplified(n)) return true;
      std::set<int> seen;
      if (expr_cost(n, seen) > kRecomputeOps) return true;
    }
    std::set<int> seen;
    const int64_t k = u.count(n), in_bytes = input_bytes(n, seen);
    return (k - 1) * in_bytes > (k + 1) * nd.results[0].bytes();
  }
  // Bytes of the memory-resident values (materialized slots, parameters,
  // results of non-fused ops) that n's fused expression reads, each once.
  int64_t input_bytes(int n, std::set<int>& seen) {
    if (seen.count(n)) return 0;
    seen.insert(n);
    const Node& nd = g.nodes[n];
    if (slot.count(ValueRef{n, 0}) || !is_fusible(nd.op)) {
      int64_t b = 0;
      for (const auto& t : nd.results) b += t.bytes();
      return b;
    }
    int64_t b = 0;
    for (const auto& o : nd.operands) b += input_bytes(o.node, seen);
    return b;
  }
  // Recompute budget in arithmetic ops (a transcendental counts 4): an HBM
  // byte costs far more than that many ops on this GPU.
  static constexpr int kRecomputeOps = 16;
  // Cost of n's fused expression, shared subexpressions counted once, stopping
  // at values that live in memory.
  int expr_cost(int n, std::set<int>& seen) {
    if (seen.count(n) || slot.count(ValueRef{n, 0})) return 0;
    seen.insert(n);
    const Node& nd = g.nodes[n];
    if (!is_fusible(nd.op)) return 0;
    int c = 0;
    switch (nd.op) {
      case Op::Exp: case Op::Expm1: case Op::Log: case Op::Log1p: case Op::Tanh:
      case Op::Logistic: case Op::Erf: case Op::Pow: case Op::Sin: case Op::Cos: case Op::Tan:
      case Op::Atan2: case Op::Cbrt:
        c = 4;
        break;
      default:
        c = is_cheap(nd) ? 0 : 1;
    }
    for (const auto& o : nd.operands) {
      c += expr_cost(o.node, seen);
      if (c > kRecomputeOps) break;
    }
    return c;
  }
  bool amplified(int n) {
    const int64_t size = g.nodes[n].results[0].numel();
    for (int c : u.users[n]) {
      const Node& cn = g.nodes[c];
      switch (cn.op) {
        case Op::ReduceWindow: case Op::SelectAndScatter: case Op::Gather: case Op::Scatter:
        case Op::Convolution: case Op::Pad: case Op::Concatenate:
          return true;
        default:
          break;
      }
      if (cn.op != Op::Reduce && !cn.results.empty() && cn.results[0].numel() > size) return true;
    }
    return false;
  }

  // Split a reduction over several blocks when its outputs alone would leave
  // most of the GPU idle (e.g. a bias gradient: 32 outputs, 200k rows each).
  // Only for init values that are the combiner's identity (0 for add, -inf /
  // +inf for max / min), which every jnp reduction uses: each block row starts
  // from the init, so a non-identity init would be counted once per split.
  int reduce_split(const Node& nd) {
    const int nin = (int)nd.operands.size() / 2;
    if (nin != 1) return 1;
    const Graph& r = *nd.regions.at(0);
    const Node& body = r.nodes.at(r.outputs.at(0).node);
    const Node& init = g.nodes[nd.operands[1].node];
    if (init.op != Op::Constant || !(init.cdata.splat || init.results[0].numel() == 1)) return 1;
    auto hv = host_eval(g, nd.operands[1]);
    if (!hv || hv->v.empty()) return 1;
    const double iv = hv->v[0];
    const bool identity = (body.op == Op::Add && iv == 0.0) ||
                          (body.op == Op::Max && std::isinf(iv) && iv < 0) ||
                          (body.op == Op::Min && std::isinf(iv) && iv > 0);
    if (!identity) return 1;
    const TensorType& it = g.type(nd.operands[0]);
    std::set<int64_t> red(nd.dims.begin(), nd.dims.end());
    int64_t OUT = 1, RED = 1;
    for (int d = 0; d < it.rank(); ++d) (red.count(d) ? RED : OUT) *= it.dims[d];
    const bool rowlike = it.rank() > 0 && red.count(it.rank() - 1);
    const int cv = rowlike ? 1 : CodeGen::column_vec(it, nd.dims);
    if (cv > 1) {
      // vector column reduction: blocks of kColWarps warps over 32 * cv
      // outputs each; split the rows until about 8 blocks per SM (a full SM
      // of loads in flight), keeping at least 4 rows per warp and at most 512
      // partial rows to combine (32 warps per combine block, 16 rows each)
      if (RED < 8 * CodeGen::kColWarps) return 1;
      const int64_t bx = (OUT / cv + 31) / 32;
      int64_t split = (148 * 8) / std::max<int64_t>(bx, 1);
      split = std::min<int64_t>(split, RED / (4 * CodeGen::kColWarps));
      split = std::min<int64_t>(split, 512);
      return (int)std::max<int64_t>(split, 1);
    }
    const int64_t threads = rowlike ? OUT * 32 : OUT * (OUT < 148 * 32 * 4 ? 32 : 8);
    if (threads >= 148 * 512 || RED < 8192) return 1;
    int64_t split = (148 * 1024) / std::max<int64_t>(threads, 1);
    split = std::min<int64_t>(split, RED / 1024);
    split = std::min<int64_t>(split, 512);
    return (int)std::max<int64_t>(split, 1);
  }

  // ---------------------------------------------------------------- GEMM --
  struct Group {
    int64_t size = 1, stride = 0;
    bool ok = true;
  };
  static Group group(const TensorType& t, const std::vector<int64_t>& dims) {
    std::vector<int64_t> st(t.rank(), 1);
    for (int i = t.rank() - 2; i >= 0; --i) st[i] = st[i + 1] * t.dims[i + 1];
    Group gr;
    int64_t prev = -1;
    for (auto d : dims) {
      if (t.dims[d] == 1) continue;
      gr.size *= t.dims[d];
      if (prev >= 0 && st[prev] != st[d] * t.dims[d]) gr.ok = false;
      prev = d;
      gr.stride = st[d];
    }
    if (gr.size == 1) gr.stride = 0;
    return gr;
  }
  void emit_gemm(int a, int b, int c, int64_t batch, int64_t M, int64_t N, int64_t K,
                 Group ab, Group am, Group ak, Group bb, Group bk, Group bn, int in_dt,
                 DType out_dt) {
    Step st;
    st.kind = StepKind::Gemm;
    st.name = "gemm";
    st.in = {a, b};
    st.out = {c};
    // strides of size-1 groups do not matter; give them a legal value
    auto fix = [](Group& x, int64_t other_unit) { if (x.size == 1) x.stride = other_unit ? 0 : 1; };
    fix(ab, 1); fix(bb, 1);
    if (am.size == 1) am.stride = ak.stride == 1 ? std::max<int64_t>(K, 1) : 1;
    if (ak.size == 1) ak.stride = am.stride == 1 ? std::max<int64_t>(M, 1) : 1;
    if (bn.size == 1) bn.stride = bk.stride == 1 ? std::max<int64_t>(K, 1) : 1;
    if (bk.size == 1) bk.stride = bn.stride == 1 ? std::max<int64_t>(N, 1) : 1;
    st.ip = {batch, M, N, K, ab.stride, am.stride, ak.stride, bb.stride, bk.stride, bn.stride, N, 0};
    st.fp = {1.0f};
    st.dtype = (int)in_dt;
    st.dtype2 = (int)out_dt;
    p.steps.push_back(st);
  }
  int permuted_copy(int src, const std::vector<int64_t>& perm, const std::string& what,
                    DType to = DType::INVALID) {
    const TensorType& t = p.slots[src].type;
    TensorType o;
    o.dtype = to == DType::INVALID ? t.dtype : to;
    for (auto d : perm) o.dims.push_back(t.dims[d]);
    int dst = new_slot(Slot::TEMP, o, what);
    add_kernel(cg.permute(src, perm, dst));
    return dst;
  }
  void lower_dot(int n) {
    const Node& nd = g.nodes[n];
    ValueRef L = nd.operands[0], R = nd.operands[1];
    int ls = slot.at(L), rs = slot.at(R);
    int llo = plane_lo.count(ls) ? plane_lo.at(ls) : -1;  // operand stored as planes
    int rlo = plane_lo.count(rs) ? plane_lo.at(rs) : -1;
    TensorType lt = g.type(L), rt = g.type(R);
    const TensorType& ot = nd.results[0];
    // Mixed f32 x bf16 operands (JAX's transpose rule for a bf16 dot with an
    // f32 preferred_element_type emits them) are computed in f32, as XLA
    // does: the GEMM splits the f32 side into bf16 hi + lo planes and reads
    // the bf16 side as it is (exact: its lo plane would be zero).
    int gemm_dt = (int)lt.dtype;
    if (lt.dtype != rt.dtype) {
      if (lt.dtype == DType::F32 && rt.dtype == DType::BF16) gemm_dt = B200_GEMM_DT_A_F32_B_BF16;
      else if (lt.dtype == DType::BF16 && rt.dtype == DType::F32) gemm_dt = B200_GEMM_DT_A_BF16_B_F32;
      else throw PjrtErr(12, "dot_general with mixed operand types");
    }
    for (DType t : {lt.dtype, rt.dtype})
      if (t != DType::F32 && t != DType::BF16)
        throw PjrtErr(12, std::string("dot_general on ") + dtype_name(t) + " is not supported");
    auto free_dims = [](int rank, const std::vector<int64_t>& a, const std::vector<int64_t>& b) {
      std::vector<int64_t> f;
      for (int64_t d = 0; d < rank; ++d)
        if (std::find(a.begin(), a.end(), d) == a.end() && std::find(b.begin(), b.end(), d) == b.end())
          f.push_back(d);
      return f;
    };
    auto lf = free_dims(lt.rank(), nd.lhs_batch, nd.lhs_contract);
    auto rf = free_dims(rt.rank(), nd.rhs_batch, nd.rhs_contract);
    Group ab = group(lt, nd.lhs_batch), am = group(lt, lf), ak = group(lt, nd.lhs_contract);
    Group bb = group(rt, nd.rhs_batch), bk = group(rt, nd.rhs_contract), bn = group(rt, rf);
    auto unit_ok = [](const Group& x, const Group& y) {
      return x.size == 1 || y.size == 1 || x.stride == 1 || y.stride == 1;
    };
    if (!(ab.ok && am.ok && ak.ok) || !unit_ok(am, ak)) {
      std::vector<int64_t> perm = nd.lhs_batch;
      perm.insert(perm.end(), lf.begin(), lf.end());
      perm.insert(perm.end(), nd.lhs_contract.begin(), nd.lhs_contract.end());
      ls = permuted_copy(ls, perm, "dot_lhs_T");
      if (llo >= 0) llo = permuted_copy(llo, perm, "dot_lhs_T.lo");
      lt = p.slots[ls].type;
      if (llo >= 0) lt.dtype = DType::F32;
      std::vector<int64_t> b(nd.lhs_batch.size()), f(lf.size()), c(nd.lhs_contract.size());
      int64_t k = 0;
      for (auto& x : b) x = k++;
      for (auto& x : f) x = k++;
      for (auto& x : c) x = k++;
      ab = group(lt, b); am = group(lt, f); ak = group(lt, c);
    }
    if (!(bb.ok && bk.ok && bn.ok) || !unit_ok(bk, bn)) {
      std::vector<int64_t> perm = nd.rhs_batch;
      perm.insert(perm.end(), rf.begin(), rf.end());
      perm.insert(perm.end(), nd.rhs_contract.begin(), nd.rhs_contract.end());
      rs = permuted_copy(rs, perm, "dot_rhs_T");
      if (rlo >= 0) rlo = permuted_copy(rlo, perm, "dot_rhs_T.lo");
      rt = p.slots[rs].type;
      if (rlo >= 0) rt.dtype = DType::F32;
      std::vector<int64_t> b(nd.rhs_batch.size()), f(rf.size()), c(nd.rhs_contract.size());
      int64_t k = 0;
      for (auto& x : b) x = k++;
      for (auto& x : f) x = k++;
      for (auto& x : c) x = k++;
      bb = group(rt, b); bn = group(rt, f); bk = group(rt, c);
    }
    if (ab.size != bb.size || ak.size != bk.size) throw PjrtErr(3, "dot_general: shape mismatch");
    int cs = temp_for(ValueRef{n, 0});
    emit_gemm(ls, rs, cs, ab.size, am.size, bn.size, ak.size, ab, am, ak, bb, bk, bn, gemm_dt,
              ot.dtype);
    if (llo >= 0 || rlo >= 0) {  // operands given as planes
      Step& gs = p.steps.back();
      Arg alo, blo;
      alo.slot = llo;
      blo.slot = rlo;
      gs.args = {alo, blo};
      for (int x : {llo, rlo})
        if (x >= 0) gs.in.push_back(x);
    }
  }

  void lower_conv(int n) {
    const Node& nd = g.nodes[n];
    if (nd.feature_groups != 1 || nd.batch_groups != 1)
      throw PjrtErr(12, "convolution with feature/batch groups is not supported");
    const ConvDims& c = nd.conv;
    const TensorType& lt = g.type(nd.operands[0]);
    const TensorType& kt = g.type(nd.operands[1]);
    const TensorType& ot = nd.results[0];
    if (lt.dtype != DType::F32 && lt.dtype != DType::BF16)
      throw PjrtErr(12, "convolution dtype not supported");
    std::vector<int64_t> k_roles, m_roles;
    for (int d = 0; d < kt.rank(); ++d)
      if (d != c.k_out) k_roles.push_back(d);
    for (int d = 0; d < ot.rank(); ++d)
      if (d != c.out_feature) m_roles.push_back(d);
    int64_t M = 1, K = 1;
    for (auto d : m_roles) M *= ot.dims[d];
    for (auto d : k_roles) K *= kt.dims[d];
    const int64_t N = kt.dims[c.k_out];
    // f32 patches go straight to the GEMM's bf16 hi / lo planes when their
    // rows are 16-byte multiples in bf16 (no f32 patch matrix, no split pass)
    const bool planes = lt.dtype == DType::F32 && K % 8 == 0;
    // A weight-gradient-shaped convolution (innermost M role = output batch,
    // read from the input's innermost dimension) writes its patches
    // transposed, [K, M] with eight channels of one input pixel per thread;
    // the GEMM reads that A MN-major.
    const bool transposed = lt.dtype == DType::F32 && !m_roles.empty() &&
                            m_roles.back() == c.out_batch && ot.dims[c.out_batch] % 8 == 0 &&
                            c.in_batch == lt.rank() - 1 &&
                            !(k_roles.back() == c.k_in && kt.dims[c.k_in] % 8 == 0 &&
                              c.in_feature == lt.rank() - 1) &&
                            slot.count(nd.operands[0]) != 0;
    int as, al = -1;
    if (transposed) {
      as = new_slot(Slot::TEMP, TensorType{DType::BF16, {K, M}}, "im2col_t_hi");
      al = new_slot(Slot::TEMP, TensorType{DType::BF16, {K, M}}, "im2col_t_lo");
      add_kernel(cg.im2col_t(n, as, k_roles, m_roles, M, K, al));
    } else if (planes) {
      as = new_slot(Slot::TEMP, TensorType{DType::BF16, {M, K}}, "im2col_hi");
      al = new_slot(Slot::TEMP, TensorType{DType::BF16, {M, K}}, "im2col_lo");
      add_kernel(cg.im2col(n, as, k_roles, m_roles, M, K, al));
    } else {
      as = new_slot(Slot::TEMP, TensorType{lt.dtype, {M, K}}, "im2col");
      add_kernel(cg.im2col(n, as, k_roles, m_roles, M, K, al));
    }
    int ks = slot.at(nd.operands[1]);
    Group bk, bn;
    if (c.k_out == kt.rank() - 1) {
      bk.size = K; bk.stride = N; bn.size = N; bn.stride = 1;
    } else if (c.k_out == 0) {
      bk.size = K; bk.stride = 1; bn.size = N; bn.stride = K;
    } else {
      std::vector<int64_t> perm = k_roles;
      perm.push_back(c.k_out);
      ks = permuted_copy(ks, perm, "conv_kernel_T");
      bk.size = K; bk.stride = N; bn.size = N; bn.stride = 1;
    }
    Group ab, am, ak, bb;
    am.size = M; am.stride = K; ak.size = K; ak.stride = 1;
    if (transposed) { am.stride = 1; ak.stride = M; }
    const bool direct = c.out_feature == ot.rank() - 1;
    int cs;
    if (direct) {
      cs = temp_for(ValueRef{n, 0});
    } else {
      cs = new_slot(Slot::TEMP, TensorType{ot.dtype, {M, N}}, "conv_out_MN");
    }
    emit_gemm(as, ks, cs, 1, M, N, K, ab, am, ak, bb, bk, bn, (int)lt.dtype, ot.dtype);
    if (planes || transposed) {  // A arrives split: its lo plane (see the executor's GEMM step)
      Step& g = p.steps.back();
      Arg alo, blo;
      alo.slot = al;
      blo.slot = -1;
      g.args = {alo, blo};
      g.in.push_back(al);
    }
    if (!direct) {
      // [M..., N] -> output dims: out dim d takes (m_roles position | feature)
      TensorType mn;
      mn.dtype = ot.dtype;
      for (auto d : m_roles) mn.dims.push_back(ot.dims[d]);
      mn.dims.push_back(N);
      p.slots[cs].type = mn;
      std::vector<int64_t> perm(ot.rank());
      for (int d = 0; d < ot.rank(); ++d) {
        if (d == c.out_feature) { perm[d] = (int64_t)m_roles.size(); continue; }
        perm[d] = std::find(m_roles.begin(), m_roles.end(), d) - m_roles.begin();
      }
      int os = temp_for(ValueRef{n, 0});
      add_kernel(cg.permute(cs, perm, os));
    }
  }

  // ------------------------------------------------------------ fused ops --
  void lower_sdpa_custom(int n, const Node& nd) {
    // custom_call @mlx_sdpa(Q, K, V), layout (B, T, N, H), backend_config {"scale": s}
    const TensorType& qt = g.type(nd.operands[0]);
    const TensorType& kt = g.type(nd.operands[1]);
    if (qt.rank() != 4) throw PjrtErr(3, "mlx_sdpa expects rank-4 (B,T,N,H) operands");
    float scale = 1.0f / std::sqrt((float)qt.dims[3]);
    auto pos = nd.backend_config.find("scale");
    if (pos != std::string::npos) {
      pos = nd.backend_config.find(':', pos);
      if (pos != std::string::npos) scale = std::stof(nd.backend_config.substr(pos + 1));
    }
    Step st;
    st.kind = StepKind::Sdpa;
    st.name = "sdpa";
    const int64_t B = qt.dims[0], T = qt.dims[1], N = qt.dims[2], D = qt.dims[3], S = kt.dims[1];
    st.in = {slot.at(nd.operands[0]), slot.at(nd.operands[1]), slot.at(nd.operands[2])};
    st.out = {temp_for(ValueRef{n, 0})};
    st.ip = {B, T, S, N, D, T * N * D, N * D, D, S * N * D, N * D, D, S * N * D, N * D, D,
             T * N * D, N * D, D, 0};
    st.fp = {scale};
    st.dtype = (int)qt.dtype;
    p.steps.push_back(st);
    p.num_sdpa++;
  }
  void lower_fused_sdpa(int n, const Node& nd) {
    Step st;
    st.kind = StepKind::Sdpa;
    st.name = "sdpa";
    st.in = {slot.at(nd.operands[0]), slot.at(nd.operands[1]), slot.at(nd.operands[2])};
    st.out = {temp_for(ValueRef{n, 0})};
    if (nd.i_flags & 2) st.out.push_back(temp_for(ValueRef{n, 1}));  // row statistics
    st.ip = nd.dims;  // B T S N D
    st.ip.insert(st.ip.end(), nd.strides.begin(), nd.strides.end());
    st.ip.push_back(nd.i_flags & 1);
    st.fp = {nd.f_scale};
    st.dtype = (int)g.type(nd.operands[0]).dtype;
    p.steps.push_back(st);
    p.num_sdpa++;
  }
  // Attention backward (b200_sdpa_bwd): in q, k, v, o, dO, row statistics;
  // out dQ, dK, dV.  ip: B T N D, 24 strides, causal.
  void lower_fused_sdpa_bwd(int n, const Node& nd) {
    Step st;
    st.kind = StepKind::SdpaBwd;
    st.name = "sdpa_bwd";
    for (const auto& o : nd.operands) st.in.push_back(slot.at(o));
    st.out = {temp_for(ValueRef{n, 0}), temp_for(ValueRef{n, 1}), temp_for(ValueRef{n, 2})};
    st.ip = {nd.dims[0], nd.dims[1], nd.dims[3], nd.dims[4]};
    st.ip.insert(st.ip.end(), nd.strides.begin(), nd.strides.end());
    st.ip.push_back(nd.i_flags & 1);
    st.fp = {nd.f_scale};
    st.dtype = (int)g.type(nd.operands[0]).dtype;
    p.steps.push_back(st);
    p.num_sdpa++;
  }
  void lower_fused_ln(int n, const Node& nd) {
    Step st;
    st.kind = StepKind::LayerNorm;
    st.name = "layer_norm";
    int k = 0;
    const int x = slot.at(nd.operands[k++]);
    const int r = (nd.i_flags & 2) ? slot.at(nd.operands[k++]) : -1;
    const int ga = (nd.i_flags & 4) ? slot.at(nd.operands[k++]) : -1;
    const int be = (nd.i_flags & 8) ? slot.at(nd.operands[k++]) : -1;
    const TensorType& yt = nd.results[0];
    st.in = {x, r, ga, be};
    st.out = {temp_for(ValueRef{n, 0}), (nd.i_flags & 16) ? temp_for(ValueRef{n, 1}) : -1};
    const int64_t cols = yt.dims.back();
    st.ip = {yt.numel() / cols, cols, nd.i_flags & 1};
    st.fp = {nd.f_eps};
    st.dtype = (int)yt.dtype;
    p.steps.push_back(st);
    p.num_ln++;
  }
  void lower_ln_custom(int n, const Node& nd) {
    // custom_call @mlx_layer_norm(x, w, b) {"eps": e}: LayerNorm over the last axis
    float eps = 1e-5f;
    auto pos = nd.backend_config.find("eps");
    if (pos != std::string::npos) {
      pos = nd.backend_config.find(':', pos);
      if (pos != std::string::npos) eps = std::stof(nd.backend_config.substr(pos + 1));
    }
    Step st;
    st.kind = StepKind::LayerNorm;
    st.name = "layer_norm";
    const TensorType& yt = nd.results[0];
    st.in = {slot.at(nd.operands[0]), -1, nd.operands.size() > 1 ? slot.at(nd.operands[1]) : -1,
             nd.operands.size() > 2 ? slot.at(nd.operands[2]) : -1};
    st.out = {temp_for(ValueRef{n, 0}), -1};
    const int64_t cols = yt.dims.back();
    st.ip = {yt.numel() / cols, cols, 0};
    st.fp = {eps};
    st.dtype = (int)yt.dtype;
    p.steps.push_back(st);
    p.num_ln++;
  }

  void lower_all_reduce(int n, const Node& nd) {
    const Graph& r = *nd.regions.at(0);
    const Node& b = r.nodes.at(r.outputs.at(0).node);
    int op = 0;  // 0 sum, 1 prod, 2 max, 3 min
    if (b.op == Op::Add) op = 0;
    else if (b.op == Op::Mul) op = 1;
    else if (b.op == Op::Max) op = 2;
    else if (b.op == Op::Min) op = 3;
    else throw PjrtErr(12, "all_reduce with an unsupported reduction body");
    for (size_t k = 0; k < nd.operands.size(); ++k) {
      Step st;
      st.kind = StepKind::AllReduce;
      st.name = "all_reduce";
      st.in = {slot.at(nd.operands[k])};
      st.out = {temp_for(ValueRef{n, (int)k})};
      st.ip = {nd.results[k].numel(), op, (int64_t)nd.replica_groups.size(),
               nd.replica_groups.empty() ? 0 : (int64_t)nd.replica_groups[0].size()};
      for (auto& grp : nd.replica_groups) st.ip.insert(st.ip.end(), grp.begin(), grp.end());
      st.dtype = (int)nd.results[k].dtype;
      p.steps.push_back(st);
    }
  }

  // Consecutive all_reduce steps over the same replica groups, reduction and
  // element type become one NCCL call on a flat bucket (data-parallel gradient
  // means: one collective instead of one per parameter).  args[2k] = (input
  // slot, offset in elements), args[2k+1] = (output slot, element count); the
  // bucket is the last output slot.
  void bucket_all_reduces() {
    std::map<int, int> readers;  // slot -> steps reading it
    for (const Step& s : p.steps)
      for (int x : s.in)
        if (x >= 0) ++readers[x];
    std::vector<Step> merged;
    for (size_t i = 0; i < p.steps.size();) {
      const Step& a = p.steps[i];
      size_t j = i + 1;
      if (a.kind == StepKind::AllReduce && a.args.empty()) {
        auto same = [&](const Step& b) {
          return b.kind == StepKind::AllReduce && b.args.empty() && b.dtype == a.dtype &&
                 std::vector<int64_t>(b.ip.begin() + 1, b.ip.end()) ==
                     std::vector<int64_t>(a.ip.begin() + 1, a.ip.end());
        };
        while (j < p.steps.size() && same(p.steps[j])) ++j;
      }
      if (j - i < 2) {
        merged.push_back(p.steps[i]);
        i = j;
        continue;
      }
      Step b;
      b.kind = StepKind::AllReduce;
      b.name = "all_reduce_bucket";
      b.dtype = a.dtype;
      int64_t off = 0;
      for (size_t k = i; k < j; ++k) {
        const Step& s = p.steps[k];
        Arg in;
        in.slot = s.in[0];
        in.i = off;
        Arg out;
        out.slot = s.out[0];
        out.i = s.ip[0];
        b.args.push_back(in);
        b.args.push_back(out);
        b.in.push_back(s.in[0]);
        b.out.push_back(s.out[0]);
        off += (s.ip[0] + 63) / 64 * 64;  // 256-byte aligned pieces
      }
      TensorType bt;
      bt.dtype = (DType)a.dtype;
      bt.dims = {off};
      const int bucket = new_slot(Slot::TEMP, bt, "all_reduce_bucket");
      b.out.push_back(bucket);
      // A gradient that only this collective reads is computed in its piece
      // of the bucket and its reduced value read from there (f = 1: no
      // copies); outputs and parameters keep their own buffers.
      const int64_t es = dtype_size(bt.dtype);
      for (size_t k = 0; k < b.args.size(); k += 2) {
        const int si = b.args[k].slot, so = b.args[k + 1].slot;
        if (p.slots[si].kind != Slot::TEMP || p.slots[so].kind != Slot::TEMP || readers[si] != 1 ||
            p.slots[si].parent >= 0 || p.slots[so].parent >= 0)
          continue;
        for (int x : {si, so}) {
          p.slots[x].parent = bucket;
          p.slots[x].offset = b.args[k].i * es;
        }
        b.args[k].f = 1.f;
      }
      b.ip = a.ip;
      b.ip[0] = off;
      merged.push_back(b);
      i = j;
    }
    p.steps.swap(merged);
  }

  // ------------------------------------------------------------ row groups --
  // Consecutive row-wise kernels over the same OUT rows of RED elements --
  // reductions of the last dimension and loops whose last dimension is RED --
  // are gathered into one row-group kernel (CodeGen::rowgroup) when every
  // value a phase reads from an earlier phase is read at its own row.  A
  // softmax (max, sum of exponentials, normalise), a cross-entropy (max, sum,
  // target logit, gradient) or a layer norm (mean, variance, normalise) then
  // reads each row from HBM once instead of once per kernel.
  std::vector<RowPhase> rg;
  int64_t rg_out = 0, rg_red = 0;
  std::set<int> rg_nodes;  // nodes whose values the open group's phases write

  static bool elementwise_op(Op op) { return op >= Op::Neg && op <= Op::Convert; }

  // B200_ROW_GROUPS=0 emits every phase as a kernel of its own.
  static bool row_groups_on() {
    static const bool on = [] {
      const char* e = getenv("B200_ROW_GROUPS");
      return !(e && e[0] == '0');
    }();
    return on;
  }
  bool reduce_rows(int n, int64_t* out, int64_t* red) {
    if (!row_groups_on()) return false;
    const Node& nd = g.nodes[n];
    if (nd.op != Op::Reduce || nd.dims.size() != 1) return false;
    const TensorType& it = g.type(nd.operands[0]);
    if (it.rank() < 2 || nd.dims[0] != it.rank() - 1 || it.dims.back() < 2) return false;
    *red = it.dims.back();
    *out = it.numel() / *red;
    return *out > 0;
  }
  bool loop_rows(const std::vector<int>& nodes, int64_t* out, int64_t* red) {
    if (!row_groups_on()) return false;
    const TensorType& t = g.nodes[nodes[0]].results[0];
    if (t.rank() < 2 || t.dims.back() < 2) return false;
    for (int n : nodes)
      if (g.nodes[n].results[0].dims != t.dims) return false;
    *red = t.dims.back();
    *out = t.numel() / *red;
    return *out > 0;
  }
  // Does v's fused expression read a value the open group writes?
  bool reads_group(ValueRef v, std::set<int>& seen) {
    if (rg_nodes.count(v.node)) return true;
    if (slot.count(v) || !seen.insert(v.node).second) return false;
    const Node& nd = g.nodes[v.node];
    if (!is_fusible(nd.op)) return false;
    for (const auto& o : nd.operands)
      if (reads_group(o, seen)) return true;
    return false;
  }
  // True when every group value v's expression reads is read at the row of
  // the element being computed.  The row of an element of a value with
  // OUT*RED elements is its linear index / RED; of a value with OUT elements,
  // its linear index.  Elementwise ops and reshapes keep linear indices; a
  // broadcast of a per-row value along the last dimension keeps the row.
  bool row_aligned_node(int n) {
    const Node& nd = g.nodes[n];
    const TensorType& t = nd.results[0];
    auto sub = [&](ValueRef o) {
      std::set<int> seen;
      if (!reads_group(o, seen)) return true;
      if (rg_nodes.count(o.node)) return true;
      return row_aligned_node(o.node);
    };
    if (nd.op == Op::Constant || nd.op == Op::Iota) return true;
    if (elementwise_op(nd.op)) {
      for (const auto& o : nd.operands)
        if (g.type(o).numel() != t.numel() && g.type(o).numel() != 1) return false;
      for (const auto& o : nd.operands)
        if (!sub(o)) return false;
      return true;
    }
    if (nd.op == Op::Reshape) return g.type(nd.operands[0]).numel() == t.numel() && sub(nd.operands[0]);
    if (nd.op == Op::BroadcastInDim) {
      const TensorType& it = g.type(nd.operands[0]);
      {
        std::set<int> seen;
        if (!reads_group(nd.operands[0], seen)) return true;
      }
      if (it.numel() == t.numel()) {  // only size-1 dimensions added
        int last = -1;
        for (size_t i = 0; i < nd.dims.size(); ++i) {
          if (it.dims[i] == 1) continue;
          if (nd.dims[i] <= last) return false;
          last = (int)nd.dims[i];
        }
        return sub(nd.operands[0]);
      }
      // per-row value along the rows: input dims of size > 1 map, in order,
      // onto every leading output dimension of size > 1
      if (t.numel() != rg_out * rg_red || t.dims.back() != rg_red || it.numel() != rg_out) return false;
      int last = -1;
      int64_t covered = 1;
      for (size_t i = 0; i < nd.dims.size(); ++i) {
        if (it.dims[i] == 1) continue;
        const int64_t d = nd.dims[i];
        if (d <= last || d >= t.rank() - 1 || t.dims[d] != it.dims[i]) return false;
        last = (int)d;
        covered *= it.dims[i];
      }
      return covered == rg_out && sub(nd.operands[0]);
    }
    return false;
  }
  // `reads`: values the phase reads at the element it computes (a reduction's
  // operands); `roots`: nodes a loop phase computes there.
  bool phase_fits(int64_t out, int64_t red, const std::vector<ValueRef>& reads,
                  const std::vector<int>& roots) {
    if (rg.empty()) return true;
    if (out != rg_out || red != rg_red) return false;
    for (const auto& v : reads) {
      if (rg_nodes.count(v.node)) continue;
      std::set<int> seen;
      if (!reads_group(v, seen)) continue;
      if (!row_aligned_node(v.node)) return false;
    }
    for (int n : roots) {
      bool reads_any = false;
      for (const auto& o : g.nodes[n].operands) {
        std::set<int> seen;
        if (rg_nodes.count(o.node) || reads_group(o, seen)) reads_any = true;
      }
      if (reads_any && !row_aligned_node(n)) return false;
    }
    return true;
  }
  void open_phase(int64_t out, int64_t red) {
    if (rg.empty()) {
      rg_out = out;
      rg_red = red;
    }
  }
  void flush_rg() {
    if (rg.empty()) return;
    if (rg.size() == 1 && rg[0].sum_reduce < 0 &&
        !(rg[0].reduce >= 0 && cg.onehot_pick(rg[0].reduce).node >= 0)) {
      const RowPhase ph = rg[0];
      rg.clear();
      rg_nodes.clear();
      if (ph.reduce >= 0) {
        add_kernel(cg.reduce(ph.reduce, ph.out_slots));
      } else {
        for (auto& r : ph.roots) slot.erase(r);
        GenKernel k = cg.loop(ph.roots, ph.out_slots);
        for (size_t i = 0; i < ph.roots.size(); ++i) slot[ph.roots[i]] = ph.out_slots[i];
        add_kernel(std::move(k));
      }
      return;
    }
    GenKernel k = cg.rowgroup(rg, rg_out, rg_red);
    rg.clear();
    rg_nodes.clear();
    add_kernel(std::move(k));
  }
  // Reduce whose body is a single `op` and whose init is the constant `init`.
  bool simple_reduce(const Node& nd, Op op, double init) {
    if (nd.op != Op::Reduce || nd.operands.size() != 2) return false;
    const Graph& r = *nd.regions.at(0);
    if (r.outputs.size() != 1 || r.nodes.at(r.outputs[0].node).op != op) return false;
    auto hv = host_eval(g, nd.operands[1]);
    return hv && hv->v.size() == 1 && hv->v[0] == init;
  }
  // s sums exp(X - M) over the rows, where m (M) is the row max of the same
  // f32 X: the pair is computed in one pass (RowPhase::sum_reduce).
  bool softmax_sum_of(int s, int m) {
    const Node& sn = g.nodes[s];
    const Node& mn = g.nodes[m];
    if (!simple_reduce(mn, Op::Max, -INFINITY) || !simple_reduce(sn, Op::Add, 0.0)) return false;
    if (mn.results[0].dtype != DType::F32 || sn.results[0].dtype != DType::F32) return false;
    const ValueRef x = mn.operands[0];
    const ValueRef ev = sn.operands[0];
    if (slot.count(ev)) return false;
    const Node& e = g.nodes[ev.node];
    if (e.op != Op::Exp || e.results[0].dtype != DType::F32 || slot.count(e.operands[0])) return false;
    const Node& d = g.nodes[e.operands[0].node];
    if (d.op != Op::Sub || !(d.operands[0] == x)) return false;
    ValueRef b = d.operands[1];  // M broadcast along the row (alignment: phase_fits)
    while (!(b.node == m && b.idx == 0)) {
      const Node& bn = g.nodes[b.node];
      if (slot.count(b) || (bn.op != Op::BroadcastInDim && bn.op != Op::Reshape)) return false;
      b = bn.operands[0];
    }
    return true;
  }
  // A row-wise reduction (split == 1): joins or opens the row group.
  void add_reduce_phase(int n, const std::vector<int>& outs, int64_t out, int64_t red) {
    const Node& nd = g.nodes[n];
    std::vector<ValueRef> reads(nd.operands.begin(), nd.operands.end());
    if (!rg.empty() && rg.back().reduce >= 0 && rg.back().sum_reduce < 0 &&
        rg.back().out_slots.size() == 1 && phase_fits(out, red, reads, {}) &&
        softmax_sum_of(n, rg.back().reduce)) {
      rg.back().sum_reduce = n;
      rg.back().out_slots.push_back(outs[0]);
      rg_nodes.insert(n);
      return;
    }
    if (!phase_fits(out, red, reads, {})) flush_rg();
    open_phase(out, red);
    RowPhase ph;
    ph.reduce = n;
    ph.out_slots = outs;
    rg.push_back(ph);
    rg_nodes.insert(n);
  }

  std::vector<int> pending;  // materialized loop values not yet emitted
  void flush_loops() {
    if (pending.empty()) return;
    std::vector<ValueRef> roots;
    std::vector<int> outs;
    for (int n : pending) {
      roots.push_back(ValueRef{n, 0});
      outs.push_back(slot.at(ValueRef{n, 0}));
    }
    int64_t out = 0, red = 0;
    if (loop_rows(pending, &out, &red)) {
      if (!phase_fits(out, red, {}, pending)) flush_rg();
      open_phase(out, red);
      RowPhase ph;
      ph.roots = roots;
      ph.out_slots = outs;
      rg.push_back(ph);
      for (int n : pending) rg_nodes.insert(n);
      pending.clear();
      return;
    }
    flush_rg();
    // hide the slots so the kernel computes the values instead of loading them
    for (auto& r : roots) slot.erase(r);
    GenKernel k = cg.loop(roots, outs);
    for (size_t i = 0; i < roots.size(); ++i) slot[roots[i]] = outs[i];
    pending.clear();
    add_kernel(std::move(k));
  }

  // -------------------------------------------------------------- driver --
  // Schedule every all_reduce whose operands do not themselves come out of an
  // all_reduce right after the last node it does not depend on, and their
  // consumers after them: the collectives become consecutive steps that
  // bucket_all_reduces merges (one NCCL call for all of a step's gradients).
  std::vector<int> group_all_reduces(const std::vector<int>& order) {
    std::vector<char> dep(g.nodes.size(), 0);  // depends on an all_reduce output
    bool any = false;
    for (int n : order) {
      const Node& nd = g.nodes[n];
      char d = 0;
      for (auto& o : nd.operands) d |= dep[o.node];
      if (nd.op == Op::AllReduce) any = true;
      dep[n] = d || nd.op == Op::AllReduce;
    }
    if (!any) return order;
    std::vector<int> head, mid, tail;
    for (int n : order) {
      const Node& nd = g.nodes[n];
      bool in_dep = false;
      for (auto& o : nd.operands) in_dep |= dep[o.node] != 0;
      if (!dep[n]) head.push_back(n);
      else if (nd.op == Op::AllReduce && !in_dep) mid.push_back(n);
      else tail.push_back(n);
    }
    if (overlap_collectives() && mid.size() >= 2) {
      // Data-parallel gradients are ready at different points of the
      // backward pass.  Order the collectives by when their operands are
      // ready and cut them into buckets of about B200_BUCKET_MB (default 12)
      // MB; each bucket goes right after the node that completes its last
      // operand, so its all-reduce (run on the communication stream) overlaps
      // the rest of the backward pass.
      std::vector<int> pos(g.nodes.size(), -1);
      for (size_t i = 0; i < head.size(); ++i) pos[head[i]] = (int)i;
      auto ready = [&](int n) {
        int r = -1;
        for (auto& o : g.nodes[n].operands) r = std::max(r, pos[o.node]);
        return r;
      };
      std::stable_sort(mid.begin(), mid.end(), [&](int a, int b) { return ready(a) < ready(b); });
      static const int64_t limit = [] {
        const char* v = std::getenv("B200_BUCKET_MB");
        const double mb = v ? std::atof(v) : 12.0;
        return (int64_t)(std::max(mb, 0.001) * (1 << 20));
      }();
      std::map<int, std::vector<int>> after;  // head position -> collectives placed after it
      std::vector<int> cur;
      int64_t bytes = 0;
      for (int n : mid) {
        cur.push_back(n);
        for (auto& r : g.nodes[n].results) bytes += r.bytes();
        if (bytes >= limit) {
          auto& dst = after[ready(cur.back())];
          dst.insert(dst.end(), cur.begin(), cur.end());
          cur.clear();
          bytes = 0;
        }
      }
      if (!cur.empty()) {
        auto& dst = after[ready(cur.back())];
        dst.insert(dst.end(), cur.begin(), cur.end());
      }
      std::vector<int> out;
      auto it0 = after.find(-1);
      if (it0 != after.end()) out.insert(out.end(), it0->second.begin(), it0->second.end());
      for (size_t i = 0; i < head.size(); ++i) {
        out.push_back(head[i]);
        auto it = after.find((int)i);
        if (it != after.end()) out.insert(out.end(), it->second.begin(), it->second.end());
      }
      out.insert(out.end(), tail.begin(), tail.end());
      return out;
    }
    head.insert(head.end(), mid.begin(), mid.end());
    head.insert(head.end(), tail.begin(), tail.end());
    return head;
  }

  // Generated loop and reduction kernels that compile to the same code run as
  // one launch when they can meet at one place: the batched kernel takes every
  // member's pointers in one table and blockIdx.z picks the member (the
  // bodies index with blockIdx.x / .y only).  The launch goes where the last
  // member was; an earlier member may move there when no step in between
  // reads its outputs or writes its inputs or outputs.  Repeated until
  // nothing moves: an optimizer's per-parameter updates batch first (nothing
  // reads them), then the gradient reductions they read (bias and norm-gain
  // column sums, and their partial-sum combines), which now have no reader
  // before the batch.
  void batch_steps() {
    for (int pass = 0; pass < 4; ++pass)
      if (!batch_pass()) break;
  }
  bool batch_pass() {
    const size_t n = p.steps.size();
    std::vector<std::vector<int>> readers(p.slots.size()), writers(p.slots.size());
    for (size_t i = 0; i < n; ++i) {
      for (int sl : p.steps[i].in)
        if (sl >= 0) readers[sl].push_back((int)i);
      for (int sl : p.steps[i].out)
        if (sl >= 0) writers[sl].push_back((int)i);
    }
    auto between = [](const std::vector<int>& v, int lo, int hi) {
      return std::any_of(v.begin(), v.end(), [&](int x) { return x > lo && x <= hi; });
    };
    std::map<std::string, const GenKernel*> by_name;
    for (auto& k : kernels) by_name[k.name] = &k;
    auto body_key = [&](const GenKernel& k) {
      std::string key = k.code;
      const size_t at = key.find(" " + k.name + "(");
      if (at != std::string::npos) key.replace(at + 1, k.name.size(), "@");
      return key;
    };
    auto kind_ok = [](const std::string& name) {
      return name.find("_loop") != std::string::npos || name.find("_reduce") != std::string::npos;
    };
    std::map<std::string, std::vector<int>> groups;  // code -> steps, in order
    for (size_t i = 0; i < n; ++i) {
      const Step& st = p.steps[i];
      if (st.kind != StepKind::Kernel || st.table || st.grid[2] != 1 || !kind_ok(st.name)) continue;
      auto it = by_name.find(st.name);
      if (it == by_name.end()) continue;
      bool ok = true;
      for (int sl : st.out) ok = ok && sl >= 0 && writers[sl].size() == 1;
      for (int sl : st.in) ok = ok && sl >= 0;
      if (ok) groups[body_key(*it->second)].push_back((int)i);
    }
    std::set<int> removed;
    std::map<int, std::vector<Step>> placed;  // batches, at their last member
    for (auto& g : groups) {
      const std::vector<int>& members = g.second;
      if (members.size() < 2) continue;
      const GenKernel& k0 = *by_name.at(p.steps[members[0]].name);
      const size_t K = k0.ptr_slots.size();
      const int last = members.back();
      std::vector<int> ok;
      for (int m : members) {
        bool safe = true;
        const Step& ms = p.steps[m];
        for (int sl : ms.out) safe = safe && !between(readers[sl], m, last);
        for (int sl : ms.in) safe = safe && !between(writers[sl], m, last);
        if (safe) ok.push_back(m);
      }
      if (ok.size() < 2 || ok.back() != last) continue;
      // kernel parameters stay under 4 KB: at most 480 pointers per launch;
      // every chunk is placed at the last member (all members can move there)
      const size_t per = std::max<size_t>(1, 480 / std::max<size_t>(K, 1));
      for (size_t c0 = 0; c0 < ok.size(); c0 += per) {
        std::vector<int> chunk(ok.begin() + c0, ok.begin() + std::min(ok.size(), c0 + per));
        if (chunk.size() < 2) continue;
        GenKernel bk;
        bk.name = k0.name + "_x" + std::to_string(chunk.size()) + "_" + std::to_string(batched_++);
        bk.code = batched_code(k0, bk.name, (int)chunk.size());
        Step bs = p.steps[chunk.back()];
        bs.name = bk.name;
        bs.table = true;
        bs.grid[2] = (int64_t)chunk.size();
        bs.args.clear();
        bs.in.clear();
        bs.out.clear();
        for (int m : chunk) {
          const Step& ms = p.steps[m];
          bs.args.insert(bs.args.end(), ms.args.begin(), ms.args.end());
          bs.in.insert(bs.in.end(), ms.in.begin(), ms.in.end());
          bs.out.insert(bs.out.end(), ms.out.begin(), ms.out.end());
          removed.insert(m);
        }
        kernels.push_back(std::move(bk));
        placed[last].push_back(std::move(bs));
      }
    }
    if (placed.empty()) return false;
    std::vector<Step> steps;
    for (size_t i = 0; i < n; ++i) {
      auto it = placed.find((int)i);
      if (it != placed.end()) {
        for (auto& b : it->second) steps.push_back(std::move(b));
        if (!removed.count((int)i)) steps.push_back(std::move(p.steps[i]));
        continue;
      }
      if (removed.count((int)i)) continue;
      steps.push_back(std::move(p.steps[i]));
    }
    p.steps = std::move(steps);
    return true;
  }
  int batched_ = 0;
  // The code of kernel `k` as a batched kernel `name` of `count` members: its
  // pointer parameters come from a table argument (member blockIdx.z).
  static std::string batched_code(const GenKernel& k, const std::string& name, int count) {
    const std::string& c = k.code;
    const size_t np = c.find(" " + k.name + "(");
    const size_t open = np + 1 + k.name.size();
    const size_t close = c.find(") {", open);
    if (np == std::string::npos || close == std::string::npos)
      throw PjrtErr(13, "batched kernel: unexpected generated signature");
    const std::string params = c.substr(open + 1, close - open - 1);
    const std::string head = c.substr(0, np + 1);  // extern "C" __global__ ... void
    std::vector<std::string> decl;
    size_t pos = 0;
    while (pos < params.size()) {
      size_t e = params.find(", ", pos);
      if (e == std::string::npos) e = params.size();
      decl.push_back(params.substr(pos, e - pos));
      pos = e + 2;
    }
    const size_t K = decl.size();
    std::ostringstream o;
    o << "struct " << name << "_tab { void* p[" << K * count << "]; };\n";
    o << head << name << "(const __grid_constant__ " << name << "_tab t) {\n";
    o << "  const int member = blockIdx.z;\n";
    for (size_t i = 0; i < K; ++i) {
      // "<type> pN": the type without its __restrict__, for the cast
      const std::string& d = decl[i];
      const size_t sp = d.rfind(' ');
      std::string type = d.substr(0, sp), var = d.substr(sp + 1), bare = type;
      const size_t r = bare.find(" __restrict__");
      if (r != std::string::npos) bare.erase(r, 13);
      o << "  " << type << " " << var << " = (" << bare << ")t.p[member * " << K << " + " << i << "];\n";
    }
    o << c.substr(close + 3);  // the body after "{"
    return o.str();
  }

  void run() {
    auto order = group_all_reduces(topo());
    // parameters
    for (size_t i = 0; i < g.nodes.size(); ++i) {
      const Node& n = g.nodes[i];
      if (n.op != Op::Parameter || n.dead) continue;
      int s = new_slot(Slot::PARAM, n.results[0], n.name, (int)n.param_index);
      slot[ValueRef{(int)i, 0}] = s;
    }
    p.param_slots.assign(g.param_types.size(), -1);
    for (auto& kv : slot) p.param_slots.at(p.slots[kv.second].index) = kv.second;
    for (size_t i = 0; i < p.param_slots.size(); ++i)
      if (p.param_slots[i] < 0)
        p.param_slots[i] = new_slot(Slot::PARAM, g.param_types[i], "%arg" + std::to_string(i), (int)i);
    p.param_types = g.param_types;

    for (int n : order) {
      Node& nd = g.nodes[n];
      if (nd.op == Op::Parameter) continue;
      if (nd.op == Op::Constant) {
        if (!nd.cdata.splat && nd.results[0].numel() > 1) {
          int s = new_slot(Slot::CONST, nd.results[0], nd.name, (int)p.consts.size());
          p.consts.push_back(nd.cdata);
          slot[ValueRef{n, 0}] = s;
          continue;
        }
        if (!must_materialize(n)) continue;
      }
      if (is_fusible(nd.op)) {
        if (!must_materialize(n)) continue;
        // Loop outputs of one shape are emitted together: one kernel computes
        // them all (e.g. an optimizer's new parameter and both moments, or
        // every same-shaped parameter's update), sharing loads and
        // subexpressions.  Any other kernel flushes the group first.
        if (!pending.empty() &&
            (g.nodes[pending[0]].results[0].dims != nd.results[0].dims || pending.size() >= 24))
          flush_loops();
        temp_for(ValueRef{n, 0});
        maybe_planes(n);
        pending.push_back(n);
        continue;
      }
      flush_loops();
      if (nd.op != Op::Reduce) flush_rg();
      switch (nd.op) {
        case Op::Reduce: {
          std::vector<int> outs;
          for (size_t k = 0; k < nd.results.size(); ++k) outs.push_back(temp_for(ValueRef{n, (int)k}));
          const int split = reduce_split(nd);
          int64_t rows = 0, red = 0;
          if (split == 1 && reduce_rows(n, &rows, &red)) {
            add_reduce_phase(n, outs, rows, red);
            break;
          }
          flush_rg();
          if (split > 1) {
            std::vector<int> parts;
            for (size_t k = 0; k < nd.results.size(); ++k) {
              TensorType pt = nd.results[k];
              pt.dims.insert(pt.dims.begin(), split);
              if (pt.dtype == DType::BF16) pt.dtype = DType::F32;  // partials stay f32 until the final store
              parts.push_back(new_slot(Slot::TEMP, pt, "reduce_partials"));
            }
            add_kernel(cg.reduce(n, parts, split));
            add_kernel(cg.reduce_partials(n, parts, outs, split));
          } else {
            add_kernel(cg.reduce(n, outs));
          }
          break;
        }
        case Op::ReduceWindow: {
          std::vector<int> outs;
          for (size_t k = 0; k < nd.results.size(); ++k) outs.push_back(temp_for(ValueRef{n, (int)k}));
          add_kernel(cg.reduce_window(n, outs));
          break;
        }
        case Op::SelectAndScatter:
          add_kernel(cg.select_and_scatter(n, temp_for(ValueRef{n, 0})));
          break;
        case Op::Gather:
          add_kernel(cg.gather(n, temp_for(ValueRef{n, 0})));
          break;
        case Op::Scatter: {
          int out = temp_for(ValueRef{n, 0});
          auto it = slot.find(nd.operands[0]);
          const Graph& comb = *nd.regions.at(0);
          const Node& cn = comb.nodes.at(comb.outputs.at(0).node);
          if (g.type(nd.operands[0]).dtype == DType::BF16 && cn.op == Op::Add && nd.operands.size() == 3) {
            // A bf16 sum (an embedding gradient) is accumulated in an f32
            // buffer and rounded once: no per-add bf16 rounding in whatever
            // order the atomics land, only f32 addition order.
            TensorType ft = g.type(nd.operands[0]);
            ft.dtype = DType::F32;
            const int acc = new_slot(Slot::TEMP, ft, "scatter_f32_accumulator");
            std::vector<int64_t> ident(ft.rank());
            for (int d = 0; d < ft.rank(); ++d) ident[d] = d;
            if (it != slot.end()) add_kernel(cg.permute(it->second, ident, acc));
            else add_kernel(cg.loop({nd.operands[0]}, {acc}));
            add_kernel(cg.scatter(n, acc));
            add_kernel(cg.permute(acc, ident, out));
            break;
          }
          if (it != slot.end()) {
            Step c;
            c.kind = StepKind::Copy;
            c.name = "copy";
            c.in = {it->second};
            c.out = {out};
            p.steps.push_back(c);
          } else {
            add_kernel(cg.loop({nd.operands[0]}, {out}));
          }
          add_kernel(cg.scatter(n, out));
          break;
        }
        case Op::DotGeneral: lower_dot(n); break;
        case Op::Convolution: lower_conv(n); break;
        case Op::FusedSdpa: lower_fused_sdpa(n, nd); break;
        case Op::FusedSdpaBwd: lower_fused_sdpa_bwd(n, nd); break;
        case Op::FusedLayerNorm: lower_fused_ln(n, nd); break;
        case Op::AllReduce: lower_all_reduce(n, nd); break;
        case Op::CustomCall:
          if (nd.target == "mlx_sdpa") { lower_sdpa_custom(n, nd); break; }
          if (nd.target == "mlx_layer_norm") { lower_ln_custom(n, nd); break; }
          throw PjrtErr(12, "custom_call @" + nd.target + " is not supported by the B200 plugin");
        default:
          throw PjrtErr(12, std::string("op ") + op_name(nd.op) + " is not supported by the B200 plugin");
      }
    }
    flush_loops();
    flush_rg();
    bucket_all_reduces();
    // outputs
    std::set<int> used;
    for (size_t i = 0; i < g.outputs.size(); ++i) {
      ValueRef v = g.outputs[i];
      const TensorType& t = g.type(v);
      p.output_types.push_back(t);
      auto it = slot.find(v);
      if (it == slot.end()) throw PjrtErr(13, "output value was not materialized");
      int s = it->second;
      Slot& sl = p.slots[s];
      if (sl.kind == Slot::TEMP && !used.count(s)) {
        sl.kind = Slot::OUTPUT;
        sl.index = (int)i;
        used.insert(s);
        p.output_slots.push_back(s);
      } else {
        int o = new_slot(Slot::OUTPUT, t, "out" + std::to_string(i), (int)i);
        Step c;
        c.kind = StepKind::Copy;
        c.name = "copy";
        c.in = {s};
        c.out = {o};
        p.steps.push_back(c);
        p.output_slots.push_back(o);
      }
    }
    batch_steps();
    // temp lifetimes
    p.temp_first.assign(p.slots.size(), -1);
    p.temp_last.assign(p.slots.size(), -1);
    for (size_t i = 0; i < p.steps.size(); ++i) {
      for (auto* v : {&p.steps[i].in, &p.steps[i].out})
        for (int s : *v) {
          if (s < 0) continue;
          if (p.temp_first[s] < 0) p.temp_first[s] = (int)i;
          p.temp_last[s] = (int)i;
        }
    }
    // a parent slot lives from its first view's first use to its last view's last
    for (size_t s = 0; s < p.slots.size(); ++s) {
      const int par = p.slots[s].parent;
      if (par < 0 || p.temp_first[s] < 0) continue;
      if (p.temp_first[par] < 0 || p.temp_first[s] < p.temp_first[par]) p.temp_first[par] = p.temp_first[s];
      p.temp_last[par] = std::max(p.temp_last[par], p.temp_last[s]);
    }
    // distinct kernel bodies, spread over units of similar code size (kernels
    // no step launches -- members of a batched launch -- are left out)
    std::set<std::string> launched;
    for (auto& st : p.steps)
      if (st.kind == StepKind::Kernel) launched.insert(st.name);
    std::map<std::string, std::string> seen;  // code with the name blanked -> kernel
    std::vector<const GenKernel*> uniq;
    for (auto& k : kernels) {
      if (!launched.count(k.name)) continue;
      std::string key = k.code;
      const size_t at = key.find(" " + k.name + "(");
      if (at != std::string::npos) key.replace(at + 1, k.name.size(), "@");
      auto it = seen.find(key);
      if (it != seen.end()) {
        p.kernel_alias[k.name] = it->second;
        continue;
      }
      seen.emplace(std::move(key), k.name);
      uniq.push_back(&k);
    }
    std::ostringstream src;
    src << CodeGen::prelude();
    for (auto* k : uniq) src << "\n" << k->code;
    p.source = src.str();
    size_t total = 0;
    for (auto* k : uniq) total += k->code.size();
    const size_t nunits = std::min<size_t>(uniq.size(), std::max<size_t>(1, (total + 24000) / 24000));
    const size_t units = std::min<size_t>(nunits, 32);
    std::vector<std::ostringstream> us(units);
    std::vector<size_t> load(units, 0);
    p.unit_names.assign(units, {});
    for (auto& u : us) u << CodeGen::prelude();
    for (auto* k : uniq) {
      const size_t i = std::min_element(load.begin(), load.end()) - load.begin();
      us[i] << "\n" << k->code;
      load[i] += k->code.size();
      p.unit_names[i].push_back(k->name);
    }
    for (auto& u : us) p.units.push_back(u.str());
  }
};

}  // namespace

namespace {
// Dimensions of a row-major tensor that the GEMM can address as one strided
// group (they must be contiguous among themselves, in order).
bool groupable(const TensorType& t, const std::vector<int64_t>& dims, int64_t* stride) {
  std::vector<int64_t> st(t.rank(), 1);
  for (int i = t.rank() - 2; i >= 0; --i) st[i] = st[i + 1] * t.dims[i + 1];
  int64_t prev = -1, size = 1;
  *stride = 0;
  for (auto d : dims) {
    if (t.dims[d] == 1) continue;
    size *= t.dims[d];
    if (prev >= 0 && st[prev] != st[d] * t.dims[d]) return false;
    prev = d;
    *stride = st[d];
  }
  if (size == 1) *stride = 0;
  return true;
}

// A dot_general operand whose batch, free or contracting dimensions cannot be
// addressed as strided groups by the GEMM (e.g. attention over [B, T, N, H]
// with batch dims B and N) is read through an explicit transpose to batch,
// free, contracting order.  As a graph node the transpose is planned like any
// other fusible value: the kernel that produces the operand (a projection's
// bias add) writes it in the GEMM's order, instead of a copy pass afterwards.
void canonicalize_dot_operands(Graph& g) {
  std::map<std::pair<int, std::vector<int64_t>>, int> made;  // (operand node, perm) -> transpose
  const size_t n0 = g.nodes.size();
  for (size_t n = 0; n < n0; ++n) {
    if (g.nodes[n].dead || g.nodes[n].op != Op::DotGeneral) continue;
    for (int side = 0; side < 2; ++side) {
      Node& dn = g.nodes[n];
      const ValueRef v = dn.operands[side];
      const TensorType t = g.type(v);
      std::vector<int64_t>& batch = side == 0 ? dn.lhs_batch : dn.rhs_batch;
      std::vector<int64_t>& contract = side == 0 ? dn.lhs_contract : dn.rhs_contract;
      std::vector<int64_t> free_dims;
      for (int64_t d = 0; d < t.rank(); ++d)
        if (std::find(batch.begin(), batch.end(), d) == batch.end() &&
            std::find(contract.begin(), contract.end(), d) == contract.end())
          free_dims.push_back(d);
      int64_t sb, sf, sc;
      const bool ok = groupable(t, batch, &sb) && groupable(t, free_dims, &sf) &&
                      groupable(t, contract, &sc);
      // one of the two matrix dimensions must be unit-stride (or trivial)
      auto unit = [&](const std::vector<int64_t>& dims, int64_t s) {
        int64_t size = 1;
        for (auto d : dims) size *= t.dims[d];
        return size == 1 || s == 1;
      };
      if (ok && (unit(free_dims, sf) || unit(contract, sc))) continue;
      if (t.dtype != DType::F32 && t.dtype != DType::BF16) continue;
      std::vector<int64_t> perm = batch;
      perm.insert(perm.end(), free_dims.begin(), free_dims.end());
      perm.insert(perm.end(), contract.begin(), contract.end());
      int tn;
      auto key = std::make_pair(v.node * 8 + v.idx, perm);
      auto it = made.find(key);
      if (it != made.end()) {
        tn = it->second;
      } else {
        Node tr;
        tr.op = Op::Transpose;
        tr.operands = {v};
        tr.dims = perm;
        TensorType ot;
        ot.dtype = t.dtype;
        for (auto d : perm) ot.dims.push_back(t.dims[d]);
        tr.results = {ot};
        tr.name = g.nodes[v.node].name + ".T";
        g.nodes.push_back(tr);
        tn = (int)g.nodes.size() - 1;
        made[key] = tn;
      }
      Node& dn2 = g.nodes[n];  // (push_back may have moved the nodes)
      dn2.operands[side] = ValueRef{tn, 0};
      std::vector<int64_t>& b2 = side == 0 ? dn2.lhs_batch : dn2.rhs_batch;
      std::vector<int64_t>& c2 = side == 0 ? dn2.lhs_contract : dn2.rhs_contract;
      const int64_t nb = (int64_t)b2.size(), nf = (int64_t)free_dims.size();
      for (int64_t i = 0; i < nb; ++i) b2[i] = i;
      for (size_t i = 0; i < c2.size(); ++i) c2[i] = nb + nf + (int64_t)i;
    }
  }
}
}  // namespace

Plan build_plan(const Module& m) {
  Plan p;
  p.num_replicas = m.num_replicas;
  Graph g = inline_calls(m);
  simplify(g);
  dce(g);
  MatchStats ms = match_patterns(g);
  (void)ms;
  simplify(g);
  dce(g);
  canonicalize_dot_operands(g);
  p.graph_dump = dump_graph(g);
  Builder b(p, g);
  b.run();
  return p;
}

std::string dump_plan(const Plan& p) {
  std::ostringstream os;
  os << "slots:\n";
  for (size_t i = 0; i < p.slots.size(); ++i) {
    const Slot& s = p.slots[i];
    static const char* kinds[] = {"param", "output", "temp", "const"};
    os << "  s" << i << " " << kinds[s.kind] << "[" << s.index << "] " << s.type.str() << " "
       << s.what;
    if (s.parent >= 0) os << " view=s" << s.parent << "+" << s.offset;
    os << "\n";
  }
  os << "steps:\n";
  for (auto& st : p.steps) {
    os << "  " << st.name << " in=";
    for (int s : st.in) os << "s" << s << ",";
    os << " out=";
    for (int s : st.out) os << "s" << s << ",";
    if (!st.ip.empty()) os << " ip=" << join_ints(st.ip);
    os << "\n";
  }
  return os.str();
}

}  // namespace b200
