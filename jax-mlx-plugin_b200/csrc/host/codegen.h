// CUDA C generation for fused elementwise / reduce / window / gather / scatter
// kernels (compiled with NVRTC for sm_100a at PJRT_Client_Compile time).
#pragma once
#include <functional>
#include <map>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "ir.h"
#include "plan.h"

namespace b200 {

// Where the generated code reads a value from: a materialized slot, or (slot
// < 0) recomputed inline from the value's defining node.
using SlotOf = std::function<int(ValueRef)>;

// One phase of a row group: a reduction of the last dimension, or a set of
// values stored at every element of the rows.
struct RowPhase {
  int reduce = -1;               // Reduce node, or -1 for a loop phase
  // With reduce a row max M of X: a second reduce node summing exp(X - M),
  // computed in the same pass with a running maximum (out_slots: M, then the
  // sum).
  int sum_reduce = -1;
  std::vector<ValueRef> roots;   // loop phase: the values stored
  std::vector<int> out_slots;    // reduce results / loop outputs, in order
};

struct GenKernel {
  std::string name;
  std::string code;
  std::vector<int> ptr_slots;  // kernel pointer parameters, in order
  std::vector<bool> ptr_written;
  int64_t grid = 1, block = 256;
  int64_t grid_y = 1;   // >1: split reduction (blockIdx.y = split index)
  int64_t block_y = 1;  // >1: 2-D block (32, block_y) of column reductions
};

class CodeGen {
 public:
  CodeGen(const Graph& g, const std::vector<Slot>& slots, SlotOf slot_of)
      : g_(g), slots_(slots), slot_of_(std::move(slot_of)),
        round_each_op_(bf16_round_each_op_from_env()) {}

  // out = value at each index of `v`'s shape (loop fusion root).
  GenKernel loop(const std::vector<ValueRef>& roots, const std::vector<int>& out_slots);
  // Reduce node (variadic) -> out slots (one per result).  With split > 1 the
  // reduced range is divided over gridDim.y blocks and out_slots receive
  // [split, OUT] partials, combined by reduce_partials.
  GenKernel reduce(int node, const std::vector<int>& out_slots, int split = 1);
  // A reduction that keeps the input's innermost dimension (a bias or norm-gain
  // gradient: sum over tokens of [tokens, features]) is emitted with each
  // thread owning this many consecutive outputs, read as one vector load per
  // operand and row: 8 or 4 when the innermost dimension splits into such
  // groups and there are at least 32 such groups, else 1 (one output per
  // thread).
  static int column_vec(const TensorType& in, const std::vector<int64_t>& reduce_dims);
  static constexpr int kColWarps = 8;  // warps (rows in flight) per block of a vector column reduction
  GenKernel reduce_partials(int node, const std::vector<int>& partial_slots,
                            const std::vector<int>& out_slots, int split);
  GenKernel reduce_window(int node, const std::vector<int>& out_slots);
  GenKernel select_and_scatter(int node, int out_slot);
  GenKernel gather(int node, int out_slot);
  // scatter: out already holds the operand; this kernel applies the updates.
  GenKernel scatter(int node, int out_slot);
  // im2col for a convolution: A[m, k] (row-major, M x K) from the lhs operand.
  // k_roles: kernel dims (excluding k_out) in K order; m_roles: output dims
  // (excluding out_feature) in M order.
  // With lo_slot >= 0 (f32 input), out_slot / lo_slot receive the patches as
  // bf16 hi / lo planes for an f32 GEMM (x ~= hi + lo).
  GenKernel im2col(int node, int out_slot, const std::vector<int64_t>& k_roles,
                   const std::vector<int64_t>& m_roles, int64_t M, int64_t K, int lo_slot = -1);
  // The same patches stored transposed ([K, M], M innermost) as bf16 hi / lo
  // planes, eight M columns per thread; only when the innermost M role is the
  // output batch dimension, fed by the input's innermost dimension, with M a
  // multiple of 8 and the input an f32 slot (see plan.cc:lower_conv).
  GenKernel im2col_t(int node, int out_slot, const std::vector<int64_t>& k_roles,
                     const std::vector<int64_t>& m_roles, int64_t M, int64_t K, int lo_slot);
  // out[j] = src[permuted j]: out dims are src dims[perm[i]] (a transpose copy).
  GenKernel permute(int src_slot, const std::vector<int64_t>& perm, int out_slot);
  // Several row-wise phases over the same OUT rows of RED elements in one
  // kernel: one warp (or, for rows above 4096 elements read by more than one
  // phase, one 256-thread block) per row runs the phases in
  // order, with a barrier between them, so that a phase reads what earlier
  // phases wrote for its row (still in L1/L2) instead of a separate kernel
  // reading it back from HBM.  Every read of a phase output by a later phase
  // must be at the same row (the planner checks this).
  GenKernel rowgroup(const std::vector<RowPhase>& phases, int64_t OUT, int64_t RED);
  // A sum over the last dimension of one_hot * Y -- one_hot being
  // convert(compare(EQ, iota along that dimension, a value constant along it)),
  // reached through negations and float converts -- has one nonzero term per
  // row: the one at the compared value.  Returns that value (any position of
  // the row gives it), or node -1.  rowgroup evaluates such a reduction at that
  // one position instead of over the whole row.
  ValueRef onehot_pick(int reduce_node) const;

  static std::string prelude();
  int counter = 0;
  // f32 values stored as a GEMM's bf16 hi / lo planes: hi slot -> lo slot
  // (the hi slot's type is bf16); set by the planner.
  const std::map<int, int>* plane_lo = nullptr;

 private:
  // An element index: row-major linear form (lin) and/or per-dimension form
  // (multi), as C expressions.  Vector form (lane >= 0): the index is element
  // `lane` of a group of vec_ consecutive elements along the innermost
  // dimension -- lin == lin_base + lane with lin_base a multiple of vec_, and
  // multi.back() == inner_base + lane with the other entries lane-independent.
  // Loads of slots through a vector-form index become one 16-byte (or 8/32)
  // load per group, shared by the group's lanes.
  struct Idx {
    std::vector<int64_t> dims;
    std::string lin;
    std::vector<std::string> multi;
    int lane = -1;
    std::string lin_base, inner_base;
  };
  const Graph& g_;
  const std::vector<Slot>& slots_;
  SlotOf slot_of_;

  // per-kernel state
  std::ostringstream body_;
  std::vector<int> ptrs_;
  std::vector<bool> written_;
  std::vector<std::map<std::string, std::string>> memo_;
  // Values computed inline even though they have a slot (the roots a loop
  // phase is storing), and slots written earlier in the same kernel (read
  // through the coherent path, not the read-only cache).
  std::set<ValueRef> hidden_;
  std::set<int> coherent_;
  // f32 nodes whose every use in the kernel being emitted ends in a bf16 value
  // (a convert to bf16, or a bf16 output): their exp / log / tanh / divide
  // use the approximate hardware forms, as bf16-typed nodes do -- the result
  // is rounded to 8 significant bits anyway.
  std::set<int> bf16_sink_;
  // Inside a row group's loop phase (b = o * RED + r, r < RED): the row count
  // and length, else 0.
  int64_t row_loop_out_ = 0, row_loop_red_ = 0;
  // out_slots (optional, parallel to roots): a root stored as a GEMM's bf16
  // hi / lo planes (about 16 significant bits) counts as a bf16 sink too.
  void mark_bf16_sinks(const std::vector<ValueRef>& roots, const std::vector<int>* out_slots = nullptr);
  // Set while emitting a reduction's combiner: bf16 partial results stay in
  // f32 and are rounded once when stored (XLA accumulates bf16 reductions in
  // f32 rather than rounding after every add).
  bool accum_f32_ = false;
  // Round every bf16 op's result (B200_BF16_ROUND_EACH_OP=1 when compiling);
  // otherwise bf16 values stay f32 until stored or converted.
  bool round_each_op_ = false;
  static bool bf16_round_each_op_from_env();
  int vec_ = 1;  // elements per thread group in vector-form kernels
  int tmp_ = 0;
  int indent_ = 1;
  std::string idx_t_ = "int";

  void reset();
  std::string fresh(const char* p = "v");
  void line(const std::string& s);
  std::string ptr(int slot, bool write);
  void ensure_multi(Idx& idx);
  void ensure_lin(Idx& idx);
  std::string value(ValueRef v, Idx idx);
  std::string load(int slot, Idx& idx, DType dt);
  Idx vec_idx(const std::vector<int64_t>& dims, const std::string& base, int lane);
  void vec_load(const std::string& dst, int slot, const std::string& base);
  void vec_store(int slot, const std::string& base, const std::vector<std::string>& vals, DType dt);
  // Store a loop root: plain, or as hi / lo planes when the slot has a lo plane.
  void store_root(int slot, const std::string& base, const std::vector<std::string>& vals, DType dt);
  void store_root1(int slot, const std::string& at, const std::string& v, DType dt);
  std::string elementwise(const Node& n, const std::vector<std::string>& a, DType in_dt);
  std::string literal(const Node& n);
  std::string emit_region(const Graph& r, const std::vector<std::string>& args,
                          std::vector<std::string>* outs);
  std::string header(const std::string& name);
  GenKernel finish(const std::string& name, int64_t total, int64_t block, int64_t max_grid);
  GenKernel reduce_columns(int node, const std::vector<int>& out_slots, int split,
                           const std::string& name, const std::vector<std::string>& outp,
                           const std::vector<int64_t>& kdims, const std::vector<int64_t>& rdims,
                           const std::vector<int64_t>& kpos, const std::vector<int64_t>& rpos);
};

std::string ctype(DType t);     // register type
std::string stype(DType t);     // storage type
std::string store_conv(DType t, const std::string& v);  // register -> storage

}  // namespace b200
