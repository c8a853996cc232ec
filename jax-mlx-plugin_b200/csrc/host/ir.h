// Typed SSA IR for StableHLO modules.
//
// A Graph is one function body: Nodes in program order, each producing one or
// more typed results.  Operands refer to (node, result index).  Attributes are
// structured per op kind rather than kept as strings.  Replaces the reference's
// string-keyed MLXOp/MLXGraph (src/jax_mlx_pjrt.cpp:412-432).
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace b200 {

enum class DType : uint8_t {
  INVALID = 0, PRED = 1, S8 = 2, S16 = 3, S32 = 4, S64 = 5, U8 = 6, U16 = 7, U32 = 8, U64 = 9,
  F16 = 10, F32 = 11, F64 = 12, BF16 = 13, TOKEN = 23
};  // numbered as PJRT_Buffer_Type

int dtype_size(DType t);
const char* dtype_name(DType t);       // "f32", "bf16", "i32", ...
DType dtype_from_mlir(const std::string& s);  // "f32", "i1", "ui32", "bf16"
bool dtype_is_float(DType t);
bool dtype_is_int(DType t);            // signed or unsigned integer (not pred)
bool dtype_is_unsigned(DType t);

struct TensorType {
  DType dtype = DType::INVALID;
  std::vector<int64_t> dims;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
  int64_t bytes() const { return numel() * dtype_size(dtype); }
  int rank() const { return (int)dims.size(); }
  bool operator==(const TensorType& o) const { return dtype == o.dtype && dims == o.dims; }
  bool operator!=(const TensorType& o) const { return !(*this == o); }
  std::string str() const;
};

enum class Op : uint16_t {
  Parameter, Constant, Iota,
  // elementwise unary
  Neg, Abs, Exp, Expm1, Log, Log1p, Sqrt, Rsqrt, Cbrt, Tanh, Logistic, Sin, Cos, Tan, Erf,
  Floor, Ceil, RoundAfz, RoundEven, Sign, Not, IsFinite, PopCnt, Imag, Real,
  // elementwise binary
  Add, Sub, Mul, Div, Rem, Max, Min, Pow, Atan2, And, Or, Xor, ShiftLeft,
  ShiftRightArith, ShiftRightLogical,
  // other elementwise
  Compare, Select, Clamp, Convert, BitcastConvert,
  // layout
  BroadcastInDim, Reshape, Transpose, Slice, DynamicSlice, DynamicUpdateSlice, Pad,
  Concatenate, Reverse,
  // heavy
  Reduce, DotGeneral, Convolution, ReduceWindow, SelectAndScatter, Gather, Scatter,
  CustomCall, AllReduce, Sort,
  // structure
  Call, Return, OptimizationBarrier, Tuple, GetTupleElement,
  // fused ops created by the pattern matcher
  FusedSdpa, FusedLayerNorm, FusedSdpaBwd,
  NumOps
};
const char* op_name(Op op);

enum class CmpDir : uint8_t { EQ, NE, LT, LE, GT, GE };
enum class CmpType : uint8_t { FLOAT, SIGNED, UNSIGNED, TOTALORDER, NOTYPE };

struct ValueRef {
  int node = -1;
  int idx = 0;
  bool operator==(const ValueRef& o) const { return node == o.node && idx == o.idx; }
  bool operator<(const ValueRef& o) const { return node != o.node ? node < o.node : idx < o.idx; }
};

struct Graph;

// Dense constant data, stored in the element type's own byte layout.
struct ConstData {
  bool splat = false;
  std::vector<uint8_t> bytes;  // one element if splat, numel elements otherwise
};

struct ConvDims {
  int64_t in_batch = 0, in_feature = 0;
  std::vector<int64_t> in_spatial;
  int64_t k_in = 0, k_out = 0;
  std::vector<int64_t> k_spatial;
  int64_t out_batch = 0, out_feature = 0;
  std::vector<int64_t> out_spatial;
};

struct GatherDims {
  std::vector<int64_t> offset_dims, collapsed_slice_dims, start_index_map,
      operand_batching_dims, start_indices_batching_dims;
  int64_t index_vector_dim = 0;
  std::vector<int64_t> slice_sizes;
};

struct ScatterDims {
  std::vector<int64_t> update_window_dims, inserted_window_dims, scatter_dims_to_operand_dims,
      input_batching_dims, scatter_indices_batching_dims;
  int64_t index_vector_dim = 0;
};

struct Node {
  Op op = Op::Parameter;
  std::vector<ValueRef> operands;
  std::vector<TensorType> results;
  std::string name;  // SSA name of result 0, for diagnostics

  // --- attributes (which ones are meaningful depends on op) ---
  int64_t param_index = -1;        // Parameter
  ConstData cdata;                 // Constant
  int64_t iota_dim = 0;            // Iota
  CmpDir cmp_dir = CmpDir::EQ;     // Compare
  CmpType cmp_type = CmpType::NOTYPE;
  std::vector<int64_t> dims;       // BroadcastInDim dims, Transpose perm, Reduce dims, Reverse dims
  std::vector<int64_t> start, limit, strides;  // Slice; DynamicSlice sizes in `limit`
  std::vector<int64_t> pad_lo, pad_hi, pad_interior;  // Pad; conv/window padding lo/hi
  int64_t axis = 0;                // Concatenate dimension
  // dot_general
  std::vector<int64_t> lhs_batch, rhs_batch, lhs_contract, rhs_contract;
  // convolution / windows
  std::vector<int64_t> window, window_strides, lhs_dilation, rhs_dilation, base_dilation,
      window_dilation;
  std::vector<bool> window_reversal;
  ConvDims conv;
  int64_t feature_groups = 1, batch_groups = 1;
  GatherDims gather;
  ScatterDims scatter;
  // regions: reduce/reduce_window/scatter/all_reduce/select_and_scatter bodies
  std::vector<std::shared_ptr<Graph>> regions;
  // custom_call / call
  std::string target;              // custom_call target or callee symbol
  std::string backend_config;
  // all_reduce
  std::vector<std::vector<int64_t>> replica_groups;
  int64_t channel_id = 0;
  // fused ops (pattern matcher): scalar parameters
  float f_scale = 1.f, f_eps = 0.f;
  int i_flags = 0;                 // FusedSdpa: bit0 causal, bit1 emits row statistics; FusedSdpaBwd: bit0 causal; FusedLayerNorm: bit0 rms, bit1 has residual, bit2 has gamma, bit3 has beta, bit4 emits h
  bool dead = false;
};

struct Graph {
  std::string name;
  std::vector<Node> nodes;
  std::vector<TensorType> param_types;
  std::vector<ValueRef> outputs;  // set by the return statement

  const TensorType& type(ValueRef v) const { return nodes.at(v.node).results.at(v.idx); }
  int add(Node n) {
    nodes.push_back(std::move(n));
    return (int)nodes.size() - 1;
  }
};

struct Module {
  std::string name;
  int64_t num_replicas = 1, num_partitions = 1;
  std::map<std::string, std::shared_ptr<Graph>> funcs;
  std::string entry = "main";
  std::shared_ptr<Graph> main() const {
    auto it = funcs.find(entry);
    if (it == funcs.end()) throw std::runtime_error("module has no @" + entry + " function");
    return it->second;
  }
};

// Parse StableHLO text (pretty or generic printing) into a Module.
Module parse_module(const std::string& text);

// Error carrying a PJRT error code.
struct PjrtErr : std::runtime_error {
  int code;
  PjrtErr(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

std::string join_ints(const std::vector<int64_t>& v);

}  // namespace b200
