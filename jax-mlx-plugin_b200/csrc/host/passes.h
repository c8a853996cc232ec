// Graph passes run at PJRT_Client_Compile time, before fusion planning.
#pragma once
#include <optional>

#include "ir.h"

namespace b200 {

// Replace func.call nodes in `main` by the callee bodies (recursively).
Graph inline_calls(const Module& m);

// Forward optimization_barrier / sdy / identity converts, reshapes, transposes
// and broadcasts to their operands.
void simplify(Graph& g);

// Mark nodes not reachable from the outputs as dead.
void dce(Graph& g);

// Consumers of every node (live nodes only). outputs_use[n] counts graph
// outputs referring to node n.
struct Uses {
  std::vector<std::vector<int>> users;
  std::vector<int> output_refs;
  int count(int n) const { return (int)users[n].size() + output_refs[n]; }
};
Uses compute_uses(const Graph& g);

// Host evaluation of a constant subgraph (constants, iota and elementwise/
// layout ops on them), values widened to double.  nullopt if the value depends
// on a parameter, uses an unsupported op or exceeds `max_elems`.
struct HostTensor {
  TensorType type;
  std::vector<double> v;
};
std::optional<HostTensor> host_eval(const Graph& g, ValueRef v, int64_t max_elems = 1 << 22);

// Pattern matchers (the fusion rules of the north star):
//   dot_general -> [scale] -> [causal select] -> softmax -> dot_general -> FusedSdpa
//   the same chain plus its backward (dV, dP, softmax vjp, dQ, dK)
//                                           -> FusedSdpa (with row statistics) + FusedSdpaBwd
//   [residual add] -> mean/var -> normalize -> [gamma] -> [beta]  -> FusedLayerNorm
// Both refuse to fuse when an intermediate value has a consumer outside the
// pattern (reference src/jax_mlx_pjrt.cpp:1843-1855 applies the same guard).
struct MatchStats {
  int sdpa = 0, sdpa_train = 0, layer_norm = 0;
};
MatchStats match_patterns(Graph& g);

// Text dump of the live graph (for B200_DUMP and the inspection entry point).
std::string dump_graph(const Graph& g);

}  // namespace b200
