// Compile-time expansion of the reference's backward custom calls into
// StableHLO (see custom_calls.cc).
#pragma once
#include <string>
#include <vector>

#include "ir.h"

namespace b200 {

// True for custom-call targets that are expanded into StableHLO at compile time.
bool expands_custom_call(const std::string& target);

// A module whose @main takes the custom call's operands (types as given) and
// returns its results, written in StableHLO text.
std::string custom_call_expansion(const Node& n, const std::vector<TensorType>& operand_types);

// mlx_sdpa_bwd on the fused attention kernels: when the operands `ops` (in
// `dst`) are bf16 [B, T, N, 64] with T <= 256, adds the attention forward
// with row statistics and the fused backward to `dst`, sets `outs` to
// (dQ, dK, dV) and returns true; otherwise adds nothing and returns false.
bool fused_sdpa_bwd_call(const Node& n, const std::vector<ValueRef>& ops, Graph& dst,
                         std::vector<ValueRef>& outs);

}  // namespace b200
