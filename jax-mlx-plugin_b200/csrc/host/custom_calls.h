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

}  // namespace b200
