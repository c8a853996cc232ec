// Compiled, device-independent program of one executable: memory slots and an
// ordered list of launch steps.  Built from the IR by plan.cc (fusion planning,
// GEMM/conv lowering) with NVRTC sources from codegen.cc; run by runtime.cc.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "ir.h"

namespace b200 {

struct Slot {
  enum Kind { PARAM, OUTPUT, TEMP, CONST } kind = TEMP;
  int index = -1;  // parameter / output / constant index
  TensorType type;
  int64_t bytes = 0;
  std::string what;  // producing value, for dumps
  // A view into another TEMP slot (byte offset): a gradient computed straight
  // into its piece of an all-reduce bucket, and the reduced value read back
  // from there.  The parent's lifetime covers its views'.
  int parent = -1;
  int64_t offset = 0;
};

struct Arg {
  enum Kind { PTR, I64, F32 } kind = PTR;
  int slot = -1;
  int64_t i = 0;
  float f = 0.f;
};

enum class StepKind {
  Kernel,     // NVRTC-generated kernel: name, grid/block, args
  LayerNorm,  // b200_ln_residual_fwd
  Sdpa,       // tcgen05 attention (with row statistics when it has a second output)
  SdpaBwd,    // tcgen05 attention backward
  Gemm,       // tcgen05 or SIMT GEMM
  AllReduce,  // NCCL sum over replicas
  Copy,       // device-to-device copy of slot bytes
};

struct Step {
  StepKind kind = StepKind::Kernel;
  std::string name;
  int64_t grid[3] = {1, 1, 1}, block[3] = {1, 1, 1};
  int smem = 0;
  std::vector<Arg> args;
  std::vector<int> in, out;  // slots read / written (liveness; kernel-specific order)
  std::vector<int64_t> ip;   // integer parameters
  std::vector<float> fp;     // float parameters
  int dtype = 0, dtype2 = 0;
  // Kernel: the pointer arguments go to the kernel as one table (an array of
  // pointers passed by value), as a batched launch of several steps' work
  // takes them (blockIdx.z selects a member's set).
  bool table = false;
};

struct Plan {
  std::vector<Slot> slots;
  std::vector<Step> steps;
  std::vector<int> param_slots, output_slots;
  std::vector<ConstData> consts;
  std::vector<TensorType> param_types, output_types;
  std::string source;  // NVRTC program (all generated kernels, each body once)
  std::vector<std::string> kernel_names;  // every step's kernel name
  // Compilation units (prelude + a share of the distinct kernels), compiled in
  // parallel, and the kernel names each defines.  A kernel whose code equals an
  // earlier one's (e.g. the same layer norm in every block) is compiled once:
  // kernel_alias maps its name to the compiled one.
  std::vector<std::string> units;
  std::vector<std::vector<std::string>> unit_names;
  std::map<std::string, std::string> kernel_alias;
  int64_t num_replicas = 1;
  std::vector<int> temp_first, temp_last;  // per slot: first/last step touching it
  std::string graph_dump;
  int num_sdpa = 0, num_ln = 0;
};

// Compile a parsed module into a Plan (throws PjrtErr on unsupported input).
// B200_OVERLAP_COLLECTIVES (runtime.cc): gradient all-reduces in buckets
// placed where their gradients are ready, run on a communication stream.
bool overlap_collectives();
Plan build_plan(const Module& m);

// Human-readable listing of the plan (steps, kernels, slots).
std::string dump_plan(const Plan& p);

}  // namespace b200
