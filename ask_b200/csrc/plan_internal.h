// The plan object behind the C ABI's opaque ask_b200_plan, shared by the plan
// layer (plan.cpp) and the kernel-artifact generator (artifact.cpp).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "kernels.h"

namespace askb {

enum Family { FAM_ELEMENTWISE = 0, FAM_REDUCE, FAM_GATHER, FAM_SCATTER, FAM_SOFTMAX };

struct PortInfo {
  int dtype;
  uint64_t elements;
  int map;
};

}  // namespace askb

struct ask_b200_plan {
  int family = askb::FAM_ELEMENTWISE;
  int device = -1;
  int num_sms = 148;
  std::vector<askb::PortInfo> inputs, outputs;
  askb::Program prog{};
  askb::Program ssa{};  // the canonical SSA program before register assignment (artifact generation)
  int spec = 0;
  int strategy = 0;
  int grid = 1;
  int launches = 1;
  size_t scratch = 0;
  size_t record_offset = 0;  // sharded reduce: where the per-rank records live in scratch
  uint64_t count = 0, inner = 1;
  askb::RedArgs red{};
  askb::IndexArgs idx{};
  askb::SoftmaxArgs sm{};
  bool views = false;  // elementwise step with IM_VIEW ports or coordinate instructions
  askb::ViewSet vs{};
  bool shardable = false;
  std::string kernel;
  int block = 256;  // threads per CTA where the family fixes it (softmax)
  int col_chunks = 1;  // RS_COLUMN: chunks of the extent over grid.y (1 = the one-pass column kernel)
  int blocks_per_sm = 0;  // recipe cap on resident CTAs per SM of a persistent grid (0 = occupancy)
  int sm_step = 0;   // reduce matched to a softmax step run by the softmax row kernel (SoftmaxMode), else 0
  int red_grid = 1;  // sm_step: the warp-row kernel's grid for a launch whose x is not 16-byte aligned
};

