// Execution-plan verification and workspace slot assignment for the runtime
// layer (runtime.cpp).
//
// A program is a list of steps over logical buffers: public inputs are
// caller-owned, every other buffer has exactly one producing step, and the
// non-public buffers live in workspace "slots" that later buffers may reuse.
// The rules follow the reference's plan verifier (lib/Pass/Pass.h:13-55,
// lib/Pass/Pass.cpp:12-208) and its two slot assigners, one for stream order
// and one for a dependency graph (lib/Runtime/CUDA.cpp:609-677, 794-813):
//
//   - a step may read only buffers that are public inputs or were produced
//     by an earlier step (diagnostic READ_<step>_<port>);
//   - a slot holds each assigned buffer (CAPACITY_<buffer>);
//   - stream order: two consecutive occupants of one slot must not be live at
//     the same step (ADJACENT_<a>_<b>);
//   - graph order: each step's data producers, and every access of the
//     previous occupant of each slot the step writes, must precede the step
//     through the declared dependency edges (GRAPH_ORDER_<step>).
//
// Diagnostics are "verify <NAME> FAIL\n" lines in that order (reads,
// capacities in assignment order, slot obligations in slot order, graph
// orders in step order), the format the reference reports, so callers that
// parse them keep working.
#pragma once

#include <cstddef>
#include <string>
#include <vector>

namespace askb {
namespace check {

struct StepPorts {
  std::vector<size_t> inputs, outputs;
};

struct Plan {
  size_t buffer_count = 0;
  std::vector<size_t> public_inputs, public_outputs;
  std::vector<StepPorts> steps;
};

struct SlotAssignment {
  size_t buffer = 0, slot = 0;
};

struct Allocation {
  Plan plan;
  std::vector<size_t> buffer_sizes;
  std::vector<SlotAssignment> assignments;
  std::vector<size_t> slot_capacity_bytes;
  bool graph = false;
  std::vector<std::vector<size_t>> dependencies;  // graph mode: predecessor steps of each step
};

struct Verdict {
  bool pass = false;
  std::string explanation;  // first structural error, or the list of failed obligations
};

// Availability only: every read and public output has a producer before it.
Verdict check_plan(const Plan& plan);

// Everything check_plan checks, plus the mapping (each non-public buffer in
// exactly one slot, no empty slot, no public buffer in a slot), capacities and
// the stream- or graph-order reuse obligations.
Verdict check_allocation(const Allocation& allocation);

// Fill assignments and slot capacities for stream order: a slot is reused by
// the first later buffer produced after its occupant's last access.
void assign_stream_slots(Allocation& allocation);

// Fill dependencies (each step depends on the producers of its inputs) and
// assignments for graph order: a slot is reused only when every access of its
// occupant is an ancestor of the new producer in that dependency graph.
void assign_graph_slots(Allocation& allocation);

}  // namespace check
}  // namespace askb
