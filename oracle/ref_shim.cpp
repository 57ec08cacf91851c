// Test-only C binding of the REFERENCE's own Runtime and PASS checker, built
// from the reference sources (lib/Runtime/CUDA.cpp, lib/Runtime/CUBLASLt.cpp,
// lib/Pass/Pass.cpp; include/ask/Runtime/CUDA.h, lib/Pass/Pass.h) by
// oracle/ref_build.py into oracle/_ref/libask_ref.so.  This file is this
// project's code; it only calls the reference's public C++ API:
//   - askref_pass_check: ask::pass::checkPlan / checkAllocationPlan
//     (lib/Pass/Pass.h:48-53) on the allocation JSON that
//     ask_b200_allocation_check takes, so the tests can compare the two
//     verifiers case by case;
//   - askref_run_step: Session::create, Session::load (cubin, entry, element
//     types, arch, parameter widths), prepareProgram with one kernel PlanStep,
//     run, copyToHost and stats (include/ask/Runtime/CUDA.h:64-175) -- the
//     reference's own loader running an ask_b200 kernel artifact;
//   - askref_run_program: a whole program of kernel steps in the JSON form
//     ask_b200_program_prepare_kernels takes, so the tests can run one
//     program through both runtimes and compare outputs and counters.
// Like everything under oracle/, it is a checker for the tests, never part of
// the product path.
#include <array>
#include <cstdint>
#include <cstring>
#include <exception>
#include <sstream>
#include <string>
#include <vector>

#include "Pass.h"
#include "ask/Runtime/CUDA.h"
#include "../ask_b200/csrc/json.h"

namespace {

void write_text(const std::string& s, char* buf, size_t cap) {
  if (buf && cap) {
    const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
}

std::vector<size_t> list(const askb::json::Value& v, const char* what) {
  std::vector<size_t> out;
  for (const auto& x : v.as_array(what)) out.push_back(size_t(uint64_t(x.as_int(what))));
  return out;
}

ask::pass::Plan parse_plan(const askb::json::Value& v) {
  ask::pass::Plan p;
  p.buffer_count = size_t(v.at("buffer_count").as_int("buffer_count"));
  p.public_inputs = list(v.at("public_inputs"), "public_inputs");
  p.public_outputs = list(v.at("public_outputs"), "public_outputs");
  for (const auto& s : v.at("steps").as_array("steps"))
    p.steps.push_back({list(s.at("inputs"), "inputs"), list(s.at("outputs"), "outputs")});
  return p;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int askref_pass_check(const char* allocation_json, int* pass, char* buf,
                                                             size_t cap) {
  try {
    const askb::json::Value v = askb::json::Parser(allocation_json).parse();
    ask::pass::Decision d;
    if (!v.get("buffer_sizes")) {
      d = ask::pass::checkPlan(parse_plan(v));
    } else {
      ask::pass::AllocationPlan a;
      a.plan = parse_plan(v);
      a.buffer_sizes = list(v.at("buffer_sizes"), "buffer_sizes");
      if (const auto* as = v.get("assignments"))
        for (const auto& e : as->as_array("assignments")) {
          const auto pair = list(e, "assignment");
          a.assignments.push_back({pair.at(0), pair.at(1)});
        }
      if (const auto* c = v.get("slot_capacity_bytes")) a.slot_capacity_bytes = list(*c, "slot_capacity_bytes");
      if (const auto* g = v.get("graph")) a.graph = g->kind == askb::json::Value::Bool && g->b;
      if (const auto* dd = v.get("dependencies"))
        for (const auto& e : dd->as_array("dependencies")) a.dependencies.push_back(list(e, "dependencies"));
      d = ask::pass::checkAllocationPlan(a);
    }
    *pass = d.verdict == ask::pass::Verdict::Pass ? 1 : 0;
    write_text(d.explanation, buf, cap);
    return 0;
  } catch (const std::exception& e) {
    write_text(e.what(), buf, cap);
    return -1;
  }
}

// One kernel step through the reference Runtime.  Buffers 0..n_in-1 are the
// program inputs, n_in..n_in+n_out-1 its outputs; parameter i binds buffer
// arg_buffer[i] (-1: null) or, when widths[i] > 0, the scalar bytes
// scalars[8*i .. 8*i+widths[i]).  The program runs `repeats` times (fresh
// inputs each time after the first, so graph mode updates its nodes); the
// outputs of the last run are copied to host_out.  stats receives the
// session counters as JSON.
__attribute__((visibility("default"))) int askref_run_step(
    int device, const void* image, size_t image_bytes, const char* entry, const char* types_csv, int arch,
    const unsigned* widths, size_t n_params, const int64_t* arg_buffer, const unsigned char* scalars,
    const unsigned grid[3], const unsigned block[3], unsigned shared, const size_t* buffer_sizes, size_t n_in,
    size_t n_out, const void* const* host_in, void* const* host_out, int graph, int repeats, char* stats,
    size_t stats_cap, char* err, size_t err_cap) {
  try {
    using namespace ask::runtime;
    auto session = Session::create(device);
    std::vector<std::string> types;
    std::stringstream ts(types_csv ? types_csv : "");
    for (std::string t; std::getline(ts, t, ',');)
      if (!t.empty()) types.push_back(t);
    const std::string cubin(static_cast<const char*>(image), image_bytes);
    auto kernel = session->load(cubin, entry, types, arch, std::vector<unsigned>(widths, widths + n_params));
    PlanStep step;
    step.kernel = kernel;
    for (size_t i = 0; i < n_params; ++i) {
      PlanArgument a;
      if (widths[i]) a.scalar.assign(reinterpret_cast<const char*>(scalars + 8 * i), widths[i]);
      else a.buffer = arg_buffer[i];
      step.arguments.push_back(a);
    }
    step.grid = {grid[0], grid[1], grid[2]};
    step.block = {block[0], block[1], block[2]};
    step.sharedBytes = shared;
    std::vector<size_t> sizes(buffer_sizes, buffer_sizes + n_in + n_out), ins, outs;
    for (size_t k = 0; k < n_in; ++k) ins.push_back(k);
    for (size_t k = 0; k < n_out; ++k) outs.push_back(n_in + k);
    step.inputs = ins;
    step.outputs = outs;
    auto program = session->prepareProgram(sizes, ins, outs, {step}, graph != 0);
    std::vector<std::shared_ptr<DeviceBuffer>> results;
    for (int r = 0; r < (repeats > 0 ? repeats : 1); ++r) {
      std::vector<std::shared_ptr<DeviceBuffer>> bufs;
      for (size_t k = 0; k < n_in; ++k) {
        auto b = session->allocate(sizes[k]);
        if (sizes[k]) b->copyFromHost(host_in[k], sizes[k]);
        bufs.push_back(b);
      }
      auto out = program->run(bufs);
      out.second->wait();
      results = out.first;
    }
    for (size_t k = 0; k < n_out; ++k)
      if (sizes[n_in + k]) results[k]->copyToHost(host_out[k], sizes[n_in + k]);
    std::ostringstream o;
    o << "{";
    bool first = true;
    for (const auto& [name, value] : session->stats()) {
      o << (first ? "" : ",") << "\"" << name << "\":" << value;
      first = false;
    }
    o << "}";
    write_text(o.str(), stats, stats_cap);
    session->close();
    return 0;
  } catch (const std::exception& e) {
    write_text(e.what(), err, err_cap);
    return -1;
  }
}

// program_json: {"buffer_sizes", "inputs", "outputs",
//   "kernels": [{"entry", "types": [...], "arch", "widths": [...]}],
//   "steps": [{"kernel": k, "inputs", "outputs", "grid", "block", "shared_bytes",
//              "arguments": [{"buffer": b} | {"scalar": "<hex>"}]}]}
// images[k] / image_bytes[k]: the cubin of kernels[k].  Runs the program
// `repeats` times with the same host inputs uploaded to fresh buffers.
__attribute__((visibility("default"))) int askref_run_program(int device, const char* program_json,
                                                              const void* const* images, const size_t* image_bytes,
                                                              const void* const* host_in, void* const* host_out,
                                                              int graph, int repeats, char* stats, size_t stats_cap,
                                                              char* err, size_t err_cap) {
  try {
    using namespace ask::runtime;
    const askb::json::Value v = askb::json::Parser(program_json).parse();
    auto session = Session::create(device);
    std::vector<std::shared_ptr<Kernel>> kernels;
    const auto& ks = v.at("kernels").as_array("kernels");
    for (size_t k = 0; k < ks.size(); ++k) {
      std::vector<std::string> types;
      for (const auto& t : ks[k].at("types").as_array("types")) types.push_back(t.as_str("type"));
      std::vector<unsigned> widths;
      for (const auto& w : ks[k].at("widths").as_array("widths")) widths.push_back(unsigned(w.as_int("width")));
      kernels.push_back(session->load(std::string(static_cast<const char*>(images[k]), image_bytes[k]),
                                      ks[k].at("entry").as_str("entry"), types, int(ks[k].at("arch").as_int("arch")),
                                      widths));
    }
    auto triple = [](const askb::json::Value& a) {
      const auto& x = a.as_array("dims");
      return std::array<unsigned, 3>{unsigned(x.at(0).as_int("d")), unsigned(x.at(1).as_int("d")),
                                     unsigned(x.at(2).as_int("d"))};
    };
    std::vector<PlanStep> steps;
    for (const auto& sv : v.at("steps").as_array("steps")) {
      PlanStep st;
      st.kernel = kernels.at(size_t(sv.at("kernel").as_int("kernel")));
      st.inputs = list(sv.at("inputs"), "inputs");
      st.outputs = list(sv.at("outputs"), "outputs");
      st.grid = triple(sv.at("grid"));
      st.block = triple(sv.at("block"));
      st.sharedBytes = sv.get("shared_bytes") ? unsigned(sv.at("shared_bytes").as_int("shared_bytes")) : 0;
      for (const auto& a : sv.at("arguments").as_array("arguments")) {
        PlanArgument pa;
        if (const auto* sc = a.get("scalar")) {
          const std::string hex = sc->as_str("scalar");
          for (size_t i = 0; i + 1 < hex.size(); i += 2) pa.scalar.push_back(char(std::stoi(hex.substr(i, 2), nullptr, 16)));
        } else {
          pa.buffer = a.at("buffer").as_int("buffer");
        }
        st.arguments.push_back(pa);
      }
      steps.push_back(st);
    }
    const std::vector<size_t> sizes = list(v.at("buffer_sizes"), "buffer_sizes");
    const std::vector<size_t> ins = list(v.at("inputs"), "inputs"), outs = list(v.at("outputs"), "outputs");
    auto program = session->prepareProgram(sizes, ins, outs, steps, graph != 0);
    std::vector<std::shared_ptr<DeviceBuffer>> results;
    for (int r = 0; r < (repeats > 0 ? repeats : 1); ++r) {
      std::vector<std::shared_ptr<DeviceBuffer>> bufs;
      for (size_t k = 0; k < ins.size(); ++k) {
        auto b = session->allocate(sizes[ins[k]]);
        if (sizes[ins[k]]) b->copyFromHost(host_in[k], sizes[ins[k]]);
        bufs.push_back(b);
      }
      auto out = program->run(bufs);
      out.second->wait();
      results = out.first;
    }
    for (size_t k = 0; k < outs.size(); ++k)
      if (sizes[outs[k]]) results[k]->copyToHost(host_out[k], sizes[outs[k]]);
    std::ostringstream o;
    o << "{";
    bool first = true;
    for (const auto& [name, value] : session->stats()) {
      o << (first ? "" : ",") << "\"" << name << "\":" << value;
      first = false;
    }
    o << "}";
    write_text(o.str(), stats, stats_cap);
    session->close();
    return 0;
  } catch (const std::exception& e) {
    write_text(e.what(), err, err_cap);
    return -1;
  }
}

}  // extern "C"
