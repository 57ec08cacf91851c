// Execution-plan verification and slot assignment (see plan_check.h).
//
// The verdicts and the diagnostic texts (and the order in which they are
// reported) are the contract with callers of the reference's plan verifier
// (lib/Pass/Pass.cpp:13-49, 96-209); the checks are organised here around
// buffer lifetimes: each buffer's life runs from the step that writes it to
// the last step that touches it, and a slot is a sequence of such lives.
#include "plan_check.h"

#include <algorithm>
#include <cstdint>
#include <utility>

namespace askb {
namespace check {

namespace {

constexpr size_t kNone = SIZE_MAX;          // no writer (yet)
constexpr size_t kCaller = SIZE_MAX - 1;    // public input: written by the caller before step 0

// Who writes each buffer.  Returns the first structural error of the plan, or
// "" when every buffer has exactly one writer (a step or the caller).  The
// checks run in the order the reference reports them, so a plan with several
// defects gets the same message.
std::string find_writers(const Plan& p, std::vector<size_t>& writer) {
  writer.assign(p.buffer_count, kNone);
  const auto in_range = [&](size_t b) { return b < p.buffer_count; };
  for (size_t b : p.public_inputs) {
    if (!in_range(b)) return "public input buffer index is out of range";
    if (writer[b] == kCaller) return "public input buffer is repeated";
    writer[b] = kCaller;
  }
  for (size_t s = 0; s < p.steps.size(); ++s) {
    const StepPorts& step = p.steps[s];
    if (!std::all_of(step.inputs.begin(), step.inputs.end(), in_range))
      return "step input buffer index is out of range";
    for (size_t b : step.outputs) {
      if (!in_range(b)) return "step output buffer index is out of range";
      if (writer[b] != kNone) return "buffer has multiple writers or aliases a public input";
      writer[b] = s;
    }
  }
  if (p.public_outputs.empty()) return "plan must have a public output";
  if (!std::all_of(p.public_outputs.begin(), p.public_outputs.end(), in_range))
    return "public output buffer index is out of range";
  if (std::find(writer.begin(), writer.end(), kNone) != writer.end()) return "plan contains a buffer without a writer";
  return {};
}

void report(std::string& out, const std::string& name) {
  out += "verify ";
  out += name;
  out += " FAIL\n";
}

// A step may read a buffer only once the caller or an earlier step wrote it.
void report_early_reads(const Plan& p, const std::vector<size_t>& writer, std::string& out) {
  for (size_t s = 0; s < p.steps.size(); ++s) {
    const std::vector<size_t>& in = p.steps[s].inputs;
    for (size_t port = 0; port < in.size(); ++port) {
      const size_t w = writer[in[port]];
      if (w != kCaller && w >= s) report(out, "READ_" + std::to_string(s) + "_" + std::to_string(port));
    }
  }
}

// Ancestor marking over a dependency DAG: mark(step, floor) visits every
// ancestor of `step` whose index is >= floor (no ancestor of a node is
// larger than the node, so the floor prunes whole prefixes of a long chain).
class Ancestors {
 public:
  explicit Ancestors(const std::vector<std::vector<size_t>>& deps) : deps_(deps), mark_(deps.size(), kNone) {}
  void mark(size_t step, size_t floor) {
    stack_.assign(deps_[step].begin(), deps_[step].end());
    while (!stack_.empty()) {
      const size_t x = stack_.back();
      stack_.pop_back();
      if (x < floor || mark_[x] == step) continue;
      mark_[x] = step;
      stack_.insert(stack_.end(), deps_[x].begin(), deps_[x].end());
    }
  }
  bool is_ancestor(size_t x, size_t step) const { return mark_[x] == step; }

 private:
  const std::vector<std::vector<size_t>>& deps_;
  std::vector<size_t> mark_;
  std::vector<size_t> stack_;
};

// The life of one slot occupant: written at `from`, last touched at `to`.
struct Life {
  size_t from, to, buffer;
  bool operator<(const Life& o) const { return from != o.from ? from < o.from : buffer < o.buffer; }
};

// Shape of the mapping itself: every internal buffer in exactly one slot, no
// public buffer in a slot, no empty slot.  Fills the occupants of each slot.
std::string place_buffers(const Allocation& a, std::vector<std::vector<size_t>>& occupants) {
  const Plan& p = a.plan;
  std::vector<char> role(p.buffer_count, 0);  // 1 public, 2 placed internal
  for (size_t b : p.public_inputs) role[b] = 1;
  for (size_t b : p.public_outputs) role[b] = 1;
  occupants.assign(a.slot_capacity_bytes.size(), {});
  for (const SlotAssignment& e : a.assignments) {
    if (e.buffer >= p.buffer_count || e.slot >= occupants.size()) return "allocation assignment index is out of range";
    if (role[e.buffer] == 1) return "public port cannot use an internal slot";
    if (role[e.buffer] == 2) return "internal buffer has multiple slot assignments";
    role[e.buffer] = 2;
    occupants[e.slot].push_back(e.buffer);
  }
  if (std::find(role.begin(), role.end(), 0) != role.end()) return "internal buffer has no slot assignment";
  for (const auto& o : occupants)
    if (o.empty()) return "allocation contains an unused slot";
  return {};
}

// Graph mode: each step lists earlier steps, each at most once; stream mode
// has no edges (stream order is the order).
std::string check_edges(const Allocation& a) {
  const size_t n = a.plan.steps.size();
  if (!a.graph) return a.dependencies.empty() ? std::string() : "stream plan contains graph dependencies";
  if (a.dependencies.size() != n) return "graph dependency count differs from the plan";
  for (size_t s = 0; s < n; ++s) {
    const std::vector<size_t>& d = a.dependencies[s];
    if (std::any_of(d.begin(), d.end(), [s](size_t x) { return x >= s; }))
      return "graph dependency is not topologically ordered";
    std::vector<size_t> sorted(d);
    std::sort(sorted.begin(), sorted.end());
    if (std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end()) return "graph dependency is repeated";
  }
  return {};
}

}  // namespace

Verdict check_plan(const Plan& plan) {
  std::vector<size_t> writer;
  std::string error = find_writers(plan, writer);
  if (!error.empty()) return {false, error};
  std::string out;
  report_early_reads(plan, writer, out);
  return {out.empty(), out};
}

Verdict check_allocation(const Allocation& a) {
  const Plan& p = a.plan;
  const size_t n = p.steps.size();
  std::vector<size_t> writer;
  std::string error = find_writers(p, writer);
  if (error.empty() && a.buffer_sizes.size() != p.buffer_count) error = "allocation buffer sizes differ from the plan";
  std::vector<std::vector<size_t>> occupants;
  if (error.empty()) error = place_buffers(a, occupants);
  if (error.empty()) error = check_edges(a);
  if (!error.empty()) return {false, error};

  // Steps touching each buffer, ascending (a writer counts: an unread buffer
  // is alive at the step that writes it).
  std::vector<std::vector<size_t>> touches(p.buffer_count);
  for (size_t s = 0; s < n; ++s)
    for (const auto* ports : {&p.steps[s].outputs, &p.steps[s].inputs})
      for (size_t b : *ports)
        if (touches[b].empty() || touches[b].back() != s) touches[b].push_back(s);

  std::string out;
  report_early_reads(p, writer, out);
  for (const SlotAssignment& e : a.assignments)
    if (a.buffer_sizes[e.buffer] > a.slot_capacity_bytes[e.slot]) report(out, "CAPACITY_" + std::to_string(e.buffer));

  // Each slot's lives in the order they begin.  A life must not begin before
  // the previous one in its slot has ended: in stream order that is a
  // comparison of step indices; in graph order every step that touched the
  // previous occupant must be an ancestor of the new writer.
  std::vector<std::vector<size_t>> must_precede(a.graph ? n : 0);
  for (const auto& slot : occupants) {
    std::vector<Life> lives;
    lives.reserve(slot.size());
    for (size_t b : slot) lives.push_back({writer[b], touches[b].back(), b});
    std::sort(lives.begin(), lives.end());
    for (size_t i = 1; i < lives.size(); ++i) {
      const Life& prev = lives[i - 1];
      const Life& next = lives[i];
      if (a.graph) {
        const auto& t = touches[prev.buffer];
        must_precede[next.from].insert(must_precede[next.from].end(), t.begin(), t.end());
      } else if (prev.to >= next.from) {
        report(out, "ADJACENT_" + std::to_string(prev.buffer) + "_" + std::to_string(next.buffer));
      }
    }
  }
  if (!a.graph) return {out.empty(), out};

  // Graph order: a step also needs a path from the writer of everything it
  // reads.  One ancestor walk per step, cut off below its earliest need.
  Ancestors anc(a.dependencies);
  for (size_t s = 0; s < n; ++s) {
    std::vector<size_t>& need = must_precede[s];
    for (size_t b : p.steps[s].inputs)
      if (writer[b] != kCaller) need.push_back(writer[b]);
    if (need.empty()) continue;
    const auto [lo, hi] = std::minmax_element(need.begin(), need.end());
    bool ordered = *hi < s;
    if (ordered) {
      anc.mark(s, *lo);
      ordered = std::all_of(need.begin(), need.end(), [&](size_t x) { return anc.is_ancestor(x, s); });
    }
    if (!ordered) report(out, "GRAPH_ORDER_" + std::to_string(s));
  }
  return {out.empty(), out};
}

namespace {

struct Lifetimes {
  std::vector<char> is_public;
  std::vector<size_t> last;  // last step touching the buffer
};

Lifetimes lifetimes(const Plan& p) {
  Lifetimes l;
  l.is_public.assign(p.buffer_count, 0);
  for (size_t b : p.public_inputs) l.is_public[b] = 1;
  for (size_t b : p.public_outputs) l.is_public[b] = 1;
  l.last.assign(p.buffer_count, 0);
  for (size_t s = 0; s < p.steps.size(); ++s)
    for (const auto* list : {&p.steps[s].outputs, &p.steps[s].inputs})
      for (size_t b : *list) l.last[b] = std::max(l.last[b], s);
  return l;
}

}  // namespace

void assign_stream_slots(Allocation& a) {
  const Plan& p = a.plan;
  const Lifetimes l = lifetimes(p);
  a.graph = false;
  a.dependencies.clear();
  a.assignments.clear();
  a.slot_capacity_bytes.clear();
  std::vector<size_t> busy_until;  // last access of each slot's current occupant
  for (size_t s = 0; s < p.steps.size(); ++s)
    for (size_t b : p.steps[s].outputs) {
      if (l.is_public[b]) continue;
      size_t k = 0;
      while (k < busy_until.size() && busy_until[k] >= s) ++k;
      if (k == busy_until.size()) {
        busy_until.push_back(l.last[b]);
        a.slot_capacity_bytes.push_back(a.buffer_sizes[b]);
      } else {
        busy_until[k] = l.last[b];
        a.slot_capacity_bytes[k] = std::max(a.slot_capacity_bytes[k], a.buffer_sizes[b]);
      }
      a.assignments.push_back({b, k});
    }
}

void assign_graph_slots(Allocation& a) {
  const Plan& p = a.plan;
  const size_t n = p.steps.size();
  const Lifetimes l = lifetimes(p);
  a.graph = true;
  a.assignments.clear();
  a.slot_capacity_bytes.clear();
  a.dependencies.assign(n, {});
  std::vector<size_t> producer(p.buffer_count, kNone);
  std::vector<std::vector<size_t>> touched(p.buffer_count);
  for (size_t s = 0; s < n; ++s) {
    auto& d = a.dependencies[s];
    for (size_t b : p.steps[s].inputs)
      if (producer[b] != kNone) d.push_back(producer[b]);
    std::sort(d.begin(), d.end());
    d.erase(std::unique(d.begin(), d.end()), d.end());
    for (size_t b : p.steps[s].outputs) producer[b] = s;
    for (const auto* list : {&p.steps[s].outputs, &p.steps[s].inputs})
      for (size_t b : *list)
        if (touched[b].empty() || touched[b].back() != s) touched[b].push_back(s);
  }
  Ancestors anc(a.dependencies);
  std::vector<size_t> occupant;  // current buffer of each slot
  for (size_t s = 0; s < n; ++s) {
    bool marked = false;
    for (size_t b : p.steps[s].outputs) {
      if (l.is_public[b]) continue;
      // a slot is free for step s when its occupant's every access is an
      // ancestor of s; the occupant's producer bounds how far back to look
      size_t pick = kNone, floor = kNone;
      for (size_t k = 0; k < occupant.size(); ++k)
        if (l.last[occupant[k]] < s) floor = std::min(floor, touched[occupant[k]].front());
      if (floor != kNone) {
        if (!marked) {
          anc.mark(s, floor);
          marked = true;
        }
        for (size_t k = 0; k < occupant.size() && pick == kNone; ++k) {
          const size_t old = occupant[k];
          if (l.last[old] >= s) continue;
          bool ok = true;
          for (size_t x : touched[old])
            if (!anc.is_ancestor(x, s)) { ok = false; break; }
          if (ok) pick = k;
        }
      }
      if (pick == kNone) {
        pick = occupant.size();
        occupant.push_back(b);
        a.slot_capacity_bytes.push_back(a.buffer_sizes[b]);
      } else {
        occupant[pick] = b;
        a.slot_capacity_bytes[pick] = std::max(a.slot_capacity_bytes[pick], a.buffer_sizes[b]);
      }
      a.assignments.push_back({b, pick});
    }
  }
}

}  // namespace check
}  // namespace askb
