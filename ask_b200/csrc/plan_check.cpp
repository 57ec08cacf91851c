// Execution-plan verification and slot assignment (see plan_check.h).
#include "plan_check.h"

#include <algorithm>
#include <cstdint>
#include <utility>

namespace askb {
namespace check {

namespace {

constexpr size_t kNone = SIZE_MAX;

// birth[b]: 0 for a public input, producing step + 1 otherwise.  Returns the
// first structural error, or "" when every buffer has exactly one source.
std::string births(const Plan& p, std::vector<size_t>& birth) {
  birth.assign(p.buffer_count, kNone);
  for (size_t b : p.public_inputs) {
    if (b >= p.buffer_count) return "public input buffer index is out of range";
    if (birth[b] != kNone) return "public input buffer is repeated";
    birth[b] = 0;
  }
  for (size_t s = 0; s < p.steps.size(); ++s) {
    for (size_t b : p.steps[s].inputs)
      if (b >= p.buffer_count) return "step input buffer index is out of range";
    for (size_t b : p.steps[s].outputs) {
      if (b >= p.buffer_count) return "step output buffer index is out of range";
      if (birth[b] != kNone) return "buffer has multiple writers or aliases a public input";
      birth[b] = s + 1;
    }
  }
  if (p.public_outputs.empty()) return "plan must have a public output";
  for (size_t b : p.public_outputs)
    if (b >= p.buffer_count) return "public output buffer index is out of range";
  for (size_t v : birth)
    if (v == kNone) return "plan contains a buffer without a writer";
  return {};
}

void fail(std::string& out, const std::string& name) {
  out += "verify ";
  out += name;
  out += " FAIL\n";
}

void check_reads(const Plan& p, const std::vector<size_t>& birth, std::string& out) {
  for (size_t s = 0; s < p.steps.size(); ++s)
    for (size_t port = 0; port < p.steps[s].inputs.size(); ++port)
      if (birth[p.steps[s].inputs[port]] > s) fail(out, "READ_" + std::to_string(s) + "_" + std::to_string(port));
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

}  // namespace

Verdict check_plan(const Plan& plan) {
  std::vector<size_t> birth;
  std::string error = births(plan, birth);
  if (!error.empty()) return {false, error};
  std::string out;
  check_reads(plan, birth, out);
  return {out.empty(), out};
}

Verdict check_allocation(const Allocation& a) {
  const Plan& p = a.plan;
  const size_t n = p.steps.size();
  std::vector<size_t> birth;
  std::string error = births(p, birth);
  if (!error.empty()) return {false, error};
  if (a.buffer_sizes.size() != p.buffer_count) return {false, "allocation buffer sizes differ from the plan"};

  std::vector<char> is_public(p.buffer_count, 0), placed(p.buffer_count, 0);
  for (size_t b : p.public_inputs) is_public[b] = 1;
  for (size_t b : p.public_outputs) is_public[b] = 1;
  std::vector<std::vector<size_t>> occupants(a.slot_capacity_bytes.size());
  for (const SlotAssignment& e : a.assignments) {
    if (e.buffer >= p.buffer_count || e.slot >= occupants.size())
      return {false, "allocation assignment index is out of range"};
    if (is_public[e.buffer]) return {false, "public port cannot use an internal slot"};
    if (placed[e.buffer]) return {false, "internal buffer has multiple slot assignments"};
    placed[e.buffer] = 1;
    occupants[e.slot].push_back(e.buffer);
  }
  for (size_t b = 0; b < p.buffer_count; ++b)
    if (!is_public[b] && !placed[b]) return {false, "internal buffer has no slot assignment"};
  for (const auto& o : occupants)
    if (o.empty()) return {false, "allocation contains an unused slot"};

  if (a.graph) {
    if (a.dependencies.size() != n) return {false, "graph dependency count differs from the plan"};
    for (size_t s = 0; s < n; ++s) {
      std::vector<size_t> d = a.dependencies[s];
      for (size_t x : d)
        if (x >= s) return {false, "graph dependency is not topologically ordered"};
      std::sort(d.begin(), d.end());
      if (std::adjacent_find(d.begin(), d.end()) != d.end()) return {false, "graph dependency is repeated"};
    }
  } else if (!a.dependencies.empty()) {
    return {false, "stream plan contains graph dependencies"};
  }

  // Last access of each buffer (its producer counts as an access, so an
  // unread buffer is live at its producing step); graph mode keeps them all.
  std::vector<size_t> last(p.buffer_count, 0);
  std::vector<std::vector<size_t>> touched(a.graph ? p.buffer_count : 0);
  for (size_t s = 0; s < n; ++s) {
    for (const auto* list : {&p.steps[s].outputs, &p.steps[s].inputs})
      for (size_t b : *list) {
        last[b] = std::max(last[b], s);
        if (a.graph) touched[b].push_back(s);
      }
  }

  std::string out;
  check_reads(p, birth, out);
  for (const SlotAssignment& e : a.assignments)
    if (a.buffer_sizes[e.buffer] > a.slot_capacity_bytes[e.slot]) fail(out, "CAPACITY_" + std::to_string(e.buffer));

  std::vector<std::vector<size_t>> precede(a.graph ? n : 0);  // steps that must come before step s
  if (a.graph)
    for (size_t s = 0; s < n; ++s)
      for (size_t b : p.steps[s].inputs)
        if (birth[b] > 0) precede[s].push_back(birth[b] - 1);
  // Consecutive occupants of a slot in production order: the earlier one must
  // be dead before the later one is written.  Ordering each adjacent pair
  // orders every earlier occupant too, since an occupant's producer is one of
  // its accesses.
  for (auto& o : occupants) {
    std::sort(o.begin(), o.end(), [&](size_t x, size_t y) { return std::make_pair(birth[x], x) < std::make_pair(birth[y], y); });
    for (size_t i = 1; i < o.size(); ++i) {
      const size_t older = o[i - 1], newer = o[i], writer = birth[newer] - 1;
      if (a.graph)
        precede[writer].insert(precede[writer].end(), touched[older].begin(), touched[older].end());
      else if (last[older] >= writer)
        fail(out, "ADJACENT_" + std::to_string(older) + "_" + std::to_string(newer));
    }
  }
  if (a.graph) {
    Ancestors anc(a.dependencies);
    for (size_t s = 0; s < n; ++s) {
      auto& req = precede[s];
      if (req.empty()) continue;
      std::sort(req.begin(), req.end());
      req.erase(std::unique(req.begin(), req.end()), req.end());
      if (req.back() >= s) {
        fail(out, "GRAPH_ORDER_" + std::to_string(s));
        continue;
      }
      anc.mark(s, req.front());
      for (size_t x : req)
        if (!anc.is_ancestor(x, s)) {
          fail(out, "GRAPH_ORDER_" + std::to_string(s));
          break;
        }
    }
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
