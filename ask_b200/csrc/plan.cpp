// C-ABI plan layer: recipe parsing and validation, kernel selection, launch.
//
// A recipe is the JSON form of one owned ASK execution-plan step.  It plays the
// role of the step source that ask::lowerToCUDALLVM consumes
// (lib/Lowering/CUDA.cpp:152-419): ports in the pointer-ABI order (inputs,
// then outputs, CUDA.cpp:177-208), static sizes, and the step's computation as
// an SSA op program using ASK's op names (include/ask/IR/ASKOps.h:70-145).
// Validation follows the reference's rules where they apply:
//   * at most 64 ports (CUDA.cpp:105-106);
//   * add/mul need identical operand and result types (CUDA.cpp:139-142);
//   * float-only ops (div, exp, log, ...), integer/bool-only bitwise ops and
//     i32/i64-only shifts as stated in docs/en/ir.md:77;
//   * reduce_any/all take bool, argmax/argmin need a non-empty axis
//     (lib/IR/ASKOps.cpp:297-334, docs/en/ir.md:69);
//   * gather/scatter_add index types are i32 or i64 (lib/IR/ASKOps.cpp:460-496).
#include "../../include/ask_b200.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <functional>
#include <cstring>
#include <map>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "json.h"
#include "kernels.h"
#include "plan_internal.h"

using namespace askb;

namespace {

thread_local std::string g_last_error;

struct Failure {
  int code;
  std::string message;
};

[[noreturn]] void fail(int code, const std::string& msg) { throw Failure{code, msg}; }

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(ASK_B200_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

template <class F>
int guarded(F&& body) {
  try {
    body();
    g_last_error.clear();
    return ASK_B200_OK;
  } catch (const Failure& f) {
    g_last_error = f.message;
    return f.code;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return ASK_B200_E_INVALID;
  } catch (...) {
    g_last_error = "unknown error";
    return ASK_B200_E_INVALID;
  }
}

// ---- names ----------------------------------------------------------------------
const char* const kTypeNames[kNumDTypes] = {"bool", "i32", "i64", "f32", "f16", "bf16"};

int parse_dtype(const std::string& s) {
  for (int t = 0; t < kNumDTypes; ++t)
    if (s == kTypeNames[t]) return t;
  if (s == "i1") return kBool;
  fail(ASK_B200_E_INVALID, "unknown element type '" + s + "'");
}

struct OpName {
  const char* name;
  int op;
  int arity;
};
const OpName kOpNames[] = {
    {"add", OP_ADD, 2},          {"mul", OP_MUL, 2},          {"div", OP_DIV, 2},
    {"floordiv", OP_FLOORDIV, 2}, {"mod", OP_MOD, 2},          {"pow", OP_POW, 2},
    {"maximum", OP_MAXIMUM, 2},  {"minimum", OP_MINIMUM, 2},  {"bitwise_and", OP_AND, 2},
    {"bitwise_or", OP_OR, 2},    {"bitwise_xor", OP_XOR, 2},  {"shift_left", OP_SHL, 2},
    {"shift_right", OP_SHR, 2},  {"bitwise_not", OP_NOT, 1},  {"abs", OP_ABS, 1},
    {"exp", OP_EXP, 1},          {"log", OP_LOG, 1},          {"sqrt", OP_SQRT, 1},
    {"sin", OP_SIN, 1},          {"cos", OP_COS, 1},          {"tanh", OP_TANH, 1},
    {"erf", OP_ERF, 1},          {"floor", OP_FLOOR, 1},      {"ceil", OP_CEIL, 1},
    {"round", OP_ROUND, 1},
};

std::string strip_prefix(const std::string& s) { return s.rfind("ask.", 0) == 0 ? s.substr(4) : s; }

int parse_map(const std::string& s) {
  if (s == "full") return IM_FULL;
  if (s == "scalar") return IM_SCALAR;
  if (s == "outer") return IM_OUTER;
  if (s == "inner") return IM_INNER;
  if (s == "view") return IM_VIEW;
  fail(ASK_B200_E_INVALID, "unknown index map '" + s + "'");
}
const char* map_name(int m) {
  return m == IM_FULL ? "full" : m == IM_SCALAR ? "scalar" : m == IM_OUTER ? "outer" : m == IM_INNER ? "inner" : "view";
}

// ---- constants ---------------------------------------------------------------------
// double -> binary16 / bfloat16 bits with a single round-to-nearest-even step
// (constants are rounded directly to the target width, docs/en/ir.md:108).
uint32_t double_to_small_float(double x, int exp_bits, int man_bits) {
  const uint32_t sign = std::signbit(x) ? (1u << (exp_bits + man_bits)) : 0u;
  const uint32_t exp_all = (1u << exp_bits) - 1u;
  if (std::isnan(x)) return sign | (exp_all << man_bits) | (1u << (man_bits - 1));
  const double a = std::fabs(x);
  if (std::isinf(a)) return sign | (exp_all << man_bits);
  if (a == 0.0) return sign;
  const int bias = (1 << (exp_bits - 1)) - 1;
  const int emin = 1 - bias;
  int e2;
  std::frexp(a, &e2);
  int e = e2 - 1;  // a in [2^e, 2^(e+1))
  if (e < emin) {
    const double q = std::nearbyint(std::ldexp(a, man_bits - emin));  // subnormal quantum 2^(emin-man)
    return sign | uint32_t(q);  // q == 2^man rolls into the smallest normal
  }
  double q = std::nearbyint(std::ldexp(a, man_bits - e));
  if (q == std::ldexp(1.0, man_bits + 1)) { q /= 2.0; ++e; }
  if (e > bias) return sign | (exp_all << man_bits);
  return sign | (uint32_t(e + bias) << man_bits) | (uint32_t(q) - (1u << man_bits));
}

float bits_to_float(uint32_t b) { float f; std::memcpy(&f, &b, 4); return f; }
uint32_t float_to_bits(float f) { uint32_t b; std::memcpy(&b, &f, 4); return b; }

// f16 bits -> f32 value (exact).
float half_bits_to_float(uint32_t h) {
  const uint32_t s = (h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0x1f) return bits_to_float(s | 0x7f800000u | (m << 13));
  if (e == 0) return (s ? -1.0f : 1.0f) * std::ldexp(float(m), -24);
  return bits_to_float(s | ((e + 112u) << 23) | (m << 13));
}

uint64_t constant_word(const json::Value& v, int t) {
  if (t == kBool) {
    if (v.kind == json::Value::Bool) return v.b ? 1u : 0u;
    if (v.kind == json::Value::Number) return v.num != 0.0 ? 1u : 0u;
    fail(ASK_B200_E_INVALID, "bool constant must be true/false");
  }
  if (t == kI32 || t == kI64) {
    const int64_t x = v.as_int("integer constant");
    if (t == kI32 && (x < INT32_MIN || x > INT32_MAX)) fail(ASK_B200_E_INVALID, "i32 constant out of range");
    return t == kI32 ? uint64_t(uint32_t(int32_t(x))) : uint64_t(x);
  }
  double d;
  if (v.kind == json::Value::Number) {
    d = v.num;
  } else if (v.kind == json::Value::String) {
    const std::string& s = v.str;
    if (s.rfind("bits:", 0) == 0) {
      const uint64_t bits = std::stoull(s.substr(5), nullptr, 0);
      if (t == kF32) return bits & 0xffffffffu;
      if (t == kF16) return float_to_bits(half_bits_to_float(uint32_t(bits & 0xffffu)));
      return uint64_t(uint32_t(bits & 0xffffu) << 16);
    }
    if (s == "nan") d = std::nan("");
    else if (s == "inf") d = INFINITY;
    else if (s == "-inf") d = -INFINITY;
    else d = std::stod(s);
  } else {
    fail(ASK_B200_E_INVALID, "float constant must be a number or string");
  }
  if (t == kF32) return float_to_bits(float(d));
  if (t == kF16) return float_to_bits(half_bits_to_float(double_to_small_float(d, 5, 10)));
  return uint64_t(double_to_small_float(d, 8, 7) << 16);
}

// ---- programs ------------------------------------------------------------------------
struct Ports {
  std::vector<int> type, map;
};

// Parse an SSA program.  Result: canonical SSA Program (dst == index), and the
// type of every value.
Program parse_program(const json::Value& prog_json, const json::Value& results_json, const Ports& in,
                      bool allow_inner_map) {
  const auto& insns = prog_json.as_array("program");
  if (insns.empty() || insns.size() > size_t(kMaxInsn))
    fail(ASK_B200_E_UNSUPPORTED, "program must have 1.." + std::to_string(kMaxInsn) + " instructions");
  if (in.type.size() > size_t(kMaxIn)) fail(ASK_B200_E_UNSUPPORTED, "too many inputs for one fused step");
  Program p{};
  p.n_in = uint8_t(in.type.size());
  for (size_t k = 0; k < in.type.size(); ++k) {
    p.in_type[k] = uint8_t(in.type[k]);
    if (in.map[k] == IM_INNER && !allow_inner_map) fail(ASK_B200_E_INVALID, "index map 'inner' is not valid here");
    p.in_map[k] = uint8_t(in.map[k]);
  }
  std::vector<int> vt;
  auto operand = [&](const json::Value& v, size_t i) -> uint8_t {
    const int64_t a = v.as_int("operand");
    if (a < 0 || size_t(a) >= i) fail(ASK_B200_E_INVALID, "operand must name an earlier instruction");
    return uint8_t(a);
  };
  auto need = [&](bool ok, const std::string& what) {
    if (!ok) fail(ASK_B200_E_INVALID, what);
  };
  for (size_t i = 0; i < insns.size(); ++i) {
    const auto& ins = insns[i].as_array("instruction");
    need(!ins.empty(), "empty instruction");
    const std::string name = strip_prefix(ins[0].as_str("opcode"));
    Insn x{};
    x.dst = uint8_t(i);
    int type = -1;
    if (name == "input") {
      need(ins.size() == 2, "input takes a port index");
      const int64_t k = ins[1].as_int("input port");
      need(k >= 0 && size_t(k) < in.type.size(), "input port out of range");
      x.op = OP_INPUT; x.a = uint8_t(k); type = in.type[size_t(k)];
    } else if (name == "const" || name == "constant") {
      need(ins.size() == 3, "const takes a type and a value");
      type = parse_dtype(ins[1].as_str("const type"));
      x.op = OP_CONST; x.imm = constant_word(ins[2], type); x.src_type = uint8_t(type);
    } else if (name == "cast") {
      need(ins.size() == 3, "cast takes an operand and a type");
      x.op = OP_CAST; x.a = operand(ins[1], i); type = parse_dtype(ins[2].as_str("cast type"));
      x.src_type = uint8_t(vt[x.a]);
    } else if (name == "compare") {
      need(ins.size() == 4, "compare takes a predicate and two operands");
      const std::string pred = ins[1].as_str("predicate");
      const char* preds[] = {"eq", "ne", "lt", "le", "gt", "ge"};
      int pi = -1;
      for (int q = 0; q < 6; ++q) if (pred == preds[q]) pi = q;
      need(pi >= 0, "unknown compare predicate '" + pred + "'");
      x.op = OP_CMP; x.aux = uint8_t(pi); x.a = operand(ins[2], i); x.b = operand(ins[3], i);
      need(vt[x.a] == vt[x.b], "compare operands must have identical types");
      x.src_type = uint8_t(vt[x.a]); type = kBool;
    } else if (name == "coord") {
      need(ins.size() == 2, "coord takes an axis of the iteration shape");
      const int64_t axis = ins[1].as_int("coord axis");
      need(axis >= 0 && axis < kMaxRank, "coord axis out of range");
      x.op = OP_COORD; x.aux = uint8_t(axis); type = kI64;
    } else if (name == "select") {
      need(ins.size() == 4, "select takes a condition and two operands");
      x.op = OP_SELECT; x.a = operand(ins[1], i); x.b = operand(ins[2], i); x.c = operand(ins[3], i);
      need(vt[x.a] == kBool, "select condition must be bool");
      need(vt[x.b] == vt[x.c], "select branches must have identical types");
      x.src_type = kBool; type = vt[x.b];
    } else {
      const OpName* found = nullptr;
      for (const auto& o : kOpNames) if (name == o.name) found = &o;
      if (!found) fail(ASK_B200_E_UNSUPPORTED, "op '" + name + "' is not an elementwise op of this library");
      need(int(ins.size()) == found->arity + 1, "op '" + name + "' takes " + std::to_string(found->arity) + " operand(s)");
      x.op = uint8_t(found->op);
      x.a = operand(ins[1], i);
      if (found->arity == 2) {
        x.b = operand(ins[2], i);
        need(vt[x.a] == vt[x.b], "operands of '" + name + "' must have identical types");
      }
      type = vt[x.a];
      x.src_type = uint8_t(type);
      const bool fl = dtype_is_float(type), in_ = dtype_is_int(type), bo = type == kBool;
      switch (found->op) {
        case OP_ADD: case OP_MUL: case OP_FLOORDIV: case OP_MOD: case OP_POW: case OP_ABS:
          need(fl || in_, "'" + name + "' needs a numeric type"); break;
        case OP_DIV: case OP_EXP: case OP_LOG: case OP_SQRT: case OP_SIN: case OP_COS: case OP_TANH:
        case OP_ERF: case OP_FLOOR: case OP_CEIL: case OP_ROUND:
          need(fl, "'" + name + "' needs f32, f16 or bf16"); break;
        case OP_AND: case OP_OR: case OP_XOR: case OP_NOT:
          need(in_ || bo, "'" + name + "' needs bool, i32 or i64"); break;
        case OP_SHL: case OP_SHR:
          need(in_, "'" + name + "' needs i32 or i64"); break;
        default: break;  // maximum/minimum accept all six types
      }
    }
    x.type = uint8_t(type);
    p.insn[i] = x;
    vt.push_back(type);
  }
  p.n_insn = uint8_t(insns.size());
  p.n_regs = p.n_insn;
  const auto& res = results_json.as_array("results");
  if (res.empty() || res.size() > size_t(kMaxOut)) fail(ASK_B200_E_UNSUPPORTED, "1.." + std::to_string(kMaxOut) + " results");
  p.n_out = uint8_t(res.size());
  for (size_t k = 0; k < res.size(); ++k) {
    const int64_t r = res[k].as_int("result");
    if (r < 0 || size_t(r) >= insns.size()) fail(ASK_B200_E_INVALID, "result names no instruction");
    p.out_reg[k] = uint8_t(r);
    p.out_type[k] = uint8_t(vt[size_t(r)]);
  }
  return p;
}

bool same_program(const Program& a, const Program& b) {
  if (a.n_insn != b.n_insn || a.n_in != b.n_in || a.n_out != b.n_out) return false;
  for (int k = 0; k < a.n_in; ++k)
    if (a.in_type[k] != b.in_type[k] || a.in_map[k] != b.in_map[k]) return false;
  for (int k = 0; k < a.n_out; ++k)
    if (a.out_type[k] != b.out_type[k] || a.out_reg[k] != b.out_reg[k]) return false;
  for (int i = 0; i < a.n_insn; ++i) {
    const Insn &x = a.insn[i], &y = b.insn[i];
    if (x.op != y.op || x.type != y.type || x.dst != y.dst || x.a != y.a || x.b != y.b || x.c != y.c ||
        x.aux != y.aux || x.src_type != y.src_type || x.imm != y.imm)
      return false;
  }
  return true;
}

// Linear-scan register assignment for the runtime interpreter: a value's
// register is freed after its last use (results live to the end).
int operand_count(int op) {
  if (op == OP_INPUT || op == OP_CONST || op == OP_COORD) return 0;
  if (op == OP_SELECT) return 3;
  if (op == OP_CMP || (op >= OP_ADD && op <= OP_SHR)) return 2;
  return 1;  // cast and the unary ops
}

// Canonical instruction order: every input instruction first (by port, then
// position), then what the results need, depth first with operands left to
// right; instructions no result needs are dropped.  Recipes that write the
// same expression DAG in different textual orders (hand-written, or lowered
// from a step's MLIR) then get the same program and the same specialised
// kernel.
Program canonical(const Program& p) {
  std::vector<int> id(p.n_insn, -1);
  Program q = p;
  q.n_insn = 0;
  auto remap = [&](Insn x) {
    const int n = operand_count(x.op);
    if (n >= 1) x.a = uint8_t(id[x.a]);
    if (n >= 2) x.b = uint8_t(id[x.b]);
    if (n >= 3) x.c = uint8_t(id[x.c]);
    return x;
  };
  auto push = [&](int i) {
    Insn x = remap(p.insn[i]);
    x.dst = q.n_insn;
    id[i] = q.n_insn;
    q.insn[q.n_insn++] = x;
  };
  std::vector<int> inputs;
  for (int i = 0; i < p.n_insn; ++i)
    if (p.insn[i].op == OP_INPUT) inputs.push_back(i);
  std::stable_sort(inputs.begin(), inputs.end(), [&](int x, int y) { return p.insn[x].a < p.insn[y].a; });
  for (int i : inputs) push(i);
  std::function<void(int)> visit = [&](int i) {
    if (id[i] >= 0) return;
    const Insn& x = p.insn[i];
    const int n = operand_count(x.op);
    if (n >= 1) visit(x.a);
    if (n >= 2) visit(x.b);
    if (n >= 3) visit(x.c);
    push(i);
  };
  for (int k = 0; k < p.n_out; ++k) visit(p.out_reg[k]);
  for (int k = 0; k < p.n_out; ++k) q.out_reg[k] = uint8_t(id[p.out_reg[k]]);
  q.n_regs = q.n_insn;
  return q;
}

void assign_registers(Program& p) {
  const int n = p.n_insn;
  std::vector<int> last(n, -1);
  auto use = [&](int v, int at) { if (at > last[v]) last[v] = at; };
  for (int i = 0; i < n; ++i) {
    const Insn& x = p.insn[i];
    const int k = operand_count(x.op);
    if (k >= 1) use(x.a, i);
    if (k >= 2) use(x.b, i);
    if (k >= 3) use(x.c, i);
  }
  for (int k = 0; k < p.n_out; ++k) last[p.out_reg[k]] = n;
  std::vector<int> reg(n, -1);
  std::vector<int> free_list;
  int next = 0;
  for (int i = 0; i < n; ++i) {
    Insn& x = p.insn[i];
    const int a = x.a, b = x.b, c = x.c;
    // operands are read before the destination is written, so registers whose
    // last use is this instruction may be reused for its result
    for (int v = 0; v < i; ++v)
      if (last[v] == i && reg[v] >= 0) { free_list.push_back(reg[v]); last[v] = -2; }
    int r;
    if (!free_list.empty()) { r = free_list.back(); free_list.pop_back(); }
    else r = next++;
    reg[i] = r;
    x.dst = uint8_t(r);
    if (x.op != OP_INPUT && x.op != OP_CONST) {
      x.a = uint8_t(reg[a] < 0 ? 0 : reg[a]);
      x.b = uint8_t(reg[b] < 0 ? 0 : reg[b]);
      x.c = uint8_t(reg[c] < 0 ? 0 : reg[c]);
    }
    if (last[i] == -1) { free_list.push_back(r); last[i] = -2; }  // dead value
  }
  for (int k = 0; k < p.n_out; ++k) p.out_reg[k] = uint8_t(reg[p.out_reg[k]]);
  p.n_regs = uint8_t(next);
}

// ---- plan -------------------------------------------------------------------------
const char* const kFamilyNames[] = {"elementwise", "reduce", "gather", "scatter_add", "softmax"};

uint64_t checked_count(const json::Value& v, const char* what) {
  const int64_t x = v.as_int(what);
  if (x < 0) fail(ASK_B200_E_INVALID, std::string(what) + " must be non-negative");
  return uint64_t(x);
}

uint64_t mul_checked(uint64_t a, uint64_t b) {
  if (a && b > UINT64_MAX / a) fail(ASK_B200_E_INVALID, "element count overflows");
  return a * b;
}

}  // namespace

struct ask_b200_comm {
  ncclComm_t comm = nullptr;
  int nranks = 1, rank = 0, device = 0;
  // Peer-memory exchange (when every rank's inbox could be mapped): this
  // rank's inbox, the peers' IPC mappings, and a device array of all inbox
  // addresses in rank order as this device sees them.
  bool p2p = false;
  std::string p2p_note;  // why the exchange falls back to the NCCL all-gather
  void* inbox = nullptr;
  std::vector<void*> opened;
  void** inboxes_dev = nullptr;
  uint64_t timeout_ns = 1000000000ull;
};

namespace {

constexpr int kMaxRanks = 64;

int blocks_per_sm_default(int) { return 8; }

// The grid of a softmax row-kernel launch: the launcher's own (SMs x resident
// CTAs of the instance, a CTA per row at most) when the plan has a device,
// else 8 CTAs per SM.
int softmax_grid(const ask_b200_plan& pl, const SoftmaxArgs& a) {
  if (pl.device >= 0) return softmax_rows_grid(a, pl.num_sms);
  return int(std::max<uint64_t>(1, std::min<uint64_t>(a.rows, uint64_t(pl.num_sms) * 8)));
}

void finish_elementwise(ask_b200_plan& pl) {
  // Specialisation lookup on the canonical SSA form.
  pl.spec = EW_GENERIC;
  for (int s = 1; s < EW_NUM_SPECS && !pl.views; ++s) {
    Program sp{};
    if (ew_spec_program(s, &sp) && same_program(sp, pl.prog)) { pl.spec = s; break; }
  }
  if (pl.views) {
    pl.kernel = "ew_view";
    int occ = pl.device >= 0 ? ew_view_occupancy() : 8;
    if (pl.blocks_per_sm) occ = std::min(occ, pl.blocks_per_sm);
    const uint64_t needed = (pl.count + kEwThreads - 1) / kEwThreads;
    pl.grid = int(std::max<uint64_t>(1, std::min(needed, uint64_t(std::max(occ, 1)) * uint64_t(pl.num_sms))));
    pl.launches = pl.count ? 1 : 0;
    return;
  }
  if (pl.spec == EW_GENERIC) assign_registers(pl.prog);
  const char* names[] = {"ew_generic", "ew_cfg1", "ew_cfg5b", "ew_softmax_norm_f16", "ew_softmax_norm_bf16"};
  pl.kernel = names[pl.spec];
  int occ = blocks_per_sm_default(0);
  if (pl.device >= 0) check_cuda(ew_occupancy(pl.spec, &occ), "occupancy");
  if (pl.blocks_per_sm) occ = std::min(occ, pl.blocks_per_sm);
  const uint64_t units = (pl.count + 3) / 4;
  const uint64_t needed = (units + kEwThreads - 1) / kEwThreads;
  const uint64_t cap = uint64_t(std::max(occ, 1)) * uint64_t(pl.num_sms);
  pl.grid = int(std::max<uint64_t>(1, std::min(needed, cap)));
  pl.launches = pl.count ? 1 : 0;
  // The softmax plan's normalise step runs on the fused softmax's row kernel
  // (m, s and RN(1/s) once per row, no per-unit row division) when its rows
  // fit it and no grid cap is requested.
  pl.sm_step = 0;
  const bool norm = pl.spec == EW_SOFTMAX_NORM_F16 || pl.spec == EW_SOFTMAX_NORM_BF16;
  const int vpt = norm && !pl.blocks_per_sm && pl.inner && pl.count % pl.inner == 0
                      ? softmax_vectors_per_thread(pl.inner) : 0;
  if (vpt) {
    pl.sm_step = SM_STEP_NORM;
    pl.kernel = pl.spec == EW_SOFTMAX_NORM_F16 ? "softmax_rows_norm_f16" : "softmax_rows_norm_bf16";
    pl.red_grid = pl.grid;
    pl.block = int(pl.inner / 8 / uint64_t(vpt));
    SoftmaxArgs sa{};
    sa.rows = pl.count / pl.inner;
    sa.cols = pl.inner;
    sa.type = pl.inputs[0].dtype;
    sa.mode = SM_STEP_NORM;
    pl.grid = softmax_grid(pl, sa);
  }
}

void parse_ports(const json::Value& r, const char* key, bool with_map, std::vector<int>& types, std::vector<int>& maps) {
  const auto& arr = r.at(key).as_array(key);
  for (const auto& p : arr) {
    types.push_back(parse_dtype(p.at("dtype").as_str("dtype")));
    const json::Value* m = p.get("map");
    maps.push_back(with_map && m ? parse_map(m->as_str("map")) : IM_FULL);
  }
}

// An IM_VIEW port's view (PortView) from {"elements", "offset", "lo", "step",
// "extent", "stride", "pad"}; every element it can read must lie inside the
// port's `elements`.
// One window of a view: {"offset", "lo", "step", "extent", "stride", "pad"}
// over `rank` axes, whose reads must lie in [0, elements).
void parse_window(const json::Value& v, int rank, int type, uint64_t elements, int64_t* lo_, int64_t* step_,
                  int64_t* extent_, int64_t* stride_, int64_t* offset_, uint64_t* pad_) {
  *offset_ = v.at("offset").as_int("view offset");
  const char* keys[] = {"lo", "step", "extent", "stride"};
  int64_t* dst[] = {lo_, step_, extent_, stride_};
  for (int k = 0; k < 4; ++k) {
    const auto& a = v.at(keys[k]).as_array(keys[k]);
    if (int(a.size()) != rank) fail(ASK_B200_E_INVALID, std::string("view ") + keys[k] + " must have one entry per axis");
    for (int d = 0; d < rank; ++d) dst[k][d] = a[size_t(d)].as_int(keys[k]);
  }
  bool empty = false;
  int64_t lo = *offset_, hi = *offset_;
  for (int d = 0; d < rank; ++d) {
    if (step_[d] < 1) fail(ASK_B200_E_INVALID, "view steps must be positive");
    if (extent_[d] < 0) fail(ASK_B200_E_INVALID, "view extents must be non-negative");
    if (extent_[d] == 0) empty = true;
    const int64_t span = (extent_[d] ? extent_[d] - 1 : 0) * stride_[d];
    lo += span < 0 ? span : 0;
    hi += span > 0 ? span : 0;
  }
  if (!empty && (lo < 0 || uint64_t(hi) >= elements))
    fail(ASK_B200_E_INVALID, "a view reads outside its port's elements");
  const json::Value* pad = v.get("pad");
  *pad_ = pad ? constant_word(*pad, type) : 0;
}

// An IM_VIEW port's view (PortView) from {"elements", "offset", "lo", "step",
// "extent", "stride", "pad"[, "inner": {"shape", "offset", "lo", "step",
// "extent", "stride", "pad"}]}; every element it can read must lie inside the
// port's `elements` (with "inner", the outer window's positions inside the
// inner shape, and the inner window's reads inside the port).
PortView parse_view(const json::Value& v, int rank, int type, uint64_t* elements) {
  PortView pv{};
  *elements = checked_count(v.at("elements"), "view elements");
  const json::Value* inner = v.get("inner");
  uint64_t positions = *elements;
  if (inner) {
    const auto& sh = inner->at("shape").as_array("inner shape");
    if (sh.empty() || sh.size() > size_t(kMaxRank)) fail(ASK_B200_E_INVALID, "inner view rank must be 1..6");
    pv.inner_rank = int64_t(sh.size());
    positions = 1;
    for (size_t d = 0; d < sh.size(); ++d) {
      pv.inner_shape[d] = sh[d].as_int("inner shape");
      if (pv.inner_shape[d] < 1) fail(ASK_B200_E_INVALID, "inner view extents must be positive");
      positions *= uint64_t(pv.inner_shape[d]);
    }
    parse_window(*inner, int(pv.inner_rank), type, *elements, pv.ilo, pv.istep, pv.iextent, pv.istride, &pv.ioffset,
                 &pv.ipad);
  }
  parse_window(v, rank, type, positions, pv.lo, pv.step, pv.extent, pv.stride, &pv.offset, &pv.pad);
  return pv;
}

void build_elementwise(ask_b200_plan& pl, const json::Value& r) {
  pl.count = checked_count(r.at("count"), "count");
  const json::Value* in = r.get("inner");
  pl.inner = in ? checked_count(*in, "inner") : 1;
  Ports ports;
  parse_ports(r, "inputs", true, ports.type, ports.map);
  pl.prog = canonical(parse_program(r.at("program"), r.at("results"), ports, true));
  pl.ssa = pl.prog;
  bool uses_div = false;
  bool coords = false;
  for (int i = 0; i < pl.prog.n_insn; ++i) coords = coords || pl.prog.insn[i].op == OP_COORD;
  const json::Value* shape = r.get("shape");
  int rank = 1;
  pl.vs = ViewSet{};
  if (shape) {
    const auto& a = shape->as_array("shape");
    if (a.empty() || a.size() > size_t(kMaxRank)) fail(ASK_B200_E_UNSUPPORTED, "iteration shape must have 1..6 axes");
    rank = int(a.size());
    uint64_t n = 1;
    for (int d = 0; d < rank; ++d) n = mul_checked(n, pl.vs.shape[d] = checked_count(a[size_t(d)], "shape"));
    if (n != pl.count) fail(ASK_B200_E_INVALID, "the iteration shape's element count differs from count");
  } else {
    pl.vs.shape[0] = pl.count;
  }
  pl.vs.rank = rank;
  for (int i = 0; i < pl.prog.n_insn; ++i)
    if (pl.prog.insn[i].op == OP_COORD && int(pl.prog.insn[i].aux) >= rank)
      fail(ASK_B200_E_INVALID, "coord axis beyond the iteration shape");
  const auto& in_json = r.at("inputs").as_array("inputs");
  for (size_t k = 0; k < ports.type.size(); ++k) {
    uint64_t elems = pl.count;
    if (ports.map[k] == IM_SCALAR) elems = 1;
    if (ports.map[k] == IM_OUTER || ports.map[k] == IM_INNER) uses_div = true;
    if (ports.map[k] == IM_OUTER) elems = pl.inner ? pl.count / pl.inner : 0;
    if (ports.map[k] == IM_INNER) elems = pl.inner;
    if (ports.map[k] == IM_VIEW) {
      if (!shape) fail(ASK_B200_E_INVALID, "a view port needs the step's iteration \"shape\"");
      pl.vs.port[k] = parse_view(in_json[k].at("view"), rank, ports.type[k], &elems);
      pl.views = true;
    }
    pl.inputs.push_back({ports.type[k], elems, ports.map[k]});
  }
  pl.views = pl.views || coords;
  if (uses_div && (pl.inner == 0 || pl.count % pl.inner != 0))
    fail(ASK_B200_E_INVALID, "inner must divide count when an outer/inner index map is used");
  std::vector<int> otypes, omaps;
  parse_ports(r, "outputs", false, otypes, omaps);
  if (otypes.size() != pl.prog.n_out) fail(ASK_B200_E_INVALID, "outputs and results differ in length");
  for (size_t k = 0; k < otypes.size(); ++k) {
    if (otypes[k] != pl.prog.out_type[k])
      fail(ASK_B200_E_INVALID, "output " + std::to_string(k) + " type does not match its result");
    pl.outputs.push_back({otypes[k], pl.count, IM_FULL});
  }
  finish_elementwise(pl);
}

int parse_red_op(const std::string& s) {
  const std::string n = strip_prefix(s);
  const char* names[] = {"sum", "prod", "max", "min", "any", "all", "argmax", "argmin"};
  for (int k = 0; k < kNumRedOps; ++k)
    if (n == names[k] || n == std::string("reduce_") + names[k]) return k;
  fail(ASK_B200_E_UNSUPPORTED, "unknown reduction '" + s + "'");
}

void build_reduce(ask_b200_plan& pl, const json::Value& r) {
  const uint64_t outer = checked_count(r.at("outer"), "outer");
  const uint64_t extent = checked_count(r.at("extent"), "extent");
  const json::Value* in = r.get("inner");
  const uint64_t inner = in ? checked_count(*in, "inner") : 1;
  const json::Value* ib = r.get("index_base");
  const uint64_t index_base = ib ? checked_count(*ib, "index_base") : 0;
  Ports ports;
  parse_ports(r, "inputs", true, ports.type, ports.map);
  pl.prog = canonical(parse_program(r.at("program"), r.at("results"), ports, false));
  pl.ssa = pl.prog;
  // Views (IM_VIEW ports) and coordinates are defined over the step's
  // iteration shape: the reduced operand's shape, whose axes flatten to
  // [outer, extent, inner].
  bool coords = false;
  for (int i = 0; i < pl.prog.n_insn; ++i) coords = coords || pl.prog.insn[i].op == OP_COORD;
  bool any_view = coords;
  for (int m : ports.map) {
    any_view = any_view || m == IM_VIEW;
    if (m == IM_INNER) fail(ASK_B200_E_UNSUPPORTED, "reduction prologues read full, outer, scalar or view ports");
  }
  pl.vs = ViewSet{};
  pl.vs.rank = 1;
  pl.vs.shape[0] = mul_checked(mul_checked(outer, extent), inner);
  if (const json::Value* shape = r.get("shape")) {
    const auto& sa = shape->as_array("shape");
    if (sa.empty() || sa.size() > size_t(kMaxRank)) fail(ASK_B200_E_UNSUPPORTED, "iteration shape must have 1..6 axes");
    pl.vs.rank = int(sa.size());
    uint64_t count = 1;
    for (int d = 0; d < pl.vs.rank; ++d) count = mul_checked(count, pl.vs.shape[d] = checked_count(sa[size_t(d)], "shape"));
    if (count != mul_checked(mul_checked(outer, extent), inner))
      fail(ASK_B200_E_INVALID, "the iteration shape's element count differs from outer * extent * inner");
  } else if (any_view) {
    fail(ASK_B200_E_INVALID, "a view port or coord needs the step's iteration \"shape\"");
  }
  for (int i = 0; i < pl.prog.n_insn; ++i)
    if (pl.prog.insn[i].op == OP_COORD && int(pl.prog.insn[i].aux) >= pl.vs.rank)
      fail(ASK_B200_E_INVALID, "coord axis beyond the iteration shape");
  pl.views = any_view;
  const auto& reds = r.at("reductions").as_array("reductions");
  if (reds.empty() || reds.size() > size_t(kMaxReductions))
    fail(ASK_B200_E_UNSUPPORTED, "1.." + std::to_string(kMaxReductions) + " reductions per step");
  RedArgs& a = pl.red;
  a = RedArgs{};
  a.outer = outer; a.extent = extent; a.inner = inner; a.index_base = index_base;
  a.n_red = uint8_t(reds.size());
  const uint64_t n_outputs = mul_checked(outer, inner);
  const uint64_t n_elems = mul_checked(n_outputs, extent);
  const auto& in_json = r.at("inputs").as_array("inputs");
  for (size_t k = 0; k < ports.type.size(); ++k) {
    uint64_t elems = ports.map[k] == IM_FULL ? n_elems : ports.map[k] == IM_SCALAR ? 1 : n_outputs;
    if (ports.map[k] == IM_VIEW) pl.vs.port[k] = parse_view(in_json[k].at("view"), pl.vs.rank, ports.type[k], &elems);
    pl.inputs.push_back({ports.type[k], elems, ports.map[k]});
  }
  for (size_t k = 0; k < reds.size(); ++k) {
    const int op = parse_red_op(reds[k].at("op").as_str("op"));
    const int64_t src = reds[k].get("value") ? reds[k].at("value").as_int("value") : 0;
    if (src < 0 || src >= pl.prog.n_out) fail(ASK_B200_E_INVALID, "reduction value names no result");
    const int t = pl.prog.out_type[src];
    if ((op == RED_ANY || op == RED_ALL) && t != kBool) fail(ASK_B200_E_INVALID, "reduce_any/all need bool");
    if ((op == RED_SUM || op == RED_PROD) && t == kBool) fail(ASK_B200_E_INVALID, "reduce_sum/prod need a numeric type");
    if (red_is_arg(op) && extent == 0) fail(ASK_B200_E_INVALID, "argmax/argmin need a non-empty axis");
    if ((op == RED_MAX || op == RED_MIN) && extent == 0 && n_outputs)
      fail(ASK_B200_E_INVALID, "reduce_max/min need a non-empty domain");
    a.red_op[k] = uint8_t(op);
    a.red_src[k] = uint8_t(src);
    a.red_type[k] = uint8_t(t);
    const int ot = red_is_arg(op) ? kI64 : (op == RED_ANY || op == RED_ALL) ? kBool : t;
    pl.outputs.push_back({ot, n_outputs, IM_FULL});
  }
  if (const json::Value* outs = r.get("outputs")) {
    const auto& arr = outs->as_array("outputs");
    if (arr.size() != reds.size()) fail(ASK_B200_E_INVALID, "one output per reduction");
    for (size_t k = 0; k < arr.size(); ++k)
      if (parse_dtype(arr[k].at("dtype").as_str("dtype")) != pl.outputs[k].dtype)
        fail(ASK_B200_E_INVALID, "output " + std::to_string(k) + " type does not match its reduction");
  }
  if (pl.views) {  // the view path: a warp per output, no specialisation, no scratch
    assign_registers(pl.prog);
    pl.kernel = "reduce_view";
    pl.strategy = RS_WARP_ROW;
    const int occ = std::min(pl.device >= 0 ? red_view_occupancy() : 8, pl.blocks_per_sm ? pl.blocks_per_sm : 64);
    const uint64_t needed = (n_outputs + (kRedThreads / 32) - 1) / (kRedThreads / 32);
    pl.grid = int(std::max<uint64_t>(1, std::min(needed, uint64_t(std::max(occ, 1)) * uint64_t(pl.num_sms))));
    pl.launches = n_outputs ? 1 : 0;
    pl.scratch = 0;
    return;
  }
  // Strategy.
  std::string forced = r.get("strategy") ? r.at("strategy").as_str("strategy") : "";
  if (inner != 1) pl.strategy = RS_COLUMN;
  else if (forced == "split" || (forced.empty() && outer < uint64_t(pl.num_sms) * 4 && extent >= 32768)) pl.strategy = RS_SPLIT;
  else pl.strategy = RS_WARP_ROW;
  if (forced == "warp_row" && inner == 1) pl.strategy = RS_WARP_ROW;
  // Specialisation.
  pl.spec = RED_GENERIC;
  // The specialised kernels index elements of a row with 32 bits.
  if (pl.strategy != RS_COLUMN && extent <= (uint64_t(1) << 32))
    for (int s = 1; s < RED_NUM_SPECS; ++s) {
      Program sp{};
      int nr = 0;
      uint8_t ops[kMaxReductions] = {};
      if (!red_spec_program(s, &sp, &nr, ops) || !same_program(sp, pl.prog) || nr != a.n_red) continue;
      bool same = true;
      for (int k = 0; k < nr; ++k) same = same && ops[k] == a.red_op[k] && a.red_src[k] == 0;
      if (same) { pl.spec = s; break; }
    }
  if (pl.spec == RED_GENERIC) assign_registers(pl.prog);
  const char* spec_names[] = {"generic", "rowstats_f32", "global_f32", "softmax_max_f16", "softmax_max_bf16",
                              "softmax_sum_f16", "softmax_sum_bf16"};
  const char* strat_names[] = {"warp_row", "column", "split"};
  pl.kernel = std::string("reduce_") + strat_names[pl.strategy] + "_" + spec_names[pl.spec];
  // The softmax plan's first two steps (the prologues matched above) run on the
  // fused softmax's row kernel -- a CTA per row, the next row loaded before this
  // row's reduction -- when the row length fits it and no strategy is forced.
  const int sm_vpt =
      pl.strategy == RS_WARP_ROW && forced.empty() && !pl.blocks_per_sm ? softmax_vectors_per_thread(extent) : 0;
  if (sm_vpt && (pl.spec == RED_SOFTMAX_MAX_F16 || pl.spec == RED_SOFTMAX_MAX_BF16))
    pl.sm_step = SM_STEP_MAX;
  else if (sm_vpt && (pl.spec == RED_SOFTMAX_SUM_F16 || pl.spec == RED_SOFTMAX_SUM_BF16))
    pl.sm_step = SM_STEP_SUM;
  else
    pl.sm_step = 0;
  int occ = blocks_per_sm_default(0);
  if (pl.device >= 0) check_cuda(red_occupancy(pl.spec, pl.strategy, &occ), "occupancy");
  if (pl.blocks_per_sm) occ = std::min(occ, pl.blocks_per_sm);
  const uint64_t cap = uint64_t(std::max(occ, 1)) * uint64_t(pl.num_sms);
  uint64_t needed;
  if (pl.strategy == RS_WARP_ROW) needed = (outer + (kRedThreads / 32) - 1) / (kRedThreads / 32);
  else if (pl.strategy == RS_COLUMN) needed = (n_outputs + kRedThreads - 1) / kRedThreads;
  else needed = std::max<uint64_t>(1, extent / 8192);
  pl.grid = int(std::max<uint64_t>(1, std::min(needed, cap)));
  pl.launches = n_outputs ? (pl.strategy == RS_SPLIT ? 2 : 1) : 0;
  pl.scratch = 0;
  pl.col_chunks = 1;
  if (pl.sm_step) {
    const bool f16 = pl.spec == RED_SOFTMAX_MAX_F16 || pl.spec == RED_SOFTMAX_SUM_F16;
    pl.kernel = std::string(pl.sm_step == SM_STEP_MAX ? "softmax_rows_max_" : "softmax_rows_sum_") +
                (f16 ? "f16" : "bf16");
    pl.red_grid = pl.grid;
    pl.block = int(extent / 8 / uint64_t(sm_vpt));
    SoftmaxArgs sa{};
    sa.rows = outer;
    sa.cols = extent;
    sa.type = pl.inputs[0].dtype;
    sa.mode = pl.sm_step;
    pl.grid = softmax_grid(pl, sa);
  }
  if (pl.strategy == RS_COLUMN && n_outputs && extent >= 64) {
    // Too few columns to fill the GPU (2048 threads per SM): split the extent
    // into chunks (grid.y) of at least 32 elements, none empty.
    const uint64_t threads = uint64_t(pl.num_sms) * 2048;
    if (n_outputs * 2 <= threads) {
      uint64_t chunks = std::min<uint64_t>({(threads + n_outputs - 1) / n_outputs, extent / 32, 1024});
      if (chunks > 1) {
        const uint64_t per = (extent + chunks - 1) / chunks;
        chunks = (extent + per - 1) / per;
        pl.col_chunks = int(chunks);
        pl.launches = 2;
        pl.kernel = std::string("reduce_column_chunks_") + spec_names[pl.spec];
        pl.scratch = red_column_chunks_scratch_bytes(n_outputs, pl.col_chunks, a.n_red);
      }
    }
  }
  if (pl.strategy == RS_SPLIT) {
    const size_t part = red_split_scratch_bytes(pl.grid, a.n_red) * size_t(outer);
    pl.record_offset = (part + 255) & ~size_t(255);
    pl.shardable = outer == 1;
    // Sharded launches also keep this rank's record and the gathered records.
    pl.scratch = pl.shardable ? pl.record_offset + size_t(1 + kMaxRanks) * a.n_red * sizeof(RedPartial) : part;
  }
}

void build_index(ask_b200_plan& pl, const json::Value& r, bool scatter) {
  IndexArgs& a = pl.idx;
  a = IndexArgs{};
  a.outer = r.get("outer") ? checked_count(r.at("outer"), "outer") : 1;
  a.dim = checked_count(r.at("dim"), "dim");
  a.inner = r.get("inner") ? checked_count(r.at("inner"), "inner") : 1;
  a.n = checked_count(r.at("n"), "n");
  a.elem_type = parse_dtype(r.at("dtype").as_str("dtype"));
  a.index_type = parse_dtype(r.at("index_dtype").as_str("index_dtype"));
  if (a.index_type != kI32 && a.index_type != kI64) fail(ASK_B200_E_INVALID, "indices must be i32 or i64");
  const uint64_t table = mul_checked(mul_checked(a.outer, a.dim), a.inner);
  const uint64_t rows = mul_checked(mul_checked(a.outer, a.n), a.inner);
  if (!scatter) {
    pl.inputs = {{a.elem_type, table, IM_FULL}, {a.index_type, a.n, IM_FULL}};
    pl.outputs = {{a.elem_type, rows, IM_FULL}};
    pl.kernel = "gather_rows";
    pl.launches = rows ? 1 : 0;
  } else {
    if (a.elem_type == kBool) fail(ASK_B200_E_INVALID, "scatter_add needs a numeric type");
    pl.inputs = {{a.elem_type, table, IM_FULL}, {a.index_type, a.n, IM_FULL}, {a.elem_type, rows, IM_FULL}};
    pl.outputs = {{a.elem_type, table, IM_FULL}};
    pl.kernel = scatter_sorted_ok(a) ? "scatter_add_sorted_rows" :
                a.elem_type == kF32 ? "scatter_add_rows_f32v" : "scatter_add_elems";
    if (scatter_sorted_ok(a)) pl.scratch = scatter_sorted_scratch_bytes(a);
    if (const json::Value* pc = r.get("pre_copy")) {
      if (pc->at("input").as_int("pre_copy.input") != 0 || pc->at("output").as_int("pre_copy.output") != 0)
        fail(ASK_B200_E_INVALID, "pre_copy must copy input 0 (base) to output 0");
    }
    pl.launches = (table ? 1 : 0) + (rows && a.dim ? (scatter_sorted_ok(a) ? 8 : 1) : 0);
  }
  pl.grid = pl.num_sms * 8;
}

// Family S: {"family": "softmax", "dtype": "f16"|"bf16", "rows": R, "cols": C}
// -- the reference's three softmax steps (row max, row sum of exp(x - max),
// normalise) as one step with outputs m [R] f32, s [R] f32, y [R, C].
void build_softmax(ask_b200_plan& pl, const json::Value& r) {
  SoftmaxArgs& a = pl.sm;
  a = SoftmaxArgs{};
  a.type = parse_dtype(r.at("dtype").as_str("dtype"));
  if (a.type != kF16 && a.type != kBF16) fail(ASK_B200_E_UNSUPPORTED, "the fused softmax reads f16 or bf16 rows");
  a.rows = checked_count(r.at("rows"), "rows");
  a.cols = checked_count(r.at("cols"), "cols");
  const int vpt = softmax_vectors_per_thread(a.cols);
  if (!vpt) fail(ASK_B200_E_UNSUPPORTED, "the fused softmax needs cols a multiple of 256 and at most 32768");
  const uint64_t n = mul_checked(a.rows, a.cols);
  pl.inputs = {{a.type, n, IM_FULL}};
  pl.outputs = {{kF32, a.rows, IM_FULL}, {kF32, a.rows, IM_FULL}, {a.type, n, IM_FULL}};
  pl.kernel = a.type == kF16 ? "softmax_rows_f16" : "softmax_rows_bf16";
  pl.launches = a.rows ? 1 : 0;
  pl.grid = softmax_grid(pl, a);
  pl.block = int(a.cols / 8 / uint64_t(vpt));
}

// The diagnostics the reference's CUDA lowering reports for a step
// (lib/Lowering/CUDA.cpp:408-417, "cuda_lowering"), for the kernels this plan
// launches: the same fields with the same meaning, plus the plan's strategy.
// indexing is "cooperative_grid_stride" when outputs are reduced by a warp
// each (the reference's warp reduction), else "linear_grid_stride";
// reduction_loop_count counts passes over the reduced domain (one: every
// reduction of a step folds in the same pass); input_load_count counts input
// ports, each read once per element.  pre_copy names the step's base input.
std::string cuda_lowering(const ask_b200_plan& pl, long pre_copy_input) {
  const bool reduce = pl.family == FAM_REDUCE, softmax = pl.family == FAM_SOFTMAX;
  const bool warp = (reduce && !pl.views && pl.strategy == RS_WARP_ROW) || softmax;
  const int block = pl.sm_step ? pl.block : pl.family == FAM_ELEMENTWISE ? kEwThreads : reduce ? kRedThreads
                  : softmax ? pl.block : 256;
  size_t empty = 0;
  std::ostringstream outs;
  for (size_t k = 0; k < pl.outputs.size(); ++k) {
    if (pl.outputs[k].elements == 0) { ++empty; continue; }
    outs << (outs.tellp() > 0 ? "," : "") << k;
  }
  uint64_t count = pl.outputs.empty() ? 0 : pl.outputs[0].elements;
  if (pl.family == FAM_SCATTER && pl.inputs.size() > 2) count = pl.inputs[2].elements;
  if (softmax) count = pl.sm.rows;
  uint64_t per_output = warp ? (softmax || pl.sm_step ? uint64_t(pl.block) : 32) : 1;
  if (reduce && !pl.views && pl.strategy == RS_SPLIT) per_output = uint64_t(pl.grid) * uint64_t(block);
  const char* strat[] = {"warp_row", "column", "split"};
  const char* strategy = pl.sm_step ? "row_cta" : pl.views ? "view" : strat[pl.strategy];
  std::ostringstream o;
  o << "{\"statistics_stage\":\"cuda_lowering\",\"kernel_count\":" << pl.launches << ",\"indexing\":\""
    << (warp ? "cooperative_grid_stride" : "linear_grid_stride") << "\",\"warp_reduction_groups\":" << (warp ? 1 : 0)
    << ",\"output_loop_count\":" << (pl.outputs.size() > empty ? 1 : 0) << ",\"input_load_count\":" << pl.inputs.size()
    << ",\"reduction_loop_count\":" << (reduce || softmax ? 1 : 0) << ",\"zero_element_outputs\":" << empty
    << ",\"temporary_buffer_count\":0,\"scratch_bytes\":" << pl.scratch << ",\"groups\":[";
  if (pl.outputs.size() > empty)
    o << "{\"outputs\":[" << outs.str() << "],\"element_count\":" << count << ",\"threads_per_output\":" << per_output
      << "}";
  o << "],\"bool_storage\":\"one-byte-zero-or-one\",\"cast_semantics\":\"rne-saturating-fptosi-nan-zero-v1\","
    << "\"kernel\":\"" << pl.kernel << "\",\"strategy\":\""
    << (reduce ? strategy : kFamilyNames[pl.family]) << "\"";
  if (pl.family == FAM_SCATTER) o << ",\"pre_copy\":{\"input\":" << pre_copy_input << ",\"output\":0}";
  o << "}";
  return o.str();
}

std::string describe(const ask_b200_plan& pl) {
  std::ostringstream o;
  o << "{\"format\":\"ask-b200-recipe\",\"abi_version\":" << ASK_B200_ABI_VERSION << ",\"family\":\""
    << kFamilyNames[pl.family] << "\",\"kernel\":\"" << pl.kernel << "\",\"device\":" << pl.device
    << ",\"target\":{\"backend\":\"cuda\",\"arch\":100},\"launch\":{\"grid\":[" << pl.grid << "," << pl.col_chunks << ",1],\"block\":["
    << (pl.sm_step ? pl.block : pl.family == FAM_ELEMENTWISE ? kEwThreads : pl.family == FAM_REDUCE ? kRedThreads :
        pl.family == FAM_SOFTMAX ? pl.block : 256)
    << ",1,1],\"shared_bytes\":0},\"kernels_per_launch\":" << pl.launches << ",\"scratch_bytes\":" << pl.scratch;
  if (pl.family == FAM_REDUCE) {
    const char* strat[] = {"warp_row", "column", "split"};
    o << ",\"strategy\":\"" << (pl.sm_step ? "row_cta" : pl.views ? "view" : strat[pl.strategy]) << "\",\"shardable\":" << (pl.shardable ? "true" : "false")
      << ",\"outer\":" << pl.red.outer << ",\"extent\":" << pl.red.extent << ",\"inner\":" << pl.red.inner
      << ",\"index_base\":" << pl.red.index_base;
  }
  if (pl.family == FAM_ELEMENTWISE || pl.family == FAM_REDUCE)
    o << ",\"specialized\":" << (pl.spec ? "true" : "false") << ",\"registers\":" << int(pl.prog.n_regs);
  if (pl.family == FAM_SCATTER) o << ",\"pre_copy\":{\"input\":0,\"output\":0}";
  o << ",\"port_map\":[";
  size_t arg = 0;
  auto port = [&](const PortInfo& p, const char* kind, size_t k) {
    if (arg) o << ",";
    o << "{\"argument\":" << arg++ << ",\"logical_port\":\"" << kind << ":" << k << "\",\"element_type\":\""
      << kTypeNames[p.dtype] << "\",\"elements\":" << p.elements << ",\"storage_bytes\":" << dtype_bytes(p.dtype)
      << ",\"map\":\"" << map_name(p.map) << "\",\"layout\":\"contiguous_row_major\"}";
  };
  for (size_t k = 0; k < pl.inputs.size(); ++k) port(pl.inputs[k], "input", k);
  for (size_t k = 0; k < pl.outputs.size(); ++k) port(pl.outputs[k], "output", k);
  // The reference artifact's invocation v2 and required element types
  // (lib/Lowering/CUDA.cpp:392-407): arguments are the ports in port order.
  const int block = pl.sm_step ? pl.block : pl.family == FAM_ELEMENTWISE ? kEwThreads
                    : pl.family == FAM_REDUCE ? kRedThreads
                    : pl.family == FAM_SOFTMAX ? pl.block : 256;
  o << "],\"invocation\":{\"version\":2,\"kind\":\"ask-b200-recipe\",\"grid\":[" << pl.grid
    << ",1,1],\"block\":[" << block << ",1,1],\"shared_bytes\":0,\"arguments\":[";
  for (size_t k = 0; k < pl.inputs.size() + pl.outputs.size(); ++k)
    o << (k ? "," : "") << "\"" << (k < pl.inputs.size() ? "input:" : "output:")
      << (k < pl.inputs.size() ? k : k - pl.inputs.size()) << "\"";
  o << "]},\"required_element_types\":[";
  bool used[kNumDTypes] = {}, first = true;
  for (const PortInfo& p : pl.inputs) used[p.dtype] = true;
  for (const PortInfo& p : pl.outputs) used[p.dtype] = true;
  for (int t : {kBool, kI32, kI64, kF32, kF16, kBF16})
    if (used[t]) {
      o << (first ? "" : ",") << "\"" << kTypeNames[t] << "\"";
      first = false;
    }
  o << "],\"requires_disjoint_outputs\":true,\"outputs_must_not_alias_inputs\":"
    << (pl.family == FAM_SCATTER ? "false" : "true") << ",\"cuda_lowering\":" << cuda_lowering(pl, 0) << "}";
  return o.str();
}

bool aligned16(uint64_t p) { return (p & 15u) == 0; }

void check_device(const ask_b200_plan& pl) {
  if (pl.device < 0) fail(ASK_B200_E_DEVICE, "plan was created host-only (device -1) and cannot launch");
  int cur = -1;
  check_cuda(cudaGetDevice(&cur), "cudaGetDevice");
  if (cur != pl.device)
    fail(ASK_B200_E_DEVICE, "current device " + std::to_string(cur) + " is not the plan's device " + std::to_string(pl.device));
}

void check_ports(const ask_b200_plan& pl, const uint64_t* ports, size_t n_ports) {
  const size_t want = pl.inputs.size() + pl.outputs.size();
  if (n_ports != want) fail(ASK_B200_E_INVALID, "expected " + std::to_string(want) + " ports, got " + std::to_string(n_ports));
  if (!ports && want) fail(ASK_B200_E_INVALID, "ports is NULL");
  for (size_t k = 0; k < want; ++k) {
    const PortInfo& p = k < pl.inputs.size() ? pl.inputs[k] : pl.outputs[k - pl.inputs.size()];
    if (p.elements && !ports[k]) fail(ASK_B200_E_INVALID, "port " + std::to_string(k) + " is NULL");
    if (ports[k] % uint64_t(dtype_bytes(p.dtype)))
      fail(ASK_B200_E_INVALID, "port " + std::to_string(k) + " is not aligned to its element size");
  }
}

// Launch body shared by plain and sharded launches.  `rec_out` (sharded only)
// receives this rank's per-output records instead of the outputs.
void launch_plan(const ask_b200_plan& pl, const uint64_t* ports, uint64_t scratch, cudaStream_t st, RedPartial* rec_out) {
  const size_t ni = pl.inputs.size();
  switch (pl.family) {
    case FAM_ELEMENTWISE: {
      if (pl.views) {
        EwArgs a{};
        for (size_t k = 0; k < ni; ++k) a.in[k] = reinterpret_cast<const void*>(ports[k]);
        for (size_t k = 0; k < pl.outputs.size(); ++k) a.out[k] = reinterpret_cast<void*>(ports[ni + k]);
        a.count = pl.count;
        a.inner = make_u32div(pl.inner ? pl.inner : 1, pl.count);
        check_cuda(ew_view_launch(pl.prog, a, pl.vs, pl.grid, st), "elementwise launch");
        break;
      }
      EwArgs a{};
      bool aligned = true;
      for (size_t k = 0; k < ni; ++k) {
        a.in[k] = reinterpret_cast<const void*>(ports[k]);
        if (pl.inputs[k].map == IM_FULL || pl.inputs[k].map == IM_INNER) aligned &= aligned16(ports[k]);
      }
      for (size_t k = 0; k < pl.outputs.size(); ++k) {
        a.out[k] = reinterpret_cast<void*>(ports[ni + k]);
        aligned &= aligned16(ports[ni + k]);
      }
      a.count = pl.count;
      a.inner = make_u32div(pl.inner ? pl.inner : 1, pl.count);
      if (pl.sm_step && aligned) {
        SoftmaxArgs sa{};
        sa.x = a.in[0];
        sa.m_in = static_cast<const float*>(a.in[1]);
        sa.s_in = static_cast<const float*>(a.in[2]);
        sa.y = a.out[0];
        sa.rows = pl.count / pl.inner;
        sa.cols = pl.inner;
        sa.type = pl.inputs[0].dtype;
        sa.mode = SM_STEP_NORM;
        check_cuda(softmax_rows_launch(sa, pl.num_sms, st), "elementwise launch");
        break;
      }
      check_cuda(ew_launch(pl.spec, pl.prog, a, aligned ? 1 : 0, pl.sm_step ? pl.red_grid : pl.grid, st),
                 "elementwise launch");
      break;
    }
    case FAM_REDUCE: {
      if (pl.views) {
        RedArgs a = pl.red;
        for (size_t k = 0; k < ni; ++k) a.in[k] = reinterpret_cast<const void*>(ports[k]);
        for (size_t k = 0; k < pl.outputs.size(); ++k) a.out[k] = reinterpret_cast<void*>(ports[ni + k]);
        check_cuda(red_view_launch(pl.prog, a, pl.vs, pl.grid, st), "reduce launch");
        break;
      }
      RedArgs a = pl.red;
      bool aligned = true;
      for (size_t k = 0; k < ni; ++k) {
        a.in[k] = reinterpret_cast<const void*>(ports[k]);
        if (pl.inputs[k].map == IM_FULL) {
          aligned &= aligned16(ports[k]);
          aligned &= (a.extent * uint64_t(dtype_bytes(pl.inputs[k].dtype))) % 16 == 0;
        }
      }
      for (size_t k = 0; k < pl.outputs.size(); ++k) a.out[k] = reinterpret_cast<void*>(ports[ni + k]);
      if ((pl.strategy == RS_SPLIT || pl.col_chunks > 1) && !scratch)
        fail(ASK_B200_E_INVALID, "this plan needs scratch memory");
      if (scratch && !aligned16(scratch)) fail(ASK_B200_E_INVALID, "scratch must be 16-byte aligned");
      if (pl.col_chunks > 1) {
        check_cuda(red_column_chunks_launch(pl.prog, a, pl.grid, pl.col_chunks, reinterpret_cast<void*>(scratch), st),
                   "reduce launch");
        break;
      }
      if (pl.sm_step && aligned && !rec_out) {
        SoftmaxArgs sa{};
        sa.x = a.in[0];
        sa.rows = a.outer;
        sa.cols = a.extent;
        sa.type = pl.inputs[0].dtype;
        sa.mode = pl.sm_step;
        if (pl.sm_step == SM_STEP_MAX) {
          sa.m = static_cast<float*>(a.out[0]);
        } else {
          sa.m_in = static_cast<const float*>(a.in[1]);
          sa.s = static_cast<float*>(a.out[0]);
        }
        check_cuda(softmax_rows_launch(sa, pl.num_sms, st), "reduce launch");
        break;
      }
      check_cuda(red_launch(pl.spec, pl.strategy, pl.prog, a, aligned ? 1 : 0, pl.sm_step ? pl.red_grid : pl.grid,
                            reinterpret_cast<void*>(scratch), rec_out, st),
                 "reduce launch");
      break;
    }
    case FAM_GATHER: {
      IndexArgs a = pl.idx;
      a.table = reinterpret_cast<const void*>(ports[0]);
      a.index = reinterpret_cast<const void*>(ports[1]);
      a.out = reinterpret_cast<void*>(ports[2]);
      check_cuda(gather_launch(a, 1, pl.grid, st), "gather launch");
      break;
    }
    case FAM_SCATTER: {
      IndexArgs a = pl.idx;
      a.base = reinterpret_cast<const void*>(ports[0]);
      a.index = reinterpret_cast<const void*>(ports[1]);
      a.table = reinterpret_cast<const void*>(ports[2]);
      a.out = reinterpret_cast<void*>(ports[3]);
      if (pl.scratch && !scratch) fail(ASK_B200_E_INVALID, "this plan needs scratch memory");
      if (scratch && !aligned16(scratch)) fail(ASK_B200_E_INVALID, "scratch must be 16-byte aligned");
      check_cuda(scatter_add_launch(a, 1, pl.grid, reinterpret_cast<void*>(scratch), pl.num_sms, st),
                 "scatter_add launch");
      break;
    }
    case FAM_SOFTMAX: {
      SoftmaxArgs a = pl.sm;
      a.x = reinterpret_cast<const void*>(ports[0]);
      a.m = reinterpret_cast<float*>(ports[1]);
      a.s = reinterpret_cast<float*>(ports[2]);
      a.y = reinterpret_cast<void*>(ports[3]);
      if (a.rows && (!aligned16(ports[0]) || !aligned16(ports[3])))
        fail(ASK_B200_E_INVALID, "the fused softmax needs 16-byte aligned x and y");
      check_cuda(softmax_rows_launch(a, pl.num_sms, st), "softmax launch");
      break;
    }
    default:
      fail(ASK_B200_E_INVALID, "corrupt plan");
  }
}

// ---- NCCL, loaded at run time ---------------------------------------------------------
struct Nccl {
  void* lib = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*getErrorString)(ncclResult_t) = nullptr;
};

Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW);
    if (!h) return;
    n.lib = h;
    n.getUniqueId = reinterpret_cast<decltype(n.getUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    n.commInitRank = reinterpret_cast<decltype(n.commInitRank)>(dlsym(h, "ncclCommInitRank"));
    n.commDestroy = reinterpret_cast<decltype(n.commDestroy)>(dlsym(h, "ncclCommDestroy"));
    n.allGather = reinterpret_cast<decltype(n.allGather)>(dlsym(h, "ncclAllGather"));
    n.getErrorString = reinterpret_cast<decltype(n.getErrorString)>(dlsym(h, "ncclGetErrorString"));
  });
  if (!n.lib || !n.getUniqueId || !n.commInitRank || !n.commDestroy || !n.allGather)
    fail(ASK_B200_E_NCCL, "libnccl.so.2 could not be loaded");
  return n;
}

void check_nccl(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) {
    const char* s = nccl().getErrorString ? nccl().getErrorString(r) : "error";
    fail(ASK_B200_E_NCCL, std::string(what) + ": " + s);
  }
}

// ---- Zipf tables for the generator ---------------------------------------------------------
struct ZipfKey {
  int device;
  double s;
  uint64_t n;
  bool operator<(const ZipfKey& o) const {
    if (device != o.device) return device < o.device;
    if (s != o.s) return s < o.s;
    return n < o.n;
  }
};

const double* zipf_table(int device, double s, uint64_t n) {
  static std::mutex mu;
  static std::map<ZipfKey, double*> tables;
  std::lock_guard<std::mutex> lock(mu);
  const ZipfKey key{device, s, n};
  auto it = tables.find(key);
  if (it != tables.end()) return it->second;
  // Unnormalised cumulative weights sum_{j<=k+1} j^-s, accumulated in order.
  std::vector<double> cdf(n);
  double acc = 0.0;
  for (uint64_t k = 0; k < n; ++k) {
    acc += std::pow(double(k + 1), -s);
    cdf[k] = acc;
  }
  double* dev = nullptr;
  check_cuda(cudaMalloc(&dev, n * sizeof(double)), "cudaMalloc(zipf table)");
  check_cuda(cudaMemcpy(dev, cdf.data(), n * sizeof(double), cudaMemcpyHostToDevice), "zipf table upload");
  tables[key] = dev;
  return dev;
}

}  // namespace

// Peer-memory exchange for sharded reductions.  Every rank allocates a small
// inbox, the ranks trade its IPC handle with one NCCL all-gather, and each maps
// the others'.  Any failure (no peer access, IPC refused, the variable
// ASK_B200_NO_PEER_EXCHANGE set) leaves the NCCL all-gather path in place; all
// ranks take the same decision because the outcome is all-gathered too.
// ASK_B200_EXCHANGE_TIMEOUT_MS bounds each wait for the peers' flags (default
// 1000).
void release_peer_exchange(ask_b200_comm& c) {
  if (c.p2p) {
    // This rank's exchange kernels must be done before its buffers go.  After
    // a completed exchange every peer has already stored into this inbox
    // (this rank saw their flags), so nothing stores into it later; after a
    // timed-out one a late peer still may, so the buffers stay allocated and
    // mapped until the process exits.
    (void)cudaDeviceSynchronize();
    uint32_t word = 1;
    if (cudaMemcpy(&word, static_cast<char*>(c.inbox) + kInboxStatusOffset, sizeof(word), cudaMemcpyDeviceToHost) !=
            cudaSuccess ||
        word != 0) {
      (void)cudaGetLastError();
      c.opened.clear();
      c.inboxes_dev = nullptr;
      c.inbox = nullptr;
      c.p2p = false;
      return;
    }
  }
  for (void* p : c.opened)
    if (p) (void)cudaIpcCloseMemHandle(p);
  c.opened.clear();
  if (c.inboxes_dev) (void)cudaFree(c.inboxes_dev);
  if (c.inbox) (void)cudaFree(c.inbox);
  c.inboxes_dev = nullptr;
  c.inbox = nullptr;
  c.p2p = false;
}

void setup_peer_exchange(ask_b200_comm& c) {
  if (const char* t = std::getenv("ASK_B200_EXCHANGE_TIMEOUT_MS")) {
    const long ms = std::strtol(t, nullptr, 10);
    if (ms > 0 && ms <= 60000) c.timeout_ns = uint64_t(ms) * 1000000ull;
  }
  // each rank's IPC handle and whether it can take part
  struct Card {
    cudaIpcMemHandle_t handle;
    int ok;
    int pad[15];
  };
  static_assert(sizeof(Card) == 128, "card layout");
  Card mine{};
  mine.ok = std::getenv("ASK_B200_NO_PEER_EXCHANGE") ? 0 : 1;
  if (c.nranks > kExchangeMaxRanks) mine.ok = 0;
  if (mine.ok) {
    if (cudaMalloc(&c.inbox, kInboxBytes) != cudaSuccess || cudaMemset(c.inbox, 0, kInboxBytes) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine.handle, c.inbox) != cudaSuccess) {
      (void)cudaGetLastError();
      mine.ok = 0;
      c.p2p_note = "inbox allocation or IPC handle failed";
    }
  }
  Card* cards = nullptr;
  check_cuda(cudaMalloc(&cards, sizeof(Card) * size_t(c.nranks)), "exchange card buffer");
  check_cuda(cudaMemcpy(cards + c.rank, &mine, sizeof(Card), cudaMemcpyHostToDevice), "exchange card");
  std::vector<Card> all(size_t(c.nranks));
  const ncclResult_t nr = nccl().allGather(cards + c.rank, cards, sizeof(Card), ncclUint8, c.comm, nullptr);
  cudaError_t ce = nr == ncclSuccess ? cudaStreamSynchronize(nullptr) : cudaErrorUnknown;
  if (ce == cudaSuccess) ce = cudaMemcpy(all.data(), cards, sizeof(Card) * all.size(), cudaMemcpyDeviceToHost);
  (void)cudaFree(cards);
  if (nr != ncclSuccess) fail(ASK_B200_E_NCCL, "exchange card all-gather failed");
  check_cuda(ce, "exchange card all-gather");
  bool ok = true;
  for (const Card& k : all) ok = ok && k.ok;
  std::vector<void*> addr(size_t(c.nranks), nullptr);
  if (ok) {
    addr[size_t(c.rank)] = c.inbox;
    for (int r = 0; r < c.nranks && ok; ++r) {
      if (r == c.rank) continue;
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, all[size_t(r)].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess || !p) {
        (void)cudaGetLastError();
        ok = false;
        c.p2p_note = "cudaIpcOpenMemHandle of rank " + std::to_string(r) + "'s inbox failed";
        break;
      }
      c.opened.push_back(p);
      addr[size_t(r)] = p;
    }
  } else if (c.p2p_note.empty()) {
    c.p2p_note = mine.ok ? "another rank cannot take part" : "disabled on this rank";
  }
  // every rank must agree: all-gather the mapping outcome as well
  int* flags = nullptr;
  check_cuda(cudaMalloc(&flags, sizeof(int) * size_t(c.nranks)), "exchange flag buffer");
  const int mine_ok = ok ? 1 : 0;
  check_cuda(cudaMemcpy(flags + c.rank, &mine_ok, sizeof(int), cudaMemcpyHostToDevice), "exchange flag");
  const ncclResult_t nr2 = nccl().allGather(flags + c.rank, flags, sizeof(int), ncclUint8, c.comm, nullptr);
  std::vector<int> oks(size_t(c.nranks), 0);
  cudaError_t ce2 = nr2 == ncclSuccess ? cudaStreamSynchronize(nullptr) : cudaErrorUnknown;
  if (ce2 == cudaSuccess) ce2 = cudaMemcpy(oks.data(), flags, sizeof(int) * oks.size(), cudaMemcpyDeviceToHost);
  (void)cudaFree(flags);
  if (nr2 != ncclSuccess) fail(ASK_B200_E_NCCL, "exchange outcome all-gather failed");
  check_cuda(ce2, "exchange outcome all-gather");
  for (int v : oks) ok = ok && v;
  if (ok) {
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&c.inboxes_dev), sizeof(void*) * size_t(c.nranks)), "inbox table");
    check_cuda(cudaMemcpy(c.inboxes_dev, addr.data(), sizeof(void*) * addr.size(), cudaMemcpyHostToDevice),
               "inbox table");
    c.p2p = true;
  } else {
    if (c.p2p_note.empty()) c.p2p_note = "another rank could not map an inbox";
    release_peer_exchange(c);
  }
}

// The lowering adapter's cuda_lowering report (lower.cpp): that of the
// recipe's host-only plan, with the scatter base named by the step's argument.
std::string askb_recipe_lowering_report(const std::string& recipe_json, long pre_copy_input) {
  ask_b200_plan* p = nullptr;
  if (ask_b200_plan_create(recipe_json.c_str(), -1, &p) != ASK_B200_OK)
    throw std::runtime_error(std::string("lowered recipe: ") + ask_b200_last_error());
  std::unique_ptr<ask_b200_plan> owned(p);
  return cuda_lowering(*owned, pre_copy_input);
}

extern "C" {

int ask_b200_abi_version(void) { return ASK_B200_ABI_VERSION; }

const char* ask_b200_last_error(void) { return g_last_error.c_str(); }

int ask_b200_plan_create(const char* recipe_json, int device, ask_b200_plan** out) {
  return guarded([&] {
    if (!out) fail(ASK_B200_E_INVALID, "out is NULL");
    *out = nullptr;
    if (!recipe_json) fail(ASK_B200_E_INVALID, "recipe is NULL");
    std::unique_ptr<ask_b200_plan> pl(new ask_b200_plan());
    pl->device = device;
    if (device >= 0) {
      int count = 0;
      if (cudaGetDeviceCount(&count) != cudaSuccess || device >= count)
        fail(ASK_B200_E_DEVICE, "CUDA device " + std::to_string(device) + " is not available");
      cudaDeviceProp prop{};
      check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
      if (prop.major != 10)
        fail(ASK_B200_E_DEVICE, "this library is built for sm_100a; device " + std::to_string(device) + " is sm_" +
                                    std::to_string(prop.major) + std::to_string(prop.minor));
      pl->num_sms = prop.multiProcessorCount;
    }
    const json::Value r = json::parse(recipe_json);
    if (r.kind != json::Value::Object) fail(ASK_B200_E_INVALID, "recipe must be a JSON object");
    const std::string fam = r.at("family").as_str("family");
    // Optional cap on resident CTAs per SM of the persistent grids, to leave
    // room for a kernel that must run beside this one (a collective).
    if (const json::Value* b = r.get("blocks_per_sm")) {
      const int64_t v = b->as_int("blocks_per_sm");
      if (v < 1 || v > 32) fail(ASK_B200_E_INVALID, "blocks_per_sm must be in [1, 32]");
      pl->blocks_per_sm = int(v);
    }
    if (fam == "elementwise") { pl->family = FAM_ELEMENTWISE; build_elementwise(*pl, r); }
    else if (fam == "reduce") { pl->family = FAM_REDUCE; build_reduce(*pl, r); }
    else if (fam == "gather") { pl->family = FAM_GATHER; build_index(*pl, r, false); }
    else if (fam == "scatter_add") { pl->family = FAM_SCATTER; build_index(*pl, r, true); }
    else if (fam == "softmax") { pl->family = FAM_SOFTMAX; build_softmax(*pl, r); }
    else fail(ASK_B200_E_UNSUPPORTED, "unknown family '" + fam + "'");
    if (pl->inputs.size() + pl->outputs.size() > 64)
      fail(ASK_B200_E_UNSUPPORTED, "the pointer ABI supports at most 64 input and output buffers");
    *out = pl.release();
  });
}

int ask_b200_plan_destroy(ask_b200_plan* plan) {
  delete plan;
  return ASK_B200_OK;
}

int ask_b200_plan_ports(const ask_b200_plan* plan, size_t* n_inputs, size_t* n_outputs) {
  return guarded([&] {
    if (!plan) fail(ASK_B200_E_INVALID, "plan is NULL");
    if (n_inputs) *n_inputs = plan->inputs.size();
    if (n_outputs) *n_outputs = plan->outputs.size();
  });
}

int ask_b200_plan_scratch_bytes(const ask_b200_plan* plan, size_t* bytes) {
  return guarded([&] {
    if (!plan || !bytes) fail(ASK_B200_E_INVALID, "NULL argument");
    *bytes = plan->scratch;
  });
}

int ask_b200_plan_describe(const ask_b200_plan* plan, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    if (!plan) fail(ASK_B200_E_INVALID, "plan is NULL");
    const std::string d = describe(*plan);
    if (needed) *needed = d.size() + 1;
    if (buf && cap) {
      const size_t n = std::min(cap - 1, d.size());
      std::memcpy(buf, d.data(), n);
      buf[n] = '\0';
    }
  });
}

int ask_b200_plan_kernel_launches(const ask_b200_plan* plan, int* launches) {
  return guarded([&] {
    if (!plan || !launches) fail(ASK_B200_E_INVALID, "NULL argument");
    *launches = plan->launches;
  });
}

int ask_b200_plan_launch(const ask_b200_plan* plan, const uint64_t* ports, size_t n_ports, uint64_t scratch,
                         void* stream) {
  return guarded([&] {
    if (!plan) fail(ASK_B200_E_INVALID, "plan is NULL");
    check_ports(*plan, ports, n_ports);
    check_device(*plan);
    launch_plan(*plan, ports, scratch, static_cast<cudaStream_t>(stream), nullptr);
  });
}

int ask_b200_comm_unique_id(unsigned char id[128]) {
  return guarded([&] {
    if (!id) fail(ASK_B200_E_INVALID, "id is NULL");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId layout");
    ncclUniqueId uid;
    check_nccl(nccl().getUniqueId(&uid), "ncclGetUniqueId");
    std::memcpy(id, &uid, 128);
  });
}

int ask_b200_comm_create(const unsigned char id[128], int nranks, int rank, int device, ask_b200_comm** out) {
  return guarded([&] {
    if (!id || !out) fail(ASK_B200_E_INVALID, "NULL argument");
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
      fail(ASK_B200_E_INVALID, "rank/nranks out of range (at most " + std::to_string(kMaxRanks) + " ranks)");
    int cur = -1;
    check_cuda(cudaGetDevice(&cur), "cudaGetDevice");
    if (cur != device) fail(ASK_B200_E_DEVICE, "current device must be the communicator's device");
    ncclUniqueId uid;
    std::memcpy(&uid, id, 128);
    std::unique_ptr<ask_b200_comm> c(new ask_b200_comm());
    c->nranks = nranks; c->rank = rank; c->device = device;
    check_nccl(nccl().commInitRank(&c->comm, nranks, uid, rank), "ncclCommInitRank");
    try {
      setup_peer_exchange(*c);
    } catch (...) {
      release_peer_exchange(*c);
      (void)nccl().commDestroy(c->comm);
      throw;
    }
    *out = c.release();
  });
}

int ask_b200_comm_destroy(ask_b200_comm* comm) {
  return guarded([&] {
    if (!comm) return;
    release_peer_exchange(*comm);
    if (comm->comm) check_nccl(nccl().commDestroy(comm->comm), "ncclCommDestroy");
    delete comm;
  });
}

int ask_b200_comm_status(ask_b200_comm* comm, int* status, int* peer_exchange) {
  return guarded([&] {
    if (!comm || !status) fail(ASK_B200_E_INVALID, "NULL argument");
    *status = 0;
    if (peer_exchange) *peer_exchange = comm->p2p ? 1 : 0;
    if (!comm->p2p) return;
    uint32_t word = 0;
    check_cuda(cudaMemcpy(&word, static_cast<char*>(comm->inbox) + kInboxStatusOffset, sizeof(word),
                          cudaMemcpyDeviceToHost), "read exchange status");
    *status = word ? ASK_B200_E_TIMEOUT : 0;
  });
}

int ask_b200_plan_launch_sharded(const ask_b200_plan* plan, ask_b200_comm* comm, const uint64_t* ports,
                                 size_t n_ports, uint64_t scratch, void* stream) {
  return guarded([&] {
    if (!plan || !comm) fail(ASK_B200_E_INVALID, "NULL argument");
    if (plan->family != FAM_REDUCE || !plan->shardable)
      fail(ASK_B200_E_UNSUPPORTED, "only reduce plans with 0-D outputs (split strategy) combine across ranks; "
                                   "elementwise shards need no collective and use ask_b200_plan_launch");
    check_ports(*plan, ports, n_ports);
    check_device(*plan);
    if (comm->device != plan->device) fail(ASK_B200_E_DEVICE, "communicator and plan are on different devices");
    if (!scratch) fail(ASK_B200_E_INVALID, "this plan needs scratch memory");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    char* base = reinterpret_cast<char*>(scratch);
    RedPartial* mine = reinterpret_cast<RedPartial*>(base + plan->record_offset);
    RedPartial* all = mine + plan->red.n_red;
    launch_plan(*plan, ports, scratch, st, mine);
    RedArgs a = plan->red;
    for (size_t k = 0; k < plan->outputs.size(); ++k) a.out[k] = reinterpret_cast<void*>(ports[plan->inputs.size() + k]);
    if (comm->p2p) {
      check_cuda(red_exchange_combine(a, mine, comm->inboxes_dev, comm->nranks, comm->rank, comm->timeout_ns, st),
                 "exchange launch");
      return;
    }
    const size_t rec_bytes = size_t(plan->red.n_red) * sizeof(RedPartial);
    check_nccl(nccl().allGather(mine, all, rec_bytes, ncclUint8, comm->comm, st), "ncclAllGather");
    check_cuda(red_combine_records(a, all, comm->nranks, st), "combine launch");
  });
}

// Used by the fixed-scratch entry point (noalloc.cu): launch a reduce plan with
// scratch memory the caller did not allocate, after checking it is large enough.
int askb_internal_launch_reduce_fixed_scratch(const ask_b200_plan* plan, const uint64_t* ports, size_t n_ports,
                                              void* scratch, size_t capacity, void* stream) {
  return guarded([&] {
    if (!plan) fail(ASK_B200_E_INVALID, "plan is NULL");
    if (plan->family != FAM_REDUCE)
      fail(ASK_B200_E_UNSUPPORTED, "the fixed-scratch launch serves reduce plans only");
    check_ports(*plan, ports, n_ports);
    check_device(*plan);
    const size_t needed =
        plan->strategy == RS_SPLIT ? red_split_scratch_bytes(plan->grid, plan->red.n_red) * size_t(plan->red.outer)
        : plan->col_chunks > 1     ? plan->scratch
                                   : 0;
    if (needed > capacity)
      fail(ASK_B200_E_INVALID, "plan needs " + std::to_string(needed) + " bytes of scratch; the fixed scratch array "
                               "holds at most " + std::to_string(capacity) + " bytes (use ask_b200_plan_launch "
                               "with caller-provided scratch)");
    launch_plan(*plan, ports, needed ? reinterpret_cast<uint64_t>(scratch) : 0, static_cast<cudaStream_t>(stream),
                nullptr);
  });
}

void askb_internal_set_error(const char* message) { g_last_error = message ? message : ""; }

int ask_b200_generate(int kind, uint64_t seed, uint32_t stream_id, uint64_t offset, uint64_t count, double p0,
                      double p1, uint64_t dst, void* stream) {
  return guarded([&] {
    if (kind < GEN_UNIFORM_F32 || kind > GEN_ZIPF_I32) fail(ASK_B200_E_INVALID, "unknown generator kind");
    if (count && !dst) fail(ASK_B200_E_INVALID, "dst is NULL");
    const double* cdf = nullptr;
    uint64_t zn = 0;
    if (kind == GEN_ZIPF_I64 || kind == GEN_ZIPF_I32) {
      if (!(p1 >= 1.0) || p1 > 4294967296.0) fail(ASK_B200_E_INVALID, "Zipf rank count must be in [1, 2^32]");
      zn = uint64_t(p1);
      int dev = 0;
      check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
      cdf = zipf_table(dev, p0, zn);
    }
    check_cuda(gen_launch(kind, seed, stream_id, offset, count, p0, p1, cdf, zn, reinterpret_cast<void*>(dst),
                          static_cast<cudaStream_t>(stream)),
               "generator launch");
  });
}

}  // extern "C"
