// Kernel-artifact generator: one recipe step -> the CUDA source of one
// `extern "C"` kernel with plain pointer/scalar parameters, for packaging as
// ASK's external-kernel-artifact v2 (schemas/external-kernel-artifact-v2.schema.json,
// docs/en/compilers.md "Minimal Response").  The source instantiates the
// templates of artifact_bodies.cuh with the step's sizes and op program as
// compile-time constants; ask_b200/worker.py compiles it to an sm_100a cubin.
//
// Families: elementwise (the library's compile-time program loop, or the view
// loop for general index maps and input-free programs), reduce (a warp or a CTA
// per output row, a thread per output column) and gather.  scatter_add is
// refused: its base tensor reaches the output through the Runtime's pre_copy
// (lib/Lowering/CUDA.cpp:415-417, lib/Runtime/CUDA.cpp:873-884), which an
// artifact v2 cannot declare; the fused softmax is a runtime fusion of three
// steps, each of which packages on its own.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/ask_b200.h"
#include "../../include/ask_b200_artifact.h"
#include "json.h"
#include "kernels.h"
#include "plan_internal.h"

using namespace askb;

extern "C" void askb_internal_set_error(const char* message);

namespace {

struct Failure {
  int code;
  std::string message;
};
[[noreturn]] void fail(int code, const std::string& msg) { throw Failure{code, msg}; }

// ABI scalar types of ASK's external requests (docs/en/compilers.md, "Request
// Protocol v2"): C type and launch-parameter width in bytes.
struct Scalar {
  const char* name;
  const char* ctype;
  unsigned width;
};
constexpr Scalar kScalars[] = {{"i1", "bool", 1},        {"i8", "int8_t", 1},    {"i16", "int16_t", 2},
                               {"i32", "int32_t", 4},    {"i64", "int64_t", 8},  {"u8", "uint8_t", 1},
                               {"u16", "uint16_t", 2},   {"u32", "uint32_t", 4}, {"u64", "uint64_t", 8},
                               {"fp16", "uint16_t", 2},  {"bf16", "uint16_t", 2}, {"fp32", "float", 4},
                               {"fp64", "double", 8}};

const char* const kTypeNames[] = {"bool", "i32", "i64", "f32", "f16", "bf16"};

struct Param {
  bool port = false;
  bool output = false;
  size_t index = 0;           // port index within inputs or outputs
  const Scalar* scalar = nullptr;
};

std::vector<Param> parse_parameters(const json::Value& list, size_t n_in, size_t n_out) {
  std::vector<Param> out;
  std::vector<int> seen_in(n_in, 0), seen_out(n_out, 0);
  for (const json::Value& v : list.as_array("parameters")) {
    const std::string s = v.as_str("parameter");
    Param p;
    const size_t colon = s.find(':');
    if (colon != std::string::npos) {
      const std::string kind = s.substr(0, colon), num = s.substr(colon + 1);
      if ((kind != "input" && kind != "output") || num.empty() || num.size() > 6 ||
          num.find_first_not_of("0123456789") != std::string::npos || (num.size() > 1 && num[0] == '0'))
        fail(ASK_B200_E_INVALID, "parameter '" + s + "' is neither input:N, output:N nor a scalar type");
      p.port = true;
      p.output = kind == "output";
      p.index = size_t(std::stoul(num));
      std::vector<int>& seen = p.output ? seen_out : seen_in;
      if (p.index >= seen.size()) fail(ASK_B200_E_INVALID, "parameter '" + s + "' names no port of the step");
      if (seen[p.index]++) fail(ASK_B200_E_INVALID, "parameter '" + s + "' binds a port twice");
    } else {
      for (const Scalar& sc : kScalars)
        if (s == sc.name) p.scalar = &sc;
      if (!p.scalar) fail(ASK_B200_E_INVALID, "unknown scalar parameter type '" + s + "'");
    }
    out.push_back(p);
  }
  for (size_t k = 0; k < n_in; ++k)
    if (!seen_in[k]) fail(ASK_B200_E_INVALID, "input:" + std::to_string(k) + " is bound to no parameter");
  for (size_t k = 0; k < n_out; ++k)
    if (!seen_out[k]) fail(ASK_B200_E_INVALID, "output:" + std::to_string(k) + " is bound to no parameter");
  if (out.empty() || out.size() > 64) fail(ASK_B200_E_INVALID, "an artifact kernel takes 1..64 parameters");
  return out;
}

bool valid_entry(const std::string& e) {
  if (e.empty() || e.size() > 200) return false;
  for (size_t i = 0; i < e.size(); ++i) {
    const char c = e[i];
    const bool alpha = (c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z') || c == '_';
    if (!(alpha || (i > 0 && c >= '0' && c <= '9'))) return false;
  }
  return true;
}

std::string u64(uint64_t v) { return std::to_string(v) + "ull"; }
std::string i64(int64_t v) {
  return v == INT64_MIN ? std::string("(-9223372036854775807ll - 1)") : std::to_string(v) + "ll";
}

// Named pointers of the entry: p<i> for parameter i.
std::string port_expr(const std::vector<Param>& ps, bool output, size_t index) {
  for (size_t i = 0; i < ps.size(); ++i)
    if (ps[i].port && ps[i].output == output && ps[i].index == index) return "p" + std::to_string(i);
  fail(ASK_B200_E_INVALID, "internal: unbound port");
}

std::string insn_text(const Insn& x) {
  std::ostringstream o;
  o << "askb::Insn{" << int(x.op) << ", " << int(x.type) << ", " << int(x.dst) << ", " << int(x.a) << ", " << int(x.b)
    << ", " << int(x.c) << ", " << int(x.aux) << ", " << int(x.src_type) << ", " << x.imm << "ull}";
  return o.str();
}

template <class T>
std::string list_text(const T* v, int n) {
  std::ostringstream o;
  o << "{";
  for (int i = 0; i < n; ++i) o << (i ? ", " : "") << int(v[i]);
  if (n == 0) o << "0";
  o << "}";
  return o.str();
}

// The SSA program as a compile-time program type (programs.h's format).
std::string program_struct(const Program& p, const char* name) {
  std::ostringstream o;
  o << "struct " << name << " {\n  static constexpr int kInsn = " << int(p.n_insn) << ", kIn = " << int(p.n_in)
    << ", kOut = " << int(p.n_out) << ";\n  ASKB_HD static constexpr askb::Insn insn(int i) {\n"
    << "    constexpr askb::Insn p[kInsn] = {\n";
  for (int i = 0; i < p.n_insn; ++i) o << "        " << insn_text(p.insn[i]) << (i + 1 < p.n_insn ? ",\n" : "};\n");
  o << "    return p[i];\n  }\n";
  auto table = [&](const char* fn, const uint8_t* v, int n) {
    o << "  ASKB_HD static constexpr int " << fn << "(int k) {\n    constexpr int t[] = " << list_text(v, n)
      << ";\n    return t[k];\n  }\n";
  };
  table("in_type", p.in_type, p.n_in);
  table("in_map", p.in_map, p.n_in);
  table("out_type", p.out_type, p.n_out);
  table("out_reg", p.out_reg, p.n_out);
  o << "};\n";
  return o.str();
}

std::string program_constant(const Program& p) {
  std::ostringstream o;
  o << "__constant__ askb::Program kProgram = {" << int(p.n_insn) << ", " << int(p.n_in) << ", " << int(p.n_out) << ", "
    << int(p.n_regs) << ",\n    " << list_text(p.in_type, kMaxIn) << ",\n    " << list_text(p.in_map, kMaxIn) << ",\n    "
    << list_text(p.out_type, kMaxOut) << ",\n    " << list_text(p.out_reg, kMaxOut) << ",\n    {";
  for (int i = 0; i < kMaxInsn; ++i) o << (i ? ",\n     " : "") << insn_text(p.insn[i]);
  o << "}};\n";
  return o.str();
}

std::string views_constant(const ViewSet& vs) {
  std::ostringstream o;
  auto arr = [&](const int64_t* v) {
    o << "{";
    for (int d = 0; d < kMaxRank; ++d) o << (d ? ", " : "") << i64(v[d]);
    o << "}";
  };
  o << "__constant__ askb::ViewSet kViews = {" << vs.rank << ", {";
  for (int d = 0; d < kMaxRank; ++d) o << (d ? ", " : "") << vs.shape[d] << "ull";
  o << "},\n    {";
  for (int k = 0; k < kMaxIn; ++k) {
    const PortView& v = vs.port[k];
    o << (k ? ",\n     " : "") << "{";
    arr(v.lo);
    o << ", ";
    arr(v.step);
    o << ", ";
    arr(v.extent);
    o << ", ";
    arr(v.stride);
    o << ", " << i64(v.offset) << ", " << u64(v.pad) << ", " << i64(v.inner_rank) << ", ";
    arr(v.inner_shape);
    o << ", ";
    arr(v.ilo);
    o << ", ";
    arr(v.istep);
    o << ", ";
    arr(v.iextent);
    o << ", ";
    arr(v.istride);
    o << ", " << i64(v.ioffset) << ", " << u64(v.ipad) << "}";
  }
  o << "}};\n";
  return o.str();
}

std::string reductions_struct(const RedArgs& a) {
  std::ostringstream o;
  o << "struct Reductions {\n  static constexpr int N = " << int(a.n_red) << ";\n";
  auto table = [&](const char* fn, const uint8_t* v) {
    o << "  ASKB_HD static constexpr int " << fn << "(int k) {\n    constexpr int t[] = " << list_text(v, a.n_red)
      << ";\n    return t[k];\n  }\n";
  };
  table("op", a.red_op);
  table("src", a.red_src);
  table("type", a.red_type);
  o << "};\n";
  return o.str();
}

// The library's specialised reductions as artifact template arguments: value
// source, reduction set and 16-byte loads in flight (reduce_kernels.cu's
// with_spec table).
struct FastReduction {
  int spec;
  const char* source;
  const char* set;
  int unroll;
};
constexpr FastReduction kFastReductions[] = {
    {RED_ROWSTATS_F32, "askb::red::SrcF32", "askb::red::RedSet<askb::RED_SUM, askb::RED_MAX, askb::RED_MIN, askb::RED_ARGMAX>", 8},
    {RED_GLOBAL_F32, "askb::red::SrcF32", "askb::red::RedSet<askb::RED_SUM, askb::RED_MIN, askb::RED_ARGMIN>", 8},
    {RED_SOFTMAX_MAX_F16, "askb::red::SrcCast<askb::kF16>", "askb::red::RedSet<askb::RED_MAX>", 4},
    {RED_SOFTMAX_MAX_BF16, "askb::red::SrcCast<askb::kBF16>", "askb::red::RedSet<askb::RED_MAX>", 4},
    {RED_SOFTMAX_SUM_F16, "askb::red::SrcExpShift<askb::kF16>", "askb::red::RedSet<askb::RED_SUM>", 4},
    {RED_SOFTMAX_SUM_BF16, "askb::red::SrcExpShift<askb::kBF16>", "askb::red::RedSet<askb::RED_SUM>", 4},
};

struct Generated {
  std::string source, body;
  std::vector<unsigned> widths;
};

Generated generate(const ask_b200_plan& pl, const std::string& entry, const uint64_t grid[3],
                   const std::vector<Param>& ps) {
  Generated g;
  std::ostringstream src, sig, body;
  const size_t ni = pl.inputs.size(), no = pl.outputs.size();
  for (size_t i = 0; i < ps.size(); ++i) {
    if (i) sig << ", ";
    if (ps[i].port) {
      sig << (ps[i].output ? "void* __restrict__ p" : "const void* __restrict__ p") << i;
      g.widths.push_back(0);
    } else {
      sig << ps[i].scalar->ctype << " p" << i;
      g.widths.push_back(ps[i].scalar->width);
    }
  }
  auto ins = [&](size_t k) { return port_expr(ps, false, k); };
  auto outs = [&](size_t k) { return port_expr(ps, true, k); };
  auto pointer_arrays = [&]() {
    body << "  const void* const in[] = {";
    for (size_t k = 0; k < ni; ++k) body << (k ? ", " : "") << ins(k);
    body << "};\n  void* const out[] = {";
    for (size_t k = 0; k < no; ++k) body << (k ? ", " : "") << outs(k);
    body << "};\n";
  };
  std::string decls;
  switch (pl.family) {
    case FAM_ELEMENTWISE: {
      bool ssa = pl.ssa.n_in > 0;
      for (int i = 0; i < pl.ssa.n_insn; ++i) ssa = ssa && pl.ssa.insn[i].dst == i;
      body << "  askb::EwArgs args;\n";
      for (size_t k = 0; k < ni; ++k) body << "  args.in[" << k << "] = " << ins(k) << ";\n";
      for (size_t k = 0; k < no; ++k) body << "  args.out[" << k << "] = " << outs(k) << ";\n";
      const U32Div d = make_u32div(pl.inner ? pl.inner : 1, pl.count);
      body << "  args.count = " << u64(pl.count) << ";\n  args.inner = askb::U32Div{" << u64(d.d) << ", " << d.m << "u, "
           << d.s1 << "u, " << d.s2 << "u, " << d.wide << "u};\n";
      if (pl.views || !ssa) {
        decls = program_constant(pl.ssa) + views_constant(pl.vs);
        body << "  askb::ew::ew_view_loop(kProgram, args, kViews);\n";
        g.body = "elementwise_view";
      } else {
        decls = program_struct(pl.ssa, "Program");
        body << "  const bool aligned = true";
        for (size_t k = 0; k < ni; ++k)
          if (pl.inputs[k].map == IM_FULL || pl.inputs[k].map == IM_INNER) body << " && askb::art::aligned16(" << ins(k) << ")";
        for (size_t k = 0; k < no; ++k) body << " && askb::art::aligned16(" << outs(k) << ")";
        body << ";\n";
        // The library's hand-written loops for its specialised programs
        // (ew_kernels.cu: ew_launch), when every unit is whole and aligned.
        const char* functor = pl.spec == EW_CFG1 ? "askb::ew::FnCfg1"
                              : pl.spec == EW_CFG5B ? "askb::ew::FnCfg5b"
                              : pl.spec == EW_SOFTMAX_NORM_F16 ? "askb::ew::FnSoftmaxNorm<askb::kF16>"
                              : pl.spec == EW_SOFTMAX_NORM_BF16 ? "askb::ew::FnSoftmaxNorm<askb::kBF16>" : nullptr;
        if (functor) {
          // the cfg5b functor moves 32-byte units
          std::string wide;
          if (pl.spec == EW_CFG5B) {
            for (size_t k = 0; k < ni; ++k) wide += " && askb::art::aligned32(" + ins(k) + ")";
            for (size_t k = 0; k < no; ++k) wide += " && askb::art::aligned32(" + outs(k) + ")";
          }
          body << "  using F = " << functor << ";\n  if (aligned" << wide << " && " << u64(pl.count)
               << " % F::V == 0 && (!F::kRowMapped || " << u64(d.d) << " % F::V == 0))\n    askb::ew::ew_functor_loop<F>(args, "
               << u64(pl.count) << " / F::V);\n  else\n  ";
        }
        body << "  askb::ew::ew_spec_loop<Program, 4, 2>(args, aligned ? 1 : 0);\n";
        g.body = functor ? "elementwise_functor" : "elementwise";
      }
      break;
    }
    case FAM_REDUCE: {
      const RedArgs& a = pl.red;
      if (pl.ssa.n_in == 0) fail(ASK_B200_E_UNSUPPORTED, "an artifact reduction reads at least one input port");
      if (pl.views) fail(ASK_B200_E_UNSUPPORTED, "an artifact reduction reads full, outer or scalar ports, not views");
      decls = program_struct(pl.ssa, "Program") + reductions_struct(a);
      pointer_arrays();
      const uint64_t warps = grid[0] * 256 / 32;
      const FastReduction* fast = nullptr;
      for (const FastReduction& f : kFastReductions)
        if (a.inner == 1 && pl.spec == f.spec) fast = &f;
      if (a.inner != 1) {
        body << "  askb::art::reduce_columns<Program, Reductions, " << u64(a.outer) << ", " << u64(a.extent) << ", "
             << u64(a.inner) << ", " << u64(a.index_base) << ">(in, out);\n";
        g.body = "reduce_columns";
      } else {
        body << "  const bool aligned = true";
        for (size_t k = 0; k < ni; ++k)
          if (pl.inputs[k].map == IM_FULL) {
            body << " && askb::art::aligned16(" << ins(k) << ")";
            if ((a.extent * uint64_t(dtype_bytes(pl.inputs[k].dtype))) % 16) body << " && false";
          }
        body << ";\n";
        const bool cta = a.outer * 2 <= warps && a.extent >= 1024;
        if (fast) {
          body << "  askb::RedArgs a;\n";
          for (size_t k = 0; k < ni; ++k) body << "  a.in[" << k << "] = " << ins(k) << ";\n";
          for (size_t k = 0; k < no; ++k) body << "  a.out[" << k << "] = " << outs(k) << ";\n";
          body << "  a.outer = " << u64(a.outer) << ";\n  a.extent = " << u64(a.extent) << ";\n  a.inner = 1;\n"
               << "  a.index_base = " << u64(a.index_base) << ";\n  a.n_red = " << int(a.n_red) << ";\n";
          const std::string targs = std::string("<") + fast->source + ", " + fast->set + ", " + std::to_string(fast->unroll) + ">";
          body << (cta ? "  askb::art::reduce_rows_cta_fast" : "  askb::red::red_warp_row_loop") << targs
               << "(a, aligned ? 1 : 0);\n";
          g.body = cta ? "reduce_rows_cta_fast" : "reduce_rows_warp_fast";
        } else {
          body << "  askb::art::" << (cta ? "reduce_rows_cta" : "reduce_rows_warp") << "<Program, Reductions, "
               << u64(a.outer) << ", " << u64(a.extent) << ", " << u64(a.index_base) << ">(in, out, aligned);\n";
          g.body = cta ? "reduce_rows_cta" : "reduce_rows_warp";
        }
      }
      break;
    }
    case FAM_GATHER: {
      const IndexArgs& a = pl.idx;
      const uint64_t es = uint64_t(dtype_bytes(a.elem_type)), row_bytes = a.inner * es;
      const std::string sizes = u64(a.outer) + ", " + u64(a.dim) + ", " + u64(a.n);
      const std::string elems = "askb::art::gather_elems<" + std::to_string(es) + ", " + std::to_string(a.index_type) +
                                ", " + sizes + ", " + u64(a.inner) + ">(" + ins(0) + ", " + ins(1) + ", " + outs(0) + ");\n";
      if (row_bytes % 16 == 0 && row_bytes) {
        body << "  if (askb::art::aligned16(" << ins(0) << ") && askb::art::aligned16(" << outs(0) << "))\n"
             << "    askb::art::gather_rows<" << a.index_type << ", " << sizes << ", " << u64(row_bytes) << ">(" << ins(0)
             << ", " << ins(1) << ", " << outs(0) << ");\n  else\n    " << elems;
        g.body = "gather_rows";
      } else {
        body << "  " << elems;
        g.body = "gather_elems";
      }
      break;
    }
    case FAM_SCATTER:
      fail(ASK_B200_E_UNSUPPORTED,
           "scatter_add reads its base through the Runtime's pre_copy, which an external artifact cannot declare; "
           "run it as a recipe step");
    default:
      fail(ASK_B200_E_UNSUPPORTED, "the fused softmax is a runtime fusion; package its three steps instead");
  }
  src << "// ask_b200 kernel artifact (" << g.body << "), generated from a recipe step.\n"
      << "#include \"artifact_bodies.cuh\"\n\nnamespace {\n" << decls << "}  // namespace\n\n"
      << "extern \"C\" __global__ void __launch_bounds__(askb::art::kThreads"
      << (g.body != "elementwise_functor" ? ""
          : pl.family == FAM_ELEMENTWISE && pl.spec == EW_CFG1 ? ", askb::art::kDeepFunctorMinBlocks"
                                                                : ", askb::art::kFunctorMinBlocks")
      << ") " << entry << "(" << sig.str()
      << ") {\n"
      << body.str() << "}\n";
  g.source = src.str();
  return g;
}

std::string json_string(const std::string& s) {
  std::string o = "\"";
  for (char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\t': o += "\\t"; break;
      default:
        if (static_cast<unsigned char>(c) < 0x20) {
          char b[8];
          std::snprintf(b, sizeof b, "\\u%04x", c);
          o += b;
        } else {
          o += c;
        }
    }
  }
  return o + "\"";
}

std::string artifact_source(const char* recipe_json, const char* options_json) {
  if (!recipe_json || !options_json) fail(ASK_B200_E_INVALID, "recipe and options must not be NULL");
  const json::Value opt = json::Parser(options_json).parse();
  const std::string entry = opt.at("entry").as_str("entry");
  if (!valid_entry(entry)) fail(ASK_B200_E_INVALID, "entry must match [A-Za-z_][A-Za-z0-9_]*");
  const auto& gv = opt.at("grid").as_array("grid");
  if (gv.size() != 3) fail(ASK_B200_E_INVALID, "grid must have three entries");
  uint64_t grid[3];
  for (int d = 0; d < 3; ++d) {
    const int64_t x = gv[size_t(d)].as_int("grid");
    if (x < 1 || x > 0xffffffffll) fail(ASK_B200_E_INVALID, "grid entries must be in [1, 2^32-1]");
    grid[d] = uint64_t(x);
  }
  if (grid[1] != 1 || grid[2] != 1) fail(ASK_B200_E_UNSUPPORTED, "artifact kernels stride over a one-dimensional grid");
  if (grid[0] > 0x7fffffffull) fail(ASK_B200_E_INVALID, "grid x exceeds the device limit 2^31-1");

  ask_b200_plan* raw = nullptr;
  const int rc = ask_b200_plan_create(recipe_json, -1, &raw);
  if (rc != ASK_B200_OK) fail(rc, std::string("recipe: ") + ask_b200_last_error());
  struct Holder {
    ask_b200_plan* p;
    ~Holder() { ask_b200_plan_destroy(p); }
  } holder{raw};
  const ask_b200_plan& pl = *raw;
  const std::vector<Param> ps = parse_parameters(opt.at("parameters"), pl.inputs.size(), pl.outputs.size());
  const Generated g = generate(pl, entry, grid, ps);

  std::ostringstream o;
  o << "{\"entry\":" << json_string(entry) << ",\"body\":\"" << g.body << "\",\"launch\":{\"grid\":[" << grid[0] << ","
    << grid[1] << "," << grid[2] << "],\"block\":[256,1,1],\"shared_bytes\":0},\"parameter_widths\":[";
  for (size_t i = 0; i < g.widths.size(); ++i) o << (i ? "," : "") << g.widths[i];
  // Element types the Runtime must check (lib/Lowering/CUDA.cpp:392-394 order).
  bool used[kNumDTypes] = {};
  for (const PortInfo& p : pl.inputs) used[p.dtype] = true;
  for (const PortInfo& p : pl.outputs) used[p.dtype] = true;
  o << "],\"required_element_types\":[";
  bool first = true;
  for (int t : {kBool, kI32, kI64, kF32, kF16, kBF16})
    if (used[t]) {
      o << (first ? "" : ",") << "\"" << kTypeNames[t] << "\"";
      first = false;
    }
  o << "],\"port_map\":[";
  auto port = [&](const PortInfo& p, const char* kind, size_t k, bool comma) {
    o << (comma ? "," : "") << "{\"logical_port\":\"" << kind << ":" << k << "\",\"element_type\":\"" << kTypeNames[p.dtype]
      << "\",\"elements\":" << p.elements << "}";
  };
  for (size_t k = 0; k < pl.inputs.size(); ++k) port(pl.inputs[k], "input", k, k > 0);
  for (size_t k = 0; k < pl.outputs.size(); ++k) port(pl.outputs[k], "output", k, k + pl.inputs.size() > 0);
  o << "],\"source\":" << json_string(g.source) << "}";
  return o.str();
}

void write_text(const std::string& s, char* buf, size_t cap, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (buf && cap) {
    const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
}

}  // namespace

extern "C" {

ASK_B200_API int ask_b200_artifact_source(const char* recipe_json, const char* options_json, char* buf, size_t cap,
                                          size_t* needed) {
  try {
    write_text(artifact_source(recipe_json, options_json), buf, cap, needed);
    askb_internal_set_error("");
    return ASK_B200_OK;
  } catch (const Failure& f) {
    askb_internal_set_error(f.message.c_str());
    return f.code;
  } catch (const std::exception& e) {
    askb_internal_set_error(e.what());
    return ASK_B200_E_INVALID;
  }
}

}  // extern "C"
