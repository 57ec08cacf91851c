// Lowering adapter: ASK step sources (MLIR text) -> ask_b200 recipes.
//
// The reference compiles each owned step of a partitioned graph with
// ask::lowerToCUDALLVM (lib/Lowering/CUDA.cpp:152-419).  Its partitioner
// records, for every step, the step's own module as printed MLIR
// ("step_sources", lib/Frontend/Partition.cpp:267-273) and the execution plan
// that binds steps to buffers (Partition.cpp:150-281).  This file reads that
// text for the subset of ASK ops this library runs and emits the equivalent
// recipe, so an existing partition report becomes a runtime program without
// the LLVM/MLIR toolchain:
//
//   - a step whose returned values are all ask.reduce_* / ask.argmax /
//     ask.argmin results over one shared block of contiguous axes becomes a
//     "reduce" recipe; the reduced operands (elementwise expressions of the
//     step's arguments) become its op program;
//   - a step returning one ask.gather or ask.scatter_add of its arguments
//     becomes a "gather" / "scatter_add" recipe;
//   - any other step of elementwise ops becomes an "elementwise" recipe.
// Arguments enter the op program with an index map: the full output shape,
// a scalar, a prefix of the output axes ("outer": broadcast_in_dim with
// dimensions 0..k-1), a suffix ("inner"), or -- for transpose, slice, pad,
// general broadcasts and reshapes of an argument -- a strided, windowed view
// (IM_VIEW; pad's elements outside the window read its constant pad value).
// concatenate becomes views of its operands selected by the coordinate along
// its axis, iota a cast of that coordinate -- in elementwise steps and in the
// prologues of reductions alike (a reduction's iteration shape is its
// operand's shape).  ask.constant/ask.splat become
// constants (MLIR prints each float literal so that it re-parses exactly, or
// as its bit pattern in hex; either is carried over without double rounding).
// An index map of a computed elementwise value moves onto that value's
// operands (push_index_maps); pad and concatenate of computed values become
// selects, by the coordinates, between window maps of their operands.
// matmul and external steps are reported as unsupported.
#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <map>
#include <numeric>
#include <memory>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "ask_b200.h"
#include "ask_b200_lower.h"
#include "json.h"

// plan.cpp: the cuda_lowering report of a recipe (its host-only plan's).
std::string askb_recipe_lowering_report(const std::string& recipe_json, long pre_copy_input);

extern "C" void askb_internal_set_error(const char* message);

namespace askb {
namespace lower {

namespace {

struct Failure {
  int code;
  std::string message;
};
[[noreturn]] void fail(int code, const std::string& m) { throw Failure{code, m}; }
[[noreturn]] void unsupported(const std::string& m) { fail(ASK_B200_E_UNSUPPORTED, m); }
[[noreturn]] void invalid(const std::string& m) { fail(ASK_B200_E_INVALID, m); }

// ---- MLIR text subset ---------------------------------------------------------------
struct Type {
  std::string dtype;            // bool, i32, i64, f32, f16, bf16
  std::vector<int64_t> shape;   // empty for a 0-D tensor or a scalar
  bool tensor = false;
  uint64_t numel() const {
    uint64_t n = 1;
    for (int64_t d : shape) n *= uint64_t(d);
    return n;
  }
};

struct Attr {
  enum Kind { None, Str, Int, Float, Bool, IntArray, Other } kind = None;
  std::string text;  // string contents, or the literal of a number
  int64_t i = 0;
  bool b = false;
  std::string type;  // numeric literal's type suffix
  std::vector<int64_t> arr;
};

struct Op {
  std::string result;  // "" for return
  std::string name;
  std::vector<std::string> operands;
  std::map<std::string, Attr> attrs;
  Type type;           // result type
};

struct Func {
  std::vector<std::string> args;
  std::vector<Type> arg_types;
  std::vector<Op> ops;
  std::vector<std::string> returns;
};

class Reader {
 public:
  explicit Reader(const std::string& s) : s_(s) {}

  Func read_function() {
    const size_t at = s_.find("func.func");
    if (at == std::string::npos) invalid("step source has no func.func");
    p_ = at + std::strlen("func.func");
    ws();
    symbol();
    expect('(');
    Func f;
    ws();
    if (!peek(')')) {
      for (;;) {
        f.args.push_back(value_name());
        expect(':');
        f.arg_types.push_back(type());
        ws();
        if (peek('{')) attr_dict();
        ws();
        if (peek(',')) { ++p_; continue; }
        break;
      }
    }
    expect(')');
    ws();
    if (starts("->")) {
      p_ += 2;
      ws();
      if (peek('(')) {
        ++p_;
        for (;;) {
          type();
          ws();
          if (peek('{')) attr_dict();
          ws();
          if (peek(',')) { ++p_; continue; }
          break;
        }
        expect(')');
      } else {
        type();
      }
    }
    ws();
    if (starts("attributes")) {
      p_ += std::strlen("attributes");
      ws();
      attr_dict();
    }
    expect('{');
    for (;;) {
      ws();
      if (peek('}')) break;
      if (starts("return") || starts("func.return")) {
        p_ += starts("return") ? 6 : 11;
        ws();
        while (peek('%')) {
          f.returns.push_back(value_name());
          ws();
          if (peek(',')) { ++p_; ws(); }
        }
        skip_line();
        continue;
      }
      f.ops.push_back(operation());
    }
    return f;
  }

 private:
  const std::string& s_;
  size_t p_ = 0;

  [[noreturn]] void error(const std::string& what) const {
    const size_t line_start = s_.rfind('\n', p_ ? p_ - 1 : 0);
    const size_t b = line_start == std::string::npos ? 0 : line_start + 1;
    const size_t e = s_.find('\n', p_);
    invalid("step source: " + what + " near '" + s_.substr(b, (e == std::string::npos ? s_.size() : e) - b) + "'");
  }
  void ws() {
    for (;;) {
      while (p_ < s_.size() && std::isspace(static_cast<unsigned char>(s_[p_]))) ++p_;
      if (starts("//")) { skip_line(); continue; }
      break;
    }
  }
  void skip_line() {
    while (p_ < s_.size() && s_[p_] != '\n') ++p_;
  }
  bool peek(char c) const { return p_ < s_.size() && s_[p_] == c; }
  bool starts(const char* t) const { return s_.compare(p_, std::strlen(t), t) == 0; }
  void expect(char c) {
    ws();
    if (!peek(c)) error(std::string("expected '") + c + "'");
    ++p_;
  }
  std::string ident_chars() {
    const size_t b = p_;
    while (p_ < s_.size() && (std::isalnum(static_cast<unsigned char>(s_[p_])) || s_[p_] == '_' || s_[p_] == '.' ||
                              s_[p_] == '$' || s_[p_] == '-'))
      ++p_;
    return s_.substr(b, p_ - b);
  }
  std::string value_name() {
    ws();
    if (!peek('%')) error("expected an SSA value");
    ++p_;
    std::string n = "%" + ident_chars();
    if (peek('#')) {  // %res#0
      ++p_;
      n += "#" + ident_chars();
    }
    return n;
  }
  std::string symbol() {
    ws();
    if (!peek('@')) error("expected a symbol");
    ++p_;
    if (peek('"')) return string_literal();
    return ident_chars();
  }
  std::string string_literal() {
    if (!peek('"')) error("expected a string");
    ++p_;
    std::string out;
    while (p_ < s_.size() && s_[p_] != '"') {
      if (s_[p_] == '\\' && p_ + 1 < s_.size()) {
        const char n = s_[p_ + 1];
        if (std::isxdigit(static_cast<unsigned char>(n)) && p_ + 2 < s_.size()) {
          out += char(std::stoi(s_.substr(p_ + 1, 2), nullptr, 16));
          p_ += 3;
          continue;
        }
        out += n == 'n' ? '\n' : n == 't' ? '\t' : n;
        p_ += 2;
        continue;
      }
      out += s_[p_++];
    }
    if (!peek('"')) error("unterminated string");
    ++p_;
    return out;
  }
  static std::string element_type(const std::string& t) {
    if (t == "i1") return "bool";
    if (t == "i32" || t == "i64" || t == "f32" || t == "f16" || t == "bf16") return t;
    return "";
  }
  Type type() {
    ws();
    Type t;
    if (starts("tensor<")) {
      p_ += 7;
      t.tensor = true;
      for (;;) {
        ws();
        if (peek('?')) error("dynamic tensor shapes are not supported; the step must be specialised");
        if (std::isdigit(static_cast<unsigned char>(s_[p_]))) {
          size_t e = p_;
          while (e < s_.size() && std::isdigit(static_cast<unsigned char>(s_[e]))) ++e;
          t.shape.push_back(std::stoll(s_.substr(p_, e - p_)));
          p_ = e;
          if (!peek('x')) error("malformed tensor type");
          ++p_;
          continue;
        }
        break;
      }
      t.dtype = element_type(ident_chars());
      if (t.dtype.empty()) error("unsupported element type");
      expect('>');
      return t;
    }
    t.dtype = element_type(ident_chars());
    if (t.dtype.empty()) error("unsupported type");
    return t;
  }
  // Skip a balanced (), [], {}, <> group or a string.
  void skip_group() {
    const char open = s_[p_];
    const char close = open == '(' ? ')' : open == '[' ? ']' : open == '{' ? '}' : '>';
    int depth = 0;
    while (p_ < s_.size()) {
      if (s_[p_] == '"') { string_literal(); continue; }
      if (s_[p_] == open) ++depth;
      if (s_[p_] == close && --depth == 0) { ++p_; return; }
      ++p_;
    }
    error("unbalanced brackets");
  }
  Attr attr_value() {
    ws();
    Attr a;
    if (peek('"')) {
      a.kind = Attr::Str;
      a.text = string_literal();
      return a;
    }
    if (starts("true") || starts("false")) {
      a.kind = Attr::Bool;
      a.b = starts("true");
      p_ += a.b ? 4 : 5;
      return a;
    }
    if (starts("array<")) {
      p_ += 6;
      ident_chars();  // element type
      ws();
      a.kind = Attr::IntArray;
      if (peek(':')) {
        ++p_;
        for (;;) {
          ws();
          size_t e = p_;
          if (e < s_.size() && s_[e] == '-') ++e;
          while (e < s_.size() && std::isdigit(static_cast<unsigned char>(s_[e]))) ++e;
          if (e == p_) break;
          a.arr.push_back(std::stoll(s_.substr(p_, e - p_)));
          p_ = e;
          ws();
          if (peek(',')) { ++p_; continue; }
          break;
        }
      }
      expect('>');
      return a;
    }
    if (peek('-') || std::isdigit(static_cast<unsigned char>(s_[p_]))) {
      const size_t b = p_;
      if (peek('-')) ++p_;
      while (p_ < s_.size() && (std::isalnum(static_cast<unsigned char>(s_[p_])) || s_[p_] == '.' || s_[p_] == '+' ||
                                ((s_[p_] == '-') && (s_[p_ - 1] == 'e' || s_[p_ - 1] == 'E'))))
        ++p_;
      a.text = s_.substr(b, p_ - b);
      ws();
      if (peek(':')) {
        ++p_;
        ws();
        a.type = ident_chars();
      }
      const bool hex = a.text.find("0x") != std::string::npos || a.text.find("0X") != std::string::npos;
      const bool is_float = a.type == "f32" || a.type == "f16" || a.type == "bf16" || a.type == "f64" ||
                            (!hex && a.text.find_first_of(".eE") != std::string::npos);
      if (is_float) {
        a.kind = Attr::Float;
      } else {
        a.kind = Attr::Int;
        a.i = std::stoll(a.text, nullptr, 0);
      }
      return a;
    }
    a.kind = Attr::Other;
    if (peek('(') || peek('[') || peek('{') || peek('<')) {
      skip_group();
      return a;
    }
    // #dialect<...>, @symbol, unit-like keywords, types
    while (p_ < s_.size() && !peek(',') && !peek('}')) {
      if (peek('<') || peek('(') || peek('[') || peek('{')) skip_group();
      else if (peek('"')) string_literal();
      else ++p_;
    }
    return a;
  }
  std::map<std::string, Attr> attr_dict() {
    std::map<std::string, Attr> out;
    expect('{');
    ws();
    if (peek('}')) { ++p_; return out; }
    for (;;) {
      ws();
      std::string key = peek('"') ? string_literal() : ident_chars();
      if (key.empty()) error("expected an attribute name");
      ws();
      if (peek('=')) {
        ++p_;
        out[key] = attr_value();
      } else {
        out[key] = Attr{};  // unit attribute
      }
      ws();
      if (peek(',')) { ++p_; continue; }
      break;
    }
    expect('}');
    return out;
  }
  Op operation() {
    Op op;
    op.result = value_name();
    ws();
    if (peek(':')) error("multi-result operations are not supported");
    expect('=');
    ws();
    op.name = string_literal();
    expect('(');
    ws();
    while (!peek(')')) {
      op.operands.push_back(value_name());
      ws();
      if (peek(',')) ++p_;
      ws();
    }
    ++p_;
    ws();
    if (starts("<{")) { ++p_; op.attrs = attr_dict(); expect('>'); ws(); }  // properties
    if (peek('{')) {
      auto more = attr_dict();
      op.attrs.insert(more.begin(), more.end());
    }
    expect(':');
    ws();
    expect('(');
    ws();
    while (!peek(')')) {
      type();
      ws();
      if (peek(',')) ++p_;
      ws();
    }
    ++p_;
    ws();
    if (!starts("->")) error("expected '->'");
    p_ += 2;
    op.type = type();
    return op;
  }
};

// ---- lowering ----------------------------------------------------------------------
std::string json_str(const std::string& s) {
  std::string o = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\') { o += '\\'; o += c; }
    else if (static_cast<unsigned char>(c) < 0x20) {
      char b[8];
      std::snprintf(b, sizeof b, "\\u%04x", c);
      o += b;
    } else {
      o += c;
    }
  }
  return o + "\"";
}

uint64_t product(const std::vector<int64_t>& v, size_t b, size_t e) {
  uint64_t n = 1;
  for (size_t i = b; i < e; ++i) n *= uint64_t(v[i]);
  return n;
}

const std::set<std::string> kUnary = {"exp", "log", "sqrt", "sin", "cos", "tanh", "erf", "abs",
                                      "floor", "ceil", "round", "bitwise_not"};
const std::set<std::string> kBinary = {"add", "mul", "div", "floordiv", "mod", "pow", "maximum", "minimum",
                                       "bitwise_and", "bitwise_or", "bitwise_xor", "shift_left", "shift_right"};

std::string strip(const std::string& n) { return n.rfind("ask.", 0) == 0 ? n.substr(4) : n; }

// Synthetic ops the lowering adds while moving index maps onto operands: a
// window map reads its operand at (c - lo) / step per axis (a pad's window
// without the pad value), a window mask is true where that coordinate is
// valid (non-negative, divisible, below the operand's extent).
constexpr const char* kWindow = "ask_b200_window";
constexpr const char* kWindowMask = "ask_b200_window_mask";

struct Lowered {
  std::string recipe;
  std::vector<size_t> input_args;  // recipe input k reads function argument input_args[k]
};

// A value that is only an index map of a step argument: for each axis of the
// value's shape the argument coordinate (c - lo) / step (valid while
// non-negative, divisible and below extent) and its element stride, plus a
// base offset and the value outside the window (ScalarEmitter.h:626-730).
struct ArgView {
  size_t arg = 0;
  std::vector<int64_t> lo, step, extent, stride;
  int64_t offset = 0;
  std::string pad = "0";  // JSON constant for elements outside the window
  std::vector<int64_t> shape;  // the viewed value's shape (its coordinate ranges)
  // A reshape that no strided window expresses: the window above yields a
  // row-major position in a value of shape inner->shape (the reshape's
  // operand), whose coordinates are read through *inner.
  std::shared_ptr<const ArgView> inner;
  // Whether axis d reads pad at some coordinate: an offset or strided window,
  // or one that ends before the axis does (a high pad).
  bool windowed(size_t d) const { return lo[d] != 0 || step[d] != 1 || extent[d] < shape[d]; }
};

class Lowering {
 public:
  explicit Lowering(const Func& f) : f_(f) {
    for (size_t k = 0; k < f.args.size(); ++k) arg_[f.args[k]] = k;
    for (size_t k = 0; k < f.ops.size(); ++k) def_[f.ops[k].result] = k;
    erase_marks();
    gather_reduced_axes();
    push_index_maps();
  }

  Lowered run() {
    if (f_.returns.empty()) invalid("step returns nothing");
    for (const Op& op : f_.ops) {
      const std::string n = strip(op.name);
      if (n == "matmul") unsupported("matmul steps run on the library (cuBLASLt) path, not on recipes");
      if (n == "external") unsupported("external steps run their own artifact, not a recipe");
    }
    const Op* first = producer(f_.returns[0]);
    const std::string fam = first ? strip(first->name) : "";
    if (fam == "gather" || fam == "scatter_add") return indexed(*first, fam == "scatter_add");
    bool reduce = false;
    for (const std::string& r : f_.returns) {
      const Op* p = producer(r);
      if (p && is_reduction(strip(p->name))) reduce = true;
    }
    return reduce ? reduction() : elementwise();
  }

 private:
  struct Port {
    size_t arg;
    std::string map;   // full, scalar, outer, inner, view
    std::string view;  // the view's JSON for map == view
    ArgView w;         // and the view itself
  };
  Func f_;  // the step, with index maps of computed values moved onto their operands
  std::map<std::string, size_t> arg_, def_;
  // op program under construction; insn_port_[i] >= 0 marks an input instruction
  std::vector<std::string> insns_;
  std::vector<int> insn_port_;
  std::map<std::string, int> shared_;  // emit_shared: instruction text -> its id
  std::vector<std::string> types_;
  std::map<std::string, int> memo_;
  std::vector<Port> ports_;
  std::vector<int> port_insn_;
  std::vector<int64_t> out_shape_;
  size_t lead_ = 0;            // reduce: number of leading (outer) axes
  bool uses_coord_ = false;    // the program reads iteration coordinates
  uint64_t map_inner_ = 0;     // elementwise: the 'inner' every outer/inner map shares
  bool is_reduce_ = false;
  bool uses_shape_ = false;    // a view or a coordinate needs the iteration shape

  static bool is_reduction(const std::string& n) { return n.rfind("reduce_", 0) == 0 || n == "argmax" || n == "argmin"; }

  // ask.mark is a tracing pass-through (a value's identity or port binding)
  // that the reference's prepare phase extracts and erases, connecting the
  // marked value directly to its users (docs/en/ir.md:42, 125-131); a step
  // source that still carries one lowers as if it had been erased.
  void erase_marks() {
    for (Op& op : f_.ops) {
      if (strip(op.name) != "mark" || op.operands.size() != 1) continue;
      const std::string from = op.result, to = op.operands[0];
      for (Op& o : f_.ops)
        for (std::string& x : o.operands)
          if (x == from) x = to;
      for (std::string& r : f_.returns)
        if (r == from) r = to;
      op.name = "ask.ask_b200_moved";
    }
  }

  // A reduction over axes that are not one contiguous block (say axes 0 and 2
  // of a rank-3 value) reads its operand through a transpose that puts the
  // kept axes first, in their order, and the reduced axes last, in theirs;
  // its axes become that trailing block.  The outputs keep their row-major
  // order over the kept axes, and the fold runs over the reduced index space
  // in the same row-major order.  The transpose then moves onto the operand's
  // arguments like any index map.
  void gather_reduced_axes() {
    const size_t original = f_.ops.size();
    size_t fresh = 0;
    for (size_t i = 0; i < original; ++i) {
      const std::string n = strip(f_.ops[i].name);
      if (n.rfind("reduce_", 0) != 0 || f_.ops[i].operands.empty()) continue;  // argmax/argmin take one axis
      auto ax = f_.ops[i].attrs.find("axes");
      if (ax == f_.ops[i].attrs.end()) continue;
      std::vector<int64_t> axes = ax->second.arr;
      std::sort(axes.begin(), axes.end());
      bool contiguous = true;
      for (size_t k = 1; k < axes.size(); ++k) contiguous = contiguous && axes[k] == axes[k - 1] + 1;
      const Type in = type_of(f_.ops[i].operands[0]);  // a copy: the ops may move
      const int64_t rank = int64_t(in.shape.size());
      if (contiguous || axes.empty() || axes.front() < 0 || axes.back() >= rank) continue;
      std::vector<int64_t> perm;
      for (int64_t d = 0; d < rank; ++d)
        if (!std::binary_search(axes.begin(), axes.end(), d)) perm.push_back(d);
      const int64_t kept = int64_t(perm.size());
      for (int64_t d : axes) perm.push_back(d);
      Op t;
      t.name = "ask.transpose";
      t.operands = {f_.ops[i].operands[0]};
      t.type = Type{in.dtype, {}, true};
      for (int64_t d : perm) t.type.shape.push_back(in.shape[size_t(d)]);
      Attr pa;
      pa.kind = Attr::IntArray;
      pa.arr = perm;
      t.attrs["permutation"] = pa;
      t.result = "%ask_b200.gathered" + std::to_string(fresh++);
      f_.ops.push_back(t);
      def_[t.result] = f_.ops.size() - 1;
      f_.ops[i].operands[0] = t.result;
      std::vector<int64_t> block;
      for (int64_t d = kept; d < rank; ++d) block.push_back(d);
      f_.ops[i].attrs["axes"].arr = block;
    }
  }

  const Op* producer(const std::string& v) const {
    auto it = def_.find(v);
    return it == def_.end() ? nullptr : &f_.ops[it->second];
  }
  const Type& type_of(const std::string& v) const {
    auto a = arg_.find(v);
    if (a != arg_.end()) return f_.arg_types[a->second];
    const Op* p = producer(v);
    if (!p) invalid("value " + v + " is not defined");
    return p->type;
  }
  // One axis of a window (valid coordinates c: c - lo >= 0, divisible by step,
  // (c - lo) / step < extent) read through a slice (start s, step k): the
  // output coordinate c' reads c = s + k c', valid when k c' = lo - s (mod
  // step); those c' form the progression cf, cf + step / g, ... (g =
  // gcd(k, step)) whose window index starts at qf and advances by k / g.
  struct SlicedWindow {
    int64_t lo, step, extent, qf, advance;
  };
  static SlicedWindow slice_window(int64_t lo, int64_t step, int64_t extent, int64_t start, int64_t k) {
    const int64_t diff = lo - start, g = std::gcd(k, step);
    if (((diff % g) + g) % g != 0) return {0, 1, 0, 0, 1};  // no coordinate lands on the window
    int64_t cf = diff > 0 ? (diff + k - 1) / k : 0;
    while (((k * cf - diff) % step + step) % step != 0) ++cf;  // at most step / g - 1 steps
    const int64_t qf = (start - lo + k * cf) / step, advance = k / g;
    const int64_t ext = qf >= extent ? 0 : (extent - qf + advance - 1) / advance;
    return {cf, step / g, ext, qf, advance};
  }

  // An index map (transpose, broadcast_in_dim, slice, reshape) of a computed
  // elementwise value reads that value at mapped coordinates, which the
  // reference evaluates by re-evaluating the value at the mapped index
  // (ScalarEmitter.h:626-774).  Elementwise ops commute with index maps, so
  // the map moves onto the operands -- transpose(exp(x)) = exp(transpose(x)) --
  // until it reaches step arguments (views), splats or other maps (composed by
  // view_of).  pad and concatenate of computed values first become selects
  // between window maps of their operands (a pad value must not pass through
  // the computation), and the windows move down like the other maps.
  void push_index_maps() {
    static const std::set<std::string> maps = {"transpose", "broadcast_in_dim", "slice", "reshape", kWindow};
    size_t fresh = 0;
    auto add = [&](Op op) {
      op.result = "%ask_b200.moved" + std::to_string(fresh++);
      f_.ops.push_back(op);
      def_[op.result] = f_.ops.size() - 1;
      return f_.ops.back().result;
    };
    auto replace_uses = [&](const std::string& from, const std::string& to) {
      for (Op& o : f_.ops)
        for (std::string& x : o.operands)
          if (x == from) x = to;
      for (std::string& r : f_.returns)
        if (r == from) r = to;
    };
    // pad and concatenate of computed values: select between window maps of
    // the operands (pushed below like the other maps) by the coordinates.
    auto int_array = [](const std::vector<int64_t>& v) {
      Attr a;
      a.kind = Attr::IntArray;
      a.arr = v;
      return a;
    };
    auto window = [&](const std::string& x, const Type& out, const std::vector<int64_t>& lo,
                      const std::vector<int64_t>& step) {
      Op w;
      w.name = std::string("ask.") + kWindow;
      w.operands = {x};
      w.attrs["lo"] = int_array(lo);
      w.attrs["step"] = int_array(step);
      w.type = Type{type_of(x).dtype, out.shape, true};
      return add(w);
    };
    auto mask = [&](const Type& out, const std::vector<int64_t>& lo, const std::vector<int64_t>& step,
                    const std::vector<int64_t>& extent) {
      Op m;
      m.name = std::string("ask.") + kWindowMask;
      m.attrs["lo"] = int_array(lo);
      m.attrs["step"] = int_array(step);
      m.attrs["extent"] = int_array(extent);
      m.type = Type{"bool", out.shape, true};
      return add(m);
    };
    auto select = [&](const std::string& c, const std::string& x, const std::string& y, const Type& out) {
      Op sel;
      sel.name = "ask.select";
      sel.operands = {c, x, y};
      sel.type = out;
      return add(sel);
    };
    // Consumers first: a concatenate or pad that takes the select form reads
    // its operands through windows, which the operands' own decision sees.
    const size_t original = f_.ops.size();
    for (size_t i = original; i-- > 0;) {
      const Op op = f_.ops[i];
      const std::string n = strip(op.name);
      ArgView ignored;
      if (n == "pad" && op.operands.size() == 2 && !view_of(op.result, &ignored)) {
        const std::vector<int64_t> low = arr(op, "pad_low"), interior = arr(op, "interior");
        const Type in = type_of(op.operands[0]);  // a copy: add() may move the ops
        std::vector<int64_t> step(low.size());
        bool nonneg = true;
        for (size_t d = 0; d < low.size(); ++d) {
          step[d] = interior[d] + 1;
          nonneg = nonneg && low[d] >= 0 && interior[d] >= 0;
        }
        if (!nonneg) continue;  // stays unsupported
        Op sp;
        sp.name = "ask.splat";
        sp.operands = {op.operands[1]};
        sp.type = op.type;
        const std::string padv = add(sp);
        const std::string w = window(op.operands[0], op.type, low, step);
        replace_uses(op.result, select(mask(op.type, low, step, in.shape), w, padv, op.type));
        f_.ops[i].name = "ask.ask_b200_moved";
      } else if (n == "concatenate") {
        auto ax = op.attrs.find("axis");
        if (ax == op.attrs.end()) continue;
        const size_t axis = size_t(ax->second.i), rank = op.type.shape.size();
        // Argument views that are not padded along the axis keep the direct
        // form unless an index map reads the concatenation.
        bool direct = !mapped(op.result);
        for (const std::string& o : op.operands) {
          ArgView ow;
          direct = direct && view_of(o, &ow) && (axis >= ow.lo.size() || !ow.windowed(axis));
        }
        if (direct) continue;
        std::vector<std::pair<std::string, std::string>> parts;  // (window, mask)
        int64_t at = 0;
        for (const std::string& o : op.operands) {
          const Type ot = type_of(o);  // a copy: add() may move the ops
          if (axis >= ot.shape.size() || ot.shape[axis] == 0) continue;
          std::vector<int64_t> lo(rank, 0), step(rank, 1);
          lo[axis] = at;
          parts.emplace_back(window(o, op.type, lo, step), mask(op.type, lo, step, ot.shape));
          at += ot.shape[axis];
        }
        if (parts.empty()) continue;
        std::string v = parts.back().first;
        for (size_t k = parts.size() - 1; k-- > 0;) v = select(parts[k].second, parts[k].first, v, op.type);
        replace_uses(op.result, v);
        f_.ops[i].name = "ask.ask_b200_moved";
      }
    }
    for (size_t i = 0; i < f_.ops.size(); ++i) {
      if (f_.ops.size() > 100000) unsupported("index maps of computed values nest too deeply");
      const Op op = f_.ops[i];  // copies: f_.ops grows below
      const std::string n = strip(op.name);
      if (!maps.count(n) || op.operands.empty() || !producer(op.operands[0])) continue;
      const Op src = *producer(op.operands[0]);
      const std::string sn = strip(src.name);
      const bool elementwise = kUnary.count(sn) || kBinary.count(sn) || sn == "cast" || sn == "compare" ||
                               sn == "select";
      std::string moved;
      if (sn == "splat") {
        Op sp = src;  // a map of a splat is a splat of the mapped shape
        sp.type.shape = op.type.shape;
        moved = add(sp);
      } else if (sn == kWindowMask && n != "reshape") {
        // a transposed, sliced, broadcast or windowed window mask is a window mask
        const auto lo = arr(src, "lo"), step = arr(src, "step"), ext = arr(src, "extent");
        const size_t r = op.type.shape.size();
        std::vector<int64_t> nlo(r, 0), nstep(r, 1), next(op.type.shape.begin(), op.type.shape.end());
        if (n == "transpose") {
          const auto perm = arr(op, "permutation");
          for (size_t d = 0; d < r; ++d) {
            nlo[d] = lo[size_t(perm[d])];
            nstep[d] = step[size_t(perm[d])];
            next[d] = ext[size_t(perm[d])];
          }
        } else if (n == "slice") {
          const auto starts = arr(op, "starts"), steps = arr(op, "steps");
          for (size_t d = 0; d < r; ++d) {
            const SlicedWindow sw = slice_window(lo[d], step[d], ext[d], starts[d], steps[d]);
            nlo[d] = sw.lo;
            nstep[d] = sw.step;
            next[d] = sw.extent;
          }
        } else if (n == kWindow) {
          // the outer window's valid coordinate lo2 + step2 i reads the mask at
          // i, valid when i = lo + step j, j < extent
          const auto lo2 = arr(op, "lo"), step2 = arr(op, "step");
          for (size_t d = 0; d < r; ++d) {
            nlo[d] = lo2[d] + step2[d] * lo[d];
            nstep[d] = step2[d] * step[d];
            next[d] = ext[d];
          }
        } else {  // broadcast_in_dim: the mapped axes keep their window, a size-1 axis reads coordinate 0
          const auto dims = arr(op, "dimensions");
          const Type& in = src.type;
          for (size_t k = 0; k < dims.size(); ++k) {
            const size_t d = size_t(dims[k]);
            if (in.shape[k] == 1 && op.type.shape[d] != 1) {
              const bool on = lo[k] == 0 && ext[k] > 0;  // coordinate 0 is valid
              next[d] = on ? op.type.shape[d] : 0;
              continue;
            }
            nlo[d] = lo[k];
            nstep[d] = step[k];
            next[d] = ext[k];
          }
        }
        Op m = src;
        m.attrs["lo"].arr = nlo;
        m.attrs["step"].arr = nstep;
        m.attrs["extent"].arr = next;
        m.type.shape = op.type.shape;
        moved = add(m);
      } else if (elementwise) {
        bool same_shapes = true;
        for (const std::string& o : src.operands) same_shapes = same_shapes && type_of(o).shape == src.type.shape;
        if (!same_shapes) continue;
        Op e = src;
        e.type.shape = op.type.shape;
        for (std::string& o : e.operands) {
          Op m = op;
          m.operands = {o};
          m.type = Type{type_of(o).dtype, op.type.shape, true};
          o = add(m);
        }
        moved = add(e);
      } else {
        continue;
      }
      replace_uses(op.result, moved);
      f_.ops[i].name = "ask.ask_b200_moved";  // the original map is dead now
    }
  }
  // Whether an index map (transpose, broadcast_in_dim, slice, reshape,
  // window) reads v, directly or through elementwise ops (the maps move onto
  // their operands).
  bool mapped(const std::string& v, int depth = 0) const {
    if (depth > 64) return true;
    for (const Op& o : f_.ops) {
      if (std::find(o.operands.begin(), o.operands.end(), v) == o.operands.end()) continue;
      const std::string n = strip(o.name);
      if (n == "transpose" || n == "broadcast_in_dim" || n == "slice" || n == "reshape" || n == kWindow) {
        if (o.operands[0] == v) return true;
      } else if (kUnary.count(n) || kBinary.count(n) || n == "cast" || n == "compare" || n == "select") {
        if (mapped(o.result, depth + 1)) return true;
      }
    }
    return false;
  }
  static std::vector<int64_t> arr(const Op& p, const char* key) {
    auto it = p.attrs.find(key);
    if (it == p.attrs.end()) invalid("ask." + strip(p.name) + " needs '" + key + "'");
    return it->second.arr;
  }
  // emit() reusing an identical earlier instruction (all are pure); used for
  // the coordinate arithmetic of window masks, which repeats across masks.
  int emit_shared(const std::string& insn, const std::string& dtype) {
    const std::string key = dtype + insn;
    auto it = shared_.find(key);
    if (it != shared_.end()) return it->second;
    const int id = emit(insn, dtype);
    shared_[key] = id;
    return id;
  }
  int emit(const std::string& insn, const std::string& dtype, int port = -1) {
    insns_.push_back(insn);
    insn_port_.push_back(port);
    types_.push_back(dtype);
    return int(insns_.size()) - 1;
  }
  // One recipe input per distinct (argument, index map, view).
  int use_port(size_t arg, const std::string& map, const std::string& view = "", const ArgView* w = nullptr) {
    for (size_t k = 0; k < ports_.size(); ++k)
      if (ports_[k].arg == arg && ports_[k].map == map && ports_[k].view == view) return port_insn_[k];
    ports_.push_back({arg, map, view, w ? *w : ArgView{}});
    port_insn_.push_back(emit("", f_.arg_types[arg].dtype, int(ports_.size()) - 1));
    if (map == "view") uses_shape_ = true;
    return port_insn_.back();
  }
  std::string constant_text(const Op& op) const {
    auto it = op.attrs.find("value");
    if (it == op.attrs.end()) invalid("ask.constant without a value");
    const Attr& v = it->second;
    const std::string& dt = op.type.dtype;
    if (v.kind == Attr::Bool) return v.b ? "true" : "false";
    if (v.kind == Attr::Int && dt != "f32" && dt != "f16" && dt != "bf16") {
      if (dt == "bool") return v.i ? "true" : "false";
      return std::to_string(v.i);
    }
    if (v.kind == Attr::Int || (v.kind == Attr::Float && (v.text.find("0x") != std::string::npos ||
                                                          v.text.find("0X") != std::string::npos)))
      return json_str("bits:" + v.text);  // MLIR prints an inexact float literal as its bit pattern
    if (v.kind == Attr::Float) return json_str(v.text);  // decimal text: rounded once to the constant's type
    invalid("unsupported constant value");
  }
  // The scalar constant behind a splat / broadcast / reshape chain, if any.
  const Op* scalar_source(const std::string& v) const {
    const Op* p = producer(v);
    while (p) {
      const std::string n = strip(p->name);
      if (n == "constant") return p;
      if ((n == "splat" || n == "broadcast_in_dim" || n == "reshape") && !p->operands.empty() &&
          type_of(p->operands[0]).numel() == 1) {
        p = producer(p->operands[0]);
        continue;
      }
      return nullptr;
    }
    return nullptr;
  }

  // ---- views ---------------------------------------------------------------------------
  static std::vector<int64_t> row_major(const std::vector<int64_t>& shape) {
    std::vector<int64_t> s(shape.size(), 1);
    for (size_t d = shape.size(); d-- > 1;) s[d - 1] = s[d] * shape[d];
    return s;
  }
  bool view_of(const std::string& v, ArgView* out) const {
    if (!view_of_value(v, out)) return false;
    out->shape = type_of(v).shape;
    return true;
  }
  bool view_of_value(const std::string& v, ArgView* out) const {
    auto a = arg_.find(v);
    const Type& t = type_of(v);
    if (a != arg_.end()) {
      out->arg = a->second;
      out->lo.assign(t.shape.size(), 0);
      out->step.assign(t.shape.size(), 1);
      out->extent = t.shape;
      out->stride = row_major(t.shape);
      out->offset = 0;
      out->inner.reset();
      return true;
    }
    const Op* p = producer(v);
    if (!p) return false;
    const std::string n = strip(p->name);
    ArgView in;
    if (n == "transpose") {
      if (!view_of(p->operands.at(0), &in)) return false;
      const auto perm = arr(*p, "permutation");
      *out = in;
      for (size_t d = 0; d < perm.size(); ++d) {
        const size_t s = size_t(perm[d]);
        out->lo[d] = in.lo[s];
        out->step[d] = in.step[s];
        out->extent[d] = in.extent[s];
        out->stride[d] = in.stride[s];
      }
      return true;
    }
    if (n == "broadcast_in_dim") {
      if (!view_of(p->operands.at(0), &in)) return false;
      const auto dims = arr(*p, "dimensions");
      const Type& it = type_of(p->operands.at(0));
      const size_t r = t.shape.size();
      *out = in;
      out->lo.assign(r, 0);
      out->step.assign(r, 1);
      out->extent = t.shape;
      out->stride.assign(r, 0);
      for (size_t k = 0; k < dims.size(); ++k) {
        const size_t d = size_t(dims[k]);
        if (it.shape[k] == 1) {  // a broadcast axis: stays at the argument's coordinate 0
          if (in.windowed(k)) return false;
          continue;
        }
        out->lo[d] = in.lo[k];
        out->step[d] = in.step[k];
        out->extent[d] = in.extent[k];
        out->stride[d] = in.stride[k];
      }
      return true;
    }
    if (n == "slice") {
      if (!view_of(p->operands.at(0), &in)) return false;
      const auto starts = arr(*p, "starts");
      const auto steps = arr(*p, "steps");
      *out = in;
      for (size_t d = 0; d < t.shape.size(); ++d) {
        if (!in.windowed(d)) {
          out->offset += starts[d] * in.stride[d];
          out->stride[d] = in.stride[d] * steps[d];
          out->extent[d] = t.shape[d];
          continue;
        }
        const SlicedWindow sw = slice_window(in.lo[d], in.step[d], in.extent[d], starts[d], steps[d]);
        out->offset += sw.qf * in.stride[d];
        out->lo[d] = sw.lo;
        out->step[d] = sw.step;
        out->extent[d] = sw.extent;
        out->stride[d] = in.stride[d] * sw.advance;
      }
      return true;
    }
    if (n == "pad") {
      if (!view_of(p->operands.at(0), &in)) return false;
      const Op* c = scalar_source(p->operands.at(1));
      if (!c) return false;  // a computed pad value needs a select, not a view
      const auto low = arr(*p, "pad_low");
      const auto interior = arr(*p, "interior");
      *out = in;
      for (size_t d = 0; d < t.shape.size(); ++d) {
        if (in.windowed(d)) return false;
        out->lo[d] = low[d];
        out->step[d] = interior[d] + 1;
      }
      out->pad = constant_text(*c);
      return true;
    }
    if (n == kWindow) {
      // Coordinate lo + step i reads the operand at i; a windowed operand's i =
      // in.lo + in.step j reads its argument, so the two compose into one
      // window (the operand's pad value, if any, fills the rest of it; what
      // lies outside this window is masked by the select that made it).
      if (!view_of(p->operands.at(0), &in)) return false;
      const auto lo = arr(*p, "lo"), step = arr(*p, "step");
      *out = in;
      for (size_t d = 0; d < t.shape.size(); ++d) {
        out->lo[d] = lo[d] + step[d] * in.lo[d];
        out->step[d] = step[d] * in.step[d];
      }
      return true;
    }
    if (n == "reshape") {
      if (!view_of(p->operands.at(0), &in)) return false;
      bool plain = true;
      for (size_t d = 0; d < in.lo.size(); ++d) plain = plain && !in.windowed(d);
      std::vector<int64_t> stride;
      *out = in;
      out->lo.assign(t.shape.size(), 0);
      out->step.assign(t.shape.size(), 1);
      out->extent = t.shape;
      if (plain && reshape_strides(type_of(p->operands.at(0)).shape, in.stride, t.shape, &stride)) {
        out->stride = stride;  // the reshape is one more strided window
        return true;
      }
      // Read at the same row-major position (ScalarEmitter.h:622): the window
      // of the result yields that position in the operand, whose view becomes
      // the inner stage.  One such stage per port.
      if (in.inner) return false;
      out->inner = std::make_shared<const ArgView>(in);
      out->stride = row_major(t.shape);
      out->offset = 0;
      out->pad = "0";
      return true;
    }
    return false;
  }
  // Strides that read a strided view of shape `from` (strides `st`) in
  // row-major order as shape `to`, if a stride per axis can: the axes of
  // `from` and `to` fall into groups of equal extent products, and the axes
  // of `from` inside a group must nest (stride[k] = stride[k+1] * extent[k+1]),
  // as in a reshape without a copy.  Size-1 axes take no part.
  static bool reshape_strides(const std::vector<int64_t>& from, const std::vector<int64_t>& st,
                              const std::vector<int64_t>& to, std::vector<int64_t>* out) {
    out->assign(to.size(), 0);
    if (product(from, 0, from.size()) == 0) return true;
    std::vector<int64_t> od, os;  // `from` without its size-1 axes
    for (size_t k = 0; k < from.size(); ++k)
      if (from[k] != 1) {
        od.push_back(from[k]);
        os.push_back(st[k]);
      }
    std::vector<size_t> nd;  // indices of `to`'s axes longer than 1
    for (size_t k = 0; k < to.size(); ++k)
      if (to[k] != 1) nd.push_back(k);
    size_t oi = 0, ni = 0;
    while (oi < od.size() && ni < nd.size()) {
      size_t oj = oi + 1, nj = ni + 1;
      int64_t op = od[oi], np = to[nd[ni]];
      while (op != np) {
        if (np < op) {
          if (nj >= nd.size()) return false;
          np *= to[nd[nj++]];
        } else {
          if (oj >= od.size()) return false;
          op *= od[oj++];
        }
      }
      for (size_t k = oi; k + 1 < oj; ++k)
        if (os[k] != od[k + 1] * os[k + 1]) return false;
      (*out)[nd[nj - 1]] = os[oj - 1];
      for (size_t k = nj - 1; k > ni; --k) (*out)[nd[k - 1]] = (*out)[nd[k]] * to[nd[k]];
      oi = oj;
      ni = nj;
    }
    return oi == od.size() && ni == nd.size();
  }
  static bool is_identity(const ArgView& w, const Type& arg, const std::vector<int64_t>& shape) {
    if (w.inner || arg.numel() != product(shape, 0, shape.size()) || w.offset != 0) return false;
    return w.stride == row_major(shape) && w.extent == shape &&
           std::all_of(w.lo.begin(), w.lo.end(), [](int64_t x) { return x == 0; }) &&
           std::all_of(w.step.begin(), w.step.end(), [](int64_t x) { return x == 1; });
  }
  std::string view_json(const ArgView& w) const {
    auto list = [](const std::vector<int64_t>& v) {
      std::string o = "[";
      for (size_t i = 0; i < v.size(); ++i) o += (i ? "," : "") + std::to_string(v[i]);
      return o + "]";
    };
    auto window = [&](const ArgView& v) {
      return "\"offset\":" + std::to_string(v.offset) + ",\"lo\":" + list(v.lo) + ",\"step\":" + list(v.step) +
             ",\"extent\":" + list(v.extent) + ",\"stride\":" + list(v.stride) + ",\"pad\":" + v.pad;
    };
    std::string inner;
    if (w.inner) inner = ",\"inner\":{\"shape\":" + list(w.inner->shape) + "," + window(*w.inner) + "}";
    return "{\"elements\":" + std::to_string(f_.arg_types[w.arg].numel()) + "," + window(w) + inner + "}";
  }
  int use_view(const ArgView& w) { return use_port(w.arg, "view", view_json(w), &w); }

  // Index map of an argument broadcast to the output shape (the fast maps).
  bool simple_broadcast(const Type& from, const std::vector<int64_t>& dims, std::string* map) {
    const size_t r = out_shape_.size(), k = dims.size();
    if (from.numel() == 1) { *map = "scalar"; return true; }
    bool prefix = true, suffix = true;
    for (size_t i = 0; i < k; ++i) {
      prefix = prefix && dims[i] == int64_t(i) && from.shape[i] == out_shape_[i];
      suffix = suffix && dims[i] == int64_t(r - k + i) && from.shape[i] == out_shape_[r - k + i];
    }
    if (is_reduce_) {
      if (prefix && k == lead_) { *map = "outer"; return true; }
      return false;
    }
    if (!prefix && !suffix) return false;
    const uint64_t inner = prefix ? product(out_shape_, k, r) : product(out_shape_, r - k, r);
    if (map_inner_ && map_inner_ != inner) return false;
    map_inner_ = inner;
    *map = prefix ? "outer" : "inner";
    return true;
  }
  // An elementwise view whose addresses follow one of the fast maps: element 0
  // everywhere ("scalar"), the output's flat index divided by `inner`
  // ("outer": row-major over the leading axes, constant over the rest) or
  // modulo `inner` ("inner": constant over the leading axes) -- e.g. a
  // rank-preserving broadcast of a [rows, 1] column or a [1, cols] row.
  // Size-1 axes take no part.
  bool fast_map(const ArgView& w, std::string* map) {
    const size_t r = out_shape_.size();
    if (is_reduce_ || w.offset != 0 || w.inner) return false;
    for (size_t d = 0; d < r; ++d)
      if (w.windowed(d)) return false;
    auto nested = [&](size_t a, size_t b) {  // row-major strides over axes [a, b)
      int64_t expect = 1;
      for (size_t d = b; d-- > a;) {
        if (out_shape_[d] == 1) continue;
        if (w.stride[d] != expect) return false;
        expect *= out_shape_[d];
      }
      return true;
    };
    auto constant = [&](size_t a, size_t b) {
      for (size_t d = a; d < b; ++d)
        if (out_shape_[d] != 1 && w.stride[d] != 0) return false;
      return true;
    };
    if (constant(0, r)) {
      *map = "scalar";
      return true;
    }
    for (size_t k = 1; k < r; ++k) {
      const bool outer = nested(0, k) && constant(k, r), inner = constant(0, k) && nested(k, r);
      if (!outer && !inner) continue;
      const uint64_t n = product(out_shape_, k, r);
      if (map_inner_ && map_inner_ != n) continue;
      map_inner_ = n;
      *map = outer ? "outer" : "inner";
      return true;
    }
    return false;
  }
  int coord(int64_t axis) {
    uses_shape_ = true;
    uses_coord_ = true;
    return emit_shared("[\"coord\"," + std::to_string(axis) + "]", "i64");
  }
  int value(const std::string& v) {
    auto m = memo_.find(v);
    if (m != memo_.end()) return m->second;
    int id = -1;
    const Type& vt = type_of(v);
    auto a = arg_.find(v);
    if (a != arg_.end()) {
      if (vt.numel() == 1 && product(out_shape_, 0, out_shape_.size()) != 1) {
        id = use_port(a->second, "scalar");
      } else if (vt.numel() == product(out_shape_, 0, out_shape_.size())) {
        id = use_port(a->second, "full");
      } else {
        unsupported("argument " + v + " does not have the step's iteration shape; broadcast it explicitly");
      }
      memo_[v] = id;
      return id;
    }
    const Op* p = producer(v);
    if (!p) invalid("value " + v + " is not defined");
    const std::string n = strip(p->name);
    const std::string& dt = p->type.dtype;
    auto operand = [&](size_t k) {
      if (k >= p->operands.size()) invalid("ask." + n + " is missing an operand");
      return value(p->operands[k]);
    };
    ArgView w;
    if (n == "constant") {
      id = emit("[\"const\"," + json_str(dt) + "," + constant_text(*p) + "]", dt);
    } else if (const Op* c = (n == "splat" || n == "broadcast_in_dim" || n == "reshape") ? scalar_source(v) : nullptr) {
      id = value(c->result);
    } else if (n == "splat") {
      const std::string& src = p->operands.at(0);
      if (!arg_.count(src)) unsupported("splat of a computed scalar inside a step");
      id = use_port(arg_.at(src), "scalar");
    } else if ((n == "broadcast_in_dim" || n == "transpose" || n == "slice" || n == "pad" || n == "reshape" ||
                n == kWindow) &&
               view_of(v, &w)) {
      if (p->type.shape != out_shape_) unsupported("an index map to a shape other than the step's iteration shape");
      const Type& at = f_.arg_types[w.arg];
      std::string map;
      if (is_identity(w, at, out_shape_)) {
        id = use_port(w.arg, "full");
      } else if (n == "broadcast_in_dim" && arg_.count(p->operands.at(0)) &&
                 simple_broadcast(at, arr(*p, "dimensions"), &map)) {
        id = use_port(w.arg, map);
      } else if (fast_map(w, &map)) {
        id = use_port(w.arg, map);
      } else {
        id = use_view(w);
      }
    } else if (n == "iota") {
      auto d = p->attrs.find("dimension");
      if (d == p->attrs.end()) invalid("ask.iota without a dimension");
      if (p->type.shape != out_shape_) unsupported("iota of a shape other than the step's iteration shape");
      const int c = coord(d->second.i);
      id = dt == "i64" ? c : emit("[\"cast\"," + std::to_string(c) + "," + json_str(dt) + "]", dt);
    } else if (n == "concatenate") {
      auto ax = p->attrs.find("axis");
      if (ax == p->attrs.end()) invalid("ask.concatenate without an axis");
      if (p->type.shape != out_shape_) unsupported("concatenate to a shape other than the step's iteration shape");
      const size_t axis = size_t(ax->second.i);
      std::vector<std::pair<int, int64_t>> parts;  // (value, end coordinate along axis)
      int64_t at = 0;
      for (const std::string& o : p->operands) {
        const int64_t e = type_of(o).shape.at(axis);
        if (e == 0) continue;
        ArgView ow;
        if (!view_of(o, &ow)) unsupported("concatenate operands must be index maps of step arguments");
        if (ow.windowed(axis)) unsupported("concatenate of a padded operand along the same axis");
        ow.lo[axis] = at;
        ow.extent.resize(out_shape_.size());
        for (size_t d = 0; d < out_shape_.size(); ++d)
          if (d != axis) ow.extent[d] = std::min<int64_t>(ow.extent[d], out_shape_[d]);
        parts.emplace_back(use_view(ow), at + e);
        at += e;
      }
      if (parts.empty()) {
        id = emit("[\"const\"," + json_str(dt) + ",0]", dt);
      } else {
        const int c = parts.size() > 1 ? coord(int64_t(axis)) : -1;
        id = parts.back().first;
        for (size_t k = parts.size() - 1; k-- > 0;) {
          const int bound = emit("[\"const\",\"i64\"," + std::to_string(parts[k].second) + "]", "i64");
          const int lt = emit("[\"compare\",\"lt\"," + std::to_string(c) + "," + std::to_string(bound) + "]", "bool");
          id = emit("[\"select\"," + std::to_string(lt) + "," + std::to_string(parts[k].first) + "," +
                        std::to_string(id) + "]", dt);
        }
      }
    } else if (n == kWindowMask) {
      // AND over the axes of lo <= c <= lo + (extent - 1) step and c = lo (mod
      // step); a check the axis's coordinate range already meets is left out.
      if (p->type.shape != out_shape_) unsupported("a padded or concatenated value of another shape than the step's");
      const auto lo = arr(*p, "lo"), step = arr(*p, "step"), ext = arr(*p, "extent");
      id = -1;
      auto both = [&](int x) {
        id = id < 0 ? x : emit_shared("[\"bitwise_and\"," + std::to_string(id) + "," + std::to_string(x) + "]", "bool");
      };
      auto i64 = [&](int64_t c) { return emit_shared("[\"const\",\"i64\"," + std::to_string(c) + "]", "i64"); };
      for (size_t d = 0; d < out_shape_.size() && id != -2; ++d) {
        if (ext[d] <= 0) {
          id = -2;  // no coordinate is inside the window
          break;
        }
        const int c = coord(int64_t(d));
        const int64_t last = lo[d] + (ext[d] - 1) * step[d];
        if (lo[d] > 0) both(emit_shared("[\"compare\",\"ge\"," + std::to_string(c) + "," + std::to_string(i64(lo[d])) + "]", "bool"));
        if (last + 1 < out_shape_[d])
          both(emit_shared("[\"compare\",\"lt\"," + std::to_string(c) + "," + std::to_string(i64(last + 1)) + "]", "bool"));
        if (step[d] > 1 && ext[d] > 1) {
          const int rem = emit_shared("[\"mod\"," + std::to_string(c) + "," + std::to_string(i64(step[d])) + "]", "i64");
          const int64_t want = ((lo[d] % step[d]) + step[d]) % step[d];
          both(emit_shared("[\"compare\",\"eq\"," + std::to_string(rem) + "," + std::to_string(i64(want)) + "]", "bool"));
        }
      }
      if (id < 0) id = emit_shared(std::string("[\"const\",\"bool\",") + (id == -2 ? "false" : "true") + "]", "bool");
    } else if (n == "broadcast_in_dim" || n == "reshape" || n == "transpose" || n == "slice" || n == "pad" ||
               n == kWindow) {
      unsupported("ask." + n + " of a computed value: only index maps of step arguments are supported");
    } else if (n == "cast") {
      const int x = operand(0);
      id = emit("[\"cast\"," + std::to_string(x) + "," + json_str(dt) + "]", dt);
    } else if (n == "compare") {
      auto pr = p->attrs.find("predicate");
      if (pr == p->attrs.end() || pr->second.kind != Attr::Str) invalid("ask.compare without a predicate");
      const int x = operand(0), y = operand(1);
      id = emit("[\"compare\"," + json_str(pr->second.text) + "," + std::to_string(x) + "," + std::to_string(y) + "]", "bool");
    } else if (n == "select") {
      const int c = operand(0), x = operand(1), y = operand(2);
      id = emit("[\"select\"," + std::to_string(c) + "," + std::to_string(x) + "," + std::to_string(y) + "]", dt);
    } else if (kUnary.count(n)) {
      const int x = operand(0);
      id = emit("[" + json_str(n) + "," + std::to_string(x) + "]", dt);
    } else if (kBinary.count(n)) {
      const int x = operand(0), y = operand(1);
      id = emit("[" + json_str(n) + "," + std::to_string(x) + "," + std::to_string(y) + "]", dt);
    } else {
      unsupported("ask." + n + " inside an elementwise step");
    }
    if (p->type.shape != out_shape_ && p->type.numel() != 1)
      unsupported("ask." + n + " changes the iteration shape inside the step");
    memo_[v] = id;
    return id;
  }
  void start_program() {
    insns_.clear();
    insn_port_.clear();
    types_.clear();
    memo_.clear();
    shared_.clear();
    ports_.clear();
    port_insn_.clear();
    uses_shape_ = false;
    uses_coord_ = false;
  }
  // Ports in argument order (then first use); input instructions name them.
  std::vector<size_t> port_order() const {
    std::vector<size_t> order(ports_.size());
    for (size_t k = 0; k < order.size(); ++k) order[k] = k;
    std::stable_sort(order.begin(), order.end(), [&](size_t x, size_t y) { return ports_[x].arg < ports_[y].arg; });
    return order;
  }
  std::string inputs_json(const std::vector<size_t>& order) const {
    std::string o = "[";
    for (size_t k = 0; k < order.size(); ++k) {
      const Port& pt = ports_[order[k]];
      o += (k ? "," : "");
      o += "{\"dtype\":" + json_str(f_.arg_types[pt.arg].dtype) + ",\"map\":" + json_str(pt.map);
      if (pt.map == "view") o += ",\"view\":" + pt.view;
      o += "}";
    }
    return o + "]";
  }
  std::string program_json(const std::vector<size_t>& order) const {
    std::vector<size_t> rank(order.size());
    for (size_t k = 0; k < order.size(); ++k) rank[order[k]] = k;
    std::string o = "[";
    for (size_t k = 0; k < insns_.size(); ++k) {
      o += (k ? "," : "");
      o += insn_port_[k] >= 0 ? "[\"input\"," + std::to_string(rank[size_t(insn_port_[k])]) + "]" : insns_[k];
    }
    return o + "]";
  }
  std::vector<size_t> port_args(const std::vector<size_t>& order) const {
    std::vector<size_t> v;
    for (size_t k : order) v.push_back(ports_[k].arg);
    return v;
  }
  std::string shape_json() const {
    std::string o = "[";
    for (size_t i = 0; i < out_shape_.size(); ++i) o += (i ? "," : "") + std::to_string(out_shape_[i]);
    return o + "]";
  }

  Lowered elementwise() {
    out_shape_ = type_of(f_.returns[0]).shape;
    for (const std::string& r : f_.returns)
      if (type_of(r).shape != out_shape_) unsupported("elementwise step outputs of different shapes");
    start_program();
    std::vector<int> results;
    std::string outs = "[";
    for (size_t k = 0; k < f_.returns.size(); ++k) {
      results.push_back(value(f_.returns[k]));
      outs += (k ? "," : "") + std::string("{\"dtype\":") + json_str(type_of(f_.returns[k]).dtype) + "}";
    }
    outs += "]";
    if (uses_shape_ && (out_shape_.empty() || out_shape_.size() > 6))
      unsupported("views and coordinates need an iteration shape of 1..6 axes");
    const std::vector<size_t> order = port_order();
    std::ostringstream o;
    o << "{\"family\":\"elementwise\",\"count\":" << product(out_shape_, 0, out_shape_.size())
      << ",\"inner\":" << (map_inner_ ? map_inner_ : 1);
    if (uses_shape_) o << ",\"shape\":" << shape_json();
    o << ",\"inputs\":" << inputs_json(order) << ",\"outputs\":" << outs << ",\"program\":" << program_json(order)
      << ",\"results\":[";
    for (size_t k = 0; k < results.size(); ++k) o << (k ? "," : "") << results[k];
    o << "]}";
    return {o.str(), port_args(order)};
  }

  Lowered reduction() {
    // every returned value is a reduction over the same operand shape and axes
    std::vector<const Op*> reds;
    std::vector<int64_t> axes;
    std::vector<int64_t> in_shape;
    for (const std::string& r : f_.returns) {
      const Op* p = producer(r);
      if (!p || !is_reduction(strip(p->name)))
        unsupported("a reduction step may return only reduction results (" + r + " is not one)");
      const std::string n = strip(p->name);
      std::vector<int64_t> ax;
      if (n == "argmax" || n == "argmin") {
        auto a = p->attrs.find("axis");
        if (a == p->attrs.end()) invalid("ask." + n + " without an axis");
        ax = {a->second.i};
      } else {
        auto a = p->attrs.find("axes");
        if (a == p->attrs.end()) invalid("ask." + n + " without axes");
        ax = a->second.arr;
      }
      const std::vector<int64_t>& s = type_of(p->operands.at(0)).shape;
      if (reds.empty()) {
        axes = ax;
        in_shape = s;
      } else if (ax != axes || s != in_shape) {
        unsupported("reductions over different shapes or axes in one step");
      }
      reds.push_back(p);
    }
    if (axes.empty()) unsupported("a reduction over no axes is an elementwise copy");
    for (size_t i = 1; i < axes.size(); ++i)
      if (axes[i] != axes[i - 1] + 1) unsupported("reduction axes must be one contiguous block");
    const size_t a0 = size_t(axes.front()), a1 = size_t(axes.back()) + 1;
    if (a1 > in_shape.size()) invalid("reduction axis out of range");
    const uint64_t outer = product(in_shape, 0, a0), extent = product(in_shape, a0, a1),
                   inner = product(in_shape, a1, in_shape.size());
    out_shape_ = in_shape;
    lead_ = a0;
    is_reduce_ = true;
    start_program();
    std::vector<int> results;
    std::string reductions = "[";
    for (size_t k = 0; k < reds.size(); ++k) {
      const int v = value(reds[k]->operands.at(0));
      size_t slot = 0;
      while (slot < results.size() && results[slot] != v) ++slot;
      if (slot == results.size()) results.push_back(v);
      reductions += (k ? "," : "") + std::string("{\"op\":") + json_str(strip(reds[k]->name)) + ",\"value\":" +
                    std::to_string(slot) + "}";
    }
    reductions += "]";
    for (const Port& pt : ports_)
      if (pt.map == "inner") unsupported("reductions read no per-column operands");
    if (uses_shape_ && (out_shape_.empty() || out_shape_.size() > 6))
      unsupported("views and coordinates need an iteration shape of 1..6 axes");
    const std::vector<size_t> order = port_order();
    std::ostringstream o;
    uint64_t po = 0, pe = 0, pi = 0;
    if (uses_shape_ && permuted_reduction(a0, a1, &po, &pe, &pi)) {
      // every view reads its argument through one axis permutation: reduce
      // over the arguments' own axes instead, with full ports
      for (Port& pt : ports_)
        if (pt.map == "view") pt = Port{pt.arg, "full", "", ArgView{}};
      o << "{\"family\":\"reduce\",\"outer\":" << po << ",\"extent\":" << pe << ",\"inner\":" << pi;
    } else {
      o << "{\"family\":\"reduce\",\"outer\":" << outer << ",\"extent\":" << extent << ",\"inner\":" << inner;
      if (uses_shape_) o << ",\"shape\":" << shape_json();
    }
    o << ",\"inputs\":" << inputs_json(order) << ",\"program\":" << program_json(order) << ",\"results\":[";
    for (size_t k = 0; k < results.size(); ++k) o << (k ? "," : "") << results[k];
    o << "],\"reductions\":" << reductions << "}";
    return {o.str(), port_args(order)};
  }

  // A reduction over iteration axes [a0, a1) whose ports are scalars or views
  // that read their arguments through one axis permutation p (no window, no
  // offset; iteration axis d is argument axis p[d]) and whose program reads no
  // coordinates is the same reduction over the arguments' own layout when the
  // reduced axes map to one contiguous block of argument axes and the kept
  // axes keep their order (so the outputs keep theirs): outer/extent/inner of
  // that layout.  Axes of extent 1 take no part.  A transposed operand then
  // reads coalesced (the row, split or column kernels) instead of going
  // through the view kernel.
  bool permuted_reduction(size_t a0, size_t a1, uint64_t* po, uint64_t* pe, uint64_t* pi) const {
    if (uses_coord_) return false;
    const size_t r = out_shape_.size();
    std::vector<int64_t> perm(r, -1), arg_shape;
    bool first = true;
    for (const Port& pt : ports_) {
      if (pt.map == "scalar") continue;
      if (pt.map != "view") return false;
      const ArgView& w = pt.w;
      const std::vector<int64_t>& as = f_.arg_types[pt.arg].shape;
      if (w.offset != 0 || w.stride.size() != r || w.inner) return false;
      for (size_t d = 0; d < r; ++d)
        if (w.windowed(d) || w.extent[d] != out_shape_[d]) return false;
      const std::vector<int64_t> rm = row_major(as);
      std::vector<int64_t> p(r, -1);
      for (size_t d = 0; d < r; ++d) {
        if (out_shape_[d] == 1) continue;
        for (size_t j = 0; j < as.size(); ++j)
          if (as[j] == out_shape_[d] && rm[j] == w.stride[d]) p[d] = int64_t(j);
        if (p[d] < 0) return false;
      }
      if (first) {
        perm = p;
        arg_shape = as;
        first = false;
      } else if (p != perm || as != arg_shape) {
        return false;
      }
    }
    if (first) return false;
    // argument axes of the reduced block and of the kept axes, in iteration order
    std::vector<int64_t> red, kept;
    for (size_t d = 0; d < r; ++d) {
      if (out_shape_[d] == 1) continue;
      (d >= a0 && d < a1 ? red : kept).push_back(perm[d]);
    }
    for (size_t k = 1; k < kept.size(); ++k)
      if (kept[k] < kept[k - 1]) return false;
    if (red.empty()) return false;
    const int64_t lo = *std::min_element(red.begin(), red.end()), hi = *std::max_element(red.begin(), red.end());
    for (int64_t j = lo; j <= hi; ++j)
      if (arg_shape[size_t(j)] != 1 && std::find(red.begin(), red.end(), j) == red.end()) return false;
    for (int64_t j : kept)
      if (j > lo && j < hi) return false;
    bool identity = true;
    for (size_t d = 0, j = 0; d < r; ++d) {
      if (out_shape_[d] == 1) continue;
      while (j < arg_shape.size() && arg_shape[j] == 1) ++j;
      identity = identity && perm[d] == int64_t(j++);
    }
    if (identity) return false;  // the views already read in order
    *po = product(arg_shape, 0, size_t(lo));
    *pe = product(arg_shape, size_t(lo), size_t(hi) + 1);
    *pi = product(arg_shape, size_t(hi) + 1, arg_shape.size());
    return true;
  }

  Lowered indexed(const Op& op, bool scatter) {
    if (f_.returns.size() != 1) unsupported("a gather/scatter_add step returns exactly its one result");
    for (const std::string& x : op.operands)
      if (!arg_.count(x)) unsupported("gather/scatter_add operands must be step arguments (no fused prologue)");
    auto a = op.attrs.find("axis");
    if (a == op.attrs.end()) invalid("ask.gather/ask.scatter_add without an axis");
    const int64_t axis = a->second.i;
    const Type& table = type_of(op.operands.at(0));
    const Type& index = type_of(op.operands.at(1));
    if (axis < 0 || size_t(axis) >= table.shape.size()) invalid("gather/scatter_add axis out of range");
    const uint64_t outer = product(table.shape, 0, size_t(axis)), dim = uint64_t(table.shape[size_t(axis)]),
                   inner = product(table.shape, size_t(axis) + 1, table.shape.size());
    std::ostringstream o;
    o << "{\"family\":" << (scatter ? "\"scatter_add\"" : "\"gather\"") << ",\"dtype\":" << json_str(table.dtype)
      << ",\"index_dtype\":" << json_str(index.dtype) << ",\"outer\":" << outer << ",\"dim\":" << dim
      << ",\"inner\":" << inner << ",\"n\":" << index.numel();
    if (scatter) o << ",\"pre_copy\":{\"input\":0,\"output\":0}";
    o << "}";
    std::vector<size_t> ports;
    for (const std::string& x : op.operands) ports.push_back(arg_.at(x));
    return {o.str(), ports};
  }
};

Lowered lower_source(const std::string& text) {
  Reader r(text);
  const Func f = r.read_function();
  return Lowering(f).run();
}

size_t element_bytes(const std::string& t);

// One program step of a lowered source: per recipe input, the function
// argument it reads (>= 0) or internal buffer k (-1 - k); per recipe output,
// the function result it writes (>= 0) or internal buffer k (-1 - k).
struct Part {
  Lowered l;
  std::vector<int64_t> ins, outs;
};
struct Split {
  std::vector<Part> parts;
  std::vector<uint64_t> internal_bytes;  // sizes of the internal buffers the parts exchange
};

// A step lowers to one recipe when it can; otherwise:
//   - results one recipe cannot hold together (elementwise results of
//     different shapes, reductions over different operand shapes or axes, or
//     both kinds) lower as one recipe per group, the way the reference emits
//     one batch per output shape in a step's kernel (lib/Lowering/CUDA.cpp:
//     210-244); groups keep the order of their first result;
//   - a gather or scatter_add whose operands are computed in the step reads
//     them from internal buffers that elementwise recipes write first (the
//     reference evaluates such operands per element inside its kernel,
//     lib/Lowering/ScalarEmitter.h:775-815).
// ask.mark pass-throughs (erased by the reference's prepare phase): every use
// of a mark's result, and every return of it, reads the marked value itself.
Func without_marks(Func f) {
  std::map<std::string, std::string> to;
  for (const Op& op : f.ops)
    if (strip(op.name) == "mark" && op.operands.size() == 1) to[op.result] = op.operands[0];
  auto resolve = [&](std::string v) {
    for (auto it = to.find(v); it != to.end(); it = to.find(v)) v = it->second;
    return v;
  };
  std::vector<Op> kept;
  for (Op& op : f.ops) {
    if (to.count(op.result)) continue;
    for (std::string& x : op.operands) x = resolve(x);
    kept.push_back(op);
  }
  f.ops = kept;
  for (std::string& r : f.returns) r = resolve(r);
  return f;
}

Split lower_source_split(const std::string& text) {
  Reader r(text);
  const Func f = without_marks(r.read_function());
  std::map<std::string, const Op*> def;
  std::map<std::string, size_t> arg;
  for (const Op& op : f.ops) def[op.result] = &op;
  for (size_t k = 0; k < f.args.size(); ++k) arg[f.args[k]] = k;
  auto shape_key = [](const std::vector<int64_t>& v) {
    std::string o;
    for (int64_t d : v) o += std::to_string(d) + ",";
    return o;
  };
  std::vector<std::string> keys;
  std::vector<std::vector<size_t>> groups;
  for (size_t k = 0; k < f.returns.size(); ++k) {
    std::string key;
    auto d = def.find(f.returns[k]);
    if (d == def.end()) {
      auto a = arg.find(f.returns[k]);
      key = "E|" + (a != arg.end() ? shape_key(f.arg_types[a->second].shape) : std::string("?"));
    } else {
      const Op& op = *d->second;
      const std::string n = strip(op.name);
      if (n == "gather" || n == "scatter_add") {
        key = "X|" + std::to_string(k);
      } else if (n.rfind("reduce_", 0) == 0 || n == "argmax" || n == "argmin") {
        std::vector<int64_t> axes;
        auto ax = op.attrs.find(n == "argmax" || n == "argmin" ? "axis" : "axes");
        if (ax != op.attrs.end()) axes = ax->second.kind == Attr::IntArray ? ax->second.arr
                                                                          : std::vector<int64_t>{ax->second.i};
        std::sort(axes.begin(), axes.end());
        auto od = op.operands.empty() ? def.end() : def.find(op.operands[0]);
        auto oa = op.operands.empty() ? arg.end() : arg.find(op.operands[0]);
        const std::vector<int64_t> in = od != def.end() ? od->second->type.shape
                                        : oa != arg.end() ? f.arg_types[oa->second].shape : std::vector<int64_t>{};
        key = "R|" + shape_key(in) + "|" + shape_key(axes);
      } else {
        key = "E|" + shape_key(op.type.shape);
      }
    }
    size_t g = 0;
    while (g < keys.size() && keys[g] != key) ++g;
    if (g == keys.size()) {
      keys.push_back(key);
      groups.emplace_back();
    }
    groups[g].push_back(k);
  }
  Split out;
  std::map<std::string, int64_t> internal_of_value;  // a computed operand's internal buffer, written once
  auto plain = [](const Lowered& l, const std::vector<size_t>& results) {
    Part p{l, {}, {}};
    for (size_t a : l.input_args) p.ins.push_back(int64_t(a));
    for (size_t k : results) p.outs.push_back(int64_t(k));
    return p;
  };
  for (size_t g = 0; g < groups.size(); ++g) {
    Func part = f;
    part.returns.clear();
    for (size_t k : groups[g]) part.returns.push_back(f.returns[k]);
    const bool indexed = keys[g].rfind("X|", 0) == 0;
    if (!indexed) {
      out.parts.push_back(plain(Lowering(part).run(), groups[g]));
      continue;
    }
    // a gather/scatter_add: computed operands first, into internal buffers
    const Op& op = *def.at(f.returns[groups[g][0]]);
    size_t op_index = 0;
    while (part.ops[op_index].result != op.result) ++op_index;
    std::vector<int64_t> internal_of_arg;  // per extra argument of `part`, its internal buffer
    std::map<std::string, std::string> arg_of_value;  // within this part: one extra argument per value
    for (size_t j = 0; j < op.operands.size(); ++j) {
      const std::string v = op.operands[j];
      if (arg.count(v)) continue;
      auto pd = def.find(v);
      if (pd == def.end()) invalid("value " + v + " is not defined");
      const Type t = pd->second->type;
      auto known = internal_of_value.find(v);
      int64_t k;
      if (known != internal_of_value.end()) {
        k = known->second;
      } else {
        Func pre = f;
        pre.returns = {v};
        const Lowered lp = Lowering(pre).run();
        k = int64_t(out.internal_bytes.size());
        out.internal_bytes.push_back(t.numel() * element_bytes(t.dtype));
        Part pp{lp, {}, {-1 - k}};
        for (size_t a : lp.input_args) pp.ins.push_back(int64_t(a));
        out.parts.push_back(pp);
        internal_of_value[v] = k;
      }
      auto named = arg_of_value.find(v);
      if (named == arg_of_value.end()) {
        const std::string name = "%ask_b200.internal" + std::to_string(k);
        part.args.push_back(name);
        part.arg_types.push_back(t);
        internal_of_arg.push_back(k);
        named = arg_of_value.emplace(v, name).first;
      }
      part.ops[op_index].operands[j] = named->second;
    }
    const Lowered l = Lowering(part).run();
    Part p{l, {}, {}};
    for (size_t a : l.input_args)
      p.ins.push_back(a < f.args.size() ? int64_t(a) : -1 - internal_of_arg[a - f.args.size()]);
    for (size_t k : groups[g]) p.outs.push_back(int64_t(k));
    out.parts.push_back(p);
  }
  return out;
}

size_t element_bytes(const std::string& t) {
  if (t == "bool") return 1;
  if (t == "i32" || t == "f32") return 4;
  if (t == "i64") return 8;
  if (t == "f16" || t == "bf16") return 2;
  invalid("unknown element type '" + t + "'");
}

std::string lower_report(const char* report_json) {
  const json::Value root = json::parse(report_json);
  const json::Value& plan = root.get("execution_plan") ? root.at("execution_plan") : root;
  const json::Value* sources = root.get("step_sources");
  if (!sources) invalid("the report has no step_sources");
  std::map<std::string, size_t> index;
  std::vector<uint64_t> sizes;
  for (const auto& b : plan.at("buffers").as_array("buffers")) {
    const std::string id = b.at("id").as_str("buffer id");
    uint64_t n = 1;
    for (const auto& d : b.at("shape").as_array("shape")) n *= uint64_t(d.as_int("shape"));
    index[id] = sizes.size();
    sizes.push_back(n * element_bytes(b.at("element_type").as_str("element_type")));
  }
  auto ids = [&](const json::Value& list, const char* what) {
    std::vector<size_t> out;
    for (const auto& x : list.as_array(what)) {
      auto it = index.find(x.as_str(what));
      if (it == index.end()) invalid(std::string(what) + " names an undeclared buffer '" + x.str + "'");
      out.push_back(it->second);
    }
    return out;
  };
  auto list = [](const std::vector<size_t>& v) {
    std::string o = "[";
    for (size_t i = 0; i < v.size(); ++i) o += (i ? "," : "") + std::to_string(v[i]);
    return o + "]";
  };
  std::ostringstream steps;
  std::vector<std::string> unresolved;
  bool first = true;
  for (const auto& step : plan.at("steps").as_array("steps")) {
    const std::string id = step.at("id").as_str("step id");
    const json::Value* kind = step.get("kind");
    if (kind && kind->as_str("kind") != "owned") {
      // An external or library step keeps its place and its buffers; the
      // caller binds a loaded kernel to it ("kernel", "grid", "block",
      // "arguments") before preparing the program.
      const std::string k = kind->str;
      if (k != "external" && k != "library") invalid("step " + id + " has unknown kind '" + k + "'");
      std::string what = "{\"kind\":" + json_str(k);
      for (const char* key : {"function", "external_id", "library"})
        if (const json::Value* v = step.get(key)) what += std::string(",\"") + key + "\":" + json_str(v->as_str(key));
      what += "}";
      steps << (first ? "" : ",") << "{\"id\":" << json_str(id) << ",\"unresolved\":" << what
            << ",\"inputs\":" << list(ids(step.at("inputs"), "step inputs"))
            << ",\"outputs\":" << list(ids(step.at("outputs"), "step outputs")) << "}";
      first = false;
      unresolved.push_back(id);
      continue;
    }
    const json::Value* src = sources->get(id);
    if (!src) invalid("no step source for " + id);
    Split split;
    try {
      split = lower_source_split(src->as_str("step source"));
    } catch (const Failure& f) {
      fail(f.code, "step " + id + ": " + f.message);
    }
    const std::vector<size_t> ins = ids(step.at("inputs"), "step inputs");
    const std::vector<size_t> outs = ids(step.at("outputs"), "step outputs");
    const size_t internal0 = sizes.size();  // this step's internal buffers follow the plan's
    for (uint64_t b : split.internal_bytes) sizes.push_back(b);
    auto buffer = [&](int64_t x, const std::vector<size_t>& bound, const char* what) {
      if (x < 0) return internal0 + size_t(-1 - x);
      if (size_t(x) >= bound.size()) invalid("step " + id + " source has more " + what + " than the plan binds");
      return bound[size_t(x)];
    };
    for (size_t g = 0; g < split.parts.size(); ++g) {
      const Part& part = split.parts[g];
      std::vector<size_t> read, written;
      for (int64_t x : part.ins) read.push_back(buffer(x, ins, "arguments"));
      for (int64_t x : part.outs) written.push_back(buffer(x, outs, "results"));
      const std::string sid = split.parts.size() > 1 ? id + "#" + std::to_string(g) : id;
      const long base_arg = part.ins.empty() ? 0 : long(part.ins[0]);
      steps << (first ? "" : ",") << "{\"id\":" << json_str(sid) << ",\"recipe\":" << json_str(part.l.recipe)
            << ",\"inputs\":" << list(read) << ",\"outputs\":" << list(written)
            << ",\"cuda_lowering\":" << askb_recipe_lowering_report(part.l.recipe, base_arg) << "}";
      first = false;
    }
  }
  std::ostringstream o;
  o << "{\"buffer_sizes\":[";
  for (size_t i = 0; i < sizes.size(); ++i) o << (i ? "," : "") << sizes[i];
  o << "],\"inputs\":" << list(ids(plan.at("inputs"), "inputs")) << ",\"outputs\":" << list(ids(plan.at("outputs"), "outputs"))
    << ",\"steps\":[" << steps.str() << "]";
  if (!unresolved.empty()) {
    o << ",\"unresolved_steps\":[";
    for (size_t i = 0; i < unresolved.size(); ++i) o << (i ? "," : "") << json_str(unresolved[i]);
    o << "]";
  }
  o << "}";
  return o.str();
}

void write_text(const std::string& s, char* buf, size_t cap, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (buf && cap) {
    const size_t n = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
}

template <class F>
int guarded(F&& body) {
  try {
    body();
    askb_internal_set_error("");
    return ASK_B200_OK;
  } catch (const Failure& f) {
    askb_internal_set_error(f.message.c_str());
    return f.code;
  } catch (const std::exception& e) {
    askb_internal_set_error(e.what());
    return ASK_B200_E_INVALID;
  } catch (...) {
    askb_internal_set_error("unknown error");
    return ASK_B200_E_INVALID;
  }
}

}  // namespace
}  // namespace lower
}  // namespace askb

extern "C" {

int ask_b200_lower_step(const char* step_source, char* buf, size_t cap, size_t* needed) {
  using namespace askb::lower;
  return guarded([&] {
    if (!step_source) invalid("step source is NULL");
    const Lowered l = lower_source(step_source);
    std::string ports = "[";
    for (size_t k = 0; k < l.input_args.size(); ++k) ports += (k ? "," : "") + std::to_string(l.input_args[k]);
    ports += "]";
    const long base_arg = l.input_args.empty() ? 0 : long(l.input_args[0]);
    write_text("{\"recipe\":" + l.recipe + ",\"input_arguments\":" + ports +
                   ",\"cuda_lowering\":" + askb_recipe_lowering_report(l.recipe, base_arg) + "}",
               buf, cap, needed);
  });
}

int ask_b200_lower_report(const char* report_json, char* buf, size_t cap, size_t* needed) {
  using namespace askb::lower;
  return guarded([&] {
    if (!report_json) invalid("report is NULL");
    write_text(lower_report(report_json), buf, cap, needed);
  });
}

}  // extern "C"
