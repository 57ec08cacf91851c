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
// dimensions 0..k-1) or a suffix ("inner").  ask.constant/ask.splat become
// constants (MLIR prints each float literal so that it re-parses exactly, or
// as its bit pattern in hex; either is carried over without double rounding),
// ask.reshape of an argument is the argument itself.  Ops this library has no
// index map for (transpose, slice, pad, concatenate, iota) and matmul or
// external steps are reported as unsupported.
#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "ask_b200.h"
#include "ask_b200_lower.h"
#include "json.h"

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

struct Lowered {
  std::string recipe;
  std::vector<size_t> input_args;  // recipe input k reads function argument input_args[k]
};

class Lowering {
 public:
  explicit Lowering(const Func& f) : f_(f) {
    for (size_t k = 0; k < f.args.size(); ++k) arg_[f.args[k]] = k;
    for (size_t k = 0; k < f.ops.size(); ++k) def_[f.ops[k].result] = k;
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
  const Func& f_;
  std::map<std::string, size_t> arg_, def_;
  // op program under construction
  std::vector<std::string> insns_;
  std::vector<std::string> types_;
  std::map<std::string, int> memo_;
  std::vector<std::string> arg_map_;   // per argument: "", full, scalar, outer, inner
  std::vector<int> arg_insn_;
  std::vector<int64_t> out_shape_;
  size_t lead_ = 0;                    // reduce: number of leading (outer) axes
  uint64_t map_inner_ = 0;             // elementwise: the 'inner' every outer/inner map shares
  bool is_reduce_ = false;

  static bool is_reduction(const std::string& n) { return n.rfind("reduce_", 0) == 0 || n == "argmax" || n == "argmin"; }

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
  int emit(const std::string& insn, const std::string& dtype) {
    insns_.push_back(insn);
    types_.push_back(dtype);
    return int(insns_.size()) - 1;
  }
  // Argument `a` read with index map `map`: one recipe input per argument.
  int use_arg(size_t a, const std::string& map) {
    if (arg_map_[a].empty()) arg_map_[a] = map;
    if (arg_map_[a] != map)
      unsupported("argument " + std::to_string(a) + " is read through two index maps (" + arg_map_[a] + ", " + map + ")");
    return arg_insn_[a];
  }
  std::string constant(const Op& op) {
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
    if (v.kind == Attr::Float) {
      if (v.text == "nan" || v.text == "inf" || v.text == "-inf") return json_str(v.text);
      return json_str(v.text);  // decimal text: rounded once to the constant's type
    }
    invalid("unsupported constant value");
  }
  // The scalar value behind a splat / broadcast of a constant, if any.
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
  // Index map of an argument broadcast to the output shape.
  std::string broadcast_map(const Type& from, const std::vector<int64_t>& dims) {
    const size_t r = out_shape_.size(), k = dims.size();
    if (from.numel() == 1) return "scalar";
    bool prefix = true, suffix = true;
    for (size_t i = 0; i < k; ++i) {
      prefix = prefix && dims[i] == int64_t(i);
      suffix = suffix && dims[i] == int64_t(r - k + i);
    }
    if (is_reduce_) {
      if (prefix && k == lead_) return "outer";
      unsupported("a broadcast operand of a reduction must be indexed by exactly the kept leading axes");
    }
    const uint64_t inner = prefix ? product(out_shape_, k, r) : product(out_shape_, r - k, r);
    if (!prefix && !suffix) unsupported("broadcast_in_dim over non-leading, non-trailing axes needs a general index map");
    if (map_inner_ && map_inner_ != inner)
      unsupported("outer/inner broadcasts of different extents in one step");
    map_inner_ = inner;
    return prefix ? "outer" : "inner";
  }
  int value(const std::string& v) {
    auto m = memo_.find(v);
    if (m != memo_.end()) return m->second;
    int id;
    auto a = arg_.find(v);
    if (a != arg_.end()) {
      const Type& t = f_.arg_types[a->second];
      if (t.shape != out_shape_ && t.numel() != product(out_shape_, 0, out_shape_.size()))
        unsupported("argument " + v + " does not have the step's iteration shape; broadcast it explicitly");
      id = use_arg(a->second, t.numel() == 1 && product(out_shape_, 0, out_shape_.size()) != 1 ? "scalar" : "full");
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
    if (n == "constant") {
      id = emit("[\"const\"," + json_str(dt) + "," + constant(*p) + "]", dt);
    } else if (n == "splat" || n == "broadcast_in_dim" || n == "reshape") {
      if (const Op* c = scalar_source(v)) {
        id = value(c->result);
      } else if (n == "reshape") {
        const std::string& src = p->operands.at(0);
        if (!arg_.count(src) || type_of(src).numel() != p->type.numel())
          unsupported("reshape of a computed value inside a step");
        id = use_arg(arg_.at(src), "full");
      } else if (n == "broadcast_in_dim") {
        const std::string& src = p->operands.at(0);
        if (!arg_.count(src)) unsupported("broadcast_in_dim of a computed value inside a step");
        if (p->type.shape != out_shape_) unsupported("broadcast to a shape other than the step's iteration shape");
        auto d = p->attrs.find("dimensions");
        id = use_arg(arg_.at(src), broadcast_map(type_of(src), d == p->attrs.end() ? std::vector<int64_t>{} : d->second.arr));
      } else {  // splat of a non-constant scalar argument
        const std::string& src = p->operands.at(0);
        if (!arg_.count(src)) unsupported("splat of a computed scalar inside a step");
        id = use_arg(arg_.at(src), "scalar");
      }
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
    } else if (n == "transpose" || n == "slice" || n == "pad" || n == "concatenate" || n == "iota") {
      unsupported("ask." + n + " needs a general index map, which this library's kernels do not have");
    } else {
      unsupported("ask." + n + " inside an elementwise step");
    }
    if (p->type.shape != out_shape_ && p->type.numel() != 1 && n != "reshape")
      unsupported("ask." + n + " changes the iteration shape inside the step");
    memo_[v] = id;
    return id;
  }
  void start_program() {
    insns_.clear();
    types_.clear();
    memo_.clear();
    arg_map_.assign(f_.args.size(), "");
    arg_insn_.clear();
    for (size_t k = 0; k < f_.args.size(); ++k)
      arg_insn_.push_back(emit("[\"input\"," + std::to_string(k) + "]", f_.arg_types[k].dtype));
  }
  std::string inputs_json() const {
    std::string o = "[";
    for (size_t k = 0; k < f_.args.size(); ++k) {
      o += (k ? "," : "");
      o += "{\"dtype\":" + json_str(f_.arg_types[k].dtype) + ",\"map\":" +
           json_str(arg_map_[k].empty() ? "full" : arg_map_[k]) + "}";
    }
    return o + "]";
  }
  std::string program_json() const {
    std::string o = "[";
    for (size_t k = 0; k < insns_.size(); ++k) o += (k ? "," : "") + insns_[k];
    return o + "]";
  }
  std::vector<size_t> identity_args() const {
    std::vector<size_t> v(f_.args.size());
    for (size_t k = 0; k < v.size(); ++k) v[k] = k;
    return v;
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
    std::ostringstream o;
    o << "{\"family\":\"elementwise\",\"count\":" << product(out_shape_, 0, out_shape_.size())
      << ",\"inner\":" << (map_inner_ ? map_inner_ : 1) << ",\"inputs\":" << inputs_json() << ",\"outputs\":" << outs
      << ",\"program\":" << program_json() << ",\"results\":[";
    for (size_t k = 0; k < results.size(); ++k) o << (k ? "," : "") << results[k];
    o << "]}";
    return {o.str(), identity_args()};
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
    for (size_t k = 0; k < f_.args.size(); ++k)
      if (arg_map_[k] == "inner") unsupported("reductions read no per-column operands");
    std::ostringstream o;
    o << "{\"family\":\"reduce\",\"outer\":" << outer << ",\"extent\":" << extent << ",\"inner\":" << inner
      << ",\"inputs\":" << inputs_json() << ",\"program\":" << program_json() << ",\"results\":[";
    for (size_t k = 0; k < results.size(); ++k) o << (k ? "," : "") << results[k];
    o << "],\"reductions\":" << reductions << "}";
    return {o.str(), identity_args()};
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
  std::ostringstream o;
  o << "{\"buffer_sizes\":[";
  for (size_t i = 0; i < sizes.size(); ++i) o << (i ? "," : "") << sizes[i];
  o << "],\"inputs\":" << list(ids(plan.at("inputs"), "inputs")) << ",\"outputs\":" << list(ids(plan.at("outputs"), "outputs"))
    << ",\"steps\":[";
  bool first = true;
  for (const auto& step : plan.at("steps").as_array("steps")) {
    const std::string id = step.at("id").as_str("step id");
    const json::Value* kind = step.get("kind");
    if (kind && kind->as_str("kind") != "owned")
      unsupported("step " + id + " is a '" + kind->str + "' step; only owned steps lower to recipes");
    const json::Value* src = sources->get(id);
    if (!src) invalid("no step source for " + id);
    Lowered l;
    try {
      l = lower_source(src->as_str("step source"));
    } catch (const Failure& f) {
      fail(f.code, "step " + id + ": " + f.message);
    }
    const std::vector<size_t> ins = ids(step.at("inputs"), "step inputs");
    std::vector<size_t> bound;
    for (size_t a : l.input_args) {
      if (a >= ins.size()) invalid("step " + id + " source has more arguments than the plan binds");
      bound.push_back(ins[a]);
    }
    o << (first ? "" : ",") << "{\"id\":" << json_str(id) << ",\"recipe\":" << json_str(l.recipe)
      << ",\"inputs\":" << list(bound) << ",\"outputs\":" << list(ids(step.at("outputs"), "step outputs")) << "}";
    first = false;
  }
  o << "]}";
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
    write_text("{\"recipe\":" + l.recipe + ",\"input_arguments\":" + ports + "}", buf, cap, needed);
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
