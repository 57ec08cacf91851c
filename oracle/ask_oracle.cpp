// ask_oracle -- TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline).
//
// A CPU restatement of ASK's host-path semantics for the data-parallel hot path
// (fused elementwise loops, reductions, gather, scatter_add).  Only tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may load
// it; nothing in the ask_b200 product links, imports or calls it.
//
// Parity status: PARTIALLY PINNED.  The reference's own tests hold no numeric
// golden vectors for this path (tests/cpp/primitives.cpp pins only emitted-IR
// structure) and its compiler half needs an LLVM/MLIR 23.1 SDK that is absent
// here, so the reference cannot be run to produce vectors.  The restatement is
// pinned against the known answers the reference documents in prose
// (docs/en/ir.md:69, 77, 108-121; include/ask/LLIR/Numeric.h:36-37) via
// tests/golden/, and is otherwise unpinned; transcendental results (expf, tanhf,
// ...) come from the host libm exactly as the reference's host path calls them
// (lib/Lowering/ScalarEmitter.h:149, 153, 246-259).
//
// Each function cites the reference code it restates.  Build flags mirror the
// reference's host codegen: no floating-point contraction
// (lib/Lowering/Host.cpp:51, -ffp-contract=off), no fast-math.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// Element types and opcodes (numbering private to the oracle; callers use the
// names through orc_op_code / orc_dtype_code).
enum { T_BOOL = 0, T_I32, T_I64, T_F32, T_F16, T_BF16 };
const char* const kTypes[] = {"bool", "i32", "i64", "f32", "f16", "bf16"};

enum {
  O_INPUT = 0, O_CONST, O_CAST, O_ADD, O_MUL, O_DIV, O_FLOORDIV, O_MOD, O_POW, O_MAXIMUM, O_MINIMUM,
  O_AND, O_OR, O_XOR, O_SHL, O_SHR, O_NOT, O_ABS, O_EXP, O_LOG, O_SQRT, O_SIN, O_COS, O_TANH, O_ERF,
  O_FLOOR, O_CEIL, O_ROUND, O_CMP, O_SELECT, O_COUNT
};
const char* const kOps[] = {"input", "const", "cast", "add", "mul", "div", "floordiv", "mod", "pow",
                            "maximum", "minimum", "bitwise_and", "bitwise_or", "bitwise_xor",
                            "shift_left", "shift_right", "bitwise_not", "abs", "exp", "log", "sqrt",
                            "sin", "cos", "tanh", "erf", "floor", "ceil", "round", "compare", "select"};

enum { R_SUM = 0, R_PROD, R_MAX, R_MIN, R_ANY, R_ALL, R_ARGMAX, R_ARGMIN };
const char* const kReds[] = {"sum", "prod", "max", "min", "any", "all", "argmax", "argmin"};

bool is_float(int t) { return t == T_F32 || t == T_F16 || t == T_BF16; }

float f_of(uint32_t b) { float f; std::memcpy(&f, &b, 4); return f; }
uint32_t b_of(float f) { uint32_t b; std::memcpy(&b, &f, 4); return b; }

// bf16: extend is a 16-bit shift; truncation rounds to nearest even and a NaN
// keeps its top bits with the quiet bit set (include/ask/LLIR/Numeric.h:21-34).
uint32_t bf16_round_bits(float f) {
  const uint32_t x = b_of(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (x >> 16) | 0x40u;
  return (x + 0x7fffu + ((x >> 16) & 1u)) >> 16;
}
float bf16_value(uint32_t h) { return f_of(h << 16); }

// f16 through the compiler's IEEE binary16 type (libgcc conversion routines):
// fptrunc/fpext semantics of Numeric.h:107-110.
uint32_t f16_round_bits(float f) {
  _Float16 h = static_cast<_Float16>(f);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}
float f16_value(uint32_t bits) {
  uint16_t b = uint16_t(bits);
  _Float16 h;
  std::memcpy(&h, &b, 2);
  return static_cast<float>(h);
}

float round_type(int t, float f) {
  if (t == T_F16) return f16_value(f16_round_bits(f));
  if (t == T_BF16) return bf16_value(bf16_round_bits(f));
  return f;
}

// llvm.maximum / llvm.minimum (ScalarEmitter.h:181-200): NaN if either operand
// is NaN, and -0 orders below +0.
float maximum_f(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}
float minimum_f(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  if (a == b) return std::signbit(a) ? a : b;
  return a < b ? a : b;
}

// Integer semantics on a signed value of `bits` width held in int64.
int64_t wrap(int64_t v, int bits) { return bits == 32 ? int64_t(int32_t(uint32_t(uint64_t(v)))) : v; }

int64_t int_op(int op, int bits, int64_t x, int64_t y) {
  const int64_t mn = bits == 32 ? int64_t(INT32_MIN) : INT64_MIN;
  switch (op) {
    case O_ADD: return wrap(int64_t(uint64_t(x) + uint64_t(y)), bits);             // ScalarEmitter.h:140
    case O_MUL: return wrap(int64_t(uint64_t(x) * uint64_t(y)), bits);             // ScalarEmitter.h:141
    case O_MAXIMUM: return x > y ? x : y;                                           // ScalarEmitter.h:183-184
    case O_MINIMUM: return x < y ? x : y;                                           // ScalarEmitter.h:193-194
    case O_AND: return x & y;
    case O_OR: return x | y;
    case O_XOR: return x ^ y;
    case O_NOT: return wrap(~x, bits);
    case O_ABS: return x < 0 ? wrap(int64_t(0ull - uint64_t(x)), bits) : x;          // ScalarEmitter.h:225-229
    case O_SHL:  // ScalarEmitter.h:100-108: in-range counts shift, all others give 0
      return (y >= 0 && y < bits) ? wrap(int64_t(uint64_t(x) << y), bits) : 0;
    case O_SHR:  // ScalarEmitter.h:109-113: arithmetic; counts >= width sign-fill, negative give 0
      if (y >= 0 && y < bits) return x >> y;
      return y >= 0 ? (x < 0 ? -1 : 0) : 0;
    case O_FLOORDIV:
    case O_MOD: {  // ScalarEmitter.h:117-139
      const bool zero = y == 0, overflow = x == mn && y == -1;
      if (zero) return 0;
      if (overflow) return op == O_FLOORDIV ? mn : 0;
      const int64_t q = x / y, r = x % y;
      const bool adj = r != 0 && ((r ^ y) < 0);
      return op == O_FLOORDIV ? (adj ? q - 1 : q) : (adj ? r + y : r);
    }
    case O_POW: {  // ScalarEmitter.h:57-93
      if (y < 0) return x == 1 ? 1 : x == -1 ? ((y & 1) ? -1 : 1) : 0;
      int64_t res = 1, cur = x;
      for (uint64_t k = uint64_t(y); k; k >>= 1) {
        if (k & 1) res = wrap(int64_t(uint64_t(res) * uint64_t(cur)), bits);
        cur = wrap(int64_t(uint64_t(cur) * uint64_t(cur)), bits);
      }
      return res;
    }
    default: return 0;
  }
}

// Floored float modulo (ScalarEmitter.h:152-158).
float fmod_floor(float l, float r) {
  const float rem = std::fmod(l, r);
  const bool nonzero = !std::isnan(rem) && rem != 0.0f;
  const bool diff = (rem < 0.0f) != (r < 0.0f);
  return (nonzero && diff) ? rem + r : rem;
}

float float_op(int op, float x, float y) {
  switch (op) {
    case O_ADD: return x + y;
    case O_MUL: return x * y;
    case O_DIV: return x / y;
    case O_FLOORDIV: return std::floor(x / y);
    case O_MOD: return fmod_floor(x, y);
    case O_POW: return std::pow(x, y);
    case O_MAXIMUM: return maximum_f(x, y);
    case O_MINIMUM: return minimum_f(x, y);
    case O_ABS: return std::fabs(x);
    case O_EXP: return std::exp(x);
    case O_LOG: return std::log(x);
    case O_SQRT: return std::sqrt(x);
    case O_SIN: return std::sin(x);
    case O_COS: return std::cos(x);
    case O_TANH: return std::tanh(x);
    case O_ERF: return std::erf(x);
    case O_FLOOR: return std::floor(x);
    case O_CEIL: return std::ceil(x);
    case O_ROUND: return std::nearbyint(x);  // rint: ties to even
    default: return x;
  }
}

// Integer -> f16/bf16 in one rounding step from the exact integer
// (Numeric.h:36-76).  Written from the definition: round the magnitude to the
// destination's significand width, ties to even.
float int_to_small_float(int64_t v, int t) {
  if (v == 0) return 0.0f;
  const int man = t == T_F16 ? 10 : 7;
  const bool neg = v < 0;
  uint64_t m = neg ? 0ull - uint64_t(v) : uint64_t(v);
  int e = 63;
  while (!(m >> e)) --e;
  const int drop = e > man ? e - man : 0;
  uint64_t sig = m >> drop;
  if (drop) {
    const uint64_t rem = m & ((1ull << drop) - 1), half = 1ull << (drop - 1);
    if (rem > half || (rem == half && (sig & 1))) ++sig;
  }
  const double mag = std::ldexp(double(sig), drop);
  if (t == T_F16) {
    if (mag > 65504.0) return neg ? -INFINITY : INFINITY;  // rounded past the largest finite f16
    return neg ? -float(mag) : float(mag);
  }
  return neg ? -float(mag) : float(mag);  // bf16 magnitudes here are exact in f32
}

// Numeric cast on a value word (Numeric.h:78-111).  Words: ints as int64,
// floats as the f32 value (f16/bf16 already rounded), bool 0/1.
struct Word {
  int64_t i;
  float f;
};

Word cast_word(int st, int dt, Word a) {
  Word r{0, 0.0f};
  if (st == dt) return a;
  if (dt == T_BOOL) {
    r.i = is_float(st) ? !(a.f == 0.0f) : (a.i != 0);  // une: NaN -> true
    return r;
  }
  if (st == T_BOOL) {
    if (dt == T_I32 || dt == T_I64) r.i = a.i & 1;
    else r.f = (a.i & 1) ? 1.0f : 0.0f;
    return r;
  }
  if (st == T_I32 || st == T_I64) {
    if (dt == T_I32) r.i = wrap(a.i, 32);
    else if (dt == T_I64) r.i = a.i;
    else if (dt == T_F32) r.f = float(a.i);  // sitofp, round to nearest even
    else r.f = int_to_small_float(a.i, dt);
    return r;
  }
  if (dt == T_I32 || dt == T_I64) {  // fptosi.sat (Numeric.h:100-102)
    const float x = a.f;
    const double lim = dt == T_I32 ? 2147483648.0 : 9223372036854775808.0;
    if (std::isnan(x)) r.i = 0;
    else if (double(x) >= lim) r.i = dt == T_I32 ? INT32_MAX : INT64_MAX;
    else if (double(x) < -lim) r.i = dt == T_I32 ? INT32_MIN : INT64_MIN;
    else r.i = int64_t(x);
    return r;
  }
  r.f = round_type(dt, a.f);  // f32/f16/bf16 conversions, all via the f32 value
  return r;
}

bool compare_word(int st, int pred, Word a, Word b) {
  if (is_float(st)) {
    const float x = a.f, y = b.f;
    switch (pred) {
      case 0: return x == y;
      case 1: return !(x == y);  // une
      case 2: return x < y;
      case 3: return x <= y;
      case 4: return x > y;
      default: return x >= y;
    }
  }
  int64_t x = a.i, y = b.i;
  if (st == T_BOOL) { x &= 1; y &= 1; }  // unsigned, values 0/1
  switch (pred) {
    case 0: return x == y;
    case 1: return x != y;
    case 2: return x < y;
    case 3: return x <= y;
    case 4: return x > y;
    default: return x >= y;
  }
}

struct Insn {
  int32_t op, type, a, b, c, aux, src_type, pad;
  uint64_t imm;
};

Word const_word(int t, uint64_t imm) {
  Word w{0, 0.0f};
  if (t == T_BOOL) w.i = imm & 1;
  else if (t == T_I32) w.i = int64_t(int32_t(uint32_t(imm)));
  else if (t == T_I64) w.i = int64_t(imm);
  else w.f = f_of(uint32_t(imm));
  return w;
}

Word eval(const Insn& x, Word a, Word b, Word c) {
  switch (x.op) {
    case O_CONST: return const_word(x.type, x.imm);
    case O_CAST: return cast_word(x.src_type, x.type, a);
    case O_SELECT: return (a.i & 1) ? b : c;
    case O_CMP: { Word r{compare_word(x.src_type, x.aux, a, b) ? 1 : 0, 0.0f}; return r; }
    default: break;
  }
  Word r{0, 0.0f};
  if (x.type == T_BOOL) {
    const int64_t p = a.i & 1, q = b.i & 1;
    switch (x.op) {
      case O_AND: case O_MINIMUM: r.i = p & q; break;  // ScalarEmitter.h:192
      case O_OR: case O_MAXIMUM: r.i = p | q; break;   // ScalarEmitter.h:182
      case O_XOR: r.i = p ^ q; break;
      case O_NOT: r.i = p ^ 1; break;
      default: break;
    }
    return r;
  }
  if (x.type == T_I32 || x.type == T_I64) {
    r.i = int_op(x.op, x.type == T_I32 ? 32 : 64, a.i, b.i);
    return r;
  }
  // float: f16/bf16 widen to f32, compute, round back (ScalarEmitter.h:161-179, 234, 261)
  r.f = round_type(x.type, float_op(x.op, a.f, b.f));
  return r;
}

Word load_word(int t, const void* p, uint64_t i) {
  Word w{0, 0.0f};
  switch (t) {
    case T_BOOL: w.i = static_cast<const uint8_t*>(p)[i] != 0; break;
    case T_I32: w.i = static_cast<const int32_t*>(p)[i]; break;
    case T_I64: w.i = static_cast<const int64_t*>(p)[i]; break;
    case T_F32: w.f = static_cast<const float*>(p)[i]; break;
    case T_F16: w.f = f16_value(static_cast<const uint16_t*>(p)[i]); break;
    default: w.f = bf16_value(static_cast<const uint16_t*>(p)[i]); break;
  }
  return w;
}
void store_word(int t, void* p, uint64_t i, Word w) {
  switch (t) {
    case T_BOOL: static_cast<uint8_t*>(p)[i] = uint8_t(w.i & 1); break;
    case T_I32: static_cast<int32_t*>(p)[i] = int32_t(w.i); break;
    case T_I64: static_cast<int64_t*>(p)[i] = w.i; break;
    case T_F32: static_cast<float*>(p)[i] = w.f; break;
    case T_F16: static_cast<uint16_t*>(p)[i] = uint16_t(f16_round_bits(w.f)); break;
    default: static_cast<uint16_t*>(p)[i] = uint16_t(bf16_round_bits(w.f)); break;
  }
}

// Index maps of the oracle's program ports: 0 full, 1 scalar, 2 outer (i / inner
// for elementwise; the output index for reductions), 3 inner (i % inner).
uint64_t map_ew(int m, uint64_t i, uint64_t inner) {
  return m == 0 ? i : m == 1 ? 0 : m == 2 ? i / inner : i % inner;
}

void run_program(const Insn* prog, int n, const int* in_types, const void* const* inputs,
                 std::vector<Word>& r, const uint64_t* in_index) {
  for (int k = 0; k < n; ++k) {
    const Insn& x = prog[k];
    if (x.op == O_INPUT) r[k] = load_word(in_types[x.a], inputs[x.a], in_index[x.a]);
    else r[k] = eval(x, r[x.a], r[x.b], r[x.c]);
  }
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) and the input mappings.
void philox(uint64_t seed, uint32_t stream, uint64_t index, uint32_t out[4]) {
  uint32_t c0 = uint32_t(index), c1 = uint32_t(index >> 32), c2 = stream, c3 = 0;
  uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
  for (int round = 0; round < 10; ++round) {
    const uint64_t p0 = uint64_t(0xD2511F53u) * c0, p1 = uint64_t(0xCD9E8D57u) * c2;
    const uint32_t hi0 = uint32_t(p0 >> 32), lo0 = uint32_t(p0), hi1 = uint32_t(p1 >> 32), lo1 = uint32_t(p1);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

std::vector<double> zipf_cdf(double s, uint64_t n) {
  std::vector<double> cdf(n);
  double acc = 0.0;
  for (uint64_t k = 0; k < n; ++k) { acc += std::pow(double(k + 1), -s); cdf[k] = acc; }
  return cdf;
}

template <class F>
void parallel_for(uint64_t n, int threads, F&& body) {
  if (threads <= 1 || n < 4096) { body(0, n, 0); return; }
  std::vector<std::thread> pool;
  const uint64_t per = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const uint64_t b = std::min(n, per * t), e = std::min(n, b + per);
    pool.emplace_back([&, b, e, t] { body(b, e, t); });
  }
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

int orc_dtype_code(const char* name) {
  for (int t = 0; t < 6; ++t) if (!std::strcmp(name, kTypes[t])) return t;
  return -1;
}
int orc_op_code(const char* name) {
  for (int o = 0; o < O_COUNT; ++o) if (!std::strcmp(name, kOps[o])) return o;
  return -1;
}
int orc_red_code(const char* name) {
  for (int o = 0; o < 8; ++o) if (!std::strcmp(name, kReds[o])) return o;
  return -1;
}

// ---- scalar semantics, exposed for known-answer tests ----------------------
uint32_t orc_f32_to_bf16(float f) { return bf16_round_bits(f); }
float orc_bf16_to_f32(uint32_t h) { return bf16_value(h); }
uint32_t orc_f32_to_f16(float f) { return f16_round_bits(f); }
float orc_f16_to_f32(uint32_t h) { return f16_value(h); }
float orc_maximum(float a, float b) { return maximum_f(a, b); }
float orc_minimum(float a, float b) { return minimum_f(a, b); }
int64_t orc_int_op(int op, int type, int64_t a, int64_t b) { return int_op(op, type == T_I32 ? 32 : 64, a, b); }
// Cast of one value; `in` and `out` hold the source/destination word as
// (int64, f32 value).  Returns the destination's storage bits.
uint64_t orc_cast_bits(int st, int dt, int64_t ival, float fval) {
  Word w = cast_word(st, dt, Word{ival, fval});
  uint8_t buf[8] = {0};
  store_word(dt, buf, 0, w);
  uint64_t bits = 0;
  std::memcpy(&bits, buf, 8);
  return bits;
}

void orc_philox(uint64_t seed, uint32_t stream, uint64_t index, uint32_t* out) { philox(seed, stream, index, out); }

// Same mappings as the device generator (kinds as in ask_b200_generate).
void orc_generate(int kind, uint64_t seed, uint32_t stream, uint64_t offset, uint64_t count, double p0, double p1,
                  void* dst, int threads) {
  std::vector<double> cdf;
  if (kind == 5 || kind == 6) cdf = zipf_cdf(p0, uint64_t(p1));
  parallel_for(count, threads, [&](uint64_t b, uint64_t e, int) {
    for (uint64_t t = b; t < e; ++t) {
      uint32_t r[4];
      philox(seed, stream, offset + t, r);
      switch (kind) {
        case 0: static_cast<float*>(dst)[t] = float(p0 + (p1 - p0) * (double(r[0] >> 8) * (1.0 / 16777216.0))); break;
        case 4: static_cast<int32_t*>(dst)[t] = int32_t(r[0]); break;
        case 5:
        case 6: {
          const uint64_t bits = (uint64_t(r[0] >> 5) << 26) | uint64_t(r[1] >> 6);
          const double target = double(bits) * (1.0 / 9007199254740992.0) * cdf.back();
          const uint64_t k = uint64_t(std::upper_bound(cdf.begin(), cdf.end(), target) - cdf.begin());
          const uint64_t idx = k < cdf.size() ? k : cdf.size() - 1;
          if (kind == 5) static_cast<int64_t*>(dst)[t] = int64_t(idx);
          else static_cast<int32_t*>(dst)[t] = int32_t(idx);
          break;
        }
        default: {
          const double u1 = (double(r[0]) + 1.0) * (1.0 / 4294967296.0);
          const double u2 = double(r[1]) * (1.0 / 4294967296.0);
          const double x = p0 + p1 * (std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
          if (kind == 1) static_cast<float*>(dst)[t] = float(x);
          else if (kind == 2) static_cast<uint16_t*>(dst)[t] = uint16_t(f16_round_bits(float(x)));
          else static_cast<uint16_t*>(dst)[t] = uint16_t(bf16_round_bits(float(x)));
          break;
        }
      }
    }
  });
}

// ---- fused elementwise step (lib/Lowering/Host.cpp:825-877: one shared i64
// loop over the batch, every output stored per index) ------------------------
int orc_elementwise(const Insn* prog, int n_insn, const int* in_types, const int* in_maps, int n_in,
                    const void* const* inputs, const int* out_regs, const int* out_types, int n_out,
                    void* const* outputs, uint64_t count, uint64_t inner, int threads) {
  if (n_in > 64 || n_insn <= 0) return -1;
  parallel_for(count, threads, [&](uint64_t b, uint64_t e, int) {
    std::vector<Word> r(static_cast<size_t>(n_insn));
    uint64_t idx[64];
    for (uint64_t i = b; i < e; ++i) {
      for (int k = 0; k < n_in; ++k) idx[k] = map_ew(in_maps[k], i, inner);
      run_program(prog, n_insn, in_types, inputs, r, idx);
      for (int k = 0; k < n_out; ++k) store_word(out_types[k], outputs[k], i, r[size_t(out_regs[k])]);
    }
  });
  return 0;
}

// ---- reductions over [outer, extent, inner] ------------------------------------
// sum_mode 0: float sums accumulate in f64 and round once (ground truth for
//             tolerance checks);
// sum_mode 1: float sums in f32 over 16 interleaved lanes combined pairwise --
//             the shape LLVM's reassoc vectorisation gives the host loop
//             (ScalarEmitter.h:167-176);
// sum_mode 2: float sums strictly sequential in f32 (the reference CUDA
//             thread-per-output loop, ScalarEmitter.h:263-287, 464-471).
// Everything else follows ScalarEmitter::reduce/argmaxmin exactly: initial
// values (426-439), NaN-propagating max/min, argmax/argmin taking a candidate
// iff it is NaN and the best is not, or strictly better (506-517).
int orc_reduce(const Insn* prog, int n_insn, const int* in_types, const int* in_maps, int n_in,
               const void* const* inputs, const int* val_regs, int n_red, const int* red_ops,
               const int* red_src, void* const* outputs, uint64_t outer, uint64_t extent, uint64_t inner,
               uint64_t index_base, int sum_mode, int threads) {
  if (n_in > 64 || n_insn <= 0 || n_red > 8) return -1;
  const uint64_t n_out = outer * inner;
  parallel_for(n_out, threads, [&](uint64_t b, uint64_t e, int) {
    std::vector<Word> r(static_cast<size_t>(n_insn));
    uint64_t idx[64];
    for (uint64_t oi = b; oi < e; ++oi) {
      const uint64_t o = oi / inner, n = oi % inner;
      for (int k = 0; k < n_red; ++k) {
        const int op = red_ops[k];
        const int vreg = val_regs[red_src[k]];
        const int vt = prog[vreg].type;
        const bool fl = is_float(vt);
        auto value_at = [&](uint64_t ei) -> Word {
          const uint64_t full = (o * extent + ei) * inner + n;
          for (int q = 0; q < n_in; ++q) idx[q] = in_maps[q] == 0 ? full : in_maps[q] == 1 ? 0 : oi;
          run_program(prog, n_insn, in_types, inputs, r, idx);
          return r[size_t(vreg)];
        };
        Word res{0, 0.0f};
        int out_t = vt;
        if (op == R_ARGMAX || op == R_ARGMIN) {
          out_t = T_I64;
          const bool mx = op == R_ARGMAX;
          Word best = value_at(0);
          int64_t bi = 0;
          for (uint64_t ei = 1; ei < extent; ++ei) {
            const Word c = value_at(ei);
            bool take;
            if (fl) {
              const bool cn = std::isnan(c.f), bn = std::isnan(best.f);
              take = (cn && !bn) || (mx ? c.f > best.f : c.f < best.f);
            } else if (vt == T_BOOL) {
              take = mx ? (c.i & 1) > (best.i & 1) : (c.i & 1) < (best.i & 1);
            } else {
              take = mx ? c.i > best.i : c.i < best.i;
            }
            if (take) { best = c; bi = int64_t(ei); }
          }
          res.i = bi + int64_t(index_base);
        } else if (op == R_SUM && fl) {
          if (sum_mode == 0) {
            double acc = 0.0;
            for (uint64_t ei = 0; ei < extent; ++ei) acc += double(value_at(ei).f);
            res.f = round_type(vt, float(acc));
          } else if (sum_mode == 1) {
            float lanes[16] = {0};
            for (uint64_t ei = 0; ei < extent; ++ei) lanes[ei % 16] = lanes[ei % 16] + value_at(ei).f;
            for (int w = 8; w; w >>= 1)
              for (int l = 0; l < w; ++l) lanes[l] = lanes[l] + lanes[l + w];
            res.f = round_type(vt, lanes[0]);
          } else {
            float acc = 0.0f;
            for (uint64_t ei = 0; ei < extent; ++ei) acc = acc + value_at(ei).f;
            res.f = round_type(vt, acc);
          }
        } else {
          // initial values: ScalarEmitter.h:426-439 (bool max/min start from the
          // i1 signed min/max, true/false, and fold with or/and)
          Word acc{0, 0.0f};
          switch (op) {
            case R_SUM: acc.i = 0; break;
            case R_PROD: acc.i = 1; acc.f = 1.0f; break;
            case R_MAX: acc.i = vt == T_I32 ? INT32_MIN : vt == T_I64 ? INT64_MIN : 1; acc.f = -INFINITY; break;
            case R_MIN: acc.i = vt == T_I32 ? INT32_MAX : vt == T_I64 ? INT64_MAX : 0; acc.f = INFINITY; break;
            case R_ANY: acc.i = 0; break;
            default: acc.i = 1; break;
          }
          if (op == R_ANY || op == R_ALL) out_t = T_BOOL;
          for (uint64_t ei = 0; ei < extent; ++ei) {
            const Word v = value_at(ei);
            switch (op) {
              case R_SUM: acc.i = int_op(O_ADD, vt == T_I32 ? 32 : 64, acc.i, v.i); break;
              case R_PROD:
                if (fl) acc.f = acc.f * v.f;  // f32 accumulation (warp path, ScalarEmitter.h:311-336)
                else acc.i = int_op(O_MUL, vt == T_I32 ? 32 : 64, acc.i, v.i);
                break;
              case R_MAX:
                if (fl) acc.f = maximum_f(acc.f, v.f);
                else if (vt == T_BOOL) acc.i = (acc.i | v.i) & 1;
                else acc.i = v.i > acc.i ? v.i : acc.i;
                break;
              case R_MIN:
                if (fl) acc.f = minimum_f(acc.f, v.f);
                else if (vt == T_BOOL) acc.i = (acc.i & v.i) & 1;
                else acc.i = v.i < acc.i ? v.i : acc.i;
                break;
              case R_ANY: acc.i = (acc.i | v.i) & 1; break;
              default: acc.i = (acc.i & v.i) & 1; break;
            }
          }
          if (fl) acc.f = round_type(vt, acc.f);
          res = acc;
        }
        store_word(out_t, outputs[k], oi, res);
      }
    }
  });
  return 0;
}

// ---- gather / scatter_add over [outer, dim, inner] with n indices -----------------
// gather: out-of-bounds index -> zeros (ScalarEmitter.h:787-815); i32 indices
// sign-extend (786).  Raw element copy.
int orc_gather(const void* table, const void* index, int index_is_i32, void* out, uint64_t outer, uint64_t dim,
               uint64_t inner, uint64_t n, int elem_bytes, int threads) {
  parallel_for(outer * n, threads, [&](uint64_t b, uint64_t e, int) {
    for (uint64_t row = b; row < e; ++row) {
      const uint64_t o = row / n, j = row % n;
      const int64_t idx = index_is_i32 ? int64_t(static_cast<const int32_t*>(index)[j])
                                       : static_cast<const int64_t*>(index)[j];
      char* dst = static_cast<char*>(out) + row * inner * elem_bytes;
      if (idx < 0 || uint64_t(idx) >= dim) std::memset(dst, 0, inner * elem_bytes);
      else std::memcpy(dst, static_cast<const char*>(table) + (o * dim + uint64_t(idx)) * inner * elem_bytes,
                       inner * elem_bytes);
    }
  });
  return 0;
}

// scatter_add: copy base, then add every in-bounds update in update order
// (lib/Lowering/Host.cpp:677-772).  mode 0: accumulate in the element type
// (the reference host path); mode 1 (f32 only): accumulate in f64 into `out64`
// together with sum|upd| into `abs64`, for tolerance checks.
int orc_scatter_add(int type, const void* base, const void* index, int index_is_i32, const void* upd, void* out,
                    double* out64, double* abs64, uint64_t outer, uint64_t dim, uint64_t inner, uint64_t n, int mode) {
  const uint64_t table = outer * dim * inner;
  const int es = type == T_I64 ? 8 : (type == T_F16 || type == T_BF16) ? 2 : type == T_BOOL ? 1 : 4;
  if (mode == 0) std::memcpy(out, base, table * es);
  else for (uint64_t i = 0; i < table; ++i) { out64[i] = static_cast<const float*>(base)[i]; abs64[i] = 0.0; }
  for (uint64_t o = 0; o < outer; ++o)
    for (uint64_t j = 0; j < n; ++j) {
      const int64_t idx = index_is_i32 ? int64_t(static_cast<const int32_t*>(index)[j])
                                       : static_cast<const int64_t*>(index)[j];
      if (idx < 0 || uint64_t(idx) >= dim) continue;
      const uint64_t d0 = (o * dim + uint64_t(idx)) * inner, s0 = (o * n + j) * inner;
      for (uint64_t c = 0; c < inner; ++c) {
        if (mode == 1) {
          const double u = static_cast<const float*>(upd)[s0 + c];
          out64[d0 + c] += u;
          abs64[d0 + c] += std::fabs(u);
          continue;
        }
        const Word cur = load_word(type, out, d0 + c), u = load_word(type, upd, s0 + c);
        Word r{0, 0.0f};
        if (type == T_I32 || type == T_I64) r.i = int_op(O_ADD, type == T_I32 ? 32 : 64, cur.i, u.i);
        else r.f = round_type(type, cur.f + u.f);
        store_word(type, out, d0 + c, r);
      }
    }
  return 0;
}

// ---- whole-config restatements used by the CPU baseline ----------------------------
// cfg1: y0 = exp(a)*b + c, y1 = max(a,b) + tanh(c)*(-1), one fused loop.
void orc_cfg1(const float* a, const float* b, const float* c, float* y0, float* y1, uint64_t n, int threads) {
  parallel_for(n, threads, [&](uint64_t lo, uint64_t hi, int) {
    for (uint64_t i = lo; i < hi; ++i) {
      const float e = std::exp(a[i]);
      y0[i] = e * b[i] + c[i];
      y1[i] = maximum_f(a[i], b[i]) + std::tanh(c[i]) * -1.0f;
    }
  });
}

// cfg5b: ((x << 3) ^ (x >> 5)) & 0x7fffffff + y on i32 (wrapping add).
void orc_cfg5b(const int32_t* x, const int32_t* y, int32_t* z, uint64_t n, int threads) {
  parallel_for(n, threads, [&](uint64_t lo, uint64_t hi, int) {
    for (uint64_t i = lo; i < hi; ++i) {
      const uint32_t v = uint32_t(x[i]);
      const uint32_t t = ((v << 3) ^ uint32_t(x[i] >> 5)) & 0x7fffffffu;
      z[i] = int32_t(t + uint32_t(y[i]));
    }
  });
}

// cfg5a: sum, min and argmin over a flat f32 vector.  sum64 is the f64 ground
// truth; sum_ref is the reference host loop's f32 result (16 interleaved f32
// lanes per thread partition, see orc_reduce sum_mode 1); min/argmin follow
// ScalarEmitter.h:473-529 (first NaN wins, ties keep the lowest index).
void orc_cfg5a(const float* x, uint64_t n, uint64_t index_base, double* sum64, float* sum_ref, float* mn,
               int64_t* argmin, int threads) {
  const int T = threads < 1 ? 1 : threads;
  std::vector<double> s64(T, 0.0);
  std::vector<float> sref(T, 0.0f), mv(T, INFINITY);
  std::vector<int64_t> mi(T, -1);
  parallel_for(n, T, [&](uint64_t lo, uint64_t hi, int t) {
    double acc = 0.0;
    float lanes[16] = {0};
    float best = 0.0f;
    int64_t bi = -1;
    for (uint64_t i = lo; i < hi; ++i) {
      const float v = x[i];
      acc += double(v);
      lanes[i & 15] = lanes[i & 15] + v;
      if (bi < 0) { best = v; bi = int64_t(i); continue; }
      if ((std::isnan(v) && !std::isnan(best)) || v < best) { best = v; bi = int64_t(i); }
    }
    for (int w = 8; w; w >>= 1)
      for (int l = 0; l < w; ++l) lanes[l] = lanes[l] + lanes[l + w];
    s64[t] = acc; sref[t] = lanes[0]; mv[t] = best; mi[t] = bi;
  });
  double total = 0.0;
  float tref = 0.0f;
  float best = 0.0f;
  int64_t bi = -1;
  for (int t = 0; t < T; ++t) {
    total += s64[t];
    tref = tref + sref[t];
    if (mi[t] < 0) continue;
    if (bi < 0 || (std::isnan(mv[t]) && !std::isnan(best)) || mv[t] < best) { best = mv[t]; bi = mi[t]; }
  }
  *sum64 = total;
  *sum_ref = tref;
  *mn = best;
  *argmin = bi < 0 ? -1 : bi + int64_t(index_base);
}

// Canonical softmax partition (three owned steps; lib/Frontend/Partition.cpp:126-132):
//   m = max_j cast(x, f32); s = sum_j exp(cast(x) + m*(-1)); y = cast(exp(cast(x) + m*(-1)) / s, T)
// s accumulates in f64 and rounds to f32 once (the reference folds it in f32
// on the warp path; the tolerance covers the difference).  type: 4 f16, 5 bf16.
void orc_softmax(int type, const uint16_t* x, uint64_t rows, uint64_t cols, float* m, float* s, uint16_t* y,
                 int threads) {
  parallel_for(rows, threads, [&](uint64_t lo, uint64_t hi, int) {
    for (uint64_t r = lo; r < hi; ++r) {
      const uint16_t* xr = x + r * cols;
      auto val = [&](uint64_t j) { return type == T_F16 ? f16_value(xr[j]) : bf16_value(xr[j]); };
      float mx = -INFINITY;
      for (uint64_t j = 0; j < cols; ++j) mx = maximum_f(mx, val(j));
      double acc = 0.0;
      for (uint64_t j = 0; j < cols; ++j) acc += double(std::exp(val(j) + mx * -1.0f));
      const float sum = float(acc);
      m[r] = mx;
      s[r] = sum;
      if (y)
        for (uint64_t j = 0; j < cols; ++j) {
          const float q = std::exp(val(j) + mx * -1.0f) / sum;
          y[r * cols + j] = uint16_t(type == T_F16 ? f16_round_bits(q) : bf16_round_bits(q));
        }
    }
  });
}

// cfg2 row statistics: sum (f64 ground truth), max, min, argmax per row.
void orc_rowstats(const float* x, uint64_t rows, uint64_t cols, float* sum, float* mx, float* mn, int64_t* am,
                  int threads) {
  parallel_for(rows, threads, [&](uint64_t lo, uint64_t hi, int) {
    for (uint64_t r = lo; r < hi; ++r) {
      const float* xr = x + r * cols;
      double acc = 0.0;
      float a = -INFINITY, b = INFINITY, best = xr[0];
      int64_t bi = 0;
      for (uint64_t j = 0; j < cols; ++j) {
        const float v = xr[j];
        acc += double(v);
        a = maximum_f(a, v);
        b = minimum_f(b, v);
        if (j && ((std::isnan(v) && !std::isnan(best)) || v > best)) { best = v; bi = int64_t(j); }
      }
      sum[r] = float(acc);
      mx[r] = a;
      mn[r] = b;
      am[r] = bi;
    }
  });
}

}  // extern "C"
