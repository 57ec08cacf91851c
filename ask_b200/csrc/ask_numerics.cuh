// Device-side element semantics of ASK's owned CUDA path, restated for sm_100a.
//
// Every function here follows one rule of the reference and cites it:
//   * maximum/minimum: llvm.maximum/llvm.minimum in f32 -- NaN propagates and
//     -0 < +0 (lib/Lowering/ScalarEmitter.h:181-200, docs/en/ir.md:69).
//   * guarded shifts (ScalarEmitter.h:100-114), total integer floordiv/mod
//     (ScalarEmitter.h:117-139), wrapping add/mul (ScalarEmitter.h:140-141),
//     integer pow by squaring with the negative-exponent rule (ScalarEmitter.h:57-93).
//   * casts (include/ask/LLIR/Numeric.h:78-111): bf16 RNE with NaN quieting
//     (Numeric.h:25-34), integer -> f16/bf16 by a single rounding
//     (Numeric.h:36-76), saturating float -> int with NaN -> 0 (Numeric.h:100-102).
//   * float ops run in f32 and round back to f16/bf16 (ScalarEmitter.h:161-179).
// Floating add/mul/div use the explicit _rn intrinsics, so no multiply-add is
// ever contracted (the reference compiles with fp-contract=off,
// docs/en/codegen.md:55-57); the library is also built with -fmad=false.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "ask_types.h"

namespace askb {

// ---- bit helpers ------------------------------------------------------------
__device__ __forceinline__ float f32_of(uint64_t w) { return __uint_as_float(uint32_t(w)); }
__device__ __forceinline__ uint64_t w_of_f32(float f) { return uint64_t(__float_as_uint(f)); }
__device__ __forceinline__ int32_t i32_of(uint64_t w) { return int32_t(uint32_t(w)); }
__device__ __forceinline__ uint64_t w_of_i32(int32_t v) { return uint64_t(uint32_t(v)); }

// f32 -> bf16 bits, round to nearest even; NaN keeps its sign and top payload
// bits with the quiet bit forced (Numeric.h:25-34).
__device__ __forceinline__ uint32_t bf16_bits_rne(float f) {
  const uint32_t bits = __float_as_uint(f);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return (bits >> 16) | 0x40u;
  const uint32_t lsb = (bits >> 16) & 1u;
  return (bits + 0x7fffu + lsb) >> 16;
}
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float round_bf16(float f) { return bf16_bits_to_f32(bf16_bits_rne(f)); }
// f32 -> f16 is LLVM fptrunc, i.e. cvt.rn.f16.f32 on NVPTX (Numeric.h:107-110).
__device__ __forceinline__ float round_f16(float f) { return __half2float(__float2half_rn(f)); }

__device__ __forceinline__ float round_to(int type, float f) {
  return type == kF16 ? round_f16(f) : type == kBF16 ? round_bf16(f) : f;
}

// llvm.maximum / llvm.minimum on f32.  The NaN produced is the canonical
// 0x7fffffff that NVPTX's max.NaN/min.NaN return.
__device__ __forceinline__ float ask_maximum(float a, float b) {
  if (a != a || b != b) return __uint_as_float(0x7fffffffu);
  if (a == b) return __uint_as_float(__float_as_uint(a) & __float_as_uint(b));  // max(-0,+0)=+0
  return a > b ? a : b;
}
__device__ __forceinline__ float ask_minimum(float a, float b) {
  if (a != a || b != b) return __uint_as_float(0x7fffffffu);
  if (a == b) return __uint_as_float(__float_as_uint(a) | __float_as_uint(b));  // min(-0,+0)=-0
  return a < b ? a : b;
}

// ---- integers -----------------------------------------------------------------
template <class T> struct IntTraits;
template <> struct IntTraits<int32_t> { using U = uint32_t; static constexpr int kBits = 32; static constexpr int32_t kMin = INT32_MIN; };
template <> struct IntTraits<int64_t> { using U = uint64_t; static constexpr int kBits = 64; static constexpr int64_t kMin = INT64_MIN; };

template <class T> __device__ __forceinline__ T int_add(T a, T b) {
  using U = typename IntTraits<T>::U; return T(U(a) + U(b));
}
template <class T> __device__ __forceinline__ T int_mul(T a, T b) {
  using U = typename IntTraits<T>::U; return T(U(a) * U(b));
}
template <class T> __device__ __forceinline__ T int_shl(T x, T s) {
  using U = typename IntTraits<T>::U;
  return (s >= 0 && s < IntTraits<T>::kBits) ? T(U(x) << s) : T(0);
}
template <class T> __device__ __forceinline__ T int_shr(T x, T s) {
  if (s >= 0 && s < IntTraits<T>::kBits) return x >> s;  // arithmetic
  return s >= 0 ? (x < 0 ? T(-1) : T(0)) : T(0);
}
template <class T> __device__ __forceinline__ T int_floordiv(T l, T r) {
  const bool zero = r == 0, overflow = (l == IntTraits<T>::kMin) && (r == T(-1));
  if (zero) return 0;
  if (overflow) return IntTraits<T>::kMin;
  const T q = l / r, rem = l % r;
  return (rem != 0 && ((rem ^ r) < 0)) ? T(q - 1) : q;
}
template <class T> __device__ __forceinline__ T int_mod(T l, T r) {
  const bool zero = r == 0, overflow = (l == IntTraits<T>::kMin) && (r == T(-1));
  if (zero || overflow) return 0;
  const T rem = l % r;
  return (rem != 0 && ((rem ^ r) < 0)) ? T(rem + r) : rem;
}
template <class T> __device__ __forceinline__ T int_pow(T base, T e) {
  if (e < 0) {
    if (base == 1) return 1;
    if (base == -1) return (e & 1) ? T(-1) : T(1);
    return 0;
  }
  T result = 1, cur = base;
  for (T k = e; k != 0; k = T(typename IntTraits<T>::U(k) >> 1)) {
    if (k & 1) result = int_mul(result, cur);
    cur = int_mul(cur, cur);
  }
  return result;
}
template <class T> __device__ __forceinline__ T int_abs(T x) {
  using U = typename IntTraits<T>::U; return x < 0 ? T(U(0) - U(x)) : x;
}

// Saturating float -> signed integer, NaN -> 0 (llvm.fptosi.sat).
__device__ __forceinline__ int32_t f32_to_i32_sat(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x < -2147483648.0f) return INT32_MIN;
  return int32_t(x);
}
__device__ __forceinline__ int64_t f32_to_i64_sat(float x) {
  if (x != x) return 0;
  if (x >= 9223372036854775808.0f) return INT64_MAX;
  if (x < -9223372036854775808.0f) return INT64_MIN;
  return int64_t(x);
}

// Signed integer -> f16/bf16 with one round-to-nearest-even step on the
// 64-bit magnitude (the double-rounding hazard is described at
// Numeric.h:36-37).  Returns the f32 value of the rounded result.
__device__ __forceinline__ float int_to_low_float(int64_t v, int type) {
  const int frac = type == kF16 ? 10 : 7;
  const int bias = type == kF16 ? 15 : 127;
  if (v == 0) return 0.0f;
  const bool neg = v < 0;
  uint64_t mag = neg ? (0ull - uint64_t(v)) : uint64_t(v);
  int e = 63 - __clzll(mag);
  uint64_t sig;
  if (e > frac) {
    const int sh = e - frac;
    sig = mag >> sh;
    const uint64_t rem = mag & ((1ull << sh) - 1), half = 1ull << (sh - 1);
    if (rem > half || (rem == half && (sig & 1))) ++sig;
    if (sig == (1ull << (frac + 1))) { sig >>= 1; ++e; }
  } else {
    sig = mag << (frac - e);
  }
  uint32_t bits;
  if (type == kF16) {
    const int biased = e + bias;
    bits = biased >= 31 ? 0x7c00u : uint32_t((biased << frac) | int(sig & ((1u << frac) - 1)));
    bits |= neg ? 0x8000u : 0u;
    return __half2float(__ushort_as_half(uint16_t(bits)));
  }
  bits = uint32_t(((e + bias) << frac) | int(sig & ((1u << frac) - 1))) | (neg ? 0x8000u : 0u);
  return bf16_bits_to_f32(bits);
}

// createNumericCast (Numeric.h:78-111) on register words.
__device__ __forceinline__ uint64_t cast_word(int st, int dt, uint64_t a) {
  if (st == dt) return a;
  if (dt == kBool) {
    if (dtype_is_float(st)) return !(f32_of(a) == 0.0f) ? 1u : 0u;  // fcmp une: NaN is true
    if (st == kI32) return i32_of(a) != 0 ? 1u : 0u;
    return a != 0 ? 1u : 0u;
  }
  if (st == kBool) {
    const uint64_t one = a & 1u;
    if (dt == kI32 || dt == kI64) return one;
    return w_of_f32(one ? 1.0f : 0.0f);
  }
  if (st == kI32 || st == kI64) {
    const int64_t v = st == kI32 ? int64_t(i32_of(a)) : int64_t(a);
    if (dt == kI32) return w_of_i32(int32_t(v));
    if (dt == kI64) return uint64_t(v);
    if (dt == kF32) return w_of_f32(st == kI32 ? __int2float_rn(int32_t(v)) : __ll2float_rn(v));
    return w_of_f32(int_to_low_float(v, dt));
  }
  const float x = f32_of(a);  // f32, or an f16/bf16 value already widened
  if (dt == kI32) return w_of_i32(f32_to_i32_sat(x));
  if (dt == kI64) return uint64_t(f32_to_i64_sat(x));
  if (dt == kBF16) return w_of_f32(round_bf16(x));
  if (dt == kF16) return w_of_f32(round_f16(x));
  return a;  // f16/bf16 -> f32 is exact
}

__device__ __forceinline__ uint64_t compare_word(int st, int pred, uint64_t a, uint64_t b) {
  bool r;
  if (dtype_is_float(st)) {
    const float x = f32_of(a), y = f32_of(b);
    switch (pred) {
      case CMP_EQ: r = x == y; break;
      case CMP_NE: r = !(x == y); break;  // fcmp une: NaN satisfies only ne
      case CMP_LT: r = x < y; break;
      case CMP_LE: r = x <= y; break;
      case CMP_GT: r = x > y; break;
      default: r = x >= y; break;
    }
  } else if (st == kBool) {
    const uint32_t x = uint32_t(a & 1u), y = uint32_t(b & 1u);  // unsigned for bool
    switch (pred) {
      case CMP_EQ: r = x == y; break;
      case CMP_NE: r = x != y; break;
      case CMP_LT: r = x < y; break;
      case CMP_LE: r = x <= y; break;
      case CMP_GT: r = x > y; break;
      default: r = x >= y; break;
    }
  } else {
    const int64_t x = st == kI32 ? int64_t(i32_of(a)) : int64_t(a);
    const int64_t y = st == kI32 ? int64_t(i32_of(b)) : int64_t(b);
    switch (pred) {
      case CMP_EQ: r = x == y; break;
      case CMP_NE: r = x != y; break;
      case CMP_LT: r = x < y; break;
      case CMP_LE: r = x <= y; break;
      case CMP_GT: r = x > y; break;
      default: r = x >= y; break;
    }
  }
  return r ? 1u : 0u;
}

template <class T>
__device__ __forceinline__ T int_binary(int op, T x, T y) {
  switch (op) {
    case OP_ADD: return int_add(x, y);
    case OP_MUL: return int_mul(x, y);
    case OP_FLOORDIV: return int_floordiv(x, y);
    case OP_MOD: return int_mod(x, y);
    case OP_POW: return int_pow(x, y);
    case OP_MAXIMUM: return x > y ? x : y;
    case OP_MINIMUM: return x < y ? x : y;
    case OP_AND: return x & y;
    case OP_OR: return x | y;
    case OP_XOR: return x ^ y;
    case OP_SHL: return int_shl(x, y);
    case OP_SHR: return int_shr(x, y);
    case OP_NOT: return ~x;
    case OP_ABS: return int_abs(x);
    default: return 0;
  }
}

// Floored float modulo: fmod, then move a non-zero remainder whose sign
// differs from the divisor's into the divisor's sign (ScalarEmitter.h:152-158).
__device__ __forceinline__ float float_mod(float l, float r) {
  const float rem = fmodf(l, r);
  const bool nonzero = (rem == rem) && rem != 0.0f;  // fcmp one
  const bool diff = (rem < 0.0f) != (r < 0.0f);
  return (nonzero && diff) ? __fadd_rn(rem, r) : rem;
}

__device__ __forceinline__ float float_op(int op, float x, float y) {
  switch (op) {
    case OP_ADD: return __fadd_rn(x, y);
    case OP_MUL: return __fmul_rn(x, y);
    case OP_DIV: return __fdiv_rn(x, y);
    case OP_FLOORDIV: return floorf(__fdiv_rn(x, y));
    case OP_MOD: return float_mod(x, y);
    case OP_POW: return powf(x, y);
    case OP_MAXIMUM: return ask_maximum(x, y);
    case OP_MINIMUM: return ask_minimum(x, y);
    case OP_ABS: return fabsf(x);
    case OP_EXP: return expf(x);
    case OP_LOG: return logf(x);
    case OP_SQRT: return __fsqrt_rn(x);
    case OP_SIN: return sinf(x);
    case OP_COS: return cosf(x);
    case OP_TANH: return tanhf(x);
    case OP_ERF: return erff(x);
    case OP_FLOOR: return floorf(x);
    case OP_CEIL: return ceilf(x);
    case OP_ROUND: return rintf(x);  // ties to even
    default: return x;
  }
}

// Evaluate one instruction on register words.  With constant arguments (the
// specialised kernels) every switch folds away.
__device__ __forceinline__ uint64_t eval_insn(int op, int type, int st, int aux, uint64_t imm,
                                              uint64_t a, uint64_t b, uint64_t c) {
  if (op == OP_CONST) return imm;
  if (op == OP_CAST) return cast_word(st, type, a);
  if (op == OP_SELECT) return (a & 1u) ? b : c;
  if (op == OP_CMP) return compare_word(st, aux, a, b);
  if (type == kBool) {
    const uint64_t x = a & 1u, y = b & 1u;
    switch (op) {
      case OP_AND: case OP_MINIMUM: return x & y;
      case OP_OR: case OP_MAXIMUM: return x | y;
      case OP_XOR: return x ^ y;
      case OP_NOT: return x ^ 1u;
      default: return 0;
    }
  }
  if (type == kI32) return w_of_i32(int_binary<int32_t>(op, i32_of(a), i32_of(b)));
  if (type == kI64) return uint64_t(int_binary<int64_t>(op, int64_t(a), int64_t(b)));
  return w_of_f32(round_to(type, float_op(op, f32_of(a), f32_of(b))));
}

// ---- storage <-> register words ------------------------------------------------
__device__ __forceinline__ uint64_t word_from_storage(int type, const void* p, uint64_t i) {
  switch (type) {
    case kBool: return static_cast<const uint8_t*>(p)[i] != 0 ? 1u : 0u;
    case kI32: return w_of_i32(static_cast<const int32_t*>(p)[i]);
    case kI64: return static_cast<const uint64_t*>(p)[i];
    case kF32: return uint64_t(static_cast<const uint32_t*>(p)[i]);
    case kF16: return w_of_f32(__half2float(__ushort_as_half(static_cast<const uint16_t*>(p)[i])));
    default: return w_of_f32(bf16_bits_to_f32(static_cast<const uint16_t*>(p)[i]));
  }
}
__device__ __forceinline__ void word_to_storage(int type, void* p, uint64_t i, uint64_t w) {
  switch (type) {
    case kBool: static_cast<uint8_t*>(p)[i] = uint8_t(w & 1u); break;
    case kI32: static_cast<uint32_t*>(p)[i] = uint32_t(w); break;
    case kI64: static_cast<uint64_t*>(p)[i] = w; break;
    case kF32: static_cast<uint32_t*>(p)[i] = uint32_t(w); break;
    case kF16: static_cast<uint16_t*>(p)[i] = __half_as_ushort(__float2half_rn(f32_of(w))); break;
    default: static_cast<uint16_t*>(p)[i] = uint16_t(bf16_bits_rne(f32_of(w))); break;
  }
}

}  // namespace askb
