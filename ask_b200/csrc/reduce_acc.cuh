// Reduction accumulators with ASK's semantics, shared by the library's
// reduction kernels (reduce_kernels.cu) and the generated kernel artifacts
// (artifact.cpp): initial values (lib/Lowering/ScalarEmitter.h:426-439), the
// fold of one value or of another accumulator, and the output word.
#pragma once

#include <float.h>

#include "ask_numerics.cuh"
#include "kernels.h"
#include "vec_io.cuh"

namespace askb {
namespace red {

__device__ constexpr U32Div kNoDiv{1, 1, 0, 0, 0};  // unused by full-map loads

__device__ __forceinline__ double d_of(uint64_t w) { return __longlong_as_double(int64_t(w)); }
__device__ __forceinline__ uint64_t w_of_d(double d) { return uint64_t(__double_as_longlong(d)); }

__device__ __forceinline__ int64_t signed_of(int t, uint64_t w) {
  return t == kI32 ? int64_t(i32_of(w)) : int64_t(w);
}

__device__ __forceinline__ void acc_init(int op, int t, uint64_t& v, int64_t& i) {
  i = -1;
  const bool fl = dtype_is_float(t);
  switch (op) {
    case RED_SUM: v = fl ? w_of_d(0.0) : 0; break;
    case RED_PROD: v = fl ? w_of_f32(1.0f) : 1; break;
    // bool max/min start from APInt::getSigned{Min,Max}Value(1) = true / false
    // and fold with or / and (ScalarEmitter.h:182, 192, 433-439).
    case RED_MAX: v = fl ? w_of_f32(-INFINITY) : t == kI32 ? w_of_i32(INT32_MIN) : t == kI64 ? uint64_t(INT64_MIN) : 1; break;
    case RED_MIN: v = fl ? w_of_f32(INFINITY) : t == kI32 ? w_of_i32(INT32_MAX) : t == kI64 ? uint64_t(INT64_MAX) : 0; break;
    case RED_ANY: v = 0; break;
    case RED_ALL: v = 1; break;
    default: v = 0; break;  // arg reductions start empty (i = -1)
  }
}

// true when candidate (v2, i2) beats the current best (v, i).
__device__ __forceinline__ bool arg_better(bool is_max, int t, uint64_t v2, int64_t i2, uint64_t v, int64_t i) {
  if (i2 < 0) return false;
  if (i < 0) return true;
  if (dtype_is_float(t)) {
    const float a = f32_of(v2), b = f32_of(v);
    const bool na = a != a, nb = b != b;
    if (na || nb) return (na && nb) ? i2 < i : na;
    if (is_max ? a > b : a < b) return true;
    if (is_max ? a < b : a > b) return false;
    return i2 < i;
  }
  const int64_t a = t == kBool ? int64_t(v2 & 1u) : signed_of(t, v2);
  const int64_t b = t == kBool ? int64_t(v & 1u) : signed_of(t, v);
  if (is_max ? a > b : a < b) return true;
  if (is_max ? a < b : a > b) return false;
  return i2 < i;
}

// Fold (x, xi) into the accumulator.  `partial` means x is itself an
// accumulator (float sums then carry f64 bits instead of an f32 element).
template <bool kPartial>
__device__ __forceinline__ void acc_fold(int op, int t, uint64_t& v, int64_t& i, uint64_t x, int64_t xi) {
  switch (op) {
    case RED_SUM:
      if (dtype_is_float(t)) v = w_of_d(d_of(v) + (kPartial ? d_of(x) : double(f32_of(x))));
      else if (t == kI32) v = w_of_i32(int_add(i32_of(v), i32_of(x)));
      else v = uint64_t(int_add(int64_t(v), int64_t(x)));
      break;
    case RED_PROD:
      if (dtype_is_float(t)) v = w_of_f32(__fmul_rn(f32_of(v), f32_of(x)));
      else if (t == kI32) v = w_of_i32(int_mul(i32_of(v), i32_of(x)));
      else v = uint64_t(int_mul(int64_t(v), int64_t(x)));
      break;
    case RED_MAX:
      if (dtype_is_float(t)) v = w_of_f32(ask_maximum(f32_of(v), f32_of(x)));
      else if (t == kBool) v = (v | x) & 1u;
      else v = signed_of(t, x) > signed_of(t, v) ? x : v;
      break;
    case RED_MIN:
      if (dtype_is_float(t)) v = w_of_f32(ask_minimum(f32_of(v), f32_of(x)));
      else if (t == kBool) v = (v & x) & 1u;
      else v = signed_of(t, x) < signed_of(t, v) ? x : v;
      break;
    case RED_ANY: v = (v | x) & 1u; break;
    case RED_ALL: v = (v & x) & 1u; break;
    default:
      if (arg_better(op == RED_ARGMAX, t, x, xi, v, i)) { v = x; i = xi; }
      break;
  }
}

// Output word of a finished accumulator, in the output's storage type.
__device__ __forceinline__ uint64_t acc_result(int op, int t, uint64_t v, int64_t i) {
  if (red_is_arg(op)) return uint64_t(i);
  if (op == RED_SUM && dtype_is_float(t)) return w_of_f32(round_to(t, float(d_of(v))));
  if (op == RED_PROD && dtype_is_float(t)) return w_of_f32(round_to(t, f32_of(v)));
  return v;
}
__device__ __forceinline__ int out_type_of(int op, int t) {
  return red_is_arg(op) ? int(kI64) : (op == RED_ANY || op == RED_ALL) ? int(kBool) : t;
}

}  // namespace red
}  // namespace askb
