// Paired f32 arithmetic and 16-bit float helpers shared by the softmax kernels:
// the fused row softmax (softmax_kernels.cu) and the plan's normalise step
// (ew_body.cuh, FnSoftmaxNorm).  The plan's sum step keeps CUDA's expf: on a
// B200 the paired exp measured no faster there (69.7 against 68.5 us for the
// bf16 step of [32768, 4096], 75.8 against 68.5 for f16), while the normalise
// step went from 139.4 to 104.4 us (f16) and 135.2 to 101.4 (bf16).
//
// sm_100 executes add/mul/fma.rn.f32x2 on two f32 values held in one 64-bit
// register, two elements an instruction, each half rounded exactly as the
// scalar .rn instruction rounds it.
//
// exp_pair(t) for -69 <= t <= 0:
//   exp(t) = 2^hi * 2^lo, hi = RN(t * L) with L = RN(log2 e); the residual
//   t*L - hi is exact by one fused multiply-add (the FMA two-product of
//   Ogita, Rump and Oishi, 2005), to which t * (log2 e - L) is added, so
//   |lo| <= 2^-17 and 2^lo = 1 + lo*ln2 within 2^-35; 2^hi is ex2.approx.ftz.f32
//   (relative error about 2^-22).  The result is a normal f32 within about 3
//   ulps of exp(t).
#ifndef ASK_B200_PAIR_F32_CUH
#define ASK_B200_PAIR_F32_CUH

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ask_numerics.cuh"

namespace askb {

// 16-bit storage (f16 or bf16) to f32, exactly: the low and high halves of a word.
template <int T>
__device__ __forceinline__ float widen_lo(uint32_t w) {
  if constexpr (T == kF16) return __half2float(__ushort_as_half(uint16_t(w & 0xffffu)));
  else return __uint_as_float(w << 16);
}
template <int T>
__device__ __forceinline__ float widen_hi(uint32_t w) {
  if constexpr (T == kF16) return __half2float(__ushort_as_half(uint16_t(w >> 16)));
  else return __uint_as_float(w & 0xffff0000u);
}
// One value rounded to nearest even (any input; bf16 keeps NaN payloads).
template <int T>
__device__ __forceinline__ uint32_t narrow_one(float f) {
  if constexpr (T == kF16) return __half_as_ushort(__float2half_rn(f));
  else return bf16_bits_rne(f);
}
// Two non-NaN values rounded to nearest even and packed, lo in bits 0..15:
// one cvt.rn.{f16,bf16}x2.f32, equal to narrow_one on each.
template <int T>
__device__ __forceinline__ uint32_t narrow_two(float lo, float hi) {
  uint32_t r;
  if constexpr (T == kF16)
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// llvm.maximum / llvm.minimum on f32 in one instruction: NaN if either
// operand is NaN (the canonical NaN), otherwise the larger (smaller), with
// -0 < +0.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float min_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// The same on two packed f16/bf16 values at once (NaN-propagating max), the
// plain packed minimum and the NaN-propagating one; widening to f32 is exact
// and monotone, so the max/min of the widened values equals the widened max/min.
template <int T>
__device__ __forceinline__ uint32_t max2_nan(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (T == kF16)
    asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <int T>
__device__ __forceinline__ uint32_t min2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (T == kF16)
    asm("min.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <int T>
__device__ __forceinline__ uint32_t min2_nan(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (T == kF16)
    asm("min.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("min.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Pairs of f32 values in one 64-bit register (element 0 in the low half).
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// 2^a for -100 <= a <= 0 (exp_pair's range): a and 2^a are normal f32 values
// or zero, so the flush-to-zero form, which skips the subnormal handling of
// the plain one, computes the same value.
__device__ __forceinline__ float ex2_approx(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// exp(t) of a pair with -69 <= t <= 0 (the file comment gives the error bound).
constexpr float kLog2e = 0x1.715476p+0f;      // RN(log2 e)
constexpr float kLog2eTail = 0x1.4ae0cp-26f;  // RN(log2 e - kLog2e)
constexpr float kLn2 = 0x1.62e43p-1f;         // RN(ln 2)
__device__ __forceinline__ uint64_t exp_pair(uint64_t t) {
  const uint64_t L = pack2(kLog2e, kLog2e), nL = pack2(-kLog2e, -kLog2e);
  const uint64_t tail = pack2(kLog2eTail, kLog2eTail), ln2 = pack2(kLn2, kLn2);
  const uint64_t hi = mul2(t, L);
  uint64_t lo = fma2(t, L, mul2(t, nL));  // t*L - hi, exact
  lo = mul2(fma2(t, tail, lo), ln2);
  float h0, h1;
  unpack2(hi, h0, h1);
  const uint64_t p = pack2(ex2_approx(h0), ex2_approx(h1));
  return fma2(p, lo, p);
}

// Whether every t = RN(x + nm) of the eight 16-bit values in `w` lies in
// [-69, 0], the range of exp_pair: decided on their NaN-propagating minimum
// and maximum (RN addition is monotone), so a NaN value, a NaN nm or an
// infinite t fails it.
template <int T>
__device__ __forceinline__ bool exp_pair_range(const uint32_t (&w)[4], float nm) {
  const uint32_t lo = min2_nan<T>(min2_nan<T>(w[0], w[1]), min2_nan<T>(w[2], w[3]));
  const uint32_t hi = max2_nan<T>(max2_nan<T>(w[0], w[1]), max2_nan<T>(w[2], w[3]));
  const float tmin = __fadd_rn(min_nan(widen_lo<T>(lo), widen_hi<T>(lo)), nm);
  const float tmax = __fadd_rn(max_nan(widen_lo<T>(hi), widen_hi<T>(hi)), nm);
  return tmin >= -69.0f && tmax <= 0.0f;
}

}  // namespace askb

#endif  // ASK_B200_PAIR_F32_CUH
