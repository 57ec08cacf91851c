// Family S: the reference's three-step softmax plan fused into one pass.
//
// ASK partitions a row softmax into three owned steps (lib/Frontend/
// Partition.cpp:100-148; the recompute form, in which each step casts x itself):
//   step 0  m = reduce_max(cast(x, f32))                     over each row
//   step 1  s = reduce_sum(exp(cast(x) + m*(-1)))            over each row
//   step 2  y = cast(exp(cast(x) + m*(-1)) / s, T)
// Run as three kernels the plan reads x three times and computes exp twice.
// Here a CTA owns a whole row (cols / 8 vectors of 8 f16/bf16 elements,
// VPT vectors per thread): it loads the row once, reduces the max across the
// CTA, computes every exp once and keeps it in registers, reduces the sum, and
// writes y (and m, s) -- 2 bytes read and 2 written per element instead of 8.
// The next row's vectors are loaded before this row's reductions.
//
// Semantics per element are those of the three steps: max folds with
// max.NaN.f32 (llvm.maximum: the canonical NaN when the row holds a NaN,
// -0 < +0); exp(x + m*(-1)) with CUDA's expf; the division is the
// correctly rounded f32 quotient (one reciprocal per row and Markstein's
// correction, with the IEEE division for any unit outside its conditions, as
// in the softmax normalise kernel); f16/bf16 rounding to nearest even.  The sum
// is accumulated per thread in f32 and across the CTA in f64 in a fixed order,
// so s is deterministic; its rounding may differ from the three-kernel plan's
// in the last place.
#include <cuda_runtime.h>

#include <algorithm>

#include "ask_numerics.cuh"
#include "kernels.h"
#include "vec_io.cuh"

namespace askb {

namespace {

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
template <int T>
__device__ __forceinline__ uint32_t narrow_one(float f) {
  if constexpr (T == kF16) return __half_as_ushort(__float2half_rn(f));
  else return bf16_bits_rne(f);
}
// Two finite values rounded to nearest even and packed, lo in bits 0..15.
template <int T>
__device__ __forceinline__ uint32_t narrow_two(float lo, float hi) {
  uint32_t r;
  if constexpr (T == kF16)
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// llvm.maximum on f32 in one instruction: NaN if either operand is NaN (the
// canonical NaN), otherwise the larger, with -0 < +0.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// The same on two packed f16/bf16 values at once (NaN-propagating max), and
// the plain packed minimum; widening to f32 is exact and monotone, so the
// max/min of the widened values equals the widened max/min.
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

constexpr int kMaxWarps = 16;
#ifndef ASKB_SOFTMAX_THREADS
#define ASKB_SOFTMAX_THREADS 128
#endif
constexpr int kPreferThreads = ASKB_SOFTMAX_THREADS;  // CTA size the row split aims for

// VPT == 4 (4096-element rows, 128-thread CTAs) is compiled for two 512-thread
// CTAs' worth of registers per SM, 64 a thread: the f16 variant then fits 8
// CTAs per SM instead of 4 without spilling (same-box A/B on cfg3: 0.111 ms
// against 0.123 ms); wider rows keep the full budget (VPT == 8 would spill).
template <int T, int VPT>
__global__ void __launch_bounds__(kMaxWarps * 32, VPT == 4 ? 2 : 1) softmax_rows_kernel(const uint4* __restrict__ x, float* __restrict__ m_out,
                                                                      float* __restrict__ s_out, uint4* __restrict__ y,
                                                                      uint64_t rows, uint32_t vecs) {
  __shared__ float red_max[2][kMaxWarps];
  __shared__ double red_sum[2][kMaxWarps];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  uint64_t row = blockIdx.x;
  uint4 v[VPT];
  if (row < rows) {
#pragma unroll
    for (int q = 0; q < VPT; ++q) v[q] = ld_stream_v4(x + row * vecs + q * blockDim.x + threadIdx.x);
  }
  for (int parity = 0; row < rows; row += gridDim.x, parity ^= 1) {
    float e[VPT * 8];
    // m = max over the row (NaN-propagating); the thread's smallest value
    // bounds its exp results from below for the division's check.  Both fold
    // on the packed 16-bit values, two elements an instruction.
    uint32_t pmax = v[0].x, pmin = v[0].x;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        e[q * 8 + 2 * j] = widen_lo<T>(w[j]);
        e[q * 8 + 2 * j + 1] = widen_hi<T>(w[j]);
        pmax = max2_nan<T>(pmax, w[j]);
        pmin = min2<T>(pmin, w[j]);
      }
    }
    const uint64_t next = row + gridDim.x;
    if (next < rows) {
#pragma unroll
      for (int q = 0; q < VPT; ++q) v[q] = ld_stream_v4(x + next * vecs + q * blockDim.x + threadIdx.x);
    }
    // max.NaN.f32 of the two halves also turns a NaN into the canonical f32 NaN
    float mx = max_nan(widen_lo<T>(pmax), widen_hi<T>(pmax));
    const float mn = fminf(widen_lo<T>(pmin), widen_hi<T>(pmin));
#pragma unroll
    for (int d = 16; d; d >>= 1) mx = max_nan(mx, __shfl_xor_sync(0xffffffffu, mx, d));
    if (lane == 0) red_max[parity][warp] = mx;
    __syncthreads();
    float m = red_max[parity][0];
    for (uint32_t k = 1; k < nwarps; ++k) m = max_nan(m, red_max[parity][k]);
    const float nm = __fmul_rn(m, -1.0f);
    // e = exp(x + m*(-1)), s = sum of e
    float part = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT * 8; ++k) {
      e[k] = expf(__fadd_rn(e[k], nm));
      part = __fadd_rn(part, e[k]);
    }
    double ps = double(part);
#pragma unroll
    for (int d = 16; d; d >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, d);
    if (lane == 0) red_sum[parity][warp] = ps;
    __syncthreads();
    double total = 0.0;
    for (uint32_t k = 0; k < nwarps; ++k) total += red_sum[parity][k];
    const float s = float(total);
    if (threadIdx.x == 0) {
      m_out[row] = m;
      s_out[row] = s;
    }
    // y = cast(e / s): the correctly rounded quotient from one reciprocal
    // (Markstein's two corrections).  Its conditions hold for the whole thread
    // when s and 1/s are normal and every e >= exp(-69) > 2^-100: then
    // 2^-100 / s <= e / s <= 1 (e <= 1 because m is the row's maximum and
    // s >= 1), so every quotient is normal.  Otherwise the IEEE division runs.
    const float r = __frcp_rn(s);
    const bool ok = s >= 1.0f && s <= 0x1p100f && __fadd_rn(mn, nm) >= -69.0f;
#pragma unroll
    for (int qv = 0; qv < VPT; ++qv) {
      float q[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float ek = e[qv * 8 + k];
        float t = __fmul_rn(ek, r);
        t = __fmaf_rn(__fmaf_rn(-t, s, ek), r, t);
        t = __fmaf_rn(__fmaf_rn(-t, s, ek), r, t);
        q[k] = t;
      }
      uint32_t o[4];
      if (ok) {
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = narrow_two<T>(q[2 * j], q[2 * j + 1]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = __fdiv_rn(e[qv * 8 + 2 * j], s), hi = __fdiv_rn(e[qv * 8 + 2 * j + 1], s);
          o[j] = narrow_one<T>(lo) | (narrow_one<T>(hi) << 16);
        }
      }
      st_stream_v4(y + row * vecs + qv * blockDim.x + threadIdx.x, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

template <int T, int VPT>
cudaError_t launch_rows(const SoftmaxArgs& a, int sms, cudaStream_t st) {
  const uint32_t vecs = uint32_t(a.cols / 8);
  const unsigned threads = vecs / VPT;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, softmax_rows_kernel<T, VPT>, int(threads), 0);
  if (e != cudaSuccess) return e;
  const uint64_t grid = std::min<uint64_t>(a.rows, uint64_t(sms) * uint64_t(per_sm > 0 ? per_sm : 1));
  softmax_rows_kernel<T, VPT><<<unsigned(grid), threads, 0, st>>>(static_cast<const uint4*>(a.x), a.m, a.s,
                                                                  static_cast<uint4*>(a.y), a.rows, vecs);
  return cudaGetLastError();
}

template <int T>
cudaError_t launch_type(const SoftmaxArgs& a, int sms, cudaStream_t st) {
  switch (softmax_vectors_per_thread(a.cols)) {
    case 1: return launch_rows<T, 1>(a, sms, st);
    case 2: return launch_rows<T, 2>(a, sms, st);
    case 4: return launch_rows<T, 4>(a, sms, st);
    case 8: return launch_rows<T, 8>(a, sms, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int softmax_vectors_per_thread(uint64_t cols) {
  if (cols == 0 || cols % 8) return 0;
  const uint64_t vecs = cols / 8;
  int best = 0;
  for (int vpt : {1, 2, 4, 8}) {
    if (vecs % uint64_t(vpt)) continue;
    const uint64_t threads = vecs / uint64_t(vpt);
    if (threads % 32 || threads > uint64_t(kMaxWarps) * 32) continue;
    if (!best || threads >= uint64_t(kPreferThreads)) best = vpt;  // the fewest threads not below the target
    if (threads <= uint64_t(kPreferThreads)) break;
  }
  return best;
}

cudaError_t softmax_rows_launch(const SoftmaxArgs& a, int sms, cudaStream_t st) {
  if (a.rows == 0) return cudaSuccess;
  return a.type == kF16 ? launch_type<kF16>(a, sms, st) : launch_type<kBF16>(a, sms, st);
}

}  // namespace askb
