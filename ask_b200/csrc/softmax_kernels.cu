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
// -0 < +0); t = x + m*(-1) rounded to f32; exp(t); e / s; f16/bf16 rounding to
// nearest even.  The sum is accumulated per thread in f32 and across the CTA
// in f64 in a fixed order, so s is deterministic.
//
// The arithmetic runs on pairs of f32 values (add/mul/fma.rn.f32x2, two
// elements an instruction on sm_100) wherever a thread's elements all have
// -69 <= t <= 0 (a finite row: every e is then a normal f32):
//   exp(t) = 2^hi * 2^lo, hi = RN(t * L) with L = RN(log2 e); the residual
//   t*L - hi is exact by one fused multiply-add (the FMA two-product of
//   Ogita, Rump and Oishi, 2005), to which t * (log2 e - L) is added, so
//   |lo| <= 2^-17 and 2^lo = 1 + lo*ln2 within 2^-35; 2^hi is ex2.approx.f32
//   (relative error about 2^-22): e is within about 3 f32 ulps of exp(t);
//   y = RN16(e * RN(1/s)), within 2 f32 ulps of e / s before the 16-bit
//   rounding, so within one 16-bit ulp of the three-step plan's RN16(e / s).
// Any other thread (a non-finite row, or t below -69) computes each element
// with CUDA's expf and the IEEE division, as the three steps do.  m is
// bit-identical to the three-step plan's; s may differ in its last places and
// y by at most one unit in the last place.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "ask_numerics.cuh"
#include "kernels.h"
#include "pair_f32.cuh"
#include "pdl.cuh"
#include "vec_io.cuh"

namespace askb {

namespace {

constexpr int kMaxWarps = 16;
#ifndef ASKB_SOFTMAX_THREADS
#define ASKB_SOFTMAX_THREADS 128
#endif
constexpr int kPreferThreads = ASKB_SOFTMAX_THREADS;  // CTA size the row split aims for

// Rows split into 128-thread CTAs with up to 4 vectors a thread (4096-element
// rows) are compiled for a number of resident CTAs per SM chosen per mode by
// measurement (same box, [32768, 4096] f16, CUDA events): the fused kernel for
// 6 (80 registers a thread: 90.2 us against 98.3 at 8 CTAs of 64 registers,
// 94.3 at 7 and 90.2-92.2 at 5), the normalise step for 5 (88.3 us against
// 94.3 at 8 and 90.2 at 6), the max and sum steps for 8 (the sum step 65.6 us
// against 66.6 at 6; the max step needs 40 registers).  Other splits keep the
// full register budget (VPT == 8 would spill at 64).
template <int kMode>
constexpr int narrow_ctas_per_sm() {
  return kMode == SM_FUSED ? 6 : kMode == SM_STEP_NORM ? 5 : 8;
}
//
// kMode selects what the row kernel computes (SoftmaxMode): SM_FUSED the
// three steps; SM_STEP_MAX the first step alone (m); SM_STEP_SUM the second
// alone, s = sum of exp(x + m*(-1)) with m read from m_in (any value: the
// pair path also checks t <= 0 on the thread's largest element);
// SM_STEP_NORM the third alone, y = cast(exp(x + m*(-1)) / s) with m and s
// read from m_in and s_in (pairs also need 2^-100 <= s <= 2^24, so that
// every product e * RN(1/s) is a normal f32; otherwise expf and the IEEE
// division, the normalise step's own scalar arithmetic).
template <int T, int VPT, bool kNarrow, int kMode>
__global__ void __launch_bounds__(kNarrow ? 128 : kMaxWarps * 32, kNarrow ? narrow_ctas_per_sm<kMode>() : 1)
    softmax_rows_kernel(const uint4* __restrict__ x, float* __restrict__ m_out, float* __restrict__ s_out,
                        uint4* __restrict__ y, const float* __restrict__ m_in, const float* __restrict__ s_in,
                        uint64_t rows, uint32_t vecs) {
  constexpr bool kGivenM = kMode == SM_STEP_SUM || kMode == SM_STEP_NORM;
  __shared__ float red_max[2][kMaxWarps];
  __shared__ double red_sum[2][kMaxWarps];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  pdl_enter();
  uint64_t row = blockIdx.x;
  uint4 v[VPT];
  float m_given = 0.0f, s_given = 0.0f;  // SM_STEP_SUM / SM_STEP_NORM: this row's m (and s), loaded with the row
  if (row < rows) {
#pragma unroll
    for (int q = 0; q < VPT; ++q) v[q] = ld_stream_v4(x + row * vecs + q * blockDim.x + threadIdx.x);
    if constexpr (kGivenM) m_given = __ldg(m_in + row);
    if constexpr (kMode == SM_STEP_NORM) s_given = __ldg(s_in + row);
  }
  for (int parity = 0; row < rows; row += gridDim.x, parity ^= 1) {
    uint64_t e[VPT * 4];  // the thread's elements as f32 pairs: x, then t, then exp(t)
    // m = max over the row (NaN-propagating); the thread's smallest value
    // decides whether all its elements take the pair path.  Both fold on the
    // packed 16-bit values, two elements an instruction.
    uint32_t pmax = v[0].x, pmin = v[0].x;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (kMode != SM_STEP_MAX) {
          e[q * 4 + j] = pack2(widen_lo<T>(w[j]), widen_hi<T>(w[j]));
          pmin = min2<T>(pmin, w[j]);
        }
        pmax = max2_nan<T>(pmax, w[j]);
      }
    }
    const float m_row = m_given, s_row = s_given;
    const uint64_t next = row + gridDim.x;
    if (next < rows) {
#pragma unroll
      for (int q = 0; q < VPT; ++q) v[q] = ld_stream_v4(x + next * vecs + q * blockDim.x + threadIdx.x);
      if constexpr (kGivenM) m_given = __ldg(m_in + next);
      if constexpr (kMode == SM_STEP_NORM) s_given = __ldg(s_in + next);
    }
    // max.NaN.f32 of the two halves also turns a NaN into the canonical f32 NaN
    float mx = max_nan(widen_lo<T>(pmax), widen_hi<T>(pmax));
    float m, nm;
    bool pairs;
    if constexpr (kGivenM) {
      // t in [-69, 0] for the thread's smallest and largest values (so for
      // all), which fails for a NaN or infinite value or m
      m = m_row;
      nm = __fmul_rn(m, -1.0f);
      const float mn = fminf(widen_lo<T>(pmin), widen_hi<T>(pmin));
      pairs = __fadd_rn(mn, nm) >= -69.0f && __fadd_rn(mx, nm) <= 0.0f;
      if constexpr (kMode == SM_STEP_NORM) pairs = pairs && s_row >= 0x1p-100f && s_row <= 0x1p24f;
    } else {
#pragma unroll
      for (int d = 16; d; d >>= 1) mx = max_nan(mx, __shfl_xor_sync(0xffffffffu, mx, d));
      if (lane == 0) red_max[parity][warp] = mx;
      __syncthreads();
      m = red_max[parity][0];
      for (uint32_t k = 1; k < nwarps; ++k) m = max_nan(m, red_max[parity][k]);
      if constexpr (kMode == SM_STEP_MAX) {
        if (threadIdx.x == 0) m_out[row] = m;
        continue;
      }
      nm = __fmul_rn(m, -1.0f);
      // e = exp(x + m*(-1)), s = sum of e.  t >= -69 for the smallest element
      // (and so for all, t <= 0 for all) holds only when m and the thread's
      // values are finite: NaN and infinities take the scalar path.
      const float mn = fminf(widen_lo<T>(pmin), widen_hi<T>(pmin));
      pairs = __fadd_rn(mn, nm) >= -69.0f;
    }
    float part;
    if (pairs) {
      const uint64_t nm2 = pack2(nm, nm);
      uint64_t acc = pack2(0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < VPT * 4; ++k) {
        e[k] = exp_pair(add2(e[k], nm2));
        acc = add2(acc, e[k]);
      }
      float a0, a1;
      unpack2(acc, a0, a1);
      part = __fadd_rn(a0, a1);
    } else {
      part = 0.0f;
#pragma unroll
      for (int k = 0; k < VPT * 4; ++k) {
        float lo, hi;
        unpack2(e[k], lo, hi);
        lo = expf(__fadd_rn(lo, nm));
        hi = expf(__fadd_rn(hi, nm));
        part = __fadd_rn(__fadd_rn(part, lo), hi);
        e[k] = pack2(lo, hi);
      }
    }
    float s;
    if constexpr (kMode == SM_STEP_NORM) {
      s = s_row;
    } else {
      double ps = double(part);
#pragma unroll
      for (int d = 16; d; d >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, d);
      if (lane == 0) red_sum[parity][warp] = ps;
      __syncthreads();
      double total = 0.0;
      for (uint32_t k = 0; k < nwarps; ++k) total += red_sum[parity][k];
      s = float(total);
      if (threadIdx.x == 0) {
        if constexpr (kMode == SM_FUSED) m_out[row] = m;
        s_out[row] = s;
      }
    }
    if constexpr (kMode == SM_FUSED || kMode == SM_STEP_NORM) {
      // y = cast(e / s).  On the pair path y = RN16(e * RN(1/s)): with e >=
      // 2^-100 and 1 <= s <= 2^100 (the fused kernel: s counts exp(0) = 1)
      // or 2^-100 <= s <= 2^24 (checked), every product is a normal f32
      // within 2 ulps of e / s.  Otherwise the IEEE division.
      const float r = __frcp_rn(s);
      const bool by_reciprocal = kMode == SM_STEP_NORM ? pairs : pairs && s >= 1.0f && s <= 0x1p100f;
      const uint64_t r2 = pack2(r, r);
#pragma unroll
      for (int qv = 0; qv < VPT; ++qv) {
        uint32_t o[4];
        if (by_reciprocal) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float lo, hi;
            unpack2(mul2(e[qv * 4 + j], r2), lo, hi);
            o[j] = narrow_two<T>(lo, hi);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float lo, hi;
            unpack2(e[qv * 4 + j], lo, hi);
            o[j] = narrow_one<T>(__fdiv_rn(lo, s)) | (narrow_one<T>(__fdiv_rn(hi, s)) << 16);
          }
        }
        st_stream_v4(y + row * vecs + qv * blockDim.x + threadIdx.x, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
  }
}

// Resident CTAs per SM of one instance for a CTA size (threads / 32 <=
// kMaxWarps), queried once: the same on every B200.
template <int T, int VPT, bool kNarrow, int kMode>
cudaError_t resident_ctas(unsigned threads, int* per_sm) {
  static std::atomic<int> cache[kMaxWarps + 1];
  int n = cache[threads / 32].load(std::memory_order_relaxed);
  if (n == 0) {
    const cudaError_t e =
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, softmax_rows_kernel<T, VPT, kNarrow, kMode>, int(threads), 0);
    if (e != cudaSuccess) return e;
    n = std::max(n, 1);
    cache[threads / 32].store(n, std::memory_order_relaxed);
  }
  *per_sm = n;
  return cudaSuccess;
}

// Launch on `st`, or with grid_out set only report the grid a launch uses.
template <int T, int VPT, bool kNarrow, int kMode>
cudaError_t launch_mode(const SoftmaxArgs& a, unsigned threads, int sms, cudaStream_t st, int* grid_out) {
  const uint32_t vecs = uint32_t(a.cols / 8);
  int per_sm = 1;
  const cudaError_t e = resident_ctas<T, VPT, kNarrow, kMode>(threads, &per_sm);
  if (e != cudaSuccess) return e;
  const uint64_t grid = std::min<uint64_t>(a.rows, uint64_t(sms) * uint64_t(per_sm));
  if (grid_out) {
    *grid_out = int(grid);
    return cudaSuccess;
  }
  (void)launch_pdl(&softmax_rows_kernel<T, VPT, kNarrow, kMode>, dim3(unsigned(grid)), dim3(threads), st,
                   static_cast<const uint4*>(a.x), a.m, a.s, static_cast<uint4*>(a.y), a.m_in, a.s_in, a.rows,
                   vecs);
  return cudaGetLastError();
}

template <int T, int VPT, bool kNarrow>
cudaError_t launch_split(const SoftmaxArgs& a, unsigned threads, int sms, cudaStream_t st, int* grid_out) {
  switch (a.mode) {
    case SM_FUSED: return launch_mode<T, VPT, kNarrow, SM_FUSED>(a, threads, sms, st, grid_out);
    case SM_STEP_MAX: return launch_mode<T, VPT, kNarrow, SM_STEP_MAX>(a, threads, sms, st, grid_out);
    case SM_STEP_SUM: return launch_mode<T, VPT, kNarrow, SM_STEP_SUM>(a, threads, sms, st, grid_out);
    case SM_STEP_NORM: return launch_mode<T, VPT, kNarrow, SM_STEP_NORM>(a, threads, sms, st, grid_out);
    default: return cudaErrorInvalidValue;
  }
}

template <int T, int VPT>
cudaError_t launch_rows(const SoftmaxArgs& a, int sms, cudaStream_t st, int* grid_out) {
  const unsigned threads = unsigned(a.cols / 8) / VPT;
  if constexpr (VPT <= 4) {
    if (threads == 128) return launch_split<T, VPT, true>(a, threads, sms, st, grid_out);
  }
  return launch_split<T, VPT, false>(a, threads, sms, st, grid_out);
}

template <int T>
cudaError_t launch_type(const SoftmaxArgs& a, int sms, cudaStream_t st, int* grid_out) {
  switch (softmax_vectors_per_thread(a.cols)) {
    case 1: return launch_rows<T, 1>(a, sms, st, grid_out);
    case 2: return launch_rows<T, 2>(a, sms, st, grid_out);
    case 4: return launch_rows<T, 4>(a, sms, st, grid_out);
    case 8: return launch_rows<T, 8>(a, sms, st, grid_out);
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
  return a.type == kF16 ? launch_type<kF16>(a, sms, st, nullptr) : launch_type<kBF16>(a, sms, st, nullptr);
}

int softmax_rows_grid(const SoftmaxArgs& a, int sms) {
  int grid = 0;
  const cudaError_t e = a.rows == 0 ? cudaErrorInvalidValue
                        : a.type == kF16 ? launch_type<kF16>(a, sms, nullptr, &grid)
                                         : launch_type<kBF16>(a, sms, nullptr, &grid);
  return e == cudaSuccess && grid > 0 ? grid : 1;
}

}  // namespace askb
