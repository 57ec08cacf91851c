// Device bodies of the generated kernel artifacts (artifact.cpp).
//
// An artifact is one `extern "C"` kernel for one owned step, compiled to an
// sm_100a cubin and packaged in ASK's external-kernel-artifact v2 form
// (schemas/external-kernel-artifact-v2.schema.json): its parameters are plain
// device pointers (one per port) and optional scalars, so ASK's
// Session::load can check them against `parameterWidths`
// (include/ask/Runtime/CUDA.h:75-78, lib/Runtime/CUDA.cpp:499-541).  Every
// size and the step's op program are compile-time constants of the generated
// source; these templates are the loops it instantiates.  The launch grid is
// the caller's (the request fixes it), so every loop is grid-stride, and an
// artifact has no scratch memory: a reduction's cross-thread combine stays
// inside one CTA.  Programs read at least one input port (the generator
// routes input-free elementwise programs to the view loop).
#pragma once

#include <type_traits>

#include "ew_body.cuh"
#include "reduce_acc.cuh"
#include "reduce_fast.cuh"

namespace askb {
namespace art {

constexpr int kThreads = 256;  // block size of every artifact kernel
// Resident CTAs an entry with a functor loop is compiled for: the functor
// loops need at most 48 registers (the library's functor kernels use 47), and
// the bound keeps the entry's compile-time-program fallback (misaligned
// ports) from raising the whole kernel's register count and lowering its
// occupancy.
constexpr int kFunctorMinBlocks = 5;
// The cfg1 functor keeps two units of loads in flight (58 registers in the
// library): its entries are compiled for 4 resident CTAs.
constexpr int kDeepFunctorMinBlocks = 4;

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
__device__ __forceinline__ bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

// ---- reductions ----------------------------------------------------------------------
// RL: the step's reductions, each folding program result src(k) of type type(k)
// with op(k) into output k.
template <class RL>
struct Acc {
  uint64_t v[RL::N];
  int64_t i[RL::N];
};

template <class RL, int K = 0>
__device__ __forceinline__ void acc_init_all(Acc<RL>& s) {
  if constexpr (K < RL::N) {
    red::acc_init(RL::op(K), RL::type(K), s.v[K], s.i[K]);
    acc_init_all<RL, K + 1>(s);
  }
}

template <class RL, int K = 0>
__device__ __forceinline__ void acc_merge_all(Acc<RL>& s, const Acc<RL>& o) {
  if constexpr (K < RL::N) {
    red::acc_fold<true>(RL::op(K), RL::type(K), s.v[K], s.i[K], o.v[K], o.i[K]);
    acc_merge_all<RL, K + 1>(s, o);
  }
}

// Fold the values of one unit (program registers r, elements e..e+V-1 of the
// row, those below `end`) into every reduction.
template <class P, class RL, int V, int K = 0>
__device__ __forceinline__ void acc_fold_unit(Acc<RL>& s, const uint64_t (&r)[P::kInsn][V], uint64_t e, uint64_t end,
                                              uint64_t index_base) {
  if constexpr (K < RL::N) {
    constexpr int reg = P::out_reg(RL::src(K));
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (e + v < end) red::acc_fold<false>(RL::op(K), RL::type(K), s.v[K], s.i[K], r[reg][v], int64_t(index_base + e + v));
    acc_fold_unit<P, RL, V, K + 1>(s, r, e, end, index_base);
  }
}

template <class RL>
__device__ __forceinline__ void acc_warp_reduce(Acc<RL>& s) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Acc<RL> o;
#pragma unroll
    for (int k = 0; k < RL::N; ++k) {
      o.v[k] = __shfl_xor_sync(0xffffffffu, s.v[k], off);
      o.i[k] = __shfl_xor_sync(0xffffffffu, s.i[k], off);
    }
    acc_merge_all<RL>(s, o);
  }
}

// Whole-CTA fold in a fixed order (warps, then warp 0 over the warp results).
// Valid in thread 0.
template <class RL>
__device__ __forceinline__ void acc_block_reduce(Acc<RL>& s) {
  __shared__ Acc<RL> part[kThreads / 32];
  acc_warp_reduce<RL>(s);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = s;
  __syncthreads();
  if (warp == 0) {
    if (lane < kThreads / 32) s = part[lane];
    else acc_init_all<RL>(s);
    acc_warp_reduce<RL>(s);
  }
  __syncthreads();
}

template <class RL, int K = 0>
__device__ __forceinline__ void acc_write(void* const* out, const Acc<RL>& s, uint64_t o_idx) {
  if constexpr (K < RL::N) {
    constexpr int op = RL::op(K), t = RL::type(K);
    word_to_storage(red::out_type_of(op, t), out[K], o_idx, red::acc_result(op, t, s.v[K], s.i[K]));
    acc_write<RL, K + 1>(out, s, o_idx);
  }
}

// Prologue inputs of one unit: full ports read elements row+e.., outer ports the
// output's element, scalar ports element 0.
template <class P, int V, int K = 0>
__device__ __forceinline__ void prologue_load(const void* const* in, uint64_t row, uint64_t e, uint64_t end,
                                              uint64_t o_idx, bool vec, uint64_t (&x)[P::kIn][V]) {
  if constexpr (K < P::kIn) {
    if constexpr (P::in_map(K) == IM_FULL) {
      load_port<P::in_type(K), IM_FULL, V>(in[K], row + e, row + end, red::kNoDiv, vec, x[K]);
    } else {
      const uint64_t w = word_from_storage(P::in_type(K), in[K], P::in_map(K) == IM_SCALAR ? 0 : o_idx);
#pragma unroll
      for (int v = 0; v < V; ++v) x[K][v] = w;
    }
    prologue_load<P, V, K + 1>(in, row, e, end, o_idx, vec, x);
  }
}

// Thread t of T folds elements t*V, (t+T)*V, ... of the row starting at
// linear element `row` (output o_idx).
template <class P, class RL, int V, uint64_t EXTENT, uint64_t BASE>
__device__ __forceinline__ void fold_row(const void* const* in, uint64_t row, uint64_t o_idx, uint32_t t, uint32_t T,
                                         bool aligned, Acc<RL>& s) {
  for (uint64_t e = uint64_t(t) * V; e < EXTENT; e += uint64_t(T) * V) {
    const bool vec = aligned && e + V <= EXTENT;
    uint64_t x[P::kIn][V];
    uint64_t r[P::kInsn][V];
    prologue_load<P, V>(in, row, e, EXTENT, o_idx, vec, x);
    ew::spec_exec<P, 0, V>(r, x);
    acc_fold_unit<P, RL, V>(s, r, e, EXTENT, BASE);
  }
}

// inner == 1, many rows: a warp per output row.
template <class P, class RL, uint64_t OUTER, uint64_t EXTENT, uint64_t BASE>
__device__ __forceinline__ void reduce_rows_warp(const void* const* in, void* const* out, bool aligned) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warp = (uint64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t(gridDim.x) * kThreads) >> 5;
  for (uint64_t o = warp; o < OUTER; o += nwarps) {
    Acc<RL> s;
    acc_init_all<RL>(s);
    fold_row<P, RL, 4, EXTENT, BASE>(in, o * EXTENT, o, lane, 32, aligned, s);
    acc_warp_reduce<RL>(s);
    if (lane == 0) acc_write<RL>(out, s, o);
  }
}

// inner == 1, few long rows: a CTA per output row.
template <class P, class RL, uint64_t OUTER, uint64_t EXTENT, uint64_t BASE>
__device__ __forceinline__ void reduce_rows_cta(const void* const* in, void* const* out, bool aligned) {
  for (uint64_t o = blockIdx.x; o < OUTER; o += gridDim.x) {
    Acc<RL> s;
    acc_init_all<RL>(s);
    fold_row<P, RL, 4, EXTENT, BASE>(in, o * EXTENT, o, threadIdx.x, kThreads, aligned, s);
    acc_block_reduce<RL>(s);
    if (threadIdx.x == 0) acc_write<RL>(out, s, o);
  }
}

// The library's specialised reductions (compile-time source S and set R, the
// exact f32 fast fold) with a CTA per output row; the warp-per-row form is
// red::red_warp_row_loop itself.
template <class S, class R, int U>
__device__ __forceinline__ void reduce_rows_cta_fast(const RedArgs& a, int aligned) {
  for (uint64_t o = blockIdx.x; o < a.outer; o += gridDim.x) {
    red::FastAcc s;
    red::fast_init(s);
    const typename S::Row rw = S::row(a, o);
    red::span_src<S, R, U>(a, rw, o * a.extent, 0, a.extent, threadIdx.x, kThreads, aligned != 0, s);
    red::fast_block_reduce<R>(s);
    if (threadIdx.x == 0) red::fast_write<R, 0>(a, s, o);
  }
}

// inner > 1: a thread per output (o, n), folding (o, e, n) for e = 0, 1, ...;
// consecutive threads read consecutive n.
template <class P, class RL, uint64_t OUTER, uint64_t EXTENT, uint64_t INNER, uint64_t BASE>
__device__ __forceinline__ void reduce_columns(const void* const* in, void* const* out) {
  constexpr uint64_t outputs = OUTER * INNER;
  for (uint64_t o_idx = uint64_t(blockIdx.x) * kThreads + threadIdx.x; o_idx < outputs;
       o_idx += uint64_t(gridDim.x) * kThreads) {
    const uint64_t o = o_idx / INNER, n = o_idx % INNER;
    Acc<RL> s;
    acc_init_all<RL>(s);
    for (uint64_t e = 0; e < EXTENT; ++e) {
      uint64_t x[P::kIn][1];
      uint64_t r[P::kInsn][1];
      prologue_load<P, 1>(in, (o * EXTENT + e) * INNER + n, 0, 1, o_idx, false, x);
      ew::spec_exec<P, 0, 1>(r, x);
      acc_fold_unit<P, RL, 1>(s, r, e, e + 1, BASE);
    }
    acc_write<RL>(out, s, o_idx);
  }
}

// ---- gather ----------------------------------------------------------------------------
// out[o, j, :] = table[o, idx[j], :], zero rows for indices outside [0, DIM).
template <int IT>
__device__ __forceinline__ int64_t index_at(const void* p, uint64_t j) {
  if constexpr (IT == kI32) return int64_t(__ldg(static_cast<const int32_t*>(p) + j));
  else return __ldg(static_cast<const int64_t*>(p) + j);
}

// Rows of ROW_BYTES (a multiple of 16): a warp per output row, 16-byte vectors.
template <int IT, uint64_t OUTER, uint64_t DIM, uint64_t N, uint64_t ROW_BYTES>
__device__ __forceinline__ void gather_rows(const void* table, const void* index, void* out) {
  constexpr uint64_t vecs = ROW_BYTES / 16, rows = OUTER * N;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warp = (uint64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t(gridDim.x) * kThreads) >> 5;
  for (uint64_t r = warp; r < rows; r += nwarps) {
    const uint64_t o = r / N, j = r % N;
    const int64_t idx = index_at<IT>(index, j);
    const bool ok = idx >= 0 && uint64_t(idx) < DIM;
    const uint4* src = static_cast<const uint4*>(table) + (o * DIM + uint64_t(ok ? idx : 0)) * vecs;
    uint4* dst = static_cast<uint4*>(out) + r * vecs;
    for (uint64_t v = lane; v < vecs; v += 32) st_stream_v4(dst + v, ok ? __ldg(src + v) : make_uint4(0, 0, 0, 0));
  }
}

// Any row size: a thread per output element of ES bytes.
template <int ES, int IT, uint64_t OUTER, uint64_t DIM, uint64_t N, uint64_t INNER>
__device__ __forceinline__ void gather_elems(const void* table, const void* index, void* out) {
  using T = typename std::conditional<ES == 1, uint8_t,
            typename std::conditional<ES == 2, uint16_t, typename std::conditional<ES == 4, uint32_t, uint64_t>::type>::type>::type;
  constexpr uint64_t total = OUTER * N * INNER;
  for (uint64_t i = uint64_t(blockIdx.x) * kThreads + threadIdx.x; i < total; i += uint64_t(gridDim.x) * kThreads) {
    const uint64_t row = i / INNER, c = i % INNER;
    const uint64_t o = row / N, j = row % N;
    const int64_t idx = index_at<IT>(index, j);
    T v = 0;
    if (idx >= 0 && uint64_t(idx) < DIM) v = static_cast<const T*>(table)[(o * DIM + uint64_t(idx)) * INNER + c];
    static_cast<T*>(out)[i] = v;
  }
}

}  // namespace art
}  // namespace askb
