// The specialised reductions' device code (family R), shared by the library's
// kernels (reduce_kernels.cu) and the generated kernel artifacts
// (artifact.cpp): compile-time reduction sets, the exact f32 fast fold on
// ordered integer keys, the value sources of the specialised programs and the
// row loops.
#pragma once

#include "programs.h"
#include "reduce_acc.cuh"

namespace askb {
namespace red {

// ---- specialised path: compile-time prologue P and reduction set R -------------
template <int... Ops>
struct RedSet {
  static constexpr int N = sizeof...(Ops);
  ASKB_HD static constexpr int op(int k) {
    constexpr int o[] = {Ops...};
    return o[k];
  }
};

template <class R>
struct AccsT {
  uint64_t v[R::N];
  int64_t i[R::N];
};

template <class R, int T, int K>
__device__ __forceinline__ void set_init(AccsT<R>& s) {
  if constexpr (K < R::N) {
    acc_init(R::op(K), T, s.v[K], s.i[K]);
    set_init<R, T, K + 1>(s);
  }
}
template <class R, int T, int K>
__device__ __forceinline__ void set_fold_value(AccsT<R>& s, uint64_t x, int64_t xi) {
  if constexpr (K < R::N) {
    acc_fold<false>(R::op(K), T, s.v[K], s.i[K], x, xi);
    set_fold_value<R, T, K + 1>(s, x, xi);
  }
}
template <class R, int T, int K>
__device__ __forceinline__ void set_merge(AccsT<R>& s, const AccsT<R>& o) {
  if constexpr (K < R::N) {
    acc_fold<true>(R::op(K), T, s.v[K], s.i[K], o.v[K], o.i[K]);
    set_merge<R, T, K + 1>(s, o);
  }
}
template <class R, int T>
__device__ __forceinline__ void set_warp_reduce(AccsT<R>& s) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    AccsT<R> o;
#pragma unroll
    for (int k = 0; k < R::N; ++k) {
      o.v[k] = __shfl_xor_sync(0xffffffffu, s.v[k], off);
      o.i[k] = __shfl_xor_sync(0xffffffffu, s.i[k], off);
    }
    set_merge<R, T, 0>(s, o);
  }
}
template <class R, int T>
__device__ __forceinline__ void set_block_reduce(AccsT<R>& s) {
  __shared__ uint64_t sv[kRedThreads / 32][R::N];
  __shared__ int64_t si[kRedThreads / 32][R::N];
  set_warp_reduce<R, T>(s);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < R::N; ++k) { sv[warp][k] = s.v[k]; si[warp][k] = s.i[k]; }
  }
  __syncthreads();
  if (warp == 0) {
    if (lane < int(blockDim.x >> 5)) {
#pragma unroll
      for (int k = 0; k < R::N; ++k) { s.v[k] = sv[lane][k]; s.i[k] = si[lane][k]; }
    } else {
      set_init<R, T, 0>(s);
    }
    set_warp_reduce<R, T>(s);
  }
  __syncthreads();
}
template <class R, int T>
__device__ __forceinline__ void set_write(const RedArgs& a, const AccsT<R>& s, uint64_t o_idx) {
#pragma unroll
  for (int k = 0; k < R::N; ++k) {
    const int op = R::op(k);
    word_to_storage(out_type_of(op, T), a.out[k], o_idx, acc_result(op, T, s.v[k], s.i[k]));
  }
}

// Prologue loads.  `row` is the linear element index of (o, 0) and `o_idx`
// the output index used by IM_OUTER ports.
template <class P, int K, int V>
__device__ __forceinline__ void spec_load(const RedArgs& a, uint64_t row, uint64_t e, uint64_t e_end, uint64_t o_idx,
                                          bool vec, uint64_t (&x)[P::kIn][V]) {
  if constexpr (K < P::kIn) {
    if constexpr (P::in_map(K) == IM_FULL) {
      load_port<P::in_type(K), IM_FULL, V>(a.in[K], row + e, row + e_end, kNoDiv, vec, x[K]);
    } else {
      const uint64_t w = word_from_storage(P::in_type(K), a.in[K], P::in_map(K) == IM_SCALAR ? 0 : o_idx);
#pragma unroll
      for (int v = 0; v < V; ++v) x[K][v] = w;
    }
    spec_load<P, K + 1, V>(a, row, e, e_end, o_idx, vec, x);
  }
}

template <class P, int I, int V>
__device__ __forceinline__ void spec_exec(uint64_t (&r)[P::kInsn][V], const uint64_t (&x)[P::kIn][V]) {
  if constexpr (I < P::kInsn) {
    constexpr Insn ins = P::insn(I);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if constexpr (ins.op == OP_INPUT) r[I][v] = x[ins.a][v];
      else r[I][v] = eval_insn(ins.op, ins.type, ins.src_type, ins.aux, ins.imm, r[ins.a][v], r[ins.b][v], r[ins.c][v]);
    }
    spec_exec<P, I + 1, V>(r, x);
  }
}

// ---- fast f32 fold: ordered integer keys ------------------------------------------
// For f32 values every reduction of the specialised kernels is folded with
// integer arithmetic on an order-preserving key of the float's bits:
//   fkey(x) = x >= +0 ? bits | 0x80000000 : ~bits
// orders -inf < ... < -0 < +0 < ... < +inf exactly as llvm.maximum/minimum do.
//   max : key, NaN -> 0xffffffff (NaN wins), empty = 0
//   min : key, NaN -> 0          (NaN wins), empty = 0xffffffff
//   argmax/argmin : (canonical key, index) where -0 is mapped onto +0 (the
//         reference's ordered compares treat them as equal) and NaN wins; a
//         lane sees its elements in increasing index order, so strict compares
//         keep the first occurrence, and lanes combine lexicographically.
//   sum : f32 tree sums per unit, flushed into an f64 accumulator every U units.
// Warp combines use redux.sync (one instruction per 32-bit key).
__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <class R, int OP>
__device__ __forceinline__ constexpr bool set_has() {
  for (int k = 0; k < R::N; ++k)
    if (R::op(k) == OP) return true;
  return false;
}
template <class R>
__device__ __forceinline__ constexpr bool fast_set() {
  for (int k = 0; k < R::N; ++k) {
    const int o = R::op(k);
    if (o != RED_SUM && o != RED_MAX && o != RED_MIN && o != RED_ARGMAX && o != RED_ARGMIN) return false;
  }
  return true;
}

struct FastAcc {
  double ds;
  float fs;
  uint32_t kmax, kmin;
  uint32_t amax_k, amax_i, amin_k, amin_i;
  // fast (all-finite) path: float extremes and arg candidates, folded into the
  // key fields above by fast_settle once a span's vector part is done
  float vmax, vmin, bmax, bmin;
  uint32_t bmax_i, bmin_i;
};

__device__ __forceinline__ void fast_init(FastAcc& s) {
  s.ds = 0.0; s.fs = 0.0f;
  s.kmax = 0u; s.kmin = 0xffffffffu;
  s.amax_k = 0u; s.amax_i = 0xffffffffu;
  s.amin_k = 0xffffffffu; s.amin_i = 0xffffffffu;
  s.vmax = -INFINITY; s.vmin = INFINITY; s.bmax = -INFINITY; s.bmin = INFINITY;
  s.bmax_i = 0xffffffffu; s.bmin_i = 0xffffffffu;
}

template <class R>
__device__ __forceinline__ void fast_fold(FastAcc& s, float x, uint32_t idx) {
  const uint32_t k = fkey(x);
  const bool nan = x != x;
  if constexpr (set_has<R, RED_MAX>()) s.kmax = max(s.kmax, nan ? 0xffffffffu : k);
  if constexpr (set_has<R, RED_MIN>()) s.kmin = min(s.kmin, nan ? 0u : k);
  if constexpr (set_has<R, RED_ARGMAX>() || set_has<R, RED_ARGMIN>()) {
    const uint32_t kc = k == 0x7fffffffu ? 0x80000000u : k;  // -0 ties with +0
    if constexpr (set_has<R, RED_ARGMAX>()) {
      const uint32_t h = nan ? 0xffffffffu : kc;
      if (h > s.amax_k) { s.amax_k = h; s.amax_i = idx; }
    }
    if constexpr (set_has<R, RED_ARGMIN>()) {
      const uint32_t h = nan ? 0u : kc;
      if (h < s.amin_k) { s.amin_k = h; s.amin_i = idx; }
    }
  }
}

// Fold a complete unit of V values with local indices idx0 .. idx0+V-1,
// assuming every value is finite (no NaN, no infinity).  Per unit: raw keys,
// the unit's extreme raw key (one min/max per value), one canonicalisation and
// one compare for each arg reduction; the arg position is located only when
// the unit beats the running best.  The integer ALU pipe is the bottleneck of
// these folds, so sums and the finiteness probe use the FMA pipe.  Callers
// check finiteness afterwards (fast_all_finite) and refold exactly otherwise.
__device__ __forceinline__ uint32_t canon_key(uint32_t k) { return k == 0x7fffffffu ? 0x80000000u : k; }

template <class R>
__device__ __forceinline__ constexpr bool needs_probe() {
  return !set_has<R, RED_SUM>() && (set_has<R, RED_MAX>() || set_has<R, RED_MIN>() ||
                                    set_has<R, RED_ARGMAX>() || set_has<R, RED_ARGMIN>());
}

template <class R, int V>
__device__ __forceinline__ void fast_fold_full(FastAcc& s, const float (&x)[V], uint32_t idx0) {
  if constexpr (set_has<R, RED_SUM>()) {
    float t[V];
#pragma unroll
    for (int v = 0; v < V; ++v) t[v] = x[v];
#pragma unroll
    for (int w = V / 2; w > 0; w >>= 1)
#pragma unroll
      for (int v = 0; v < w; ++v) t[v] = __fadd_rn(t[v], t[v + w]);
    s.fs = __fadd_rn(s.fs, t[0]);
  } else if constexpr (needs_probe<R>()) {
#pragma unroll
    for (int v = 0; v < V; ++v) s.fs = __fmaf_rn(x[v], 0.0f, s.fs);  // NaN once any value is not finite
  }
  // With finite values fmaxf/fminf (FMNMX) are llvm.maximum/minimum: on sm_100
  // they order -0 below +0 in either operand order (pinned by the GPU tests
  // whose extrema are zeros of both signs).  Ordered compares tie -0 with +0,
  // as the reference's argmax/argmin do.
  if constexpr (set_has<R, RED_MAX>() || set_has<R, RED_ARGMAX>()) {
    float m = x[0];
#pragma unroll
    for (int v = 1; v < V; ++v) m = fmaxf(m, x[v]);
    if constexpr (set_has<R, RED_MAX>()) s.vmax = fmaxf(s.vmax, m);
    if constexpr (set_has<R, RED_ARGMAX>()) {
      if (m > s.bmax) {
        uint32_t pos = V - 1;
#pragma unroll
        for (int v = V - 1; v >= 0; --v)
          if (x[v] == m) pos = v;
        s.bmax = m;
        s.bmax_i = idx0 + pos;
      }
    }
  }
  if constexpr (set_has<R, RED_MIN>() || set_has<R, RED_ARGMIN>()) {
    float m = x[0];
#pragma unroll
    for (int v = 1; v < V; ++v) m = fminf(m, x[v]);
    if constexpr (set_has<R, RED_MIN>()) s.vmin = fminf(s.vmin, m);
    if constexpr (set_has<R, RED_ARGMIN>()) {
      if (m < s.bmin) {
        uint32_t pos = V - 1;
#pragma unroll
        for (int v = V - 1; v >= 0; --v)
          if (x[v] == m) pos = v;
        s.bmin = m;
        s.bmin_i = idx0 + pos;
      }
    }
  }
}

// True when the values folded by fast_fold_full were all finite: a finite sum
// (f64 cannot overflow on f32 inputs) or a finite probe.  Sum-only sets need
// no check (NaN and infinities propagate through the sum by IEEE rules).
template <class R>
__device__ __forceinline__ bool fast_all_finite(const FastAcc& s) {
  if constexpr (set_has<R, RED_SUM>()) {
    if constexpr (needs_probe<R>() || set_has<R, RED_MAX>() || set_has<R, RED_MIN>() ||
                  set_has<R, RED_ARGMAX>() || set_has<R, RED_ARGMIN>())
      return isfinite(s.ds + double(s.fs));
    else
      return true;
  } else if constexpr (needs_probe<R>()) {
    // the probe, including what fast_flush has moved into ds
    return isfinite(s.ds + double(s.fs));
  } else {
    return true;
  }
}

// Move the fast path's float state into the key fields.  Returns false when
// the span must be refolded exactly because a value was not finite.
template <class R>
__device__ __forceinline__ bool fast_settle(FastAcc& s) {
  if (!fast_all_finite<R>(s)) return false;
  if constexpr (set_has<R, RED_MAX>()) s.kmax = max(s.kmax, fkey(s.vmax));
  if constexpr (set_has<R, RED_MIN>()) s.kmin = min(s.kmin, fkey(s.vmin));
  if constexpr (set_has<R, RED_ARGMAX>())
    if (s.bmax_i != 0xffffffffu) { s.amax_k = canon_key(fkey(s.bmax)); s.amax_i = s.bmax_i; }
  if constexpr (set_has<R, RED_ARGMIN>())
    if (s.bmin_i != 0xffffffffu) { s.amin_k = canon_key(fkey(s.bmin)); s.amin_i = s.bmin_i; }
  return true;
}

// Fold one value (tails).
template <class R>
__device__ __forceinline__ void fast_fold_one(FastAcc& s, float x, uint32_t idx) {
  if constexpr (set_has<R, RED_SUM>()) s.fs = __fadd_rn(s.fs, x);
  fast_fold<R>(s, x, idx);
}

__device__ __forceinline__ void fast_flush(FastAcc& s) {
  s.ds += double(s.fs);
  s.fs = 0.0f;
}

template <class R>
__device__ __forceinline__ void fast_warp_reduce(FastAcc& s) {
  constexpr unsigned kAll = 0xffffffffu;
  fast_flush(s);
  if constexpr (set_has<R, RED_SUM>()) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s.ds += __shfl_xor_sync(kAll, s.ds, off);
  }
  if constexpr (set_has<R, RED_MAX>()) s.kmax = __reduce_max_sync(kAll, s.kmax);
  if constexpr (set_has<R, RED_MIN>()) s.kmin = __reduce_min_sync(kAll, s.kmin);
  if constexpr (set_has<R, RED_ARGMAX>()) {
    const uint32_t h = __reduce_max_sync(kAll, s.amax_k);
    s.amax_i = __reduce_min_sync(kAll, s.amax_k == h ? s.amax_i : 0xffffffffu);
    s.amax_k = h;
  }
  if constexpr (set_has<R, RED_ARGMIN>()) {
    const uint32_t h = __reduce_min_sync(kAll, s.amin_k);
    s.amin_i = __reduce_min_sync(kAll, s.amin_k == h ? s.amin_i : 0xffffffffu);
    s.amin_k = h;
  }
}

// Block-wide: warps reduce, then warp 0 reduces the per-warp results (fixed
// order for the f64 sum).  Valid in thread 0.
template <class R>
__device__ __forceinline__ void fast_block_reduce(FastAcc& s) {
  __shared__ FastAcc sh[kRedThreads / 32];
  fast_warp_reduce<R>(s);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = s;
  __syncthreads();
  if (warp == 0) {
    if (lane < int(blockDim.x >> 5)) s = sh[lane];
    else fast_init(s);
    fast_warp_reduce<R>(s);
  }
  __syncthreads();
}

// Result of reduction `op` as a record in the generic (value word, index)
// form used by the combine kernels.
template <int OP>
__device__ __forceinline__ RedPartial fast_record(const FastAcc& s, uint64_t index_base) {
  if constexpr (OP == RED_SUM) {
    return RedPartial{uint64_t(__double_as_longlong(s.ds)), -1};
  } else if constexpr (OP == RED_MAX) {
    const float v = s.kmax == 0u ? -INFINITY : s.kmax == 0xffffffffu ? __uint_as_float(0x7fffffffu) : fkey_value(s.kmax);
    return RedPartial{w_of_f32(v), -1};
  } else if constexpr (OP == RED_MIN) {
    const float v = s.kmin == 0xffffffffu ? INFINITY : s.kmin == 0u ? __uint_as_float(0x7fffffffu) : fkey_value(s.kmin);
    return RedPartial{w_of_f32(v), -1};
  } else if constexpr (OP == RED_ARGMAX) {
    if (s.amax_k == 0u) return RedPartial{0, -1};
    const float v = s.amax_k == 0xffffffffu ? __uint_as_float(0x7fffffffu) : fkey_value(s.amax_k);
    return RedPartial{w_of_f32(v), int64_t(index_base + s.amax_i)};
  } else {
    if (s.amin_k == 0xffffffffu) return RedPartial{0, -1};
    const float v = s.amin_k == 0u ? __uint_as_float(0x7fffffffu) : fkey_value(s.amin_k);
    return RedPartial{w_of_f32(v), int64_t(index_base + s.amin_i)};
  }
}

template <class R, int K>
__device__ __forceinline__ void fast_records(const FastAcc& s, uint64_t index_base, RedPartial* dst) {
  if constexpr (K < R::N) {
    dst[K] = fast_record<R::op(K)>(s, index_base);
    fast_records<R, K + 1>(s, index_base, dst);
  }
}

// Write the outputs of one output index from a finished fast accumulator.
template <class R, int K>
__device__ __forceinline__ void fast_write(const RedArgs& a, const FastAcc& s, uint64_t o_idx) {
  if constexpr (K < R::N) {
    constexpr int op = R::op(K);
    const RedPartial r = fast_record<op>(s, a.index_base);
    word_to_storage(out_type_of(op, kF32), a.out[K], o_idx, acc_result(op, kF32, r.v, r.idx));
    fast_write<R, K + 1>(a, s, o_idx);
  }
}

// ---- value sources of the specialised reductions -------------------------------
// Each source turns one 16-byte load into V f32 values exactly as the matching
// program in programs.h does (the program is what the plan is matched on).
struct SrcF32 {  // ProgIdentity<f32>
  static constexpr int V = 4;
  struct Row {};
  __device__ static Row row(const RedArgs&, uint64_t) { return {}; }
  __device__ static void values(const Row&, uint4 r, float (&x)[V]) {
    x[0] = __uint_as_float(r.x); x[1] = __uint_as_float(r.y); x[2] = __uint_as_float(r.z); x[3] = __uint_as_float(r.w);
  }
  __device__ static float value_at(const RedArgs& a, const Row&, uint64_t i) {
    return static_cast<const float*>(a.in[0])[i];
  }
  static constexpr int kBytes = 4;
  static constexpr int kUnroll = 8;
};

template <int T>
__device__ __forceinline__ float half_to_f32(uint32_t h) {
  if constexpr (T == kF16) return __half2float(__ushort_as_half(uint16_t(h)));
  else return __uint_as_float(h << 16);
}

template <int T>
struct SrcCast {  // ProgSoftmaxMax<T>: cast(x, f32)
  static constexpr int V = 8;
  struct Row {};
  __device__ static Row row(const RedArgs&, uint64_t) { return {}; }
  __device__ static void values(const Row&, uint4 r, float (&x)[V]) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) { x[2 * j] = half_to_f32<T>(w[j] & 0xffffu); x[2 * j + 1] = half_to_f32<T>(w[j] >> 16); }
  }
  __device__ static float value_at(const RedArgs& a, const Row&, uint64_t i) {
    return half_to_f32<T>(static_cast<const uint16_t*>(a.in[0])[i]);
  }
  static constexpr int kBytes = 2;
  static constexpr int kUnroll = 4;
};

template <int T>
struct SrcExpShift {  // ProgSoftmaxSum<T>: exp(cast(x, f32) + m*(-1)), m indexed by the row
  static constexpr int V = 8;
  struct Row { float nm; };
  __device__ static Row row(const RedArgs& a, uint64_t o) {
    return Row{__fmul_rn(static_cast<const float*>(a.in[1])[o], -1.0f)};
  }
  __device__ static void values(const Row& rw, uint4 r, float (&x)[V]) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[2 * j] = expf(__fadd_rn(half_to_f32<T>(w[j] & 0xffffu), rw.nm));
      x[2 * j + 1] = expf(__fadd_rn(half_to_f32<T>(w[j] >> 16), rw.nm));
    }
  }
  __device__ static float value_at(const RedArgs& a, const Row& rw, uint64_t i) {
    return expf(__fadd_rn(half_to_f32<T>(static_cast<const uint16_t*>(a.in[0])[i]), rw.nm));
  }
  static constexpr int kBytes = 2;
  static constexpr int kUnroll = 4;
};

// Scalar fold of elements [e, e1) of a row, stepping by `step` (tails, unaligned rows).
template <class S, class R>
__device__ __forceinline__ void span_scalar(const RedArgs& a, const typename S::Row& rw, uint64_t row, uint64_t e,
                                            uint64_t e1, uint64_t step, FastAcc& s) {
  for (; e < e1; e += step) {
#pragma unroll
    for (int v = 0; v < S::V; ++v)
      if (e + v < e1) fast_fold_one<R>(s, S::value_at(a, rw, row + e + v), uint32_t(e + v));
    fast_flush(s);
  }
}

// Contiguous span [e0, e1) of row `row` (element index of (o, 0)), processed by
// thread t of T cooperating threads in units of S::V elements (e0 a multiple of
// S::V), U 16-byte loads in flight per thread.  Local indices (e) fit 32 bits:
// the plan layer guarantees extent <= 2^32.
template <class S, class R, int U>
__device__ __forceinline__ void span_src(const RedArgs& a, const typename S::Row& rw, uint64_t row, uint64_t e0,
                                         uint64_t e1, uint32_t t, uint32_t T, bool aligned, FastAcc& s) {
  constexpr int V = S::V;
  const char* base = static_cast<const char*>(a.in[0]) + row * S::kBytes;
  uint64_t e = e0 + uint64_t(t) * V;
  if (aligned) {
    const uint64_t step = uint64_t(T) * V;
    for (; e + (U - 1) * step + V <= e1; e += step * U) {
      uint4 raw[U];
#pragma unroll
      for (int q = 0; q < U; ++q) raw[q] = ld_stream_v4(base + (e + q * step) * S::kBytes);
#pragma unroll
      for (int q = 0; q < U; ++q) {
        float x[V];
        S::values(rw, raw[q], x);
        fast_fold_full<R, V>(s, x, uint32_t(e + q * step));
      }
      fast_flush(s);
    }
    for (; e + V <= e1; e += step) {
      float x[V];
      S::values(rw, ld_stream_v4(base + e * S::kBytes), x);
      fast_fold_full<R, V>(s, x, uint32_t(e));
    }
    fast_flush(s);
    if (!fast_settle<R>(s)) {
      // NaN or infinity among this thread's values, or a zero extremum:
      // refold them exactly (NaN-aware keys) in the same increasing order.
      fast_init(s);
      span_scalar<S, R>(a, rw, row, e0 + uint64_t(t) * V, e1, uint64_t(T) * V, s);
      return;
    }
  }
  span_scalar<S, R>(a, rw, row, e, e1, uint64_t(T) * V, s);
}

// inner == 1: a warp per output row (RS_WARP_ROW), compile-time source S and set R.
template <class S, class R, int U>
__device__ __forceinline__ void red_warp_row_loop(const RedArgs& a, int aligned) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warp = (uint64_t(blockIdx.x) * kRedThreads + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t(gridDim.x) * kRedThreads) >> 5;
  for (uint64_t o = warp; o < a.outer; o += nwarps) {
    FastAcc s;
    fast_init(s);
    const typename S::Row rw = S::row(a, o);
    span_src<S, R, U>(a, rw, o * a.extent, 0, a.extent, lane, 32, aligned != 0, s);
    fast_warp_reduce<R>(s);
    if (lane == 0) fast_write<R, 0>(a, s, o);
  }
}

}  // namespace red
}  // namespace askb
