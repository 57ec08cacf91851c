// Families R and T: map-reduce over a canonical [outer, extent, inner] domain.
//
// One launch evaluates a prologue op program per element and folds every
// requested reduction (sum, prod, max, min, any, all, argmax, argmin) in a
// single pass over the input.  Reference behaviour it replaces:
//   * ScalarEmitter::reduce / accumulate (lib/Lowering/ScalarEmitter.h:263-287,
//     420-472): initial values sum 0, prod 1, min +inf/INT_MAX, max -inf/INT_MIN,
//     any false, all true (ScalarEmitter.h:426-439);
//   * the warp-cooperative reduction (ScalarEmitter.h:288-415) -- one warp per
//     output, butterfly shuffles -- which the reference only picks when no
//     argmax/argmin shares the batch (lib/Lowering/CUDA.cpp:51-88);
//   * argmax/argmin (ScalarEmitter.h:473-529): a candidate wins iff it is NaN
//     and the best is not, or it is strictly better in an ordered compare, so
//     ties keep the lowest index and the first NaN wins.  The parallel combine
//     used here is the lexicographic order (NaN first, better value, lower
//     index), which is associative and gives the sequential answer bit-exactly.
// Each reduction's result is written once per output; float sums accumulate in
// f64 (B200's FP64 rate is far above what an HBM-bound pass needs) and are
// rounded to the output type at the end, f16/bf16 operands are folded in f32
// like the reference's warp path (ScalarEmitter.h:311, 335, 414).
//
// Strategies (chosen by the plan layer):
//   RS_WARP_ROW  inner == 1: a warp owns an output row, lanes stride the row
//                with 16-byte loads, U loads in flight per lane.
//   RS_COLUMN    inner > 1: a thread owns an output column, loads coalesce
//                across the inner axis.
//   RS_SPLIT     few outputs over a huge extent (0-D reductions such as cfg5):
//                every CTA folds one contiguous chunk into a partial record in
//                scratch; a second single-CTA-per-output kernel combines the
//                records in a fixed order, so the result is deterministic.
#include <cuda_runtime.h>
#include <float.h>

#include "ask_numerics.cuh"
#include "kernels.h"
#include "programs.h"
#include "vec_io.cuh"
#include "reduce_acc.cuh"

namespace askb {

namespace {

using namespace red;

struct Accs {
  uint64_t v[kMaxReductions];
  int64_t i[kMaxReductions];
};

__device__ __forceinline__ void accs_init(const RedArgs& a, Accs& s) {
#pragma unroll
  for (int k = 0; k < kMaxReductions; ++k)
    if (k < a.n_red) acc_init(a.red_op[k], a.red_type[k], s.v[k], s.i[k]);
}

__device__ __forceinline__ void accs_merge(const RedArgs& a, Accs& s, const Accs& o) {
#pragma unroll
  for (int k = 0; k < kMaxReductions; ++k)
    if (k < a.n_red) acc_fold<true>(a.red_op[k], a.red_type[k], s.v[k], s.i[k], o.v[k], o.i[k]);
}

// Butterfly over the 32 lanes; every lane ends with the warp's result.
__device__ __forceinline__ void accs_warp_reduce(const RedArgs& a, Accs& s) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Accs o;
#pragma unroll
    for (int k = 0; k < kMaxReductions; ++k) {
      if (k < a.n_red) {
        o.v[k] = __shfl_xor_sync(0xffffffffu, s.v[k], off);
        o.i[k] = __shfl_xor_sync(0xffffffffu, s.i[k], off);
      }
    }
    accs_merge(a, s, o);
  }
}

// Block-wide fold in a fixed order: warps butterfly, then warp 0 folds the
// per-warp results.  Result valid in thread 0.
__device__ __forceinline__ void accs_block_reduce(const RedArgs& a, Accs& s) {
  __shared__ uint64_t sv[kRedThreads / 32][kMaxReductions];
  __shared__ int64_t si[kRedThreads / 32][kMaxReductions];
  accs_warp_reduce(a, s);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < kMaxReductions; ++k)
      if (k < a.n_red) { sv[warp][k] = s.v[k]; si[warp][k] = s.i[k]; }
  }
  __syncthreads();
  if (warp == 0) {
    if (lane < int(blockDim.x >> 5)) {
#pragma unroll
      for (int k = 0; k < kMaxReductions; ++k)
        if (k < a.n_red) { s.v[k] = sv[lane][k]; s.i[k] = si[lane][k]; }
    } else {
      accs_init(a, s);
    }
    accs_warp_reduce(a, s);
  }
  __syncthreads();
}

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
    return isfinite(s.fs);
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

// Runtime-program version of span_spec (one unit in flight, registers in local memory).
template <int V>
__device__ __forceinline__ void span_generic(const Program& prog, const RedArgs& a, uint64_t row, uint64_t o_idx,
                                             uint64_t e0, uint64_t e1, uint32_t t, uint32_t T, bool aligned, Accs& s,
                                             uint64_t (*r)[V]) {
  for (uint64_t e = e0 + uint64_t(t) * V; e < e1; e += uint64_t(T) * V) {
    const bool vec = aligned && e + V <= e1;
    for (int i = 0; i < prog.n_insn; ++i) {
      const Insn& ins = prog.insn[i];
      if (ins.op == OP_INPUT) {
        const int map = prog.in_map[ins.a];
        uint64_t w[V];
        if (map == IM_FULL) {
          rt_load<V>(prog.in_type[ins.a], IM_FULL, a.in[ins.a], row + e, row + e1, kNoDiv, vec, w);
        } else {
          const uint64_t sv = word_from_storage(prog.in_type[ins.a], a.in[ins.a], map == IM_SCALAR ? 0 : o_idx);
#pragma unroll
          for (int v = 0; v < V; ++v) w[v] = sv;
        }
#pragma unroll
        for (int v = 0; v < V; ++v) r[ins.dst][v] = w[v];
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v)
          r[ins.dst][v] = eval_insn(ins.op, ins.type, ins.src_type, ins.aux, ins.imm, r[ins.a][v], r[ins.b][v], r[ins.c][v]);
      }
    }
#pragma unroll
    for (int k = 0; k < kMaxReductions; ++k) {
      if (k < a.n_red) {
        const int reg = prog.out_reg[a.red_src[k]];
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (e + v < e1)
            acc_fold<false>(a.red_op[k], a.red_type[k], s.v[k], s.i[k], r[reg][v], int64_t(a.index_base + e + v));
      }
    }
  }
}

__device__ __forceinline__ void write_outputs(const RedArgs& a, const Accs& s, uint64_t o_idx) {
#pragma unroll
  for (int k = 0; k < kMaxReductions; ++k) {
    if (k < a.n_red) {
      const int op = a.red_op[k], t = a.red_type[k];
      word_to_storage(out_type_of(op, t), a.out[k], o_idx, acc_result(op, t, s.v[k], s.i[k]));
    }
  }
}

// ---- kernels ---------------------------------------------------------------------
template <class S, class R, int U>
__global__ void __launch_bounds__(kRedThreads)
    red_warp_row_kernel(const __grid_constant__ RedArgs a, int aligned) {
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

template <int V>
__global__ void __launch_bounds__(kRedThreads)
    red_warp_row_generic(const __grid_constant__ Program prog, const __grid_constant__ RedArgs a, int aligned) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warp = (uint64_t(blockIdx.x) * kRedThreads + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t(gridDim.x) * kRedThreads) >> 5;
  uint64_t r[kMaxRegs][V];
  for (uint64_t o = warp; o < a.outer; o += nwarps) {
    Accs s;
    accs_init(a, s);
    span_generic<V>(prog, a, o * a.extent, o, 0, a.extent, lane, 32, aligned != 0, s, r);
    accs_warp_reduce(a, s);
    if (lane == 0) write_outputs(a, s, o);
  }
}

// inner > 1: thread per output (o, n); element (o, e, n) at (o*extent + e)*inner + n.
__global__ void __launch_bounds__(kRedThreads)
    red_column_generic(const __grid_constant__ Program prog, const __grid_constant__ RedArgs a) {
  const uint64_t n_outputs = a.outer * a.inner;
  uint64_t r[kMaxRegs][1];
  for (uint64_t o_idx = uint64_t(blockIdx.x) * kRedThreads + threadIdx.x; o_idx < n_outputs;
       o_idx += uint64_t(gridDim.x) * kRedThreads) {
    const uint64_t o = o_idx / a.inner, n = o_idx % a.inner;
    Accs s;
    accs_init(a, s);
    for (uint64_t e = 0; e < a.extent; ++e) {
      const uint64_t idx = (o * a.extent + e) * a.inner + n;
      for (int i = 0; i < prog.n_insn; ++i) {
        const Insn& ins = prog.insn[i];
        if (ins.op == OP_INPUT) {
          const int map = prog.in_map[ins.a];
          r[ins.dst][0] = word_from_storage(prog.in_type[ins.a], a.in[ins.a],
                                            map == IM_FULL ? idx : map == IM_SCALAR ? 0 : o_idx);
        } else {
          r[ins.dst][0] = eval_insn(ins.op, ins.type, ins.src_type, ins.aux, ins.imm, r[ins.a][0], r[ins.b][0], r[ins.c][0]);
        }
      }
#pragma unroll
      for (int k = 0; k < kMaxReductions; ++k)
        if (k < a.n_red)
          acc_fold<false>(a.red_op[k], a.red_type[k], s.v[k], s.i[k], r[prog.out_reg[a.red_src[k]]][0],
                          int64_t(a.index_base + e));
    }
    write_outputs(a, s, o_idx);
  }
}

// Chunk of the extent owned by CTA c of G, aligned to whole units of V*U*blockDim.
__device__ __forceinline__ void split_chunk(uint64_t extent, uint32_t c, uint32_t g, uint64_t granule, uint64_t& e0,
                                            uint64_t& e1) {
  const uint64_t granules = (extent + granule - 1) / granule;
  const uint64_t per = (granules + g - 1) / g;
  e0 = min(extent, uint64_t(c) * per * granule);
  e1 = min(extent, e0 + per * granule);
}

template <class S, class R, int U>
__global__ void __launch_bounds__(kRedThreads)
    red_split_kernel(const __grid_constant__ RedArgs a, int aligned, RedPartial* __restrict__ part) {
  for (uint64_t o = 0; o < a.outer; ++o) {
    uint64_t e0, e1;
    split_chunk(a.extent, blockIdx.x, gridDim.x, uint64_t(S::V) * 32, e0, e1);
    FastAcc s;
    fast_init(s);
    const typename S::Row rw = S::row(a, o);
    span_src<S, R, U>(a, rw, o * a.extent, e0, e1, threadIdx.x, kRedThreads, aligned != 0, s);
    fast_block_reduce<R>(s);
    if (threadIdx.x == 0) fast_records<R, 0>(s, a.index_base, part + (o * gridDim.x + blockIdx.x) * R::N);
  }
}

// Fold n partial records of each output (layout [outer][n][N]) in a fixed
// order; the reduction set is a compile-time constant.
template <class R, int VT>
__global__ void __launch_bounds__(kRedThreads)
    red_combine_set_kernel(const __grid_constant__ RedArgs a, const RedPartial* __restrict__ part, int n,
                           RedPartial* __restrict__ rec_out) {
  const uint64_t o = blockIdx.x;
  AccsT<R> s;
  set_init<R, VT, 0>(s);
  for (int j = threadIdx.x; j < n; j += kRedThreads) {
    const RedPartial* src = part + (o * n + j) * R::N;
    AccsT<R> x;
#pragma unroll
    for (int k = 0; k < R::N; ++k) { x.v[k] = src[k].v; x.i[k] = src[k].idx; }
    set_merge<R, VT, 0>(s, x);
  }
  set_block_reduce<R, VT>(s);
  if (threadIdx.x == 0) {
    if (rec_out) {
#pragma unroll
      for (int k = 0; k < R::N; ++k) rec_out[o * R::N + k] = RedPartial{s.v[k], s.i[k]};
    } else {
      set_write<R, VT>(a, s, o);
    }
  }
}

template <int V>
__global__ void __launch_bounds__(kRedThreads)
    red_split_generic(const __grid_constant__ Program prog, const __grid_constant__ RedArgs a, int aligned,
                      RedPartial* __restrict__ part) {
  uint64_t r[kMaxRegs][V];
  for (uint64_t o = 0; o < a.outer; ++o) {
    uint64_t e0, e1;
    split_chunk(a.extent, blockIdx.x, gridDim.x, uint64_t(V) * 32, e0, e1);
    Accs s;
    accs_init(a, s);
    span_generic<V>(prog, a, o * a.extent, o, e0, e1, threadIdx.x, kRedThreads, aligned != 0, s, r);
    accs_block_reduce(a, s);
    if (threadIdx.x == 0) {
      RedPartial* dst = part + (o * gridDim.x + blockIdx.x) * a.n_red;
      for (int k = 0; k < a.n_red; ++k) dst[k] = RedPartial{s.v[k], s.i[k]};
    }
  }
}

// Fold n partial records of output o (layout [outer][n][n_red]) in a fixed
// order.  Writes the outputs, or one record per output when `rec_out` is set.
__global__ void __launch_bounds__(kRedThreads)
    red_combine_kernel(const __grid_constant__ RedArgs a, const RedPartial* __restrict__ part, int n,
                       RedPartial* __restrict__ rec_out) {
  const uint64_t o = blockIdx.x;
  Accs s;
  accs_init(a, s);
  for (int j = threadIdx.x; j < n; j += kRedThreads) {
    const RedPartial* src = part + (o * n + j) * a.n_red;
    Accs x;
#pragma unroll
    for (int k = 0; k < kMaxReductions; ++k)
      if (k < a.n_red) { x.v[k] = src[k].v; x.i[k] = src[k].idx; }
    accs_merge(a, s, x);
  }
  accs_block_reduce(a, s);
  if (threadIdx.x == 0) {
    if (rec_out) {
      for (int k = 0; k < a.n_red; ++k) rec_out[o * a.n_red + k] = RedPartial{s.v[k], s.i[k]};
    } else {
      write_outputs(a, s, o);
    }
  }
}

// ---- specialisation table ------------------------------------------------------------
using SetRowStats = RedSet<RED_SUM, RED_MAX, RED_MIN, RED_ARGMAX>;
using SetGlobal = RedSet<RED_SUM, RED_MIN, RED_ARGMIN>;
using SetMax = RedSet<RED_MAX>;
using SetSum = RedSet<RED_SUM>;

// 16-byte loads in flight per lane per iteration (S::kUnroll): 8 (128 bytes)
// where the fold is light on registers, 4 for the widening f16/bf16 source.
template <class S> struct Unroll { static constexpr int U = S::kUnroll; };

// Calls f(program, source, set) for the specialisation `spec`.
template <class F>
bool with_spec(int spec, F&& f) {
  switch (spec) {
    case RED_ROWSTATS_F32: f(ProgIdentity<kF32>{}, SrcF32{}, SetRowStats{}); return true;
    case RED_GLOBAL_F32: f(ProgIdentity<kF32>{}, SrcF32{}, SetGlobal{}); return true;
    case RED_SOFTMAX_MAX_F16: f(ProgSoftmaxMax<kF16>{}, SrcCast<kF16>{}, SetMax{}); return true;
    case RED_SOFTMAX_MAX_BF16: f(ProgSoftmaxMax<kBF16>{}, SrcCast<kBF16>{}, SetMax{}); return true;
    case RED_SOFTMAX_SUM_F16: f(ProgSoftmaxSum<kF16>{}, SrcExpShift<kF16>{}, SetSum{}); return true;
    case RED_SOFTMAX_SUM_BF16: f(ProgSoftmaxSum<kBF16>{}, SrcExpShift<kBF16>{}, SetSum{}); return true;
    default: return false;
  }
}

const void* kernel_ptr(int spec, int strategy) {
  const void* ptr = nullptr;
  const bool found = with_spec(spec, [&](auto, auto src, auto r) {
    using S = decltype(src);
    using R = decltype(r);
    ptr = strategy == RS_WARP_ROW ? reinterpret_cast<const void*>(&red_warp_row_kernel<S, R, Unroll<S>::U>)
                                  : reinterpret_cast<const void*>(&red_split_kernel<S, R, Unroll<S>::U>);
  });
  if (found && strategy != RS_COLUMN) return ptr;
  if (strategy == RS_WARP_ROW) return reinterpret_cast<const void*>(&red_warp_row_generic<4>);
  if (strategy == RS_COLUMN) return reinterpret_cast<const void*>(&red_column_generic);
  return reinterpret_cast<const void*>(&red_split_generic<4>);
}

}  // namespace

bool red_spec_program(int spec, Program* out, int* n_red, uint8_t* ops) {
  return with_spec(spec, [&](auto p, auto, auto r) {
    using P = decltype(p);
    using R = decltype(r);
    *out = program_of<P>();
    *n_red = R::N;
    for (int k = 0; k < R::N; ++k) ops[k] = uint8_t(R::op(k));
  });
}

cudaError_t red_occupancy(int spec, int strategy, int* blocks_per_sm) {
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kernel_ptr(spec, strategy), kRedThreads, 0);
}

size_t red_split_scratch_bytes(int grid, int n_red) { return size_t(grid) * size_t(n_red) * sizeof(RedPartial); }

cudaError_t red_launch(int spec, int strategy, const Program& prog, const RedArgs& a, int aligned, int grid,
                       void* scratch, RedPartial* rec_out, cudaStream_t st) {
  if (a.outer == 0 || a.inner == 0) return cudaSuccess;
  if (strategy == RS_COLUMN) {
    red_column_generic<<<grid, kRedThreads, 0, st>>>(prog, a);
    return cudaGetLastError();
  }
  cudaError_t err = cudaSuccess;
  const bool found = with_spec(spec, [&](auto, auto src, auto r) {
    using S = decltype(src);
    using R = decltype(r);
    constexpr int U = Unroll<S>::U;
    if (strategy == RS_WARP_ROW) {
      red_warp_row_kernel<S, R, U><<<grid, kRedThreads, 0, st>>>(a, aligned);
      err = cudaGetLastError();
      return;
    }
    RedPartial* part = static_cast<RedPartial*>(scratch);
    red_split_kernel<S, R, U><<<grid, kRedThreads, 0, st>>>(a, aligned, part);
    err = cudaGetLastError();
    if (err != cudaSuccess) return;
    red_combine_set_kernel<R, kF32><<<unsigned(a.outer), kRedThreads, 0, st>>>(a, part, grid, rec_out);
    err = cudaGetLastError();
  });
  if (found) return err;
  if (strategy == RS_WARP_ROW) {
    red_warp_row_generic<4><<<grid, kRedThreads, 0, st>>>(prog, a, aligned);
    return cudaGetLastError();
  }
  RedPartial* part = static_cast<RedPartial*>(scratch);
  red_split_generic<4><<<grid, kRedThreads, 0, st>>>(prog, a, aligned, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  red_combine_kernel<<<unsigned(a.outer), kRedThreads, 0, st>>>(a, part, grid, rec_out);
  return cudaGetLastError();
}

cudaError_t red_combine_records(const RedArgs& a, const RedPartial* records, int n, cudaStream_t st) {
  red_combine_kernel<<<unsigned(a.outer), kRedThreads, 0, st>>>(a, records, n, nullptr);
  return cudaGetLastError();
}

}  // namespace askb
