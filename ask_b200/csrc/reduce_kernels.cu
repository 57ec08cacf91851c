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

#include <algorithm>

#include "ask_numerics.cuh"
#include "kernels.h"
#include "programs.h"
#include "vec_io.cuh"
#include "pdl.cuh"
#include "reduce_acc.cuh"
#include "reduce_fast.cuh"
#include "ew_body.cuh"

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
  pdl_enter();
  red_warp_row_loop<S, R, U>(a, aligned);
}

template <int V>
__global__ void __launch_bounds__(kRedThreads)
    red_warp_row_generic(const __grid_constant__ Program prog, const __grid_constant__ RedArgs a, int aligned) {
  pdl_enter();
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

// Fold elements e0 <= e < e1 of column (o, n) -- element (o, e, n) at
// (o*extent + e)*inner + n -- into s, in order.  A program reading one full
// port (the common prologue) has four elements' loads issued before it
// interprets them, so more than one load per thread is in flight.
__device__ __forceinline__ void column_fold(const Program& prog, const RedArgs& a, uint64_t o, uint64_t n,
                                            uint64_t o_idx, uint64_t e0, uint64_t e1, Accs& s) {
  uint64_t r[kMaxRegs][1];
  auto run = [&](uint64_t e, bool loaded, uint64_t w) {
    const uint64_t idx = (o * a.extent + e) * a.inner + n;
    for (int i = 0; i < prog.n_insn; ++i) {
      const Insn& ins = prog.insn[i];
      if (ins.op == OP_INPUT) {
        const int map = prog.in_map[ins.a];
        r[ins.dst][0] = loaded ? w : word_from_storage(prog.in_type[ins.a], a.in[ins.a],
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
  };
  uint64_t e = e0;
  if (prog.n_in == 1 && prog.in_map[0] == IM_FULL) {
    const int t = prog.in_type[0];
    const void* p = a.in[0];
    for (; e + 4 <= e1; e += 4) {
      uint64_t w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) w[u] = word_from_storage(t, p, (o * a.extent + e + u) * a.inner + n);
#pragma unroll
      for (int u = 0; u < 4; ++u) run(e + u, true, w[u]);
    }
  }
  for (; e < e1; ++e) run(e, false, 0);
}

// inner > 1: thread per output (o, n).
__global__ void __launch_bounds__(kRedThreads)
    red_column_generic(const __grid_constant__ Program prog, const __grid_constant__ RedArgs a) {
  pdl_enter();
  const uint64_t n_outputs = a.outer * a.inner;
  for (uint64_t o_idx = uint64_t(blockIdx.x) * kRedThreads + threadIdx.x; o_idx < n_outputs;
       o_idx += uint64_t(gridDim.x) * kRedThreads) {
    const uint64_t o = o_idx / a.inner, n = o_idx % a.inner;
    Accs s;
    accs_init(a, s);
    column_fold(prog, a, o, n, o_idx, 0, a.extent, s);
    write_outputs(a, s, o_idx);
  }
}

// inner > 1 with few outputs: the column kernel's thread per output would
// leave most of the GPU idle over a long extent, so grid.y splits the extent
// into chunks.  Thread (o_idx, chunk) folds its chunk's elements of one column
// (consecutive threads read consecutive columns) into a partial record at
// part[(chunk * n_outputs + o_idx) * n_red]; red_column_combine then folds
// each output's records in chunk order, so the result does not depend on
// timing.  No chunk is empty (the host picks the chunk count so).
__global__ void __launch_bounds__(kRedThreads)
    red_column_chunks(const __grid_constant__ Program prog, const __grid_constant__ RedArgs a,
                      RedPartial* __restrict__ part) {
  pdl_enter();
  const uint64_t n_outputs = a.outer * a.inner;
  const uint64_t chunks = gridDim.y, c = blockIdx.y;
  const uint64_t per = (a.extent + chunks - 1) / chunks;
  const uint64_t e0 = min(a.extent, c * per), e1 = min(a.extent, e0 + per);
  for (uint64_t o_idx = uint64_t(blockIdx.x) * kRedThreads + threadIdx.x; o_idx < n_outputs;
       o_idx += uint64_t(gridDim.x) * kRedThreads) {
    const uint64_t o = o_idx / a.inner, n = o_idx % a.inner;
    Accs s;
    accs_init(a, s);
    column_fold(prog, a, o, n, o_idx, e0, e1, s);
    RedPartial* dst = part + (c * n_outputs + o_idx) * a.n_red;
    for (int k = 0; k < a.n_red; ++k) dst[k] = RedPartial{s.v[k], s.i[k]};
  }
}

// A thread per output folds its `chunks` partial records in chunk order
// (records of consecutive outputs are adjacent, so the loads coalesce).
__global__ void __launch_bounds__(kRedThreads)
    red_column_combine(const __grid_constant__ RedArgs a, const RedPartial* __restrict__ part, int chunks) {
  pdl_enter();
  const uint64_t n_outputs = a.outer * a.inner;
  for (uint64_t o_idx = uint64_t(blockIdx.x) * kRedThreads + threadIdx.x; o_idx < n_outputs;
       o_idx += uint64_t(gridDim.x) * kRedThreads) {
    Accs s;
    accs_init(a, s);
    for (int c = 0; c < chunks; ++c) {
      const RedPartial* src = part + (uint64_t(c) * n_outputs + o_idx) * a.n_red;
      Accs x;
#pragma unroll
      for (int k = 0; k < kMaxReductions; ++k)
        if (k < a.n_red) { x.v[k] = src[k].v; x.i[k] = src[k].idx; }
      accs_merge(a, s, x);
    }
    write_outputs(a, s, o_idx);
  }
}

// General index maps (RS_VIEW): a warp per output (o, n); lanes stride the
// reduced extent.  A lane's coordinates in the step's iteration shape are
// computed once per output and advanced by its stride (32 elements of the
// extent) with carries; IM_VIEW ports map them through their view (transpose,
// slice, pad, general broadcast of an argument) and OP_COORD reads them, as in
// the elementwise view loop.  Scalar loads: this path serves coverage, the
// benchmark reductions read full, outer or scalar ports.
__global__ void __launch_bounds__(kRedThreads)
    red_view_generic(const __grid_constant__ Program prog, const __grid_constant__ RedArgs a,
                     const __grid_constant__ ViewSet views) {
  pdl_enter();
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warp = (uint64_t(blockIdx.x) * kRedThreads + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t(gridDim.x) * kRedThreads) >> 5;
  const uint64_t n_outputs = a.outer * a.inner;
  uint64_t r[kMaxRegs];
  int64_t by[kMaxRank];  // a lane's step e += 32 moves the linear index by 32 * inner
  ew::view_stride_digits(32 * a.inner, views, by);
  for (uint64_t o_idx = warp; o_idx < n_outputs; o_idx += nwarps) {
    const uint64_t o = o_idx / a.inner, n = o_idx % a.inner;
    Accs s;
    accs_init(a, s);
    int64_t c[kMaxRank];
    if (lane < a.extent) ew::view_coords((o * a.extent + lane) * a.inner + n, views, c);
    for (uint64_t e = lane; e < a.extent; e += 32, ew::view_advance(c, by, views)) {
      const uint64_t i = (o * a.extent + e) * a.inner + n;
      for (int k = 0; k < prog.n_insn; ++k) {
        const Insn& ins = prog.insn[k];
        if (ins.op == OP_INPUT) {
          const int port = ins.a, t = prog.in_type[port];
          const void* p = a.in[port];
          switch (prog.in_map[port]) {
            case IM_SCALAR: r[ins.dst] = word_from_storage(t, p, 0); break;
            case IM_OUTER: r[ins.dst] = word_from_storage(t, p, o_idx); break;
            case IM_VIEW: r[ins.dst] = ew::view_read(views.port[port], views.rank, c, t, p); break;
            default: r[ins.dst] = word_from_storage(t, p, i); break;
          }
        } else if (ins.op == OP_COORD) {
          r[ins.dst] = uint64_t(c[ins.aux]);
        } else {
          r[ins.dst] = eval_insn(ins.op, ins.type, ins.src_type, ins.aux, ins.imm, r[ins.a], r[ins.b], r[ins.c]);
        }
      }
#pragma unroll
      for (int k = 0; k < kMaxReductions; ++k)
        if (k < a.n_red)
          acc_fold<false>(a.red_op[k], a.red_type[k], s.v[k], s.i[k], r[prog.out_reg[a.red_src[k]]],
                          int64_t(a.index_base + e));
    }
    accs_warp_reduce(a, s);
    if (lane == 0) write_outputs(a, s, o_idx);
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
  pdl_enter();
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
  pdl_enter();
  const uint64_t o = blockIdx.x;
  AccsT<R> s;
  set_init<R, VT, 0>(s);
  for (int j = threadIdx.x; j < n; j += int(blockDim.x)) {
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
  pdl_enter();
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
  pdl_enter();
  const uint64_t o = blockIdx.x;
  Accs s;
  accs_init(a, s);
  for (int j = threadIdx.x; j < n; j += int(blockDim.x)) {
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

// A sharded reduction's record combine and its exchange run one warp per
// output: small enough (registers, threads) to be resident beside a persistent
// streaming grid that fills the SMs (a sharded step runs them beside the i32
// chain), so they need not wait for that grid to drain.  A combine that writes
// the outputs of a single-GPU launch keeps the full CTA (nothing runs beside it).
constexpr int kCombineThreads = 32;

// ---- cross-GPU record exchange over peer memory ------------------------------------------
// Inbox layout (kernels.h): records [2 parities][ranks][kMaxReductions], then
// one flag per rank, the epoch counter and the status word.  Every launch takes
// the next epoch e; rank r stores its records into slot (e & 1, r) of every
// inbox and raises flag r to e.  A rank can be at most one epoch ahead of
// another (it waits for everyone's flag before it finishes), so the parity
// keeps a fast rank's next records out of the slots a slow rank still reads.
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(kRedThreads)
    red_exchange_kernel(const __grid_constant__ RedArgs a, const RedPartial* __restrict__ mine,
                        void* const* __restrict__ inboxes, int nranks, int rank, uint64_t timeout_ns) {
  pdl_enter();
  __shared__ int s_ok;
  __shared__ uint64_t s_epoch;
  char* own = static_cast<char*>(inboxes[rank]);
  uint64_t* flags = reinterpret_cast<uint64_t*>(own + kInboxFlagsOffset);
  uint64_t* seq = reinterpret_cast<uint64_t*>(own + kInboxSeqOffset);
  if (threadIdx.x == 0) {
    const uint64_t epoch = *seq + 1;
    *seq = epoch;
    s_epoch = epoch;
    const size_t slot = (size_t(epoch & 1) * kExchangeMaxRanks + size_t(rank)) * kMaxReductions;
    // this rank's records into every inbox (plain stores; peers' over NVLink),
    // then one release store per flag orders them before the flag
    for (int r = 0; r < nranks; ++r) {
      RedPartial* dst = reinterpret_cast<RedPartial*>(inboxes[r]) + slot;
      for (int k = 0; k < a.n_red; ++k) dst[k] = mine[k];
    }
    __threadfence_system();
    for (int r = 0; r < nranks; ++r)
      st_release_sys(reinterpret_cast<uint64_t*>(static_cast<char*>(inboxes[r]) + kInboxFlagsOffset) + rank, epoch);
    // bounded wait for every rank's flag
    const uint64_t t0 = global_ns();
    int ok = 1;
    for (int r = 0; r < nranks && ok; ++r) {
      while (ld_acquire_sys(flags + r) < epoch) {
        if (global_ns() - t0 > timeout_ns) {
          ok = 0;
          break;
        }
        __nanosleep(32);
      }
    }
    if (!ok) *reinterpret_cast<uint32_t*>(own + kInboxStatusOffset) = 1u;
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  // fold the ranks' records in rank order (relaxed system-scope loads: the
  // slots were written by other GPUs after this SM may have cached older ones)
  const RedPartial* recs = reinterpret_cast<const RedPartial*>(own) + size_t(s_epoch & 1) * kExchangeMaxRanks * kMaxReductions;
  Accs s;
  accs_init(a, s);
  for (int j = threadIdx.x; j < nranks; j += int(blockDim.x)) {
    const uint64_t* src = reinterpret_cast<const uint64_t*>(recs + size_t(j) * kMaxReductions);
    Accs x;
#pragma unroll
    for (int k = 0; k < kMaxReductions; ++k)
      if (k < a.n_red) {
        x.v[k] = ld_relaxed_sys(src + 2 * k);
        x.i[k] = int64_t(ld_relaxed_sys(src + 2 * k + 1));
      }
    accs_merge(a, s, x);
  }
  accs_block_reduce(a, s);
  if (threadIdx.x == 0) write_outputs(a, s, 0);
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
    (void)launch_pdl(&red_column_generic, dim3(grid), dim3(kRedThreads), st, prog, a);
    return cudaGetLastError();
  }
  cudaError_t err = cudaSuccess;
  const bool found = with_spec(spec, [&](auto, auto src, auto r) {
    using S = decltype(src);
    using R = decltype(r);
    constexpr int U = Unroll<S>::U;
    if (strategy == RS_WARP_ROW) {
      (void)launch_pdl(&red_warp_row_kernel<S, R, U>, dim3(grid), dim3(kRedThreads), st, a, aligned);
      err = cudaGetLastError();
      return;
    }
    RedPartial* part = static_cast<RedPartial*>(scratch);
    (void)launch_pdl(&red_split_kernel<S, R, U>, dim3(grid), dim3(kRedThreads), st, a, aligned, part);
    err = cudaGetLastError();
    if (err != cudaSuccess) return;
    (void)launch_pdl(&red_combine_set_kernel<R, kF32>, dim3(unsigned(a.outer)),
                     dim3(rec_out ? kCombineThreads : kRedThreads), st, a, part, grid, rec_out);
    err = cudaGetLastError();
  });
  if (found) return err;
  if (strategy == RS_WARP_ROW) {
    (void)launch_pdl(&red_warp_row_generic<4>, dim3(grid), dim3(kRedThreads), st, prog, a, aligned);
    return cudaGetLastError();
  }
  RedPartial* part = static_cast<RedPartial*>(scratch);
  (void)launch_pdl(&red_split_generic<4>, dim3(grid), dim3(kRedThreads), st, prog, a, aligned, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  (void)launch_pdl(&red_combine_kernel, dim3(unsigned(a.outer)), dim3(rec_out ? kCombineThreads : kRedThreads), st, a,
                   part, grid, rec_out);
  return cudaGetLastError();
}

cudaError_t red_column_chunks_launch(const Program& prog, const RedArgs& a, int grid, int chunks, void* scratch,
                                     cudaStream_t st) {
  const uint64_t n_outputs = a.outer * a.inner;
  if (n_outputs == 0) return cudaSuccess;
  RedPartial* part = static_cast<RedPartial*>(scratch);
  (void)launch_pdl(&red_column_chunks, dim3(unsigned(grid), unsigned(chunks)), dim3(kRedThreads), st, prog, a, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const uint64_t blocks = (n_outputs + kRedThreads - 1) / kRedThreads;
  (void)launch_pdl(&red_column_combine, dim3(unsigned(std::min<uint64_t>(blocks, 65535))), dim3(kRedThreads), st, a,
                   static_cast<const RedPartial*>(part), chunks);
  return cudaGetLastError();
}

size_t red_column_chunks_scratch_bytes(uint64_t n_outputs, int chunks, int n_red) {
  return size_t(n_outputs) * size_t(chunks) * size_t(n_red) * sizeof(RedPartial);
}

cudaError_t red_view_launch(const Program& prog, const RedArgs& a, const ViewSet& views, int grid, cudaStream_t st) {
  if (a.outer == 0 || a.inner == 0) return cudaSuccess;
  (void)launch_pdl(&red_view_generic, dim3(grid), dim3(kRedThreads), st, prog, a, views);
  return cudaGetLastError();
}

int red_view_occupancy() {
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, red_view_generic, kRedThreads, 0) != cudaSuccess) return 1;
  return blocks > 0 ? blocks : 1;
}

cudaError_t red_exchange_combine(const RedArgs& a, const RedPartial* mine, void* const* inboxes, int nranks, int rank,
                                 uint64_t timeout_ns, cudaStream_t st) {
  if (a.outer != 1 || nranks < 1 || nranks > kExchangeMaxRanks || rank < 0 || rank >= nranks)
    return cudaErrorInvalidValue;
  (void)launch_pdl(&red_exchange_kernel, dim3(1), dim3(kCombineThreads), st, a, mine, inboxes, nranks, rank, timeout_ns);
  return cudaGetLastError();
}

cudaError_t red_combine_records(const RedArgs& a, const RedPartial* records, int n, cudaStream_t st) {
  (void)launch_pdl(&red_combine_kernel, dim3(unsigned(a.outer)), dim3(kCombineThreads), st, a, records, n, nullptr);
  return cudaGetLastError();
}

}  // namespace askb
