// Device bodies of the fused elementwise kernels (family E), shared by the
// library's kernels (ew_kernels.cu) and the generated kernel artifacts
// (artifact.cpp), so both run the same code.
#pragma once

#include "ask_numerics.cuh"
#include "kernels.h"
#include "vec_io.cuh"

namespace askb {
namespace ew {

// ---- specialised (compile-time program) path -----------------------------------
template <class P, int K, int V>
__device__ __forceinline__ void spec_load(const EwArgs& a, uint64_t base, bool vec, uint64_t (&x)[P::kIn][V]) {
  if constexpr (K < P::kIn) {
    load_port<P::in_type(K), P::in_map(K), V>(a.in[K], base, a.count, a.inner, vec, x[K]);
    spec_load<P, K + 1, V>(a, base, vec, x);
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

template <class P, int K, int V>
__device__ __forceinline__ void spec_store(const EwArgs& a, uint64_t base, bool vec, const uint64_t (&r)[P::kInsn][V]) {
  if constexpr (K < P::kOut) {
    store_port<P::out_type(K), V>(a.out[K], base, a.count, vec, r[P::out_reg(K)]);
    spec_store<P, K + 1, V>(a, base, vec, r);
  }
}

// Grid-stride loop of the compile-time program P over units of V elements,
// U units in flight per thread.  `aligned`: every port is 16-byte aligned.
template <class P, int V, int U>
__device__ __forceinline__ void ew_spec_loop(const EwArgs& args, int aligned) {
  const uint64_t n = args.count;
  const uint64_t units = (n + V - 1) / V;
  const uint64_t nthreads = uint64_t(gridDim.x) * kEwThreads;
  for (uint64_t u = uint64_t(blockIdx.x) * kEwThreads + threadIdx.x; u < units; u += nthreads * U) {
    uint64_t x[U][P::kIn][V];
#pragma unroll
    for (int q = 0; q < U; ++q) {
      const uint64_t uq = u + q * nthreads;
      if (uq < units) spec_load<P, 0, V>(args, uq * V, aligned && (uq * V + V <= n), x[q]);
    }
#pragma unroll
    for (int q = 0; q < U; ++q) {
      const uint64_t uq = u + q * nthreads;
      if (uq < units) {
        uint64_t r[P::kInsn][V];
        spec_exec<P, 0, V>(r, x[q]);
        spec_store<P, 0, V>(args, uq * V, aligned && (uq * V + V <= n), r);
      }
    }
  }
}

// One element per thread iteration: the element's coordinates in the iteration
// shape are computed once, every IM_VIEW port maps them through its view, and
// OP_COORD reads them.  Scalar loads and stores; this path serves the index
// maps the fused kernels above have no vector form for.
__device__ __forceinline__ void ew_view_loop(const Program& prog, const EwArgs& args, const ViewSet& views) {
  const uint64_t n = args.count;
  const uint64_t nthreads = uint64_t(gridDim.x) * kEwThreads;
  uint64_t r[kMaxRegs];
  for (uint64_t i = uint64_t(blockIdx.x) * kEwThreads + threadIdx.x; i < n; i += nthreads) {
    int64_t c[kMaxRank];
    uint64_t rest = i;
    for (int d = views.rank - 1; d >= 0; --d) {
      const uint64_t e = views.shape[d];
      c[d] = int64_t(rest % e);
      rest /= e;
    }
    for (int k = 0; k < prog.n_insn; ++k) {
      const Insn& ins = prog.insn[k];
      if (ins.op == OP_INPUT) {
        const int port = ins.a, t = prog.in_type[port];
        const void* p = args.in[port];
        switch (prog.in_map[port]) {
          case IM_SCALAR: r[ins.dst] = word_from_storage(t, p, 0); break;
          case IM_OUTER: r[ins.dst] = word_from_storage(t, p, i / args.inner.d); break;
          case IM_INNER: r[ins.dst] = word_from_storage(t, p, i % args.inner.d); break;
          case IM_VIEW: {
            const PortView& v = views.port[port];
            int64_t off = v.offset;
            bool ok = true;
            for (int d = 0; d < views.rank; ++d) {
              const int64_t s = c[d] - v.lo[d];
              const int64_t q = s / v.step[d];
              ok = ok && s >= 0 && q * v.step[d] == s && q < v.extent[d];
              off += q * v.stride[d];
            }
            r[ins.dst] = ok ? word_from_storage(t, p, uint64_t(off)) : v.pad;
            break;
          }
          default: r[ins.dst] = word_from_storage(t, p, i); break;
        }
      } else if (ins.op == OP_COORD) {
        r[ins.dst] = uint64_t(c[ins.aux]);
      } else {
        r[ins.dst] = eval_insn(ins.op, ins.type, ins.src_type, ins.aux, ins.imm, r[ins.a], r[ins.b], r[ins.c]);
      }
    }
    for (int k = 0; k < prog.n_out; ++k) word_to_storage(prog.out_type[k], args.out[k], i, r[prog.out_reg[k]]);
  }
}

}  // namespace ew
}  // namespace askb
