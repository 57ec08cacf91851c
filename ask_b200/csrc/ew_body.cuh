// Device bodies of the fused elementwise kernels (family E), shared by the
// library's kernels (ew_kernels.cu) and the generated kernel artifacts
// (artifact.cpp), so both run the same code.
#pragma once

#include "ask_numerics.cuh"
#include "kernels.h"
#include "pair_f32.cuh"
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

// ---- general index maps ------------------------------------------------------------
// The coordinates of linear index i in the iteration shape (row-major).
__device__ __forceinline__ void view_coords(uint64_t i, const ViewSet& views, int64_t (&c)[kMaxRank]) {
  for (int d = views.rank - 1; d >= 0; --d) {
    const uint64_t e = views.shape[d];
    c[d] = int64_t(i % e);
    i /= e;
  }
}

// The mixed-radix digits of a stride, the leading one not reduced.
__device__ __forceinline__ void view_stride_digits(uint64_t stride, const ViewSet& views, int64_t (&by)[kMaxRank]) {
  for (int d = views.rank - 1; d > 0; --d) {
    const uint64_t e = views.shape[d];
    by[d] = int64_t(stride % e);
    stride /= e;
  }
  if (views.rank > 0) by[0] = int64_t(stride);
}

// c += the mixed-radix digits `by` of a fixed stride, with carries: the
// coordinates of i + stride without a division.  The leading axis takes no
// modulus (it only leaves its range once i + stride is past the end).
__device__ __forceinline__ void view_advance(int64_t (&c)[kMaxRank], const int64_t (&by)[kMaxRank],
                                             const ViewSet& views) {
  int64_t carry = 0;
  for (int d = views.rank - 1; d > 0; --d) {
    const int64_t e = int64_t(views.shape[d]), x = c[d] + by[d] + carry;
    carry = x >= e;
    c[d] = carry ? x - e : x;
  }
  if (views.rank > 0) c[0] += by[0] + carry;
}

// An IM_VIEW port's element at coordinates c, or its pad outside the window:
// per axis q = (c - lo) / step must be a whole number in [0, extent).
__device__ __forceinline__ uint64_t view_read(const PortView& v, int rank, const int64_t (&c)[kMaxRank], int type,
                                              const void* p) {
  int64_t off = v.offset;
  bool ok = true;
  for (int d = 0; d < rank; ++d) {
    const int64_t q0 = c[d] - v.lo[d], st = v.step[d];
    const int64_t q = st == 1 ? q0 : q0 / st;
    ok = ok && q0 >= 0 && (st == 1 || q * st == q0) && q < v.extent[d];
    off += q * v.stride[d];
  }
  if (!ok) return v.pad;
  if (v.inner_rank > 0) {
    // off is a row-major position in the reshape's operand: its coordinates
    // there (one division per axis) go through the inner window
    int64_t pos = off;
    off = v.ioffset;
    for (int d = int(v.inner_rank) - 1; d >= 0; --d) {
      const int64_t e = v.inner_shape[d];
      const int64_t cd = pos % e;
      pos /= e;
      const int64_t q0 = cd - v.ilo[d], st = v.istep[d];
      const int64_t q = st == 1 ? q0 : q0 / st;
      ok = ok && q0 >= 0 && (st == 1 || q * st == q0) && q < v.iextent[d];
      off += q * v.istride[d];
    }
    if (!ok) return v.ipad;
  }
  return word_from_storage(type, p, uint64_t(off));
}

// One element per thread iteration (grid-stride): the element's coordinates
// in the iteration shape are advanced by the grid's stride with carries (no
// division per element), every IM_VIEW port maps them through its view, and
// OP_COORD reads them.  Scalar loads and stores; this path serves the index
// maps the fused kernels above have no vector form for.  (Four elements per
// thread with the generic kernel's vector loads and stores measured no
// faster: the interpreter's latency and the views' scattered reads bound it.)
__device__ __forceinline__ void ew_view_loop(const Program& prog, const EwArgs& args, const ViewSet& views) {
  const uint64_t n = args.count;
  const uint64_t nthreads = uint64_t(gridDim.x) * kEwThreads;
  uint64_t r[kMaxRegs];
  uint64_t i = uint64_t(blockIdx.x) * kEwThreads + threadIdx.x;
  if (i >= n) return;
  int64_t c[kMaxRank], by[kMaxRank];
  view_coords(i, views, c);
  view_stride_digits(nthreads, views, by);
  for (; i < n; i += nthreads, view_advance(c, by, views)) {
    for (int k = 0; k < prog.n_insn; ++k) {
      const Insn& ins = prog.insn[k];
      if (ins.op == OP_INPUT) {
        const int port = ins.a, t = prog.in_type[port];
        const void* p = args.in[port];
        switch (prog.in_map[port]) {
          case IM_SCALAR: r[ins.dst] = word_from_storage(t, p, 0); break;
          case IM_OUTER: r[ins.dst] = word_from_storage(t, p, i / args.inner.d); break;
          case IM_INNER: r[ins.dst] = word_from_storage(t, p, i % args.inner.d); break;
          case IM_VIEW: r[ins.dst] = view_read(views.port[port], views.rank, c, t, p); break;
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

// ---- hand-written functor kernels for the hottest programs ------------------------
// Software-pipelined grid-stride loop over whole 16-byte units: the loads of the
// next unit are in flight while the current unit is computed, so latency is
// hidden without depending on other warps.  Used only when every port is
// 16-byte aligned and the element count is a multiple of the unit; the
// interpreter kernels above serve every other case.
template <class F>
__device__ __forceinline__ void ew_functor_loop(const EwArgs& a, uint64_t units) {
  const uint64_t stride = uint64_t(gridDim.x) * kEwThreads;
  uint64_t u = uint64_t(blockIdx.x) * kEwThreads + threadIdx.x;
  if (u >= units) return;
  if constexpr (F::kDepth == 2) {  // the units two and one strides ahead in flight
    typename F::In cur = F::load(a, u), nxt, nxt2;
    if (u + stride < units) nxt = F::load(a, u + stride);
    for (; u < units; u += stride) {
      const uint64_t u2 = u + 2 * stride;
      if (u2 < units) nxt2 = F::load(a, u2);
      F::store(a, u, F::compute(a, cur));
      cur = nxt;
      nxt = nxt2;
    }
  } else {
    typename F::In cur = F::load(a, u), nxt;
    for (; u < units; u += stride) {
      const uint64_t un = u + stride;
      if (un < units) nxt = F::load(a, un);
      F::store(a, u, F::compute(a, cur));
      cur = nxt;
    }
  }
}

// ProgCfg5b: z = ((x << 3) ^ (x >> 5)) & 0x7fffffff + y on i32 (shifts in range,
// arithmetic right shift, wrapping add: ScalarEmitter.h:100-141), 8 elements
// per unit with 32-byte loads and stores (ports 32-byte aligned).  Measured on
// cfg5b: 3.95 ms against the compile-time program loop's 4.14 ms (16-byte
// units, no prefetch) and 4.07 ms for a 16-byte version of this functor.
struct FnCfg5b {
  static constexpr int V = 8;
  static constexpr int kDepth = 1;
  static constexpr bool kRowMapped = false;
  struct In { Vec32 x, y; };
  struct Out { Vec32 z; };
  __device__ static In load(const EwArgs& e, uint64_t u) {
    return In{ld_stream_v8(static_cast<const char*>(e.in[0]) + u * 32),
              ld_stream_v8(static_cast<const char*>(e.in[1]) + u * 32)};
  }
  __device__ static Out compute(const EwArgs&, const In& a) {
    Out o;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t x = a.x.w[k];
      o.z.w[k] = (((x << 3) ^ uint32_t(int32_t(x) >> 5)) & 0x7fffffffu) + a.y.w[k];
    }
    return o;
  }
  __device__ static void store(const EwArgs& e, uint64_t u, const Out& o) {
    st_stream_v8(static_cast<char*>(e.out[0]) + u * 32, o.z);
  }
};

// ProgCfg1: y0 = exp(a)*b + c ; y1 = maximum(a, b) + tanh(c)*(-1), 4 elements per unit.
struct FnCfg1 {
  static constexpr int V = 4;
  // loads two units ahead: 57.6 against 59.7 us on cfg1 with one (same box;
  // 58 registers, 4 CTAs an SM instead of 5, twice the bytes in flight)
  static constexpr int kDepth = 2;
  static constexpr bool kRowMapped = false;
  struct In { uint4 a, b, c; };
  struct Out { float y0[4], y1[4]; };
  __device__ static In load(const EwArgs& e, uint64_t u) {
    return In{ld_stream_v4(static_cast<const uint4*>(e.in[0]) + u), ld_stream_v4(static_cast<const uint4*>(e.in[1]) + u),
              ld_stream_v4(static_cast<const uint4*>(e.in[2]) + u)};
  }
  __device__ static Out compute(const EwArgs&, const In& x) {
    const float a[4] = {__uint_as_float(x.a.x), __uint_as_float(x.a.y), __uint_as_float(x.a.z), __uint_as_float(x.a.w)};
    const float b[4] = {__uint_as_float(x.b.x), __uint_as_float(x.b.y), __uint_as_float(x.b.z), __uint_as_float(x.b.w)};
    const float c[4] = {__uint_as_float(x.c.x), __uint_as_float(x.c.y), __uint_as_float(x.c.z), __uint_as_float(x.c.w)};
    Out o;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      o.y0[v] = __fadd_rn(__fmul_rn(expf(a[v]), b[v]), c[v]);
      o.y1[v] = __fadd_rn(ask_maximum(a[v], b[v]), __fmul_rn(tanhf(c[v]), -1.0f));
    }
    return o;
  }
  __device__ static void store(const EwArgs& e, uint64_t u, const Out& o) {
    st_stream_v4(static_cast<uint4*>(e.out[0]) + u, make_uint4(__float_as_uint(o.y0[0]), __float_as_uint(o.y0[1]),
                                                                __float_as_uint(o.y0[2]), __float_as_uint(o.y0[3])));
    st_stream_v4(static_cast<uint4*>(e.out[1]) + u, make_uint4(__float_as_uint(o.y1[0]), __float_as_uint(o.y1[1]),
                                                                __float_as_uint(o.y1[2]), __float_as_uint(o.y1[3])));
  }
};

// ProgSoftmaxNorm<T>: y = cast(exp(cast(x, f32) + m*(-1)) / s, T), 8 elements per
// unit; m and s are indexed by the row (unit*8 / inner).
//
// A unit whose eight t = x + m*(-1) all lie in [-69, 0] (every unit of a
// finite softmax row, where m is the row's maximum) with 2^-100 <= s <= 2^24
// runs on f32 pairs: e = exp_pair(t) (pair_f32.cuh; a normal f32 within about
// 3 ulps of exp(t), e >= 2^-99.6) and q = RN(e * RN(1/s)), a normal f32
// (>= 2^-123.6) within 2 ulps of e / s, so RN16(q) is within one 16-bit ulp
// of RN16(e / s).
//
// Any other unit computes exp with CUDA's expf and the correctly rounded f32
// quotient, from the row's correctly rounded reciprocal y = RN(1/s) by
// Markstein's correction: with q0 = RN(e*y) and two steps r = fma(-q, s, e)
// (exact when q is within an ulp of e/s and no value is subnormal),
// q' = fma(r, y, q), the last q equals RN(e/s) (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990).  The theorem's conditions -- s and y normal, a normal
// quotient -- are checked; a unit that fails them (a zero, subnormal,
// infinite or NaN operand or result) is recomputed with the IEEE division.
template <int T>
struct FnSoftmaxNorm {
  static constexpr int V = 8;
  static constexpr int kDepth = 1;
  static constexpr bool kRowMapped = true;  // m, s are indexed by unit*8 / inner
  struct In { uint4 x; float nm, s, y; };
  using Out = uint4;
  __device__ static In load(const EwArgs& e, uint64_t u) {
    const uint64_t row = udiv(u * V, e.inner);
    const float s = __ldg(static_cast<const float*>(e.in[2]) + row);
    return In{ld_stream_v4(static_cast<const uint4*>(e.in[0]) + u),
              __fmul_rn(__ldg(static_cast<const float*>(e.in[1]) + row), -1.0f), s, __frcp_rn(s)};
  }
  __device__ static Out compute(const EwArgs&, const In& x) {
    const uint32_t w[4] = {x.x.x, x.x.y, x.x.z, x.x.w};
    const float s = x.s, y = x.y;
    uint32_t r[4];
    if (s >= 0x1p-100f && s <= 0x1p24f && exp_pair_range<T>(w, x.nm)) {
      const uint64_t nm2 = pack2(x.nm, x.nm), y2 = pack2(y, y);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float lo, hi;
        unpack2(mul2(exp_pair(add2(pack2(widen_lo<T>(w[j]), widen_hi<T>(w[j])), nm2)), y2), lo, hi);
        r[j] = narrow_two<T>(lo, hi);
      }
      return make_uint4(r[0], r[1], r[2], r[3]);
    }
    float e[8], q[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      e[2 * j] = expf(__fadd_rn(widen_lo<T>(w[j]), x.nm));
      e[2 * j + 1] = expf(__fadd_rn(widen_hi<T>(w[j]), x.nm));
    }
    bool ok = s >= 0x1p-100f && s <= 0x1p100f;  // s and y = RN(1/s) normal (false for NaN)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float t = __fmul_rn(e[k], y);
      t = __fmaf_rn(__fmaf_rn(-t, s, e[k]), y, t);
      t = __fmaf_rn(__fmaf_rn(-t, s, e[k]), y, t);
      q[k] = t;
      ok &= (t >= 0x1p-124f && t <= 0x1p126f) || e[k] == 0.0f;
    }
    if (ok) {  // every q is finite
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = narrow_two<T>(q[2 * j], q[2 * j + 1]);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = __fdiv_rn(e[k], s);
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = narrow_one<T>(q[2 * j]) | (narrow_one<T>(q[2 * j + 1]) << 16);
    }
    return make_uint4(r[0], r[1], r[2], r[3]);
  }
  __device__ static void store(const EwArgs& e, uint64_t u, const Out& o) {
    st_stream_v4(static_cast<uint4*>(e.out[0]) + u, o);
  }
};

}  // namespace ew
}  // namespace askb
