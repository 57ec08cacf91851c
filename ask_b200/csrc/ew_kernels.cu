// Family E: multi-output fused elementwise loops.
//
// Replaces the "element.loop" kernel that lib/Lowering/CUDA.cpp:274-385 emits
// for a batch of same-shape outputs: every output of the step is computed per
// linear element index with all intermediates in registers (ScalarEmitter's
// memo, ScalarEmitter.h:599-604, 825) and each public output gets its own store
// (lib/Lowering/Host.cpp:862-866).  Differences, all B200-motivated:
//   * 16-byte vector loads/stores (the reference issues scalar 4-byte
//     accesses, CUDA.cpp:288-290, 371-373) and U independent units per thread
//     in flight;
//   * a persistent grid of (SMs x resident blocks) instead of
//     min(65535, ceil(count/128)) blocks (CUDA.cpp:256-259);
//   * the op program is a compile-time constant for the specialised plans, so
//     the interpreter folds to straight-line code; other programs run the same
//     interpreter on a runtime program held in the kernel's parameter space.
#include <cuda_runtime.h>

#include "ask_numerics.cuh"
#include "kernels.h"
#include "programs.h"
#include "vec_io.cuh"
#include "ew_body.cuh"

namespace askb {

namespace {

using ew::ew_spec_loop;
using ew::ew_view_loop;

template <class P, int V, int U>
__global__ void __launch_bounds__(kEwThreads) ew_spec_kernel(const __grid_constant__ EwArgs args, int aligned) {
  ew_spec_loop<P, V, U>(args, aligned);
}

// ---- runtime-program path -------------------------------------------------------
template <int V>
__global__ void __launch_bounds__(kEwThreads)
    ew_generic_kernel(const __grid_constant__ Program prog, const __grid_constant__ EwArgs args, int aligned) {
  const uint64_t n = args.count;
  const uint64_t units = (n + V - 1) / V;
  const uint64_t nthreads = uint64_t(gridDim.x) * kEwThreads;
  uint64_t r[kMaxRegs][V];
  for (uint64_t u = uint64_t(blockIdx.x) * kEwThreads + threadIdx.x; u < units; u += nthreads) {
    const uint64_t base = u * V;
    const bool vec = aligned && (base + V <= n);
    for (int i = 0; i < prog.n_insn; ++i) {
      const Insn& ins = prog.insn[i];
      if (ins.op == OP_INPUT) {
        uint64_t w[V];
        rt_load<V>(prog.in_type[ins.a], prog.in_map[ins.a], args.in[ins.a], base, n, args.inner, vec, w);
#pragma unroll
        for (int v = 0; v < V; ++v) r[ins.dst][v] = w[v];
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v)
          r[ins.dst][v] = eval_insn(ins.op, ins.type, ins.src_type, ins.aux, ins.imm, r[ins.a][v], r[ins.b][v], r[ins.c][v]);
      }
    }
    for (int k = 0; k < prog.n_out; ++k) {
      uint64_t w[V];
#pragma unroll
      for (int v = 0; v < V; ++v) w[v] = r[prog.out_reg[k]][v];
      rt_store<V>(prog.out_type[k], args.out[k], base, n, vec, w);
    }
  }
}

// ---- general index maps ------------------------------------------------------------
__global__ void __launch_bounds__(kEwThreads) ew_view_kernel(const __grid_constant__ Program prog,
                                                             const __grid_constant__ EwArgs args,
                                                             const __grid_constant__ ViewSet views) {
  ew_view_loop(prog, args, views);
}

// ---- hand-written functor kernels for the hottest programs ------------------------
// Software-pipelined grid-stride loop over whole 16-byte units: the loads of the
// next unit are in flight while the current unit is computed, so latency is
// hidden without depending on other warps.  Used only when every port is
// 16-byte aligned and the element count is a multiple of the unit; the
// interpreter kernels above serve every other case.
template <class F>
__global__ void __launch_bounds__(kEwThreads) ew_functor_kernel(const __grid_constant__ EwArgs a, uint64_t units) {
  const uint64_t stride = uint64_t(gridDim.x) * kEwThreads;
  uint64_t u = uint64_t(blockIdx.x) * kEwThreads + threadIdx.x;
  if (u >= units) return;
  typename F::In cur = F::load(a, u), nxt;
  for (; u < units; u += stride) {
    const uint64_t un = u + stride;
    if (un < units) nxt = F::load(a, un);
    F::store(a, u, F::compute(a, cur));
    cur = nxt;
  }
}

// ProgCfg1: y0 = exp(a)*b + c ; y1 = maximum(a, b) + tanh(c)*(-1), 4 elements per unit.
struct FnCfg1 {
  static constexpr int V = 4;
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
// The division is the correctly rounded f32 quotient, computed from the row's
// correctly rounded reciprocal y = RN(1/s) by Markstein's correction: with
// q0 = RN(e*y) and two steps r = fma(-q, s, e) (exact when q is within an ulp
// of e/s and no value is subnormal), q' = fma(r, y, q), the last q equals
// RN(e/s) (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990).  The
// theorem's conditions -- s and y normal, a normal quotient -- are checked;
// a unit that fails them (a zero, subnormal, infinite or NaN operand or
// result, which softmax rows reach only at their extremes) is recomputed with
// the IEEE division.  One reciprocal per row replaces one per element, and
// the division no longer occupies the special-function unit per element.
template <int T>
struct FnSoftmaxNorm {
  static constexpr int V = 8;
  static constexpr bool kRowMapped = true;  // m, s are indexed by unit*8 / inner
  struct In { uint4 x; float nm, s, y; };
  using Out = uint4;
  __device__ static float widen(uint32_t h) {
    if constexpr (T == kF16) return __half2float(__ushort_as_half(uint16_t(h)));
    else return __uint_as_float(h << 16);
  }
  __device__ static uint32_t narrow(float f) {
    if constexpr (T == kF16) return __half_as_ushort(__float2half_rn(f));
    else return bf16_bits_rne(f);
  }
  // Two non-NaN values rounded to nearest-even and packed (lo in bits 0..15):
  // one cvt.rn.{f16,bf16}x2.f32.  For bf16 this equals bf16_bits_rne on every
  // non-NaN input; NaN inputs take narrow() (the payload-preserving rule).
  __device__ static uint32_t narrow2(float lo, float hi) {
    uint32_t r;
    if constexpr (T == kF16)
      asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  __device__ static In load(const EwArgs& e, uint64_t u) {
    const uint64_t row = udiv(u * V, e.inner);
    const float s = __ldg(static_cast<const float*>(e.in[2]) + row);
    return In{ld_stream_v4(static_cast<const uint4*>(e.in[0]) + u),
              __fmul_rn(__ldg(static_cast<const float*>(e.in[1]) + row), -1.0f), s, __frcp_rn(s)};
  }
  __device__ static Out compute(const EwArgs&, const In& x) {
    const uint32_t w[4] = {x.x.x, x.x.y, x.x.z, x.x.w};
    float e[8], q[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      e[2 * j] = expf(__fadd_rn(widen(w[j] & 0xffffu), x.nm));
      e[2 * j + 1] = expf(__fadd_rn(widen(w[j] >> 16), x.nm));
    }
    const float s = x.s, y = x.y;
    bool ok = s >= 0x1p-100f && s <= 0x1p100f;  // s and y = RN(1/s) normal (false for NaN)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float t = __fmul_rn(e[k], y);
      t = __fmaf_rn(__fmaf_rn(-t, s, e[k]), y, t);
      t = __fmaf_rn(__fmaf_rn(-t, s, e[k]), y, t);
      q[k] = t;
      ok &= (t >= 0x1p-124f && t <= 0x1p126f) || e[k] == 0.0f;
    }
    uint32_t r[4];
    if (ok) {  // every q is finite
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = narrow2(q[2 * j], q[2 * j + 1]);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = __fdiv_rn(e[k], s);
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = narrow(q[2 * j]) | (narrow(q[2 * j + 1]) << 16);
    }
    return make_uint4(r[0], r[1], r[2], r[3]);
  }
  __device__ static void store(const EwArgs& e, uint64_t u, const Out& o) {
    st_stream_v4(static_cast<uint4*>(e.out[0]) + u, o);
  }
};

template <class P>
struct EwSpecKernels {
  static constexpr int kV = 4, kU = 2;
  static void* vec() { return reinterpret_cast<void*>(&ew_spec_kernel<P, kV, kU>); }
};

void* ew_kernel_ptr(int spec) {
  switch (spec) {
    case EW_CFG1: return reinterpret_cast<void*>(&ew_functor_kernel<FnCfg1>);
    case EW_CFG5B: return EwSpecKernels<ProgCfg5b>::vec();
    case EW_SOFTMAX_NORM_F16: return reinterpret_cast<void*>(&ew_functor_kernel<FnSoftmaxNorm<kF16>>);
    case EW_SOFTMAX_NORM_BF16: return reinterpret_cast<void*>(&ew_functor_kernel<FnSoftmaxNorm<kBF16>>);
    default: return reinterpret_cast<void*>(&ew_generic_kernel<4>);
  }
}

}  // namespace

bool ew_spec_program(int spec, Program* out) {
  switch (spec) {
    case EW_CFG1: *out = program_of<ProgCfg1>(); return true;
    case EW_CFG5B: *out = program_of<ProgCfg5b>(); return true;
    case EW_SOFTMAX_NORM_F16: *out = program_of<ProgSoftmaxNorm<kF16>>(); return true;
    case EW_SOFTMAX_NORM_BF16: *out = program_of<ProgSoftmaxNorm<kBF16>>(); return true;
    default: return false;
  }
}

int ew_num_specs() { return EW_NUM_SPECS; }

cudaError_t ew_view_launch(const Program& prog, const EwArgs& args, const ViewSet& views, int grid, cudaStream_t stream) {
  if (args.count == 0) return cudaSuccess;
  ew_view_kernel<<<dim3(grid), dim3(kEwThreads), 0, stream>>>(prog, args, views);
  return cudaGetLastError();
}

int ew_view_occupancy() {
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, ew_view_kernel, kEwThreads, 0) != cudaSuccess) return 1;
  return blocks > 0 ? blocks : 1;
}

cudaError_t ew_occupancy(int spec, int* blocks_per_sm) {
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, ew_kernel_ptr(spec), kEwThreads, 0);
}

template <class F>
bool functor_ok(const EwArgs& a, int aligned) {
  return aligned && a.count % F::V == 0 && (!F::kRowMapped || a.inner.d % F::V == 0);
}

cudaError_t ew_launch(int spec, const Program& prog, const EwArgs& args, int aligned, int grid, cudaStream_t stream) {
  if (args.count == 0) return cudaSuccess;
  const dim3 g(grid), b(kEwThreads);
  if (spec == EW_CFG1 && functor_ok<FnCfg1>(args, aligned)) {
    ew_functor_kernel<FnCfg1><<<g, b, 0, stream>>>(args, args.count / FnCfg1::V);
    return cudaGetLastError();
  }
  if (spec == EW_SOFTMAX_NORM_F16 && functor_ok<FnSoftmaxNorm<kF16>>(args, aligned)) {
    ew_functor_kernel<FnSoftmaxNorm<kF16>><<<g, b, 0, stream>>>(args, args.count / 8);
    return cudaGetLastError();
  }
  if (spec == EW_SOFTMAX_NORM_BF16 && functor_ok<FnSoftmaxNorm<kBF16>>(args, aligned)) {
    ew_functor_kernel<FnSoftmaxNorm<kBF16>><<<g, b, 0, stream>>>(args, args.count / 8);
    return cudaGetLastError();
  }
  switch (spec) {
    case EW_CFG1:
      ew_spec_kernel<ProgCfg1, 4, 2><<<g, b, 0, stream>>>(args, aligned);
      break;
    case EW_CFG5B:
      ew_spec_kernel<ProgCfg5b, 4, 2><<<g, b, 0, stream>>>(args, aligned);
      break;
    case EW_SOFTMAX_NORM_F16:
      ew_spec_kernel<ProgSoftmaxNorm<kF16>, 4, 2><<<g, b, 0, stream>>>(args, aligned);
      break;
    case EW_SOFTMAX_NORM_BF16:
      ew_spec_kernel<ProgSoftmaxNorm<kBF16>, 4, 2><<<g, b, 0, stream>>>(args, aligned);
      break;
    default:
      ew_generic_kernel<4><<<g, b, 0, stream>>>(prog, args, aligned);
      break;
  }
  return cudaGetLastError();
}

}  // namespace askb
