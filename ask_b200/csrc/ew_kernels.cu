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
#include "pdl.cuh"
#include "ew_body.cuh"

namespace askb {

namespace {

using ew::ew_functor_loop;
using ew::ew_spec_loop;
using ew::ew_view_loop;
using ew::FnCfg1;
using ew::FnCfg5b;
using ew::FnSoftmaxNorm;

template <class P, int V, int U>
__global__ void __launch_bounds__(kEwThreads) ew_spec_kernel(const __grid_constant__ EwArgs args, int aligned) {
  pdl_enter();
  ew_spec_loop<P, V, U>(args, aligned);
}

// ---- runtime-program path -------------------------------------------------------
template <int V>
__global__ void __launch_bounds__(kEwThreads)
    ew_generic_kernel(const __grid_constant__ Program prog, const __grid_constant__ EwArgs args, int aligned) {
  pdl_enter();
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
  pdl_enter();
  ew_view_loop(prog, args, views);
}

template <class F>
__global__ void __launch_bounds__(kEwThreads) ew_functor_kernel(const __grid_constant__ EwArgs a, uint64_t units) {
  pdl_enter();
  ew_functor_loop<F>(a, units);
}

template <class P>
struct EwSpecKernels {
  static constexpr int kV = 4, kU = 2;
  static void* vec() { return reinterpret_cast<void*>(&ew_spec_kernel<P, kV, kU>); }
};

void* ew_kernel_ptr(int spec) {
  switch (spec) {
    case EW_CFG1: return reinterpret_cast<void*>(&ew_functor_kernel<FnCfg1>);
    case EW_CFG5B: return reinterpret_cast<void*>(&ew_functor_kernel<FnCfg5b>);
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
  (void)launch_pdl(&ew_view_kernel, dim3(grid), dim3(kEwThreads), stream, prog, args, views);
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
    (void)launch_pdl(&ew_functor_kernel<FnCfg1>, g, b, stream, args, args.count / FnCfg1::V);
    return cudaGetLastError();
  }
  if (spec == EW_CFG5B && functor_ok<FnCfg5b>(args, aligned) &&
      ((reinterpret_cast<uintptr_t>(args.in[0]) | reinterpret_cast<uintptr_t>(args.in[1]) |
        reinterpret_cast<uintptr_t>(args.out[0])) & 31u) == 0) {
    (void)launch_pdl(&ew_functor_kernel<FnCfg5b>, g, b, stream, args, args.count / FnCfg5b::V);
    return cudaGetLastError();
  }
  if (spec == EW_SOFTMAX_NORM_F16 && functor_ok<FnSoftmaxNorm<kF16>>(args, aligned)) {
    (void)launch_pdl(&ew_functor_kernel<FnSoftmaxNorm<kF16>>, g, b, stream, args, args.count / 8);
    return cudaGetLastError();
  }
  if (spec == EW_SOFTMAX_NORM_BF16 && functor_ok<FnSoftmaxNorm<kBF16>>(args, aligned)) {
    (void)launch_pdl(&ew_functor_kernel<FnSoftmaxNorm<kBF16>>, g, b, stream, args, args.count / 8);
    return cudaGetLastError();
  }
  switch (spec) {
    case EW_CFG1:
      (void)launch_pdl(&ew_spec_kernel<ProgCfg1, 4, 2>, g, b, stream, args, aligned);
      break;
    case EW_CFG5B:
      (void)launch_pdl(&ew_spec_kernel<ProgCfg5b, 4, 2>, g, b, stream, args, aligned);
      break;
    case EW_SOFTMAX_NORM_F16:
      (void)launch_pdl(&ew_spec_kernel<ProgSoftmaxNorm<kF16>, 4, 2>, g, b, stream, args, aligned);
      break;
    case EW_SOFTMAX_NORM_BF16:
      (void)launch_pdl(&ew_spec_kernel<ProgSoftmaxNorm<kBF16>, 4, 2>, g, b, stream, args, aligned);
      break;
    default:
      (void)launch_pdl(&ew_generic_kernel<4>, g, b, stream, prog, args, aligned);
      break;
  }
  return cudaGetLastError();
}

}  // namespace askb
