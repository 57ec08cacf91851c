// Families G and X: gather and scatter_add over a canonical [outer, dim, inner]
// layout with a flat index vector of length n.
//
//   gather       out[o, j, :] = params[o, idx[j], :], zero when idx is outside
//                [0, dim) (lib/Lowering/ScalarEmitter.h:775-815; i32 indices
//                are sign-extended, ScalarEmitter.h:786).
//   scatter_add  out = base, then out[o, idx[j], :] += upd[o, j, :] for every
//                in-bounds j; out-of-bounds updates are skipped
//                (lib/Lowering/CUDA.cpp:297-352, lib/Lowering/Host.cpp:677-772).
//                The base copy is the reference Runtime's pre_copy
//                (lib/Runtime/CUDA.cpp:365-371), fused into this step's launch.
// The reference emits one thread per output/update element with a 64-bit
// udiv/urem decomposition and an index load per element; here a warp owns a
// whole row, loads its index once and moves the row with 16-byte accesses (and
// 16-byte vector atomics for f32 scatter, sm_90+).  Table rows are read through
// L1/L2 (hot Zipf rows stay resident); the 8 GiB output stream is written
// evict-first.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include <type_traits>

#include "ask_numerics.cuh"
#include "kernels.h"
#include "vec_io.cuh"

namespace askb {

namespace {

constexpr int kIdxThreads = 256;
constexpr int kRowsPerWarp = 4;

__device__ __forceinline__ int64_t load_index(int itype, const void* p, uint64_t j) {
  return itype == kI32 ? int64_t(__ldg(static_cast<const int32_t*>(p) + j)) : __ldg(static_cast<const int64_t*>(p) + j);
}

__device__ __forceinline__ uint4 ld_cached_v4(const void* p) { return __ldg(static_cast<const uint4*>(p)); }

// Rows of 16-byte vectors.  `vecs` = vectors per row.  A warp moves
// kRowsPerWarp rows per iteration: the indices first, then every lane's
// vectors of all the rows (loads through L1, where the hot rows of a skewed
// index stream stay), then evict-first stores.  (Measured on cfg4: index
// prefetching, default write-back stores, an asynchronous-copy ring through
// shared memory, smaller grids, and skipping the index division when outer is 1
// were each slower than this -- 1.83 to 2.04 ms against 1.73 ms.  Issuing the
// table-row loads sooner appears to cost L1 hits on the hot rows.  A ring of
// whole-row bulk copies (cp.async.bulk global -> shared -> global, one issuing
// thread per 32-thread CTA, mbarrier per stage) took 1.89 ms with 16 stages
// and stores 8 rows behind, and 3.52 ms with 32 stages at half the CTAs: each
// CTA refills a stage only after the bulk store that read it has finished
// reading shared memory, which under the 8 GiB write stream capped every CTA
// near 2.5 rows per microsecond.  Register stores do not hold the stage.)
__global__ void __launch_bounds__(kIdxThreads) gather_rows_vec(const __grid_constant__ IndexArgs a, uint32_t vecs) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warp = (uint64_t(blockIdx.x) * kIdxThreads + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t(gridDim.x) * kIdxThreads) >> 5;
  const uint64_t rows = a.outer * a.n;
  const uint4* table = static_cast<const uint4*>(a.table);
  uint4* out = static_cast<uint4*>(a.out);
  for (uint64_t r0 = warp * kRowsPerWarp; r0 < rows; r0 += nwarps * kRowsPerWarp) {
    int64_t src[kRowsPerWarp];
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q) {
      const uint64_t r = r0 + q;
      src[q] = -1;
      if (r < rows) {
        const uint64_t o = r / a.n, j = r - o * a.n;
        const int64_t idx = load_index(a.index_type, a.index, j);
        if (idx >= 0 && uint64_t(idx) < a.dim) src[q] = int64_t(o * a.dim + uint64_t(idx));
      }
    }
    for (uint32_t v0 = 0; v0 < vecs; v0 += 64) {
      uint4 buf[kRowsPerWarp][2];
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t v = v0 + h * 32 + lane;
          buf[q][h] = (src[q] >= 0 && v < vecs) ? ld_cached_v4(table + uint64_t(src[q]) * vecs + v) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t v = v0 + h * 32 + lane;
          if (r0 + q < rows && v < vecs) st_stream_v4(out + (r0 + q) * vecs + v, buf[q][h]);
        }
    }
  }
}

// Any element size / alignment: one thread per output element, raw copy.
template <int ES>
__global__ void __launch_bounds__(kIdxThreads) gather_elems(const __grid_constant__ IndexArgs a) {
  using T = typename std::conditional<ES == 1, uint8_t,
            typename std::conditional<ES == 2, uint16_t, typename std::conditional<ES == 4, uint32_t, uint64_t>::type>::type>::type;
  const uint64_t total = a.outer * a.n * a.inner;
  const T* table = static_cast<const T*>(a.table);
  T* out = static_cast<T*>(a.out);
  for (uint64_t i = uint64_t(blockIdx.x) * kIdxThreads + threadIdx.x; i < total; i += uint64_t(gridDim.x) * kIdxThreads) {
    const uint64_t row = i / a.inner, c = i - row * a.inner;
    const uint64_t o = row / a.n, j = row - o * a.n;
    const int64_t idx = load_index(a.index_type, a.index, j);
    T val = 0;
    if (idx >= 0 && uint64_t(idx) < a.dim) val = table[(o * a.dim + uint64_t(idx)) * a.inner + c];
    out[i] = val;
  }
}

// out = base (the step's pre_copy), 16-byte vectors plus a byte tail.
__global__ void __launch_bounds__(kIdxThreads) copy_bytes(const void* __restrict__ src, void* __restrict__ dst,
                                                          uint64_t bytes, int aligned) {
  const uint64_t tid = uint64_t(blockIdx.x) * kIdxThreads + threadIdx.x;
  const uint64_t nthreads = uint64_t(gridDim.x) * kIdxThreads;
  uint64_t done = 0;
  if (aligned) {
    const uint64_t nv = bytes / 16;
    const uint4* s = static_cast<const uint4*>(src);
    uint4* d = static_cast<uint4*>(dst);
    for (uint64_t v = tid; v < nv; v += nthreads) d[v] = ld_stream_v4(s + v);
    done = nv * 16;
  }
  for (uint64_t b = done + tid; b < bytes; b += nthreads)
    static_cast<uint8_t*>(dst)[b] = static_cast<const uint8_t*>(src)[b];
}

// f32 scatter_add, warp per update row, 16-byte vector atomics (red.global.v4.f32).
__global__ void __launch_bounds__(kIdxThreads) scatter_rows_f32v(const __grid_constant__ IndexArgs a, uint32_t vecs) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warp = (uint64_t(blockIdx.x) * kIdxThreads + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t(gridDim.x) * kIdxThreads) >> 5;
  const uint64_t rows = a.outer * a.n;
  const uint4* upd = static_cast<const uint4*>(a.table);
  float4* out = static_cast<float4*>(a.out);
  for (uint64_t r0 = warp * kRowsPerWarp; r0 < rows; r0 += nwarps * kRowsPerWarp) {
    int64_t dst[kRowsPerWarp];
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q) {
      const uint64_t r = r0 + q;
      dst[q] = -1;
      if (r < rows) {
        const uint64_t o = r / a.n, j = r - o * a.n;
        const int64_t idx = load_index(a.index_type, a.index, j);
        if (idx >= 0 && uint64_t(idx) < a.dim) dst[q] = int64_t(o * a.dim + uint64_t(idx));
      }
    }
    for (uint32_t v0 = 0; v0 < vecs; v0 += 64) {
      uint4 buf[kRowsPerWarp][2];
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t v = v0 + h * 32 + lane;
          buf[q][h] = (dst[q] >= 0 && v < vecs) ? ld_stream_v4(upd + (r0 + q) * vecs + v) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t v = v0 + h * 32 + lane;
          if (dst[q] >= 0 && v < vecs) {
            const uint4 u = buf[q][h];
            atomicAdd(out + uint64_t(dst[q]) * vecs + v,
                      make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w)));
          }
        }
    }
  }
}

// Any element type: one thread per update element, scalar atomics.
template <int T>
__global__ void __launch_bounds__(kIdxThreads) scatter_elems(const __grid_constant__ IndexArgs a) {
  const uint64_t total = a.outer * a.n * a.inner;
  for (uint64_t i = uint64_t(blockIdx.x) * kIdxThreads + threadIdx.x; i < total; i += uint64_t(gridDim.x) * kIdxThreads) {
    const uint64_t row = i / a.inner, c = i - row * a.inner;
    const uint64_t o = row / a.n, j = row - o * a.n;
    const int64_t idx = load_index(a.index_type, a.index, j);
    if (idx < 0 || uint64_t(idx) >= a.dim) continue;
    const uint64_t d = (o * a.dim + uint64_t(idx)) * a.inner + c;
    if constexpr (T == kF32) {
      atomicAdd(static_cast<float*>(a.out) + d, static_cast<const float*>(a.table)[i]);
    } else if constexpr (T == kI32) {
      atomicAdd(static_cast<int*>(a.out) + d, static_cast<const int*>(a.table)[i]);
    } else if constexpr (T == kI64) {
      atomicAdd(static_cast<unsigned long long*>(a.out) + d, static_cast<const unsigned long long*>(a.table)[i]);
    } else if constexpr (T == kF16) {
      atomicAdd(static_cast<__half*>(a.out) + d, static_cast<const __half*>(a.table)[i]);
    } else {
      atomicAdd(static_cast<__nv_bfloat16*>(a.out) + d, static_cast<const __nv_bfloat16*>(a.table)[i]);
    }
  }
}

bool ptr_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

cudaError_t gather_launch(const IndexArgs& a, int aligned, int grid, cudaStream_t st) {
  const uint64_t total = a.outer * a.n * a.inner;
  if (total == 0) return cudaSuccess;
  const int es = dtype_bytes(a.elem_type);
  const uint64_t row_bytes = a.inner * uint64_t(es);
  if (aligned && row_bytes % 16 == 0 && ptr_aligned16(a.table) && ptr_aligned16(a.out) && row_bytes >= 256) {
    gather_rows_vec<<<grid, kIdxThreads, 0, st>>>(a, uint32_t(row_bytes / 16));
  } else if (es == 1) {
    gather_elems<1><<<grid, kIdxThreads, 0, st>>>(a);
  } else if (es == 2) {
    gather_elems<2><<<grid, kIdxThreads, 0, st>>>(a);
  } else if (es == 4) {
    gather_elems<4><<<grid, kIdxThreads, 0, st>>>(a);
  } else {
    gather_elems<8><<<grid, kIdxThreads, 0, st>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t scatter_add_launch(const IndexArgs& a, int aligned, int grid, void* scratch, int sms, cudaStream_t st) {
  const int es = dtype_bytes(a.elem_type);
  const uint64_t base_bytes = a.outer * a.dim * a.inner * uint64_t(es);
  const uint64_t total = a.outer * a.n * a.inner;
  // the sorted path does its own (partial) pre_copy
  if (total && a.dim && scratch && aligned && scatter_sorted_ok(a) && ptr_aligned16(a.table) && ptr_aligned16(a.out) &&
      ptr_aligned16(a.base))
    return scatter_sorted_launch(a, scratch, sms, st);
  if (a.base != a.out && base_bytes) {
    copy_bytes<<<grid, kIdxThreads, 0, st>>>(a.base, a.out, base_bytes,
                                             ptr_aligned16(a.base) && ptr_aligned16(a.out) ? 1 : 0);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (total == 0 || a.dim == 0) return cudaSuccess;
  const uint64_t row_bytes = a.inner * uint64_t(es);
  if (a.elem_type == kF32 && aligned && row_bytes % 16 == 0 && ptr_aligned16(a.table) && ptr_aligned16(a.out) &&
      row_bytes >= 256) {
    scatter_rows_f32v<<<grid, kIdxThreads, 0, st>>>(a, uint32_t(row_bytes / 16));
  } else {
    switch (a.elem_type) {
      case kF32: scatter_elems<kF32><<<grid, kIdxThreads, 0, st>>>(a); break;
      case kI32: scatter_elems<kI32><<<grid, kIdxThreads, 0, st>>>(a); break;
      case kI64: scatter_elems<kI64><<<grid, kIdxThreads, 0, st>>>(a); break;
      case kF16: scatter_elems<kF16><<<grid, kIdxThreads, 0, st>>>(a); break;
      case kBF16: scatter_elems<kBF16><<<grid, kIdxThreads, 0, st>>>(a); break;
      default: return cudaErrorInvalidValue;
    }
  }
  return cudaGetLastError();
}

}  // namespace askb
