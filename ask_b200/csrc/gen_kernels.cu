// Seeded input synthesis on the device (Philox4x32-10, Salmon et al., SC'11).
//
// Element i of stream s under seed k is drawn from one Philox block with
// counter (lo32(i), hi32(i), s, 0) and key (lo32(k), hi32(k)), so any shard of
// a tensor can be generated independently and identically for every number of
// ranks.  Uniform, raw-i32 and Zipf draws use only integer and exact
// floating-point arithmetic and are therefore bit-identical to a host
// generator implementing the same mapping; the normal draws use Box-Muller in
// f64 (log/cos/sqrt), which is not guaranteed to match a host libm bit for bit.
// This code only synthesises benchmark/test inputs; it is not part of any plan.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"

namespace askb {

namespace {

constexpr int kGenThreads = 256;

struct Philox {
  uint32_t c[4];
};

__device__ __forceinline__ Philox philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                               uint32_t k1) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u, kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint32_t hi0 = __umulhi(kM0, c0), lo0 = kM0 * c0;
    const uint32_t hi1 = __umulhi(kM1, c2), lo1 = kM1 * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += kW0; k1 += kW1;
  }
  return Philox{{c0, c1, c2, c3}};
}

__global__ void __launch_bounds__(kGenThreads) gen_kernel(int kind, uint64_t seed, uint32_t sid, uint64_t offset,
                                                          uint64_t count, double p0, double p1,
                                                          const double* __restrict__ cdf, uint64_t zipf_n, void* dst) {
  const uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
  for (uint64_t t = uint64_t(blockIdx.x) * kGenThreads + threadIdx.x; t < count; t += uint64_t(gridDim.x) * kGenThreads) {
    const uint64_t i = offset + t;
    const Philox r = philox4x32_10(uint32_t(i), uint32_t(i >> 32), sid, 0u, k0, k1);
    switch (kind) {
      case GEN_UNIFORM_F32: {
        const double u = double(r.c[0] >> 8) * (1.0 / 16777216.0);
        static_cast<float*>(dst)[t] = float(p0 + (p1 - p0) * u);
        break;
      }
      case GEN_I32:
        static_cast<int32_t*>(dst)[t] = int32_t(r.c[0]);
        break;
      case GEN_ZIPF_I64:
      case GEN_ZIPF_I32: {
        const uint64_t bits = (uint64_t(r.c[0] >> 5) << 26) | uint64_t(r.c[1] >> 6);
        const double target = double(bits) * (1.0 / 9007199254740992.0) * cdf[zipf_n - 1];
        uint64_t lo = 0, hi = zipf_n - 1;  // smallest k with cdf[k] > target
        while (lo < hi) {
          const uint64_t mid = (lo + hi) >> 1;
          if (cdf[mid] > target) hi = mid; else lo = mid + 1;
        }
        if (kind == GEN_ZIPF_I64) static_cast<int64_t*>(dst)[t] = int64_t(lo);
        else static_cast<int32_t*>(dst)[t] = int32_t(lo);
        break;
      }
      default: {  // normals
        const double u1 = (double(r.c[0]) + 1.0) * (1.0 / 4294967296.0);
        const double u2 = double(r.c[1]) * (1.0 / 4294967296.0);
        const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
        const double x = p0 + p1 * z;
        if (kind == GEN_NORMAL_F32) static_cast<float*>(dst)[t] = float(x);
        else if (kind == GEN_NORMAL_F16) static_cast<__half*>(dst)[t] = __double2half(x);
        else static_cast<__nv_bfloat16*>(dst)[t] = __double2bfloat16(x);
        break;
      }
    }
  }
}

}  // namespace

cudaError_t gen_launch(int kind, uint64_t seed, uint32_t stream_id, uint64_t offset, uint64_t count, double p0,
                       double p1, const double* zipf_cdf, uint64_t zipf_n, void* dst, cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  uint64_t blocks = (count + kGenThreads - 1) / kGenThreads;
  if (blocks > 148 * 64) blocks = 148 * 64;
  gen_kernel<<<unsigned(blocks), kGenThreads, 0, stream>>>(kind, seed, stream_id, offset, count, p0, p1, zipf_cdf,
                                                          zipf_n, dst);
  return cudaGetLastError();
}

}  // namespace askb
