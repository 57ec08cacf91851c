// Vectorised global-memory access helpers shared by the kernel families.
//
// Loads of streamed inputs use ld.global.nc with L1::no_allocate (read-only,
// touched once); write-once outputs use st.global.cs (evict-first), so
// multi-gigabyte streams do not evict reused data such as gather tables from
// the 126 MB L2.
#pragma once

#include <stdint.h>

#include "ask_numerics.cuh"
#include "kernels.h"

namespace askb {

__device__ __forceinline__ uint64_t udiv(uint64_t n, const U32Div& q) {
  if (q.wide) return n / q.d;
  const uint32_t x = uint32_t(n);
  const uint32_t t = __umulhi(x, q.m);
  return (t + ((x - t) >> q.s1)) >> q.s2;
}
__device__ __forceinline__ uint64_t umod(uint64_t n, const U32Div& q) { return n - udiv(n, q) * q.d; }

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
// Asynchronous 16-byte global -> shared copies (cp.async, L2 only), committed
// in groups; a thread waits for its own groups with wait_group, so a stage a
// thread both fills and reads needs no other synchronisation.
__device__ __forceinline__ void copy_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void copy_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void copy_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 32-byte accesses (ld/st .v8.b32, sm_100): half the instructions of two
// 16-byte ones; the address must be 32-byte aligned.
struct Vec32 {
  uint32_t w[8];
};
__device__ __forceinline__ Vec32 ld_stream_v8(const void* p) {
  Vec32 r;
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3]), "=r"(r.w[4]), "=r"(r.w[5]), "=r"(r.w[6]),
                 "=r"(r.w[7])
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream_v8(void* p, const Vec32& v) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]),
               "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]), "r"(v.w[7])
               : "memory");
}
__device__ __forceinline__ bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

__device__ __forceinline__ void st_stream_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_stream_v2(void* p, uint2 v) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void st_stream_u32(void* p, uint32_t v) {
  asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Raw load of NB bytes (4, 8, 16, 32 or 64) into 32-bit words.
template <int NB>
__device__ __forceinline__ void load_raw(const void* p, uint32_t (&r)[NB / 4]) {
  if constexpr (NB == 4) {
    r[0] = ld_stream_u32(p);
  } else if constexpr (NB == 8) {
    const uint2 q = ld_stream_v2(p);
    r[0] = q.x; r[1] = q.y;
  } else {
#pragma unroll
    for (int k = 0; k < NB / 16; ++k) {
      const uint4 q = ld_stream_v4(static_cast<const char*>(p) + 16 * k);
      r[4 * k] = q.x; r[4 * k + 1] = q.y; r[4 * k + 2] = q.z; r[4 * k + 3] = q.w;
    }
  }
}
template <int NB>
__device__ __forceinline__ void store_raw(void* p, const uint32_t (&r)[NB / 4]) {
  if constexpr (NB == 4) {
    st_stream_u32(p, r[0]);
  } else if constexpr (NB == 8) {
    st_stream_v2(p, make_uint2(r[0], r[1]));
  } else {
#pragma unroll
    for (int k = 0; k < NB / 16; ++k)
      st_stream_v4(static_cast<char*>(p) + 16 * k, make_uint4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]));
  }
}

// Unpack element v of type T from a raw word array into a register word.
template <int T>
__device__ __forceinline__ uint64_t unpack_elem(const uint32_t* r, int v) {
  if constexpr (T == kF32 || T == kI32) {
    return uint64_t(r[v]);
  } else if constexpr (T == kI64) {
    return uint64_t(r[2 * v]) | (uint64_t(r[2 * v + 1]) << 32);
  } else if constexpr (T == kBool) {
    return ((r[v >> 2] >> (8 * (v & 3))) & 0xffu) != 0 ? 1u : 0u;
  } else {
    const uint32_t h = (r[v >> 1] >> (16 * (v & 1))) & 0xffffu;
    if constexpr (T == kF16) return w_of_f32(__half2float(__ushort_as_half(uint16_t(h))));
    else return w_of_f32(bf16_bits_to_f32(h));
  }
}
template <int T>
__device__ __forceinline__ void pack_elem(uint32_t* r, int v, uint64_t w) {
  if constexpr (T == kF32 || T == kI32) {
    r[v] = uint32_t(w);
  } else if constexpr (T == kI64) {
    r[2 * v] = uint32_t(w);
    r[2 * v + 1] = uint32_t(w >> 32);
  } else if constexpr (T == kBool) {
    const int sh = 8 * (v & 3);
    r[v >> 2] = (r[v >> 2] & ~(0xffu << sh)) | (uint32_t(w & 1u) << sh);
  } else {
    uint32_t h;
    if constexpr (T == kF16) h = __half_as_ushort(__float2half_rn(f32_of(w)));
    else h = bf16_bits_rne(f32_of(w));
    const int sh = 16 * (v & 1);
    r[v >> 1] = (r[v >> 1] & ~(0xffffu << sh)) | (h << sh);
  }
}

// V consecutive elements of type T starting at element `base` (aligned unit).
template <int T, int V>
__device__ __forceinline__ void load_unit(const void* p, uint64_t base, uint64_t (&w)[V]) {
  constexpr int NB = V * dtype_bytes(T);
  static_assert(NB % 4 == 0, "vector unit must cover whole 32-bit words");
  uint32_t r[NB / 4];
  load_raw<NB>(static_cast<const char*>(p) + base * dtype_bytes(T), r);
#pragma unroll
  for (int v = 0; v < V; ++v) w[v] = unpack_elem<T>(r, v);
}
template <int T, int V>
__device__ __forceinline__ void store_unit(void* p, uint64_t base, const uint64_t (&w)[V]) {
  constexpr int NB = V * dtype_bytes(T);
  uint32_t r[NB / 4];
#pragma unroll
  for (int k = 0; k < NB / 4; ++k) r[k] = 0;
#pragma unroll
  for (int v = 0; v < V; ++v) pack_elem<T>(r, v, w[v]);
  store_raw<NB>(static_cast<char*>(p) + base * dtype_bytes(T), r);
}

// Runtime-typed versions (uniform branch on the type).
template <int V>
__device__ __forceinline__ void load_unit_rt(int t, const void* p, uint64_t base, uint64_t (&w)[V]) {
  switch (t) {
    case kBool: load_unit<kBool, V>(p, base, w); break;
    case kI32: load_unit<kI32, V>(p, base, w); break;
    case kI64: load_unit<kI64, V>(p, base, w); break;
    case kF32: load_unit<kF32, V>(p, base, w); break;
    case kF16: load_unit<kF16, V>(p, base, w); break;
    default: load_unit<kBF16, V>(p, base, w); break;
  }
}
template <int V>
__device__ __forceinline__ void store_unit_rt(int t, void* p, uint64_t base, const uint64_t (&w)[V]) {
  switch (t) {
    case kBool: store_unit<kBool, V>(p, base, w); break;
    case kI32: store_unit<kI32, V>(p, base, w); break;
    case kI64: store_unit<kI64, V>(p, base, w); break;
    case kF32: store_unit<kF32, V>(p, base, w); break;
    case kF16: store_unit<kF16, V>(p, base, w); break;
    default: store_unit<kBF16, V>(p, base, w); break;
  }
}

// ---- ports: typed, index-mapped unit access -----------------------------------
// Load V elements of an input for the aligned unit starting at `base`.
// `vec` is true when the unit is complete and the port is 16-byte aligned.
template <int T, int MAP, int V>
__device__ __forceinline__ void load_port(const void* p, uint64_t base, uint64_t n, const U32Div& inner, bool vec,
                                          uint64_t (&w)[V]) {
  if constexpr (MAP == IM_SCALAR) {
    const uint64_t s = word_from_storage(T, p, 0);
#pragma unroll
    for (int v = 0; v < V; ++v) w[v] = s;
  } else if constexpr (MAP == IM_OUTER) {
    if (vec && inner.d % V == 0) {
      const uint64_t s = word_from_storage(T, p, udiv(base, inner));
#pragma unroll
      for (int v = 0; v < V; ++v) w[v] = s;
    } else {
#pragma unroll
      for (int v = 0; v < V; ++v) w[v] = (base + v < n) ? word_from_storage(T, p, udiv(base + v, inner)) : 0;
    }
  } else if constexpr (MAP == IM_INNER) {
    if constexpr (V > 1 && (V * dtype_bytes(T)) % 4 == 0) {
      if (vec && inner.d % V == 0) { load_unit<T, V>(p, umod(base, inner), w); return; }
    }
#pragma unroll
    for (int v = 0; v < V; ++v) w[v] = (base + v < n) ? word_from_storage(T, p, umod(base + v, inner)) : 0;
  } else {
    if constexpr (V > 1 && (V * dtype_bytes(T)) % 4 == 0) {
      if (vec) { load_unit<T, V>(p, base, w); return; }
    }
#pragma unroll
    for (int v = 0; v < V; ++v) w[v] = (base + v < n) ? word_from_storage(T, p, base + v) : 0;
  }
}

template <int T, int V>
__device__ __forceinline__ void store_port(void* p, uint64_t base, uint64_t n, bool vec, const uint64_t (&w)[V]) {
  if constexpr (V > 1 && (V * dtype_bytes(T)) % 4 == 0) {
    if (vec) { store_unit<T, V>(p, base, w); return; }
  }
#pragma unroll
  for (int v = 0; v < V; ++v)
    if (base + v < n) word_to_storage(T, p, base + v, w[v]);
}

template <int V>
__device__ __forceinline__ void rt_load(int t, int map, const void* p, uint64_t base, uint64_t n,
                                        const U32Div& inner, bool vec, uint64_t (&w)[V]) {
#define ASKB_LOAD_MAP(T)                                                         \
  switch (map) {                                                                 \
    case IM_FULL: load_port<T, IM_FULL, V>(p, base, n, inner, vec, w); break;    \
    case IM_SCALAR: load_port<T, IM_SCALAR, V>(p, base, n, inner, vec, w); break; \
    case IM_OUTER: load_port<T, IM_OUTER, V>(p, base, n, inner, vec, w); break;  \
    default: load_port<T, IM_INNER, V>(p, base, n, inner, vec, w); break;        \
  }
  switch (t) {
    case kBool: ASKB_LOAD_MAP(kBool) break;
    case kI32: ASKB_LOAD_MAP(kI32) break;
    case kI64: ASKB_LOAD_MAP(kI64) break;
    case kF32: ASKB_LOAD_MAP(kF32) break;
    case kF16: ASKB_LOAD_MAP(kF16) break;
    default: ASKB_LOAD_MAP(kBF16) break;
  }
#undef ASKB_LOAD_MAP
}
template <int V>
__device__ __forceinline__ void rt_store(int t, void* p, uint64_t base, uint64_t n, bool vec, const uint64_t (&w)[V]) {
  switch (t) {
    case kBool: store_port<kBool, V>(p, base, n, vec, w); break;
    case kI32: store_port<kI32, V>(p, base, n, vec, w); break;
    case kI64: store_port<kI64, V>(p, base, n, vec, w); break;
    case kF32: store_port<kF32, V>(p, base, n, vec, w); break;
    case kF16: store_port<kF16, V>(p, base, n, vec, w); break;
    default: store_port<kBF16, V>(p, base, n, vec, w); break;
  }
}


}  // namespace askb
