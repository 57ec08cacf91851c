// Family X, sorted path: scatter_add of whole rows grouped by destination.
//
// Semantics are those of lib/Lowering/CUDA.cpp:297-352 and
// lib/Lowering/Host.cpp:677-772: out = base, then every in-bounds update row
// j is added to out[o, idx[j], :]; out-of-bounds indices are skipped.  The
// reference issues one atomic per update element, which on a Zipf(1.1) index
// stream serialises on the hot rows and turns the 1 GiB table into a
// read-modify-write target for 2^31 atomics.  Here the updates are first
// grouped by destination row (a counting sort built from per-tile shared
// memory hash tables), then every run of updates to one row is summed in
// registers and applied once:
//
//   K1 zero the row histogram
//   K2 tile pass: each CTA aggregates its tile of indices in a shared-memory
//      hash table and adds one count per distinct row to the histogram
//   K3 exclusive scan of the histogram -> segment offsets, which also become
//      the placement cursors; then the step's pre_copy (out = base) for the
//      rows K5 does not own
//   K4 tile pass again: per distinct row of the tile reserve a range with one
//      atomicAdd on the row's cursor, write (row, update index) pairs into
//      the sorted order
//   K5 a warp per 64 sorted entries: sum each run of equal rows in registers;
//      a run that is its row's whole segment owns the row (out = base + sum,
//      no pre-copy), a run crossing a chunk boundary adds with vector atomics
//      (red.global.add.v4.f32) or scalar integer atomics.
// Float results differ from a serial order by rounding only (the reference's
// atomic order is unspecified as well); integer results are exact.
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "ask_numerics.cuh"
#include "kernels.h"
#include "vec_io.cuh"

namespace askb {

namespace {

constexpr int kTile = 2048;             // indices per CTA tile
constexpr int kHashSlots = 4096;        // shared-memory hash slots per tile (2x the tile)
constexpr uint32_t kEmpty = 0xffffffffu;
constexpr int kSortThreads = 512;
constexpr int kChunk = 64;              // sorted entries per warp in K5
constexpr int kScanThreads = 1024;

__device__ __forceinline__ int64_t index_at(const IndexArgs& a, uint64_t j) {
  return a.index_type == kI32 ? int64_t(__ldg(static_cast<const int32_t*>(a.index) + j))
                              : __ldg(static_cast<const int64_t*>(a.index) + j);
}

// Destination row key of flat update row r = (o, j), or kEmpty if skipped.
__device__ __forceinline__ uint32_t row_key(const IndexArgs& a, uint64_t r) {
  const uint64_t o = a.outer == 1 ? 0 : r / a.n, j = r - o * a.n;
  const int64_t idx = index_at(a, j);
  if (idx < 0 || uint64_t(idx) >= a.dim) return kEmpty;
  return uint32_t(o * a.dim + uint64_t(idx));
}

__device__ __forceinline__ uint32_t hash32(uint32_t k) {
  k ^= k >> 16; k *= 0x7feb352du; k ^= k >> 15; k *= 0x846ca68bu; k ^= k >> 16;
  return k;
}

// Position of a row's counter in the histogram and placement cursor.  Within
// each group of 1024 rows the 32x32 (row % 32, row / 32 % 32) layout is
// transposed, so rows that are close (the hot rows of a skewed index stream)
// land on different 128-byte lines and so on different L2 slices; with the
// plain layout the counters of the 32 hottest rows share one line and every
// tile's atomics on them serialise in one slice.
constexpr uint32_t kGroup = 1024;
__device__ __forceinline__ uint32_t counter_of(uint32_t key) {
  return (key & ~(kGroup - 1)) | ((key & 31u) << 5) | ((key >> 5) & 31u);
}

// The counters exist in `replicas` copies of mp entries; CTA b adds into copy
// b % replicas.  A hot row's counter is then the target of 1/replicas of the
// tiles' atomics (same-address atomics serialise in L2).  The scan sums the
// copies and leaves in copy q the cursor off[r] + (counts of copies < q).

// A row whose whole segment of sorted entries lies inside one K5 chunk is
// "owned" by that chunk: K5 writes it as base + sum without atomics and the
// pre-copy skips it.  The scan marks owned rows with this bit in the cursors,
// K4 carries it into the sorted keys (row keys and positions are < 2^31).
constexpr uint32_t kOwnedBit = 0x80000000u;

// Insert one key per lane of a converged warp into the tile's table; returns
// (slot, rank of this insertion), slot kEmpty for a lane whose key is kEmpty.
// Lanes holding the same key are combined first (one shared-memory atomic per
// distinct key of the warp: the hot rows of a skewed index stream recur in
// most warps), and a slot already holding the key is found by a plain read,
// so only a key's first insertion in the tile pays for the compare-and-swap.
constexpr int kRankBits = 11;  // ranks < kTile
static_assert(kTile <= (1 << kRankBits) && kHashSlots <= 4096, "tag and list packing");

__device__ __forceinline__ uint32_t tile_insert(uint32_t* keys, uint32_t* counts, uint32_t key, uint32_t* rank,
                                                bool* fresh) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t peers = __match_any_sync(0xffffffffu, key);
  const int leader = __ffs(peers) - 1;
  uint32_t s = kEmpty, r = 0;
  *fresh = false;
  if (int(lane) == leader && key != kEmpty) {
    s = hash32(key) & (kHashSlots - 1);
    for (int probe = 0; probe < kHashSlots; ++probe) {
      uint32_t prev = *reinterpret_cast<volatile uint32_t*>(&keys[s]);
      if (prev == kEmpty) {
        prev = atomicCAS(&keys[s], kEmpty, key);
        *fresh = prev == kEmpty;
      }
      if (prev == kEmpty || prev == key) break;
      s = (s + 1) & (kHashSlots - 1);  // the table has twice as many slots as a tile has keys
    }
    r = atomicAdd(&counts[s], uint32_t(__popc(peers)));
  }
  s = __shfl_sync(0xffffffffu, s, leader);
  r = __shfl_sync(0xffffffffu, r, leader);
  *rank = r + uint32_t(__popc(peers & ((1u << lane) - 1u)));
  return s;
}

__global__ void __launch_bounds__(kSortThreads) zero_u32(uint32_t* p, uint64_t n) {
  for (uint64_t i = uint64_t(blockIdx.x) * kSortThreads + threadIdx.x; i < n; i += uint64_t(gridDim.x) * kSortThreads)
    p[i] = 0;
}

// K2: per-tile aggregation into the global histogram.  Each thread loads all
// of its tile's indices before inserting any (the loads overlap), and the
// next tile's indices are loaded before this tile's counts are flushed.
constexpr int kPerThread = kTile / kSortThreads;

__device__ __forceinline__ void load_tile_keys(const IndexArgs& a, uint64_t t0, uint64_t rows,
                                               uint32_t (&k)[kPerThread]) {
#pragma unroll
  for (int q = 0; q < kPerThread; ++q) {
    const uint64_t r = t0 + uint64_t(q) * kSortThreads + threadIdx.x;
    k[q] = r < rows ? row_key(a, r) : kEmpty;
  }
}

// K2 also records, for K4, each update's tag (slot << kRankBits | rank in
// the tile; kEmpty for a skipped index) and the tile's list of distinct keys
// (key, slot | count << 12), so K4 needs neither the indices nor a hash table.
__global__ void __launch_bounds__(kSortThreads) tile_histogram(const __grid_constant__ IndexArgs a, uint64_t rows,
                                                              uint32_t* __restrict__ hist, uint64_t mp,
                                                              int replicas, uint32_t* __restrict__ tag,
                                                              uint2* __restrict__ list,
                                                              uint32_t* __restrict__ list_len) {
  __shared__ uint32_t keys[kHashSlots], counts[kHashSlots];
  __shared__ uint32_t used[kTile];  // slots claimed in this tile, in claim order
  __shared__ uint32_t n_used[2];    // claim counters of alternate tiles
  const uint32_t lane = threadIdx.x & 31u;
  for (int s = threadIdx.x; s < kHashSlots; s += kSortThreads) { keys[s] = kEmpty; counts[s] = 0; }
  if (threadIdx.x == 0) n_used[0] = 0;
  __syncthreads();
  uint64_t t0 = uint64_t(blockIdx.x) * kTile;
  const uint64_t step = uint64_t(gridDim.x) * kTile;
  uint32_t k[kPerThread];
  if (t0 < rows) load_tile_keys(a, t0, rows, k);
  for (uint32_t parity = 0; t0 < rows; t0 += step, parity ^= 1u) {
    const uint64_t tile = t0 / kTile;
    uint32_t* h = hist + (tile % unsigned(replicas)) * mp;
#pragma unroll
    for (int q = 0; q < kPerThread; ++q) {
      const uint64_t r = t0 + uint64_t(q) * kSortThreads + threadIdx.x;
      uint32_t rank;
      bool fresh;
      const uint32_t s = tile_insert(keys, counts, k[q], &rank, &fresh);
      if (r < rows) tag[r] = s == kEmpty ? kEmpty : (s << kRankBits) | rank;
      const uint32_t fb = __ballot_sync(0xffffffffu, fresh);
      if (fb) {
        uint32_t at = 0;
        if (lane == 0) at = atomicAdd(&n_used[parity], uint32_t(__popc(fb)));
        at = __shfl_sync(0xffffffffu, at, 0) + uint32_t(__popc(fb & ((1u << lane) - 1u)));
        if (fresh) used[at] = s;
      }
    }
    __syncthreads();
    if (t0 + step < rows) load_tile_keys(a, t0 + step, rows, k);
    const uint32_t len = n_used[parity];
    if (threadIdx.x == 0) { list_len[tile] = len; n_used[parity ^ 1u] = 0; }
    uint2* tl = list + tile * kTile;
    for (uint32_t e = threadIdx.x; e < len; e += kSortThreads) {
      const uint32_t s = used[e], key = keys[s], cnt = counts[s];
      atomicAdd(&h[counter_of(key)], cnt);
      tl[e] = make_uint2(key, s | (cnt << 12));
      keys[s] = kEmpty;  // ready for the next tile
      counts[s] = 0;
    }
    __syncthreads();
  }
}

// K3: exclusive scan of the histogram into off[0..m] (off[m] = number of
// valid updates), in three coalesced phases: per-block sums, a scan of the
// block sums, per-block scans.  The last phase also turns the histogram into
// the placement cursor: the counter of row r becomes off[r].  Blocks cover
// whole 1024-row groups, so the counter layout's transpose stays inside one
// block and is undone through shared memory.
__device__ __forceinline__ uint32_t block_inclusive_scan(uint32_t v, uint32_t* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += t;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < int(blockDim.x >> 5) ? warp_tot[lane] : 0u;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += t;
    }
    warp_tot[lane] = w;  // inclusive totals of warps 0..lane
  }
  __syncthreads();
  const uint32_t before = warp ? warp_tot[warp - 1] : 0u;
  __syncthreads();
  return v + before;
}

template <int kReplicas>
__global__ void __launch_bounds__(kScanThreads) scan_block_sums(const uint32_t* __restrict__ hist, uint64_t mp,
                                                               uint64_t per_block, uint32_t* __restrict__ bsum) {
  __shared__ uint32_t warp_tot[32];
  const uint64_t b0 = uint64_t(blockIdx.x) * per_block, b1 = min(mp, b0 + per_block);
  uint32_t sum = 0;
  for (uint64_t i = b0 + threadIdx.x; i < b1; i += kScanThreads) {
    uint32_t c[kReplicas];
#pragma unroll
    for (int q = 0; q < kReplicas; ++q) c[q] = hist[q * mp + i];
#pragma unroll
    for (int q = 0; q < kReplicas; ++q) sum += c[q];
  }
  sum = block_inclusive_scan(sum, warp_tot);
  if (threadIdx.x == kScanThreads - 1) bsum[blockIdx.x] = sum;
}

__global__ void __launch_bounds__(kScanThreads) scan_block_offsets(uint32_t* __restrict__ bsum, int nblocks,
                                                                  uint32_t* __restrict__ total) {
  __shared__ uint32_t warp_tot[32];
  const uint32_t v = threadIdx.x < nblocks ? bsum[threadIdx.x] : 0u;
  const uint32_t inc = block_inclusive_scan(v, warp_tot);
  if (threadIdx.x < nblocks) bsum[threadIdx.x] = inc - v;  // exclusive
  if (threadIdx.x == kScanThreads - 1) *total = inc;
}

static_assert(kScanThreads == kGroup, "one scan pass covers one counter group");

template <int kReplicas>
__global__ void __launch_bounds__(kScanThreads) scan_write_offsets(uint32_t* __restrict__ hist, uint64_t m,
                                                                  uint64_t mp, uint64_t per_block,
                                                                  const uint32_t* __restrict__ bsum,
                                                                  uint32_t* __restrict__ off) {
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t group[kReplicas][kGroup + kGroup / 32];  // padded: a column read is conflict-free
  __shared__ uint32_t last;
  const uint64_t b0 = uint64_t(blockIdx.x) * per_block, b1 = min(mp, b0 + per_block);
  const uint32_t t = threadIdx.x;
  const uint32_t col = (t & 31u) * 33u + (t >> 5);  // padded position of row t's counter
  uint32_t carry = bsum[blockIdx.x];
  for (uint64_t g = b0; g < b1; g += kGroup) {
#pragma unroll
    for (int q = 0; q < kReplicas; ++q) group[q][t + (t >> 5)] = hist[q * mp + g + t];
    __syncthreads();
    uint32_t cq[kReplicas], c = 0;
#pragma unroll
    for (int q = 0; q < kReplicas; ++q) { cq[q] = group[q][col]; c += cq[q]; }
    const uint32_t inc = block_inclusive_scan(c, warp_tot);  // (its barriers order the reads above)
    uint32_t o = carry + inc - c;
    if (g + t < m) off[g + t] = o;
    const uint32_t owned = (c && o / kChunk == (o + c - 1) / kChunk) ? kOwnedBit : 0u;
#pragma unroll
    for (int q = 0; q < kReplicas; ++q) { group[q][col] = o | owned; o += cq[q]; }
    if (t == kScanThreads - 1) last = inc;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kReplicas; ++q) hist[q * mp + g + t] = group[q][t + (t >> 5)];
    carry += last;
    __syncthreads();
  }
}

// K4: write (key, update row) pairs into sorted position.  Per tile: one
// cursor atomic per distinct key (from K2's list) reserves the key's range,
// then every update's tag gives its position in that range.
__global__ void __launch_bounds__(kSortThreads) tile_place(uint64_t rows, uint32_t* __restrict__ cursor, uint64_t mp,
                                                          int replicas, const uint32_t* __restrict__ tag,
                                                          const uint2* __restrict__ list,
                                                          const uint32_t* __restrict__ list_len,
                                                          uint2* __restrict__ sorted) {
  __shared__ uint32_t skey[kHashSlots], sbase[kHashSlots];
  constexpr int kPer = kTile / kSortThreads;  // list entries and updates per thread
  for (uint64_t t0 = uint64_t(blockIdx.x) * kTile; t0 < rows; t0 += uint64_t(gridDim.x) * kTile) {
    const uint64_t tile = t0 / kTile;
    uint32_t* c = cursor + (tile % unsigned(replicas)) * mp;
    const uint32_t len = list_len[tile];
    const uint2* tl = list + tile * kTile;
    uint2 ent[kPer];
    uint32_t tg[kPer], res[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const uint32_t e = threadIdx.x + j * kSortThreads;
      ent[j] = e < len ? tl[e] : make_uint2(kEmpty, 0);
      const uint64_t r = t0 + e;
      tg[j] = r < rows ? tag[r] : kEmpty;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j)  // all of a thread's cursor atomics in flight at once
      if (ent[j].x != kEmpty) res[j] = atomicAdd(&c[counter_of(ent[j].x)], ent[j].y >> 12);
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (ent[j].x != kEmpty) { skey[ent[j].y & 4095u] = ent[j].x; sbase[ent[j].y & 4095u] = res[j]; }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (tg[j] != kEmpty) {
        const uint32_t slot = tg[j] >> kRankBits, b = sbase[slot];
        const uint32_t pos = (b & ~kOwnedBit) + (tg[j] & ((1u << kRankBits) - 1u));
        sorted[pos] = make_uint2(skey[slot] | (b & kOwnedBit), uint32_t(t0 + threadIdx.x + j * kSortThreads));
      }
    }
    __syncthreads();
  }
  // Launched as the copy's programmatic dependent, this grid may run beside
  // it; it completes only after the copy has (K5 reads the copied rows).
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void add4(uint4& acc, uint4 v, bool fl) {
  if (fl) {
    acc.x = __float_as_uint(__fadd_rn(__uint_as_float(acc.x), __uint_as_float(v.x)));
    acc.y = __float_as_uint(__fadd_rn(__uint_as_float(acc.y), __uint_as_float(v.y)));
    acc.z = __float_as_uint(__fadd_rn(__uint_as_float(acc.z), __uint_as_float(v.z)));
    acc.w = __float_as_uint(__fadd_rn(__uint_as_float(acc.w), __uint_as_float(v.w)));
  } else {
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
}

// Write a closed run's sum at column vector `pos` of its row: an owned run
// already holds base + sum and stores it; any other run adds atomically into
// the pre-copied row.
__device__ __forceinline__ void apply(uint4* out, uint64_t pos, uint4 acc, bool fl, bool owned) {
  if (owned) {
    st_stream_v4(out + pos, acc);
  } else if (fl) {
    atomicAdd(reinterpret_cast<float4*>(out) + pos,
              make_float4(__uint_as_float(acc.x), __uint_as_float(acc.y), __uint_as_float(acc.z), __uint_as_float(acc.w)));
  } else {
    unsigned* o = reinterpret_cast<unsigned*>(out + pos);
    atomicAdd(o, acc.x); atomicAdd(o + 1, acc.y); atomicAdd(o + 2, acc.z); atomicAdd(o + 3, acc.w);
  }
}


// K5: a warp per chunk of kChunk sorted entries.  The chunk becomes a list of
// items in shared memory -- the update rows in sorted order, with the base row
// of each owned run placed before the run's first update -- and the items'
// rows stream through a per-warp ring of kDepth shared-memory stages with
// asynchronous 16-byte copies (each lane copies and later reads only its own
// column vectors, so a lane's own wait_group is all the synchronisation a
// stage needs).  Lanes own 16-byte column vectors of a row: vecs = row bytes
// / 16, kV per lane per pass.  Runs of equal keys are summed in registers.
constexpr int kRunWarps = 4;
constexpr uint32_t kBaseItem = 0xffffffffu;  // item row marker: the base row of the item's key

template <int kV, int kDepth>
constexpr size_t run_sums_smem() { return size_t(kRunWarps) * kDepth * kV * 32 * 16; }

template <int kV, int kDepth>
__global__ void __launch_bounds__(kRunWarps * 32) run_sums(const __grid_constant__ IndexArgs a, uint32_t vecs,
                                                           const uint32_t* __restrict__ total_ptr,
                                                           const uint2* __restrict__ sorted, int fl) {
  extern __shared__ uint4 ring_all[];
  __shared__ uint32_t ikey[kRunWarps][2 * kChunk], irow[kRunWarps][2 * kChunk];
  const uint64_t total = *total_ptr;  // valid (in-bounds) updates, written by the scan
  const uint32_t lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  uint4* ring = ring_all + size_t(wib) * kDepth * kV * 32;
  const uint64_t warp = uint64_t(blockIdx.x) * kRunWarps + wib;
  const uint64_t nwarps = uint64_t(gridDim.x) * kRunWarps;
  const uint4* upd = static_cast<const uint4*>(a.table);
  const uint4* base = static_cast<const uint4*>(a.base);
  uint4* out = static_cast<uint4*>(a.out);
  const uint64_t chunks = (total + kChunk - 1) / kChunk;
  for (uint64_t c = warp; c < chunks; c += nwarps) {
    const uint64_t c0 = c * kChunk;
    const int n = int(min(total, c0 + kChunk) - c0);
    // items: entry i goes to i + (owned run starts at or before i); an owned
    // run start is preceded by its base item
    uint32_t before = 0, carry_key = kEmpty;
#pragma unroll
    for (int h = 0; h < kChunk / 32; ++h) {
      const int i = h * 32 + int(lane);
      const uint2 kr = i < n ? sorted[c0 + i] : make_uint2(kEmpty, 0u);
      const uint32_t k = kr.x, r = kr.y;
      uint32_t prev = __shfl_up_sync(0xffffffffu, k, 1);
      if (lane == 0) prev = carry_key;
      const bool starts = i < n && (i == 0 || k != prev) && (k & kOwnedBit);
      const uint32_t sb = __ballot_sync(0xffffffffu, starts);
      const uint32_t at = uint32_t(i) + before + uint32_t(__popc(sb & ((2u << lane) - 1u)));
      if (i < n) {
        if (starts) { ikey[wib][at - 1] = k; irow[wib][at - 1] = kBaseItem; }
        ikey[wib][at] = k;
        irow[wib][at] = r;
      }
      before += uint32_t(__popc(sb));
      carry_key = __shfl_sync(0xffffffffu, k, 31);
    }
    __syncwarp();
    const int items = n + int(before);
    for (uint32_t v0 = 0; v0 < vecs; v0 += 32 * kV) {
      auto issue = [&](int j) {
        if (j < items) {
          const uint32_t r = irow[wib][j];
          const uint4* src = r == kBaseItem ? base + uint64_t(ikey[wib][j] & ~kOwnedBit) * vecs
                                            : upd + uint64_t(r) * vecs;
          uint4* dst = ring + (j % kDepth) * kV * 32;
#pragma unroll
          for (int q = 0; q < kV; ++q) {
            const uint32_t v = v0 + q * 32 + lane;
            if (v < vecs) copy_async16(dst + q * 32 + lane, src + v);
          }
        }
        copy_async_commit();
      };
#pragma unroll
      for (int j = 0; j < kDepth; ++j) issue(j);
      uint4 acc[kV];
#pragma unroll
      for (int q = 0; q < kV; ++q) acc[q] = make_uint4(0, 0, 0, 0);
      uint32_t cur = ikey[wib][0];
      for (int j = 0; j < items; ++j) {
        copy_async_wait<kDepth - 1>();
        const uint32_t key = ikey[wib][j];
        if (j > 0 && (key != cur || irow[wib][j] == kBaseItem)) {  // close the run of `cur`
#pragma unroll
          for (int q = 0; q < kV; ++q) {
            const uint32_t v = v0 + q * 32 + lane;
            if (v < vecs) apply(out, uint64_t(cur & ~kOwnedBit) * vecs + v, acc[q], fl != 0, (cur & kOwnedBit) != 0);
            acc[q] = make_uint4(0, 0, 0, 0);
          }
          cur = key;
        }
        const uint4* slot = ring + (j % kDepth) * kV * 32;
#pragma unroll
        for (int q = 0; q < kV; ++q) {
          const uint32_t v = v0 + q * 32 + lane;
          if (v < vecs) add4(acc[q], slot[q * 32 + lane], fl != 0);
        }
        issue(j + kDepth);  // reuses this stage: its values are already in registers
      }
#pragma unroll
      for (int q = 0; q < kV; ++q) {
        const uint32_t v = v0 + q * 32 + lane;
        if (v < vecs) apply(out, uint64_t(cur & ~kOwnedBit) * vecs + v, acc[q], fl != 0, (cur & kOwnedBit) != 0);
      }
    }
    copy_async_wait<0>();
    __syncwarp();
  }
}

// The step's pre_copy, restricted to the rows run_sums does not own: rows with
// no update, and rows whose segment crosses a chunk boundary (those receive
// atomic adds).  Rows owned by one chunk are written as base + sum there.
// A warp takes 32 consecutive rows, finds the unowned ones with one ballot,
// and streams them through a per-warp ring of kCopyDepth shared-memory stages
// with asynchronous copies, as run_sums does.  The grid is one CTA per SM and
// lets the next kernel (K4, launched as its programmatic dependent) start at
// once on the SM space it leaves free: K4 is latency-bound, this copy is
// bandwidth-bound, and they share no data.
constexpr int kCopyWarps = 8, kCopyDepth = 8;
constexpr size_t kCopySmem = size_t(kCopyWarps) * kCopyDepth * 2 * 32 * 16;

__global__ void __launch_bounds__(kCopyWarps * 32) copy_unowned_rows(const __grid_constant__ IndexArgs a, uint32_t vecs,
                                                                    const uint32_t* __restrict__ off, uint64_t m) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint4 ring_all[];
  const uint32_t lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  uint4* ring = ring_all + size_t(wib) * kCopyDepth * 2 * 32;
  const uint64_t warp = uint64_t(blockIdx.x) * kCopyWarps + wib;
  const uint64_t nwarps = uint64_t(gridDim.x) * kCopyWarps;
  const uint4* base = static_cast<const uint4*>(a.base);
  uint4* out = static_cast<uint4*>(a.out);
  for (uint64_t g = warp * 32; g < m; g += nwarps * 32) {
    bool unowned = false;
    if (g + lane < m) {
      const uint32_t s0 = off[g + lane], s1 = off[g + lane + 1];
      unowned = !(s1 > s0 && (s0 / kChunk) == ((s1 - 1) / kChunk));
    }
    const uint32_t mask = __ballot_sync(0xffffffffu, unowned);
    const int items = __popc(mask);
    for (uint32_t v0 = 0; v0 < vecs; v0 += 64) {
      auto row_of = [&](int j) { return g + uint64_t(__fns(mask, 0, j + 1)); };  // j-th set bit
      auto issue = [&](int j) {
        if (j < items) {
          const uint4* src = base + row_of(j) * vecs;
          uint4* dst = ring + (j % kCopyDepth) * 64;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const uint32_t v = v0 + q * 32 + lane;
            if (v < vecs) copy_async16(dst + q * 32 + lane, src + v);
          }
        }
        copy_async_commit();
      };
#pragma unroll
      for (int j = 0; j < kCopyDepth; ++j) issue(j);
      for (int j = 0; j < items; ++j) {
        copy_async_wait<kCopyDepth - 1>();
        const uint4* slot = ring + (j % kCopyDepth) * 64;
        uint4* dst = out + row_of(j) * vecs;
        uint4 x[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t v = v0 + q * 32 + lane;
          if (v < vecs) x[q] = slot[q * 32 + lane];
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t v = v0 + q * 32 + lane;
          if (v < vecs) st_stream_v4(dst + v, x[q]);
        }
        issue(j + kCopyDepth);  // reuses this stage: its values are already in registers
      }
    }
  }
  copy_async_wait<0>();
}

}  // namespace

constexpr int kScanBlocks = 512;

// Counter copies: 8 while they fit in 128 MiB, fewer for very large tables.
int counter_replicas(uint64_t mp) { return mp <= (uint64_t(1) << 22) ? 8 : mp <= (uint64_t(1) << 24) ? 2 : 1; }

namespace {

// Scratch layout of the sorted path (each array 256-byte aligned).
struct SortScratch {
  uint32_t* hist;      // reps copies of mp counters (counter_of layout), later the cursors
  uint32_t* off;       // m + 1 segment offsets
  uint2* sorted;       // rows (key, update index) pairs in key order (kOwnedBit marks owned rows)
  uint32_t* tag;       // rows tags from K2
  uint2* list;         // ntiles * kTile distinct-key lists from K2
  uint32_t* list_len;  // ntiles list lengths
  uint32_t* bsum;      // kScanBlocks scan block sums
  uint64_t m, rows, mp, ntiles;
  int reps;
  size_t bytes;
};

SortScratch sort_scratch(const IndexArgs& a, void* base) {
  SortScratch x{};
  x.m = a.outer * a.dim;
  x.rows = a.outer * a.n;
  x.mp = (x.m + kGroup - 1) / kGroup * kGroup;
  x.ntiles = (x.rows + kTile - 1) / kTile;
  x.reps = counter_replicas(x.mp);
  auto up = [](uint64_t b) { return (b + 255) & ~uint64_t(255); };
  char* p = static_cast<char*>(base);
  uint64_t at = 0;
  auto take = [&](uint64_t bytes) { char* q = p ? p + at : nullptr; at += up(bytes); return q; };
  x.hist = reinterpret_cast<uint32_t*>(take(4 * x.mp * x.reps));
  x.off = reinterpret_cast<uint32_t*>(take(4 * (x.m + 1)));
  x.sorted = reinterpret_cast<uint2*>(take(8 * x.rows));
  x.tag = reinterpret_cast<uint32_t*>(take(4 * x.rows));
  x.list = reinterpret_cast<uint2*>(take(8 * x.ntiles * kTile));
  x.list_len = reinterpret_cast<uint32_t*>(take(4 * x.ntiles));
  x.bsum = reinterpret_cast<uint32_t*>(take(4 * kScanBlocks));
  x.bytes = size_t(at);
  return x;
}

}  // namespace

size_t scatter_sorted_scratch_bytes(const IndexArgs& a) { return sort_scratch(a, nullptr).bytes; }

bool scatter_sorted_ok(const IndexArgs& a) {
  const uint64_t m = a.outer * a.dim, rows = a.outer * a.n;
  const uint64_t row_bytes = a.inner * uint64_t(dtype_bytes(a.elem_type));
  return (a.elem_type == kF32 || a.elem_type == kI32) && row_bytes % 16 == 0 && row_bytes >= 64 &&
         m < kOwnedBit && rows < kOwnedBit && m > 0;
}

cudaError_t scatter_sorted_launch(const IndexArgs& a, void* scratch, int sms, cudaStream_t st) {
  const SortScratch x = sort_scratch(a, scratch);
  const uint64_t m = x.m, rows = x.rows, mp = x.mp;
  const int reps = x.reps;
  uint32_t *hist = x.hist, *off = x.off, *bsum = x.bsum;
  const unsigned zgrid = unsigned(std::min<uint64_t>(uint64_t(sms) * 4, (mp * reps + kSortThreads - 1) / kSortThreads));
  zero_u32<<<zgrid, kSortThreads, 0, st>>>(hist, mp * reps);
  const unsigned tiles = unsigned(std::min<uint64_t>(uint64_t(sms) * 4, (rows + kTile - 1) / kTile));
  if (tiles) tile_histogram<<<tiles, kSortThreads, 0, st>>>(a, rows, hist, mp, reps, x.tag, x.list, x.list_len);
  // whole counter groups per scan block (sums are layout-independent)
  const uint64_t per_block = ((mp + kScanBlocks - 1) / kScanBlocks + kGroup - 1) / kGroup * kGroup;
  const int nblocks = int((mp + per_block - 1) / per_block);
  auto scan = [&](auto reps_c) {
    constexpr int R = decltype(reps_c)::value;
    scan_block_sums<R><<<nblocks, kScanThreads, 0, st>>>(hist, mp, per_block, bsum);
    scan_block_offsets<<<1, kScanThreads, 0, st>>>(bsum, nblocks, off + m);
    scan_write_offsets<R><<<nblocks, kScanThreads, 0, st>>>(hist, m, mp, per_block, bsum, off);
  };
  if (reps == 8)
    scan(std::integral_constant<int, 8>());
  else if (reps == 2)
    scan(std::integral_constant<int, 2>());
  else
    scan(std::integral_constant<int, 1>());
  const uint32_t vecs = uint32_t(a.inner * uint64_t(dtype_bytes(a.elem_type)) / 16);
  const bool copy = a.base != a.out;
  if (copy) {
    cudaError_t err = cudaFuncSetAttribute(copy_unowned_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kCopySmem));
    if (err != cudaSuccess) return err;
    copy_unowned_rows<<<unsigned(sms), kCopyWarps * 32, kCopySmem, st>>>(a, vecs, off, m);
  }
  // the scan turned hist into the placement cursors
  if (tiles) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(unsigned(std::min<uint64_t>(uint64_t(sms) * (copy ? 3 : 4), x.ntiles)));
    cfg.blockDim = dim3(kSortThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = copy ? 1 : 0;
    cudaError_t err = cudaLaunchKernelEx(&cfg, tile_place, rows, hist, mp, reps, static_cast<const uint32_t*>(x.tag),
                                         static_cast<const uint2*>(x.list), static_cast<const uint32_t*>(x.list_len),
                                         x.sorted);
    if (err != cudaSuccess) return err;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  auto run = [&](auto v_c, auto depth_c) {
    constexpr int V = decltype(v_c)::value, D = decltype(depth_c)::value;
    constexpr size_t smem = run_sums_smem<V, D>();
    cudaError_t err = cudaFuncSetAttribute(run_sums<V, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    int per_sm = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, run_sums<V, D>, kRunWarps * 32, smem);
    if (err != cudaSuccess) return err;
    const unsigned grid = unsigned(sms) * unsigned(std::max(per_sm, 1));
    run_sums<V, D><<<grid, kRunWarps * 32, smem, st>>>(a, vecs, off + m, x.sorted, a.elem_type == kF32 ? 1 : 0);
    return cudaGetLastError();
  };
  if (vecs <= 64) return run(std::integral_constant<int, 2>(), std::integral_constant<int, 16>());
  return run(std::integral_constant<int, 4>(), std::integral_constant<int, 8>());
}

}  // namespace askb
