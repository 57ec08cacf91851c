// Internal launch interface between the C-ABI plan layer (plan.cpp) and the
// kernel families.  Nothing here crosses the library boundary.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "ask_types.h"

namespace askb {

// ---- family E: fused elementwise -------------------------------------------
constexpr int kEwThreads = 256;

enum EwSpec : int {
  EW_GENERIC = 0,
  EW_CFG1,
  EW_CFG5B,
  EW_SOFTMAX_NORM_F16,
  EW_SOFTMAX_NORM_BF16,
  EW_NUM_SPECS
};

// Division by a run-time invariant divisor d with a multiply-high and shifts
// (Granlund & Montgomery, "Division by Invariant Integers using
// Multiplication", PLDI 1994, unsigned case): for dividends below 2^32,
//   t = mulhi32(m, n); q = (t + ((n - t) >> s1)) >> s2
// with l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1, s1 = min(l, 1),
// s2 = max(l - 1, 0).  `wide` falls back to 64-bit division.
struct U32Div {
  uint64_t d;
  uint32_t m, s1, s2, wide;
};

struct EwArgs {
  const void* in[kMaxIn];
  void* out[kMaxOut];
  uint64_t count;
  U32Div inner;  // IM_OUTER / IM_INNER divisor
};

inline U32Div make_u32div(uint64_t d, uint64_t max_dividend) {
  U32Div q{d ? d : 1, 0, 0, 0, 1};
  if (d == 0 || d > 0xffffffffull || max_dividend > 0xffffffffull) return q;
  uint32_t l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  const unsigned __int128 num = ((unsigned __int128)1 << 32) * ((unsigned __int128)((uint64_t(1) << l) - d));
  q.m = uint32_t(uint64_t(num / d) + 1);
  q.s1 = l < 1 ? l : 1;
  q.s2 = l > 1 ? l - 1 : 0;
  q.wide = 0;
  return q;
}

bool ew_spec_program(int spec, Program* out);
cudaError_t ew_occupancy(int spec, int* blocks_per_sm);
cudaError_t ew_launch(int spec, const Program& prog, const EwArgs& args, int aligned, int grid, cudaStream_t stream);

// ---- family R/T: map-reduce over [outer, extent, inner] ------------------------
constexpr int kRedThreads = 256;

enum RedSpec : int {
  RED_GENERIC = 0,
  RED_ROWSTATS_F32,      // cfg2: sum, max, min, argmax of f32 rows
  RED_GLOBAL_F32,        // cfg5a: sum, min, argmin of f32
  RED_SOFTMAX_MAX_F16,   // cfg3 step 0: max of cast(x, f32)
  RED_SOFTMAX_MAX_BF16,
  RED_SOFTMAX_SUM_F16,   // cfg3 step 1: sum of exp(cast(x) - m)
  RED_SOFTMAX_SUM_BF16,
  RED_NUM_SPECS
};

struct RedArgs {
  const void* in[kMaxIn];
  void* out[kMaxReductions];
  uint64_t outer, extent, inner;
  uint64_t index_base;   // added to arg-reduction indices (global offset of a shard)
  uint8_t n_red;
  uint8_t red_op[kMaxReductions];
  uint8_t red_src[kMaxReductions];   // which program output feeds each reduction
  uint8_t red_type[kMaxReductions];  // type of the reduced value (program output type)
};

// One partial accumulator as stored in scratch: value word + arg index.
struct RedPartial {
  uint64_t v;
  int64_t idx;
};

// Strategy chosen by the plan layer.
enum RedStrategy : int {
  RS_WARP_ROW = 0,   // inner == 1: one warp per output row, lanes stride the extent
  RS_COLUMN = 1,     // inner > 1: one thread per output column, loop over extent
  RS_SPLIT = 2,      // few outputs, huge extent: CTAs split the extent, partials in scratch
};

// Program and reduction list (all reductions fold program result 0) of a specialisation.
bool red_spec_program(int spec, Program* out, int* n_red, uint8_t* ops);
cudaError_t red_occupancy(int spec, int strategy, int* blocks_per_sm);
// RS_SPLIT writes grid * n_red partials to `scratch` and then combines them
// (second kernel) into the outputs, or, when `partials_out` is non-null, into
// one per-launch record per reduction (sharded plans combine those across ranks).
cudaError_t red_launch(int spec, int strategy, const Program& prog, const RedArgs& args, int aligned, int grid,
                       void* scratch, RedPartial* partials_out, cudaStream_t stream);
// Combine `n` records per reduction laid out [n][n_red] into the outputs.
cudaError_t red_combine_records(const RedArgs& args, const RedPartial* records, int n, cudaStream_t stream);
// Cross-GPU exchange of a sharded 0-D reduction's records over peer memory
// (one CTA): this rank's record `mine` (n_red records) is stored into slot
// `rank` of every rank's inbox (inboxes[r], device pointers valid on this
// device: the peers' inboxes are IPC mappings), each flag is raised with a
// release store, the rank waits (bounded by timeout_ns) for every rank's flag,
// and the records are folded in rank order into the outputs.  On a timeout the
// outputs are left as they were and the inbox's status word is set to 1.
constexpr int kExchangeMaxRanks = 64;
constexpr size_t kInboxRecordsBytes = size_t(2) * kExchangeMaxRanks * kMaxReductions * sizeof(RedPartial);
constexpr size_t kInboxFlagsOffset = kInboxRecordsBytes;                       // uint64 per rank
constexpr size_t kInboxSeqOffset = kInboxFlagsOffset + kExchangeMaxRanks * 8;  // uint64 epoch
constexpr size_t kInboxStatusOffset = kInboxSeqOffset + 8;                     // uint32, 0 = ok
constexpr size_t kInboxBytes = kInboxStatusOffset + 8;
cudaError_t red_exchange_combine(const RedArgs& args, const RedPartial* mine, void* const* inboxes, int nranks,
                                 int rank, uint64_t timeout_ns, cudaStream_t stream);
size_t red_split_scratch_bytes(int grid, int n_red);
// RS_COLUMN with few outputs: grid.y = chunks of the extent, one partial
// record per (output, chunk) in scratch, then a combine in chunk order.
cudaError_t red_column_chunks_launch(const Program& prog, const RedArgs& args, int grid, int chunks, void* scratch,
                                     cudaStream_t stream);
size_t red_column_chunks_scratch_bytes(uint64_t n_outputs, int chunks, int n_red);

// ---- family G / X: gather and scatter_add over [outer, D, inner] ------------------
struct IndexArgs {
  const void* table;     // gather: params; scatter: updates
  const void* index;
  void* out;
  const void* base;      // scatter: base tensor for the fused pre-copy (may equal out)
  uint64_t outer, dim, inner, n;  // params/base [outer, dim, inner]; index [n]
  int elem_type, index_type;
};
cudaError_t gather_launch(const IndexArgs& a, int aligned, int grid, cudaStream_t stream);
// `scratch` (scatter_sorted_scratch_bytes) enables the sorted path when
// scatter_sorted_ok holds; without it the element-atomic path runs.
cudaError_t scatter_add_launch(const IndexArgs& a, int aligned, int grid, void* scratch, int sms, cudaStream_t stream);
bool scatter_sorted_ok(const IndexArgs& a);
size_t scatter_sorted_scratch_bytes(const IndexArgs& a);
cudaError_t scatter_sorted_launch(const IndexArgs& a, void* scratch, int sms, cudaStream_t stream);

// ---- input synthesis (Philox4x32-10) -------------------------------------------------
enum GenKind : int { GEN_UNIFORM_F32 = 0, GEN_NORMAL_F32, GEN_NORMAL_F16, GEN_NORMAL_BF16, GEN_I32, GEN_ZIPF_I64, GEN_ZIPF_I32 };
// Elementwise steps with general index maps (IM_VIEW ports) or coordinate
// instructions: the runtime-program interpreter with per-element coordinates.
struct ViewSet {
  int rank;
  uint64_t shape[kMaxRank];
  PortView port[kMaxIn];
};
cudaError_t ew_view_launch(const Program& prog, const EwArgs& args, const ViewSet& views, int grid,
                           cudaStream_t stream);
int ew_view_occupancy();
// Reductions whose prologue reads IM_VIEW ports or coordinates: a warp per
// output over the [outer, extent, inner] domain of the iteration shape.
cudaError_t red_view_launch(const Program& prog, const RedArgs& a, const ViewSet& views, int grid,
                            cudaStream_t stream);
int red_view_occupancy();

// Family S: the three-step softmax plan fused (softmax_kernels.cu).  x and y
// are [rows, cols] f16/bf16 (16-byte aligned), m and s are [rows] f32.  The
// same row kernel also runs each step of the plan on its own (a reduce plan
// matched to ProgSoftmaxMax / ProgSoftmaxSum, an elementwise plan matched to
// ProgSoftmaxNorm): SM_STEP_MAX writes m only, SM_STEP_SUM reads m (m_in) and
// writes s only, SM_STEP_NORM reads m and s (m_in, s_in) and writes y only.
enum SoftmaxMode { SM_FUSED = 0, SM_STEP_MAX = 1, SM_STEP_SUM = 2, SM_STEP_NORM = 3 };
struct SoftmaxArgs {
  const void* x;
  float* m;
  float* s;
  void* y;
  const float* m_in;  // SM_STEP_SUM, SM_STEP_NORM
  const float* s_in;  // SM_STEP_NORM
  uint64_t rows, cols;
  int type;  // kF16 or kBF16
  int mode;  // SoftmaxMode
};
// 16-byte vectors each thread of a row's CTA holds, or 0 when cols has no
// fused kernel (cols must be a multiple of 256, at most 32768).
int softmax_vectors_per_thread(uint64_t cols);
cudaError_t softmax_rows_launch(const SoftmaxArgs& a, int sms, cudaStream_t stream);
// The grid softmax_rows_launch uses for `a` (SMs x resident CTAs, at most
// one CTA per row); needs the device current.
int softmax_rows_grid(const SoftmaxArgs& a, int sms);

cudaError_t gen_launch(int kind, uint64_t seed, uint32_t stream_id, uint64_t offset, uint64_t count, double p0,
                       double p1, const double* zipf_cdf, uint64_t zipf_n, void* dst, cudaStream_t stream);

}  // namespace askb
