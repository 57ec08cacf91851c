// Shared host/device definitions for the ask_b200 kernel library.
//
// Element types, the op-program encoding used by the fused elementwise (E) and
// map-reduce (R/T) kernel families, and the plan-level limits.  The encoding is
// this library's own; the op set and its semantics follow ASK's ScalarEmitter
// (lib/Lowering/ScalarEmitter.h:94-262 binary/unary/maximum/minimum/compare) and
// the element-type table of docs/en/ir.md:97-106.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define ASKB_HD __host__ __device__
#else
#define ASKB_HD
#endif

namespace askb {

// ASK's six element types (include/ask/IR/ASKOps.h:181-186, docs/en/ir.md:97-106).
// bool occupies one byte in buffers (lib/Lowering/CUDA.cpp:40-43).
enum DType : uint8_t { kBool = 0, kI32 = 1, kI64 = 2, kF32 = 3, kF16 = 4, kBF16 = 5, kNumDTypes = 6 };

ASKB_HD constexpr int dtype_bytes(int t) {
  return t == kBool ? 1 : t == kI32 ? 4 : t == kI64 ? 8 : t == kF32 ? 4 : 2;
}
ASKB_HD constexpr bool dtype_is_float(int t) { return t == kF32 || t == kF16 || t == kBF16; }
ASKB_HD constexpr bool dtype_is_int(int t) { return t == kI32 || t == kI64; }

// Program opcodes.  Each instruction produces one SSA value of type `type`.
enum Op : uint8_t {
  OP_INPUT = 0,   // a = input port index
  OP_CONST,       // imm holds the value bits (see Insn)
  OP_CAST,        // a; src_type -> type  (include/ask/LLIR/Numeric.h:78-111)
  OP_ADD, OP_MUL, OP_DIV, OP_FLOORDIV, OP_MOD, OP_POW,
  OP_MAXIMUM, OP_MINIMUM,
  OP_AND, OP_OR, OP_XOR, OP_SHL, OP_SHR,
  OP_NOT, OP_ABS, OP_EXP, OP_LOG, OP_SQRT, OP_SIN, OP_COS, OP_TANH, OP_ERF,
  OP_FLOOR, OP_CEIL, OP_ROUND,
  OP_CMP,         // aux = predicate, result bool; src_type = operand type
  OP_SELECT,      // a = bool condition, b = yes, c = no
  OP_COORD,       // i64 coordinate of the element along axis aux of the iteration shape
  kNumOps
};

enum CmpPred : uint8_t { CMP_EQ = 0, CMP_NE, CMP_LT, CMP_LE, CMP_GT, CMP_GE };

// One program instruction (16 bytes).  Register values are 64-bit words:
//   bool -> 0/1; i32 -> low 32 bits; i64 -> all bits;
//   f32/f16/bf16 -> f32 bit pattern in the low 32 bits.  f16/bf16 values are
//   held as the f32 value they represent (always exactly representable), so
//   every low-precision op is "widen, compute in f32, round back" exactly as
//   ScalarEmitter does (ScalarEmitter.h:161-179, 185-189, 234, 261).
struct Insn {
  uint8_t op, type, dst, a, b, c, aux, src_type;
  uint64_t imm;
};

// How a port is indexed relative to the step's linear element index.
enum IndexMap : uint8_t {
  IM_FULL = 0,    // same shape as the step: element i
  IM_SCALAR = 1,  // 0-D buffer: element 0
  IM_OUTER = 2,   // elementwise: i / inner      reduce: indexed by the output (o*inner + n)
  IM_INNER = 3,   // elementwise: i % inner
  IM_VIEW = 4,    // elementwise: a strided, windowed view of the port (PortView)
};

// A general index map for one port of an elementwise step over an iteration
// shape of `rank` axes (the reference's broadcast_in_dim, transpose, slice,
// pad and concatenate operand maps, ScalarEmitter.h:626-730).  For output
// coordinate c_d the port coordinate is i_d = (c_d - lo[d]) / step[d]; the
// element is valid when every c_d - lo[d] >= 0 is a multiple of step[d] and
// i_d < extent[d], and is then read at offset + sum(i_d * stride[d]);
// otherwise the port yields `pad` (a value word of the port's type).
//
// A reshape that no strided window expresses (of a transposed, sliced or
// padded value: the reference reads a reshape at the same row-major position,
// ScalarEmitter.h:622) adds a second stage: when inner_rank > 0 the window
// above yields a row-major position in a value of shape inner_shape (the
// reshape's operand), which is split into coordinates there and read through
// the inner window (ilo, istep, iextent, istride, ioffset; pad ipad).
constexpr int kMaxRank = 6;
struct PortView {
  int64_t lo[kMaxRank];
  int64_t step[kMaxRank];
  int64_t extent[kMaxRank];
  int64_t stride[kMaxRank];
  int64_t offset;
  uint64_t pad;
  int64_t inner_rank;
  int64_t inner_shape[kMaxRank];
  int64_t ilo[kMaxRank];
  int64_t istep[kMaxRank];
  int64_t iextent[kMaxRank];
  int64_t istride[kMaxRank];
  int64_t ioffset;
  uint64_t ipad;
};

constexpr int kMaxInsn = 48;
constexpr int kMaxIn = 16;
constexpr int kMaxOut = 16;
constexpr int kMaxRegs = 48;
constexpr int kMaxReductions = 8;

// A complete fused program (kernel parameter, ~840 bytes).
struct Program {
  uint8_t n_insn, n_in, n_out, n_regs;
  uint8_t in_type[kMaxIn];
  uint8_t in_map[kMaxIn];
  uint8_t out_type[kMaxOut];
  uint8_t out_reg[kMaxOut];
  Insn insn[kMaxInsn];
};

// Reduction kinds (ScalarEmitter.h:420-529).
enum RedOp : uint8_t { RED_SUM = 0, RED_PROD, RED_MAX, RED_MIN, RED_ANY, RED_ALL, RED_ARGMAX, RED_ARGMIN, kNumRedOps };

ASKB_HD constexpr bool red_is_arg(int r) { return r == RED_ARGMAX || r == RED_ARGMIN; }

}  // namespace askb
