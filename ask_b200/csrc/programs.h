// Compile-time op programs for the plans the kernels are specialised for.
//
// A plan whose parsed program is identical (instruction by instruction, ports
// and index maps included) to one of these runs the specialised instantiation
// of the same interpreter template, where every register index and opcode is a
// compile-time constant; any other program runs the runtime-interpreted
// instantiation.  Each program is the SSA form of an owned ASK step:
//
//   Cfg1      y0 = exp(a)*b + c ; y1 = max(a,b) + tanh(c)*(-1)   (f32)
//             ASK has no subtract op (include/ask/IR/ASKOps.h:70-145), so
//             "max(a,b) - tanh(c)" is add(maximum, mul(tanh, splat(-1))).
//   Cfg5b     ((x << 3) ^ (x >> 5)) & 0x7fffffff + y                 (i32)
//   SoftmaxMax<T>   step 0 of the canonical softmax partition: value cast(x, f32)
//   SoftmaxSum<T>   step 1: exp(cast(x) + m*(-1)), m indexed by the row
//   SoftmaxNorm<T>  step 2: cast(exp(cast(x) + m*(-1)) / s, T)
//   Identity<T>     value = input 0 (plain reductions such as cfg2)
// The softmax step structure follows lib/Frontend/Partition.cpp:126-132: a
// reduction result that is broadcast again is materialised, so the row max and
// the row sum each end an owned step and step 2 recomputes exp.
#pragma once

#include "ask_types.h"

namespace askb {

ASKB_HD constexpr Insn mk(uint8_t op, uint8_t type, uint8_t dst, uint8_t a = 0, uint8_t b = 0,
                          uint8_t c = 0, uint8_t aux = 0, uint8_t st = 0, uint64_t imm = 0) {
  return Insn{op, type, dst, a, b, c, aux, st, imm};
}
// f32 constant words are the IEEE bit pattern in the low 32 bits.
constexpr uint64_t kF32MinusOne = 0xbf800000ull;

struct ProgCfg1 {
  static constexpr int kInsn = 11, kIn = 3, kOut = 2;
  ASKB_HD static constexpr Insn insn(int i) {
    constexpr Insn p[kInsn] = {
        mk(OP_INPUT, kF32, 0, 0), mk(OP_INPUT, kF32, 1, 1), mk(OP_INPUT, kF32, 2, 2),
        mk(OP_EXP, kF32, 3, 0, 0, 0, 0, kF32), mk(OP_MUL, kF32, 4, 3, 1, 0, 0, kF32),
        mk(OP_ADD, kF32, 5, 4, 2, 0, 0, kF32), mk(OP_MAXIMUM, kF32, 6, 0, 1, 0, 0, kF32),
        mk(OP_TANH, kF32, 7, 2, 0, 0, 0, kF32), mk(OP_CONST, kF32, 8, 0, 0, 0, 0, kF32, kF32MinusOne),
        mk(OP_MUL, kF32, 9, 7, 8, 0, 0, kF32), mk(OP_ADD, kF32, 10, 6, 9, 0, 0, kF32)};
    return p[i];
  }
  ASKB_HD static constexpr int in_type(int) { return kF32; }
  ASKB_HD static constexpr int in_map(int) { return IM_FULL; }
  ASKB_HD static constexpr int out_type(int) { return kF32; }
  ASKB_HD static constexpr int out_reg(int k) { return k == 0 ? 5 : 10; }
};

struct ProgCfg5b {
  static constexpr int kInsn = 10, kIn = 2, kOut = 1;
  ASKB_HD static constexpr Insn insn(int i) {
    constexpr Insn p[kInsn] = {
        mk(OP_INPUT, kI32, 0, 0), mk(OP_INPUT, kI32, 1, 1),
        mk(OP_CONST, kI32, 2, 0, 0, 0, 0, kI32, 3), mk(OP_SHL, kI32, 3, 0, 2, 0, 0, kI32),
        mk(OP_CONST, kI32, 4, 0, 0, 0, 0, kI32, 5), mk(OP_SHR, kI32, 5, 0, 4, 0, 0, kI32),
        mk(OP_XOR, kI32, 6, 3, 5, 0, 0, kI32), mk(OP_CONST, kI32, 7, 0, 0, 0, 0, kI32, 0x7fffffffull),
        mk(OP_AND, kI32, 8, 6, 7, 0, 0, kI32), mk(OP_ADD, kI32, 9, 8, 1, 0, 0, kI32)};
    return p[i];
  }
  ASKB_HD static constexpr int in_type(int) { return kI32; }
  ASKB_HD static constexpr int in_map(int) { return IM_FULL; }
  ASKB_HD static constexpr int out_type(int) { return kI32; }
  ASKB_HD static constexpr int out_reg(int) { return 9; }
};

template <int T>
struct ProgIdentity {
  static constexpr int kInsn = 1, kIn = 1, kOut = 1;
  ASKB_HD static constexpr Insn insn(int) { return mk(OP_INPUT, uint8_t(T), 0, 0); }
  ASKB_HD static constexpr int in_type(int) { return T; }
  ASKB_HD static constexpr int in_map(int) { return IM_FULL; }
  ASKB_HD static constexpr int out_type(int) { return T; }
  ASKB_HD static constexpr int out_reg(int) { return 0; }
};

template <int T>
struct ProgSoftmaxMax {
  static constexpr int kInsn = 2, kIn = 1, kOut = 1;
  ASKB_HD static constexpr Insn insn(int i) {
    constexpr Insn p[kInsn] = {mk(OP_INPUT, uint8_t(T), 0, 0), mk(OP_CAST, kF32, 1, 0, 0, 0, 0, uint8_t(T))};
    return p[i];
  }
  ASKB_HD static constexpr int in_type(int) { return T; }
  ASKB_HD static constexpr int in_map(int) { return IM_FULL; }
  ASKB_HD static constexpr int out_type(int) { return kF32; }
  ASKB_HD static constexpr int out_reg(int) { return 1; }
};

template <int T>
struct ProgSoftmaxSum {
  static constexpr int kInsn = 7, kIn = 2, kOut = 1;
  ASKB_HD static constexpr Insn insn(int i) {
    constexpr Insn p[kInsn] = {
        mk(OP_INPUT, uint8_t(T), 0, 0), mk(OP_INPUT, kF32, 1, 1),
        mk(OP_CAST, kF32, 2, 0, 0, 0, 0, uint8_t(T)),
        mk(OP_CONST, kF32, 3, 0, 0, 0, 0, kF32, kF32MinusOne),
        mk(OP_MUL, kF32, 4, 1, 3, 0, 0, kF32), mk(OP_ADD, kF32, 5, 2, 4, 0, 0, kF32),
        mk(OP_EXP, kF32, 6, 5, 0, 0, 0, kF32)};
    return p[i];
  }
  ASKB_HD static constexpr int in_type(int k) { return k == 0 ? T : kF32; }
  ASKB_HD static constexpr int in_map(int k) { return k == 0 ? IM_FULL : IM_OUTER; }
  ASKB_HD static constexpr int out_type(int) { return kF32; }
  ASKB_HD static constexpr int out_reg(int) { return 6; }
};

template <int T>
struct ProgSoftmaxNorm {
  static constexpr int kInsn = 10, kIn = 3, kOut = 1;
  ASKB_HD static constexpr Insn insn(int i) {
    constexpr Insn p[kInsn] = {
        mk(OP_INPUT, uint8_t(T), 0, 0), mk(OP_INPUT, kF32, 1, 1), mk(OP_INPUT, kF32, 2, 2),
        mk(OP_CAST, kF32, 3, 0, 0, 0, 0, uint8_t(T)),
        mk(OP_CONST, kF32, 4, 0, 0, 0, 0, kF32, kF32MinusOne),
        mk(OP_MUL, kF32, 5, 1, 4, 0, 0, kF32), mk(OP_ADD, kF32, 6, 3, 5, 0, 0, kF32),
        mk(OP_EXP, kF32, 7, 6, 0, 0, 0, kF32), mk(OP_DIV, kF32, 8, 7, 2, 0, 0, kF32),
        mk(OP_CAST, uint8_t(T), 9, 8, 0, 0, 0, kF32)};
    return p[i];
  }
  ASKB_HD static constexpr int in_type(int k) { return k == 0 ? T : kF32; }
  ASKB_HD static constexpr int in_map(int k) { return k == 0 ? IM_FULL : IM_OUTER; }
  ASKB_HD static constexpr int out_type(int) { return T; }
  ASKB_HD static constexpr int out_reg(int) { return 9; }
};

// Materialise a specialised program as a runtime Program (host side, for
// matching parsed plans against the specialisations).
template <class P>
inline Program program_of() {
  Program p{};
  p.n_insn = P::kInsn;
  p.n_in = P::kIn;
  p.n_out = P::kOut;
  p.n_regs = P::kInsn;
  for (int k = 0; k < P::kIn; ++k) { p.in_type[k] = uint8_t(P::in_type(k)); p.in_map[k] = uint8_t(P::in_map(k)); }
  for (int k = 0; k < P::kOut; ++k) { p.out_type[k] = uint8_t(P::out_type(k)); p.out_reg[k] = uint8_t(P::out_reg(k)); }
  for (int i = 0; i < P::kInsn; ++i) p.insn[i] = P::insn(i);
  return p;
}

}  // namespace askb
