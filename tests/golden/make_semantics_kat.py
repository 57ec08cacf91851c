"""Write tests/golden/semantics_kat.json: known answers for ASK's element semantics.

The reference ships no numeric golden vectors for this path, and its compiler
(which needs an LLVM/MLIR 23.1 SDK) cannot run here, so these answers are
derived by hand from the semantics the reference states in prose and code.
Every case carries the citation it is derived from (paths inside the
reference project).  Run from the repository root:

    python tests/golden/make_semantics_kat.py
"""
import json
import math
import os

I32_MIN, I32_MAX = -(2 ** 31), 2 ** 31 - 1
I64_MIN, I64_MAX = -(2 ** 63), 2 ** 63 - 1
NAN, INF = "nan", "inf"

IR77 = "docs/en/ir.md:77"
IR69 = "docs/en/ir.md:69"
IR117 = "docs/en/ir.md:117-121"
SE = "lib/Lowering/ScalarEmitter.h"


def int_case(op, dtype, a, b, expect, src):
    return {"kind": "int_op", "op": op, "dtype": dtype, "a": a, "b": b, "expect": expect, "source": src}


CASES = [
    # integer divide/mod by zero returns 0; INT_MIN // -1 wraps; INT_MIN % -1 is 0
    int_case("floordiv", "i32", 7, 0, 0, IR77),
    int_case("mod", "i32", 7, 0, 0, IR77),
    int_case("floordiv", "i32", I32_MIN, -1, I32_MIN, IR77),
    int_case("mod", "i32", I32_MIN, -1, 0, IR77),
    int_case("floordiv", "i64", I64_MIN, -1, I64_MIN, IR77),
    int_case("mod", "i64", I64_MIN, -1, 0, IR77),
    # floored division and remainder take the divisor's sign (ScalarEmitter.h:130-138)
    int_case("floordiv", "i32", -7, 2, -4, SE + ":130-135"),
    int_case("mod", "i32", -7, 2, 1, SE + ":137-138"),
    int_case("floordiv", "i32", 7, -2, -4, SE + ":130-135"),
    int_case("mod", "i32", 7, -2, -1, SE + ":137-138"),
    int_case("floordiv", "i64", -6, 3, -2, SE + ":130-135"),
    # shifts: negative counts give 0; left shifts >= width give 0; right shifts
    # >= width sign-fill (-1 for negative values, else 0)
    int_case("shift_left", "i32", 5, -1, 0, IR77),
    int_case("shift_left", "i32", 5, 32, 0, IR77),
    int_case("shift_left", "i64", 5, 64, 0, IR77),
    int_case("shift_right", "i32", -8, -3, 0, IR77),
    int_case("shift_right", "i32", -8, 40, -1, IR77),
    int_case("shift_right", "i32", 8, 32, 0, IR77),
    int_case("shift_right", "i64", -1024, 70, -1, IR77),
    int_case("shift_right", "i32", -8, 1, -4, SE + ":113"),
    int_case("shift_left", "i32", 1, 31, I32_MIN, SE + ":108"),
    # add/mul wrap modulo 2^32 / 2^64 (docs/en/ir.md:21, ScalarEmitter.h:140-141)
    int_case("add", "i32", I32_MAX, 1, I32_MIN, "docs/en/ir.md:21"),
    int_case("mul", "i32", 65536, 65536, 0, "docs/en/ir.md:21"),
    int_case("add", "i64", I64_MAX, 1, I64_MIN, "docs/en/ir.md:21"),
    # integer pow: negative exponents give 1 for base 1, +-1 for base -1, else 0
    int_case("pow", "i32", 3, 4, 81, SE + ":57-93"),
    int_case("pow", "i32", 2, -1, 0, SE + ":62-67"),
    int_case("pow", "i32", 1, -5, 1, SE + ":62-67"),
    int_case("pow", "i32", -1, -3, -1, SE + ":62-67"),
    int_case("pow", "i32", -1, -4, 1, SE + ":62-67"),
    int_case("pow", "i32", 2, 31, I32_MIN, SE + ":82-86"),
    int_case("abs", "i32", I32_MIN, 0, I32_MIN, SE + ":225-229"),
    # float <-> int casts: fptosi.sat truncates toward zero, NaN -> 0, clamps
    {"kind": "cast", "src": "f32", "dst": "i32", "value": NAN, "expect": 0, "source": IR117},
    {"kind": "cast", "src": "f32", "dst": "i32", "value": INF, "expect": I32_MAX, "source": IR117},
    {"kind": "cast", "src": "f32", "dst": "i32", "value": "-inf", "expect": I32_MIN, "source": IR117},
    {"kind": "cast", "src": "f32", "dst": "i32", "value": -2.75, "expect": -2, "source": IR117},
    {"kind": "cast", "src": "f32", "dst": "i64", "value": 1e30, "expect": I64_MAX, "source": IR117},
    # any -> bool: NaN and inf are true, +-0 false
    {"kind": "cast", "src": "f32", "dst": "bool", "value": NAN, "expect": 1, "source": IR117},
    {"kind": "cast", "src": "f32", "dst": "bool", "value": "-0.0", "expect": 0, "source": IR117},
    {"kind": "cast", "src": "f32", "dst": "bool", "value": INF, "expect": 1, "source": IR117},
    {"kind": "cast", "src": "i32", "dst": "bool", "value": -3, "expect": 1, "source": IR117},
    # integer -> bf16 rounds once from the exact integer: 2^40 + 2^32 + 1 gives
    # 2^40 + 2^33 (bits 0x5381); going through f32 first would give 2^40
    # (include/ask/LLIR/Numeric.h:36-37)
    {"kind": "cast_bits", "src": "i64", "dst": "bf16", "value": 2 ** 40 + 2 ** 32 + 1, "expect_bits": 0x5381,
     "source": "include/ask/LLIR/Numeric.h:36-37"},
    {"kind": "cast_bits", "src": "i64", "dst": "f16", "value": 2049, "expect_bits": 0x6800,
     "source": "include/ask/LLIR/Numeric.h:38-76 (ties to even)"},
    {"kind": "cast_bits", "src": "i64", "dst": "f16", "value": 2051, "expect_bits": 0x6802,
     "source": "include/ask/LLIR/Numeric.h:38-76 (ties to even)"},
    {"kind": "cast_bits", "src": "i64", "dst": "f16", "value": 70000, "expect_bits": 0x7C00,
     "source": "include/ask/LLIR/Numeric.h:71-72 (overflow to inf)"},
    # f32 -> bf16: round to nearest even; NaN keeps sign/top bits, quiet bit set
    {"kind": "cast_bits", "src": "f32", "dst": "bf16", "value": 1.00390625, "expect_bits": 0x3F80,
     "source": "include/ask/LLIR/Numeric.h:25-29 (tie, even)"},
    {"kind": "cast_bits", "src": "f32", "dst": "bf16", "value": 1.01171875, "expect_bits": 0x3F82,
     "source": "include/ask/LLIR/Numeric.h:25-29 (tie, odd rounds up)"},
    {"kind": "cast_bits", "src": "f32", "dst": "bf16", "value": "-0.0", "expect_bits": 0x8000,
     "source": "docs/en/ir.md:117 (-0.0 preserved)"},
    {"kind": "bf16_nan", "f32_bits": 0x7F800001, "expect_bits": 0x7FC0,
     "source": "include/ask/LLIR/Numeric.h:30-32"},
    {"kind": "bf16_nan", "f32_bits": 0xFFA00000, "expect_bits": 0xFFE0,
     "source": "include/ask/LLIR/Numeric.h:30-32"},
    {"kind": "cast_bits", "src": "f32", "dst": "f16", "value": 65520.0, "expect_bits": 0x7C00,
     "source": "docs/en/ir.md:117 (overflow to inf)"},
    {"kind": "cast_bits", "src": "f32", "dst": "f16", "value": 65519.0, "expect_bits": 0x7BFF,
     "source": "docs/en/ir.md:117 (RNE below the overflow threshold)"},
    {"kind": "cast_bits", "src": "bool", "dst": "f32", "value": 1, "expect_bits": 0x3F800000,
     "source": "docs/en/ir.md:121"},
    # maximum/minimum propagate NaN and order -0 below +0
    {"kind": "maximum", "a": "-0.0", "b": "0.0", "expect": "0.0", "source": IR69},
    {"kind": "maximum", "a": "0.0", "b": "-0.0", "expect": "0.0", "source": IR69},
    {"kind": "minimum", "a": "0.0", "b": "-0.0", "expect": "-0.0", "source": IR69},
    {"kind": "maximum", "a": NAN, "b": "1.0", "expect": NAN, "source": IR69},
    {"kind": "minimum", "a": "3.0", "b": NAN, "expect": NAN, "source": IR69},
    {"kind": "maximum", "a": "-inf", "b": "-3.5", "expect": "-3.5", "source": IR69},
    # compare: NaN satisfies only ne
    {"kind": "compare", "pred": "eq", "a": NAN, "b": NAN, "expect": 0, "source": IR77},
    {"kind": "compare", "pred": "ne", "a": NAN, "b": NAN, "expect": 1, "source": IR77},
    {"kind": "compare", "pred": "lt", "a": NAN, "b": "1.0", "expect": 0, "source": IR77},
    {"kind": "compare", "pred": "ge", "a": "1.0", "b": NAN, "expect": 0, "source": IR77},
    {"kind": "compare", "pred": "eq", "a": "-0.0", "b": "0.0", "expect": 1, "source": IR77},
    # argmax/argmin: first occurrence; the first NaN wins; -0 and +0 tie
    {"kind": "arg", "op": "argmax", "values": ["1.0", "3.0", "3.0", "2.0"], "expect": 1, "source": IR69},
    {"kind": "arg", "op": "argmin", "values": ["1.0", "0.5", "0.5"], "expect": 1, "source": IR69},
    {"kind": "arg", "op": "argmax", "values": ["1.0", NAN, "5.0", NAN], "expect": 1, "source": IR69},
    {"kind": "arg", "op": "argmin", "values": [NAN, "-5.0"], "expect": 0, "source": SE + ":506-512"},
    {"kind": "arg", "op": "argmax", "values": ["-0.0", "0.0"], "expect": 0, "source": SE + ":511"},
    # reductions: empty-domain / initial values and NaN propagation
    {"kind": "reduce", "op": "sum", "dtype": "f32", "values": [], "expect": "0.0", "source": IR69},
    {"kind": "reduce", "op": "prod", "dtype": "f32", "values": [], "expect": "1.0", "source": IR69},
    {"kind": "reduce", "op": "max", "dtype": "f32", "values": ["1.0", NAN, "2.0"], "expect": NAN, "source": IR69},
    {"kind": "reduce", "op": "min", "dtype": "f32", "values": ["0.0", "-0.0"], "expect": "-0.0", "source": IR69},
    {"kind": "reduce", "op": "max", "dtype": "i32", "values": [-5, -7], "expect": -5, "source": IR69},
    {"kind": "reduce", "op": "sum", "dtype": "i32", "values": [I32_MAX, 1], "expect": I32_MIN, "source": IR69},
    {"kind": "reduce", "op": "any", "dtype": "bool", "values": [], "expect": 0, "source": IR69},
    {"kind": "reduce", "op": "all", "dtype": "bool", "values": [], "expect": 1, "source": IR69},
    {"kind": "reduce", "op": "any", "dtype": "bool", "values": [0, 1, 0], "expect": 1, "source": IR69},
    {"kind": "reduce", "op": "all", "dtype": "bool", "values": [1, 0, 1], "expect": 0, "source": IR69},
    # float floordiv / mod are floored (docs/en/ir.md:77; ScalarEmitter.h:150-158)
    {"kind": "float_op", "op": "floordiv", "a": "-7.0", "b": "2.0", "expect": "-4.0", "source": IR77},
    {"kind": "float_op", "op": "mod", "a": "-7.0", "b": "2.0", "expect": "1.0", "source": IR77},
    {"kind": "float_op", "op": "mod", "a": "7.0", "b": "-2.0", "expect": "-1.0", "source": IR77},
    {"kind": "float_op", "op": "round", "a": "2.5", "b": "0.0", "expect": "2.0", "source": "docs/en/ir.md:77 (ties to even)"},
    {"kind": "float_op", "op": "round", "a": "-3.5", "b": "0.0", "expect": "-4.0", "source": "docs/en/ir.md:77 (ties to even)"},
]


def main():
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "semantics_kat.json")
    with open(out, "w") as f:
        json.dump({"description": __doc__.strip().splitlines()[0], "cases": CASES}, f, indent=1)
        f.write("\n")
    print(out, len(CASES), "cases")


if __name__ == "__main__":
    main()
