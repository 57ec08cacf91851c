"""Turn the golden known-answer cases into (recipe, inputs, check) triples.

The same recipe runs through the CPU oracle (test_oracle_golden.py) and the
CUDA kernels (test_gpu_parity.py), so both are held to the documented answers.
"""
import json
import math
import os

import numpy as np

from ask_b200 import recipes as R

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "semantics_kat.json")
NP = {"bool": np.uint8, "i32": np.int32, "i64": np.int64, "f32": np.float32, "f16": np.uint16, "bf16": np.uint16}


def load_cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def fval(x) -> float:
    return float(x)


def f32_array(values):
    return np.array([fval(v) for v in values], np.float32)


def _bits(x: np.ndarray) -> int:
    return int(np.ascontiguousarray(x).view({1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[x.itemsize])[0])


def same_float(got: float, want) -> bool:
    w = fval(want)
    if math.isnan(w):
        return math.isnan(got)
    return got == w and math.copysign(1.0, got) == math.copysign(1.0, w)


def build(case):
    """Return (kind, recipe, inputs, check) where check(outputs) -> bool."""
    k = case["kind"]
    if k == "int_op":
        p = R.Program()
        a, b = p.input(case["dtype"]), p.input(case["dtype"])
        r = p.op(case["op"], a) if case["op"] == "abs" else p.op(case["op"], a, b)
        rec = R.elementwise(p, [r], 1)
        ins = [np.array([case["a"]], NP[case["dtype"]]), np.array([case["b"]], NP[case["dtype"]])]
        return "elementwise", rec, ins, lambda o: int(o[0][0]) == case["expect"]
    if k in ("cast", "cast_bits", "bf16_nan"):
        src = "f32" if k == "bf16_nan" else case["src"]
        dst = "bf16" if k == "bf16_nan" else case["dst"]
        p = R.Program()
        x = p.input(src)
        rec = R.elementwise(p, [p.cast(x, dst)], 1)
        if k == "bf16_nan":
            inp = np.array([case["f32_bits"]], np.uint32).view(np.float32)
        elif src in ("f32",):
            inp = np.array([fval(case["value"])], np.float32)
        elif src in ("f16", "bf16"):
            raise ValueError("no f16/bf16 sources in the fixture")
        else:
            inp = np.array([case["value"]], NP[src])
        if k == "cast":
            return "elementwise", rec, [inp], lambda o: int(o[0][0]) == case["expect"]
        return "elementwise", rec, [inp], lambda o: _bits(o[0]) == case["expect_bits"]
    if k in ("maximum", "minimum", "float_op"):
        p = R.Program()
        a, b = p.input("f32"), p.input("f32")
        op = case["op"] if k == "float_op" else k
        r = p.op(op, a) if op in ("round", "floor", "ceil", "abs") else p.op(op, a, b)
        rec = R.elementwise(p, [r], 1)
        ins = [f32_array([case["a"]]), f32_array([case["b"]])]
        return "elementwise", rec, ins, lambda o: same_float(float(o[0][0]), case["expect"])
    if k == "compare":
        p = R.Program()
        a, b = p.input("f32"), p.input("f32")
        rec = R.elementwise(p, [p.compare(case["pred"], a, b)], 1)
        return "elementwise", rec, [f32_array([case["a"]]), f32_array([case["b"]])], \
            lambda o: int(o[0][0]) == case["expect"]
    if k == "arg":
        p = R.Program()
        x = p.input("f32")
        vals = f32_array(case["values"])
        rec = R.reduce(p, x, [case["op"]], 1, len(vals))
        return "reduce", rec, [vals], lambda o: int(o[0][0]) == case["expect"]
    if k == "reduce":
        p = R.Program()
        x = p.input(case["dtype"])
        dt = case["dtype"]
        vals = f32_array(case["values"]) if dt == "f32" else np.array(case["values"], NP[dt])
        if vals.size == 0:
            vals = np.zeros(1, NP[dt])  # a valid pointer for an empty domain
            rec = R.reduce(p, x, [case["op"]], 1, 0)
        else:
            rec = R.reduce(p, x, [case["op"]], 1, len(case["values"]))
        if dt == "f32":
            return "reduce", rec, [vals], lambda o: same_float(float(o[0][0]), case["expect"])
        return "reduce", rec, [vals], lambda o: int(o[0][0]) == case["expect"]
    raise ValueError(k)
