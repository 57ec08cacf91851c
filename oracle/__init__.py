"""TEST INFRASTRUCTURE ONLY: ctypes/numpy wrapper of the CPU oracle.

The oracle (oracle/ask_oracle.cpp) restates ASK's host-path semantics for the
hot path and is the parity checker for the CUDA kernels and the timed CPU
baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference legs may import it.  Parity status: partially pinned (see the header
of ask_oracle.cpp and tests/golden/).
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np

from . import build as _build

_lib = None

_DTYPES = {"bool": np.uint8, "i32": np.int32, "i64": np.int64, "f32": np.float32, "f16": np.uint16,
           "bf16": np.uint16}
_MAPS = {"full": 0, "scalar": 1, "outer": 2, "inner": 3}
_PRED = {"eq": 0, "ne": 1, "lt": 2, "le": 3, "gt": 4, "ge": 5}


class _Insn(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int32), ("type", ctypes.c_int32), ("a", ctypes.c_int32), ("b", ctypes.c_int32),
                ("c", ctypes.c_int32), ("aux", ctypes.c_int32), ("src_type", ctypes.c_int32),
                ("pad", ctypes.c_int32), ("imm", ctypes.c_uint64)]


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        vp, u64, i32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int
        L.orc_dtype_code.restype = i32
        L.orc_dtype_code.argtypes = [ctypes.c_char_p]
        L.orc_op_code.restype = i32
        L.orc_op_code.argtypes = [ctypes.c_char_p]
        L.orc_red_code.restype = i32
        L.orc_red_code.argtypes = [ctypes.c_char_p]
        L.orc_f32_to_bf16.restype = ctypes.c_uint32
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_bf16_to_f32.restype = ctypes.c_float
        L.orc_bf16_to_f32.argtypes = [ctypes.c_uint32]
        L.orc_f32_to_f16.restype = ctypes.c_uint32
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint32]
        L.orc_maximum.restype = ctypes.c_float
        L.orc_maximum.argtypes = [ctypes.c_float, ctypes.c_float]
        L.orc_minimum.restype = ctypes.c_float
        L.orc_minimum.argtypes = [ctypes.c_float, ctypes.c_float]
        L.orc_int_op.restype = ctypes.c_int64
        L.orc_int_op.argtypes = [i32, i32, ctypes.c_int64, ctypes.c_int64]
        L.orc_cast_bits.restype = u64
        L.orc_cast_bits.argtypes = [i32, i32, ctypes.c_int64, ctypes.c_float]
        L.orc_philox.restype = None
        L.orc_philox.argtypes = [u64, ctypes.c_uint32, u64, ctypes.POINTER(ctypes.c_uint32)]
        L.orc_generate.restype = None
        L.orc_generate.argtypes = [i32, u64, ctypes.c_uint32, u64, u64, ctypes.c_double, ctypes.c_double, vp, i32]
        L.orc_elementwise.restype = i32
        L.orc_elementwise.argtypes = [vp, i32, vp, vp, i32, vp, vp, vp, i32, vp, u64, u64, i32]
        L.orc_reduce.restype = i32
        L.orc_reduce.argtypes = [vp, i32, vp, vp, i32, vp, vp, i32, vp, vp, vp, u64, u64, u64, u64, i32, i32]
        L.orc_gather.restype = i32
        L.orc_gather.argtypes = [vp, vp, i32, vp, u64, u64, u64, u64, i32, i32]
        L.orc_scatter_add.restype = i32
        L.orc_scatter_add.argtypes = [i32, vp, vp, i32, vp, vp, vp, vp, u64, u64, u64, u64, i32]
        L.orc_cfg1.restype = None
        L.orc_cfg1.argtypes = [vp, vp, vp, vp, vp, u64, i32]
        L.orc_cfg5b.restype = None
        L.orc_cfg5b.argtypes = [vp, vp, vp, u64, i32]
        L.orc_cfg5a.restype = None
        L.orc_cfg5a.argtypes = [vp, u64, u64, vp, vp, vp, vp, i32]
        L.orc_softmax.restype = None
        L.orc_softmax.argtypes = [i32, vp, u64, u64, vp, vp, vp, i32]
        L.orc_rowstats.restype = None
        L.orc_rowstats.argtypes = [vp, u64, u64, vp, vp, vp, vp, i32]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _ptrs(arrays):
    arr = (ctypes.c_void_p * max(1, len(arrays)))(*[a.ctypes.data for a in arrays])
    return arr


# ---- scalars -----------------------------------------------------------------------
def dtype_code(name: str) -> int:
    return lib().orc_dtype_code(name.encode())


def f32_to_bf16(x: float) -> int:
    return lib().orc_f32_to_bf16(x)


def bf16_to_f32(h: int) -> float:
    return lib().orc_bf16_to_f32(h)


def f32_to_f16(x: float) -> int:
    return lib().orc_f32_to_f16(x)


def maximum(a: float, b: float) -> float:
    return lib().orc_maximum(a, b)


def minimum(a: float, b: float) -> float:
    return lib().orc_minimum(a, b)


def int_op(op: str, dtype: str, a: int, b: int = 0) -> int:
    return lib().orc_int_op(lib().orc_op_code(op.encode()), dtype_code(dtype), a, b)


def cast_bits(src: str, dst: str, ival: int = 0, fval: float = 0.0) -> int:
    return lib().orc_cast_bits(dtype_code(src), dtype_code(dst), ival, fval)


def philox(seed: int, stream: int, index: int) -> list:
    out = (ctypes.c_uint32 * 4)()
    lib().orc_philox(seed, stream, index, out)
    return list(out)


def generate(kind: int, seed: int, stream: int, offset: int, count: int, p0: float, p1: float,
             threads: int = 1) -> np.ndarray:
    dt = {0: np.float32, 1: np.float32, 2: np.uint16, 3: np.uint16, 4: np.int32, 5: np.int64, 6: np.int32}[kind]
    out = np.empty(count, dtype=dt)
    lib().orc_generate(kind, seed, stream, offset, count, p0, p1, _p(out), threads)
    return out


# ---- programs ------------------------------------------------------------------------
def _double_to_small(x: float, exp_bits: int, man_bits: int) -> int:
    sign = (1 << (exp_bits + man_bits)) if math.copysign(1.0, x) < 0 else 0
    exp_all = (1 << exp_bits) - 1
    if math.isnan(x):
        return sign | (exp_all << man_bits) | (1 << (man_bits - 1))
    a = abs(x)
    if math.isinf(a):
        return sign | (exp_all << man_bits)
    if a == 0.0:
        return sign
    bias = (1 << (exp_bits - 1)) - 1
    emin = 1 - bias
    e = math.frexp(a)[1] - 1
    if e < emin:
        return sign | int(round(math.ldexp(a, man_bits - emin)))  # round(): ties to even
    q = round(math.ldexp(a, man_bits - e))
    if q == 1 << (man_bits + 1):
        q //= 2
        e += 1
    if e > bias:
        return sign | (exp_all << man_bits)
    return sign | ((e + bias) << man_bits) | (q - (1 << man_bits))


def _const_imm(dtype: str, value) -> int:
    if dtype == "bool":
        return 1 if value else 0
    if dtype in ("i32", "i64"):
        v = int(value)
        return v & 0xFFFFFFFF if dtype == "i32" else v & 0xFFFFFFFFFFFFFFFF
    if isinstance(value, str):
        if value.startswith("bits:"):
            bits = int(value[5:], 0)
            if dtype == "f32":
                return bits
            if dtype == "f16":
                return int(np.array([bits], np.uint16).view(np.float16).astype(np.float32).view(np.uint32)[0])
            return (bits & 0xFFFF) << 16
        value = float(value)  # also parses "nan", "inf", "-inf"
    value = float(value)
    if dtype == "f32":
        return int(np.array([value], np.float32).view(np.uint32)[0])
    if dtype == "f16":
        h = _double_to_small(value, 5, 10)
        return int(np.array([h], np.uint16).view(np.float16).astype(np.float32).view(np.uint32)[0])
    return _double_to_small(value, 8, 7) << 16


def compile_program(program: list, inputs: list):
    """Recipe program (ASK op names) -> oracle instruction array + value types."""
    L = lib()
    types = []
    insns = (_Insn * len(program))()
    for i, ins in enumerate(program):
        name = ins[0][4:] if ins[0].startswith("ask.") else ins[0]
        x = insns[i]
        if name == "input":
            x.op, x.a = L.orc_op_code(b"input"), ins[1]
            t = inputs[ins[1]]["dtype"]
        elif name in ("const", "constant"):
            t = ins[1]
            x.op, x.imm = L.orc_op_code(b"const"), _const_imm(t, ins[2])
            x.src_type = dtype_code(t)
        elif name == "cast":
            x.op, x.a = L.orc_op_code(b"cast"), ins[1]
            x.src_type = dtype_code(types[ins[1]])
            t = ins[2]
        elif name == "compare":
            x.op, x.aux, x.a, x.b = L.orc_op_code(b"compare"), _PRED[ins[1]], ins[2], ins[3]
            x.src_type = dtype_code(types[ins[2]])
            t = "bool"
        elif name == "select":
            x.op, x.a, x.b, x.c = L.orc_op_code(b"select"), ins[1], ins[2], ins[3]
            t = types[ins[2]]
        else:
            code = L.orc_op_code(name.encode())
            if code < 0:
                raise ValueError(f"oracle does not know op {name}")
            x.op, x.a = code, ins[1]
            if len(ins) > 2:
                x.b = ins[2]
            t = types[ins[1]]
            x.src_type = dtype_code(t)
        x.type = dtype_code(t)
        types.append(t)
    return insns, types


def _port_arrays(inputs, recipe_inputs):
    out = []
    for a, spec in zip(inputs, recipe_inputs):
        a = np.ascontiguousarray(a, dtype=_DTYPES[spec["dtype"]])
        out.append(a)
    return out


def elementwise(recipe: dict, inputs: list, threads: int = 1) -> list:
    insns, types = compile_program(recipe["program"], recipe["inputs"])
    ins = _port_arrays(inputs, recipe["inputs"])
    n = recipe["count"]
    outs = [np.empty(n, dtype=_DTYPES[types[r]]) for r in recipe["results"]]
    in_t = np.array([dtype_code(s["dtype"]) for s in recipe["inputs"]], np.int32)
    in_m = np.array([_MAPS[s.get("map", "full")] for s in recipe["inputs"]], np.int32)
    out_r = np.array(recipe["results"], np.int32)
    out_t = np.array([dtype_code(types[r]) for r in recipe["results"]], np.int32)
    rc = lib().orc_elementwise(ctypes.cast(insns, ctypes.c_void_p), len(insns), _p(in_t), _p(in_m), len(ins),
                               _ptrs(ins), _p(out_r), _p(out_t), len(outs), _ptrs(outs), n,
                               max(1, recipe.get("inner", 1)), threads)
    assert rc == 0
    return outs


def reduce(recipe: dict, inputs: list, sum_mode: int = 0, threads: int = 1) -> list:
    insns, types = compile_program(recipe["program"], recipe["inputs"])
    ins = _port_arrays(inputs, recipe["inputs"])
    outer, extent, inner = recipe["outer"], recipe["extent"], recipe.get("inner", 1)
    reds = recipe["reductions"]
    L = lib()
    ops = np.array([L.orc_red_code(r["op"].encode()) for r in reds], np.int32)
    src = np.array([r.get("value", 0) for r in reds], np.int32)
    vregs = np.array(recipe["results"], np.int32)
    outs = []
    for r in reds:
        vt = types[recipe["results"][r.get("value", 0)]]
        ot = "i64" if r["op"] in ("argmax", "argmin") else "bool" if r["op"] in ("any", "all") else vt
        outs.append(np.empty(outer * inner, dtype=_DTYPES[ot]))
    in_t = np.array([dtype_code(s["dtype"]) for s in recipe["inputs"]], np.int32)
    in_m = np.array([_MAPS[s.get("map", "full")] for s in recipe["inputs"]], np.int32)
    rc = L.orc_reduce(ctypes.cast(insns, ctypes.c_void_p), len(insns), _p(in_t), _p(in_m), len(ins), _ptrs(ins),
                      _p(vregs), len(reds), _p(ops), _p(src), _ptrs(outs), outer, extent, inner,
                      recipe.get("index_base", 0), sum_mode, threads)
    assert rc == 0
    return outs


def gather(table: np.ndarray, index: np.ndarray, outer: int, dim: int, inner: int, threads: int = 1, out=None):
    n = index.size
    if out is None:
        out = np.empty(outer * n * inner, dtype=table.dtype)
    lib().orc_gather(_p(table), _p(index), 1 if index.dtype == np.int32 else 0, _p(out), outer, dim, inner, n,
                     table.dtype.itemsize, threads)
    return out


def scatter_add(dtype: str, base: np.ndarray, index: np.ndarray, upd: np.ndarray, outer: int, dim: int,
                inner: int, out=None):
    """Reference-order scatter_add in the element type (lib/Lowering/Host.cpp:677-772)."""
    if out is None:
        out = np.empty_like(base)
    lib().orc_scatter_add(dtype_code(dtype), _p(base), _p(index), 1 if index.dtype == np.int32 else 0, _p(upd),
                          _p(out), None, None, outer, dim, inner, index.size, 0)
    return out


def scatter_add_f64(base: np.ndarray, index: np.ndarray, upd: np.ndarray, outer: int, dim: int, inner: int):
    """f32 scatter_add accumulated in f64; also returns sum |upd| per element."""
    out64 = np.empty(base.size, np.float64)
    abs64 = np.empty(base.size, np.float64)
    lib().orc_scatter_add(dtype_code("f32"), _p(base), _p(index), 1 if index.dtype == np.int32 else 0, _p(upd),
                          None, _p(out64), _p(abs64), outer, dim, inner, index.size, 1)
    return out64, abs64


def cfg1(a, b, c, threads: int = 1, out=None):
    y0, y1 = out if out is not None else (np.empty_like(a), np.empty_like(a))
    lib().orc_cfg1(_p(a), _p(b), _p(c), _p(y0), _p(y1), a.size, threads)
    return y0, y1


def cfg5b(x, y, threads: int = 1, out=None):
    z = np.empty_like(x) if out is None else out
    lib().orc_cfg5b(_p(x), _p(y), _p(z), x.size, threads)
    return z


def cfg5a(x, index_base: int = 0, threads: int = 1):
    s64, sref, mn, am = (np.zeros(1, np.float64), np.zeros(1, np.float32), np.zeros(1, np.float32),
                         np.zeros(1, np.int64))
    lib().orc_cfg5a(_p(x), x.size, index_base, _p(s64), _p(sref), _p(mn), _p(am), threads)
    return float(s64[0]), float(sref[0]), float(mn[0]), int(am[0])


def softmax(dtype: str, x: np.ndarray, rows: int, cols: int, with_output: bool = True, threads: int = 1,
            out=None):
    m = np.empty(rows, np.float32)
    s = np.empty(rows, np.float32)
    y = (np.empty(rows * cols, np.uint16) if out is None else out) if with_output else None
    lib().orc_softmax(dtype_code(dtype), _p(x), rows, cols, _p(m), _p(s), _p(y) if y is not None else None,
                      threads)
    return m, s, y


def rowstats(x: np.ndarray, rows: int, cols: int, threads: int = 1):
    s, mx, mn = np.empty(rows, np.float32), np.empty(rows, np.float32), np.empty(rows, np.float32)
    am = np.empty(rows, np.int64)
    lib().orc_rowstats(_p(x), rows, cols, _p(s), _p(mx), _p(mn), _p(am), threads)
    return s, mx, mn, am
