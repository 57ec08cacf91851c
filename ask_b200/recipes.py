"""Recipe builders: the JSON form of owned ASK steps that Plan consumes.

A recipe is what ASK's CUDA lowering would receive for one owned step of an
execution plan (lib/Frontend/Partition.cpp:183-273 clones each part into its
own function; lib/Lowering/CUDA.cpp:152-419 lowers it).  Values are built with
:class:`Program`, an SSA builder whose method names are ASK's op names
(include/ask/IR/ASKOps.h:70-145, docs/en/ir.md:16-44).

The five benchmark configurations are provided as step recipes:

* :func:`cfg1_step` -- fused y0 = exp(a)*b + c, y1 = max(a,b) - tanh(c) (f32);
  ASK has no subtract, so "- t" is "+ t * (-1)".
* :func:`cfg2_step` -- row sum/max/min/argmax (one owned step, 4 outputs).
* :func:`cfg3_steps` -- the canonical three-step softmax partition
  (row max; row sum of exp(x - m); normalise), f16 or bf16 in, f32 math.
* :func:`cfg4_gather_step`, :func:`cfg4_scatter_step` -- embedding gather and
  scatter_add (with the runtime pre_copy of the base into the output).
* :func:`cfg5a_step`, :func:`cfg5b_step` -- the sharded plan's two parts.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class Value:
    index: int
    dtype: str


@dataclass
class Program:
    """SSA op program over the step's inputs."""

    inputs: list = field(default_factory=list)     # [{"dtype":..., "map":...}]
    insns: list = field(default_factory=list)
    types: list = field(default_factory=list)

    def _emit(self, insn, dtype) -> Value:
        self.insns.append(insn)
        self.types.append(dtype)
        return Value(len(self.insns) - 1, dtype)

    def input(self, dtype: str, map: str = "full") -> Value:
        port = len(self.inputs)
        self.inputs.append({"dtype": dtype, "map": map})
        return self._emit(["input", port], dtype)

    def const(self, dtype: str, value) -> Value:
        return self._emit(["const", dtype, value], dtype)

    def cast(self, x: Value, dtype: str) -> Value:
        return self._emit(["cast", x.index, dtype], dtype)

    def compare(self, pred: str, x: Value, y: Value) -> Value:
        return self._emit(["compare", pred, x.index, y.index], "bool")

    def select(self, c: Value, x: Value, y: Value) -> Value:
        return self._emit(["select", c.index, x.index, y.index], x.dtype)

    def op(self, name: str, *args: Value) -> Value:
        return self._emit([name] + [a.index for a in args], args[0].dtype)

    def __getattr__(self, name):
        if name in _UNARY or name in _BINARY:
            return lambda *a: self.op(name, *a)
        raise AttributeError(name)


_UNARY = {"bitwise_not", "abs", "exp", "log", "sqrt", "sin", "cos", "tanh", "erf", "floor", "ceil", "round"}
_BINARY = {"add", "mul", "div", "floordiv", "mod", "pow", "maximum", "minimum", "bitwise_and", "bitwise_or",
           "bitwise_xor", "shift_left", "shift_right"}


def elementwise(prog: Program, results: list, count: int, inner: int = 1) -> dict:
    return {
        "family": "elementwise",
        "count": int(count),
        "inner": int(inner),
        "inputs": prog.inputs,
        "outputs": [{"dtype": r.dtype} for r in results],
        "program": prog.insns,
        "results": [r.index for r in results],
    }


def reduce(prog: Program, value: Value, ops: list, outer: int, extent: int, inner: int = 1,
           index_base: int = 0, strategy: str | None = None) -> dict:
    r = {
        "family": "reduce",
        "outer": int(outer),
        "extent": int(extent),
        "inner": int(inner),
        "index_base": int(index_base),
        "inputs": prog.inputs,
        "program": prog.insns,
        "results": [value.index],
        "reductions": [{"op": op, "value": 0} for op in ops],
    }
    if strategy:
        r["strategy"] = strategy
    return r


def gather(dtype: str, index_dtype: str, dim: int, inner: int, n: int, outer: int = 1) -> dict:
    return {"family": "gather", "dtype": dtype, "index_dtype": index_dtype, "outer": int(outer), "dim": int(dim),
            "inner": int(inner), "n": int(n)}


def scatter_add(dtype: str, index_dtype: str, dim: int, inner: int, n: int, outer: int = 1) -> dict:
    return {"family": "scatter_add", "dtype": dtype, "index_dtype": index_dtype, "outer": int(outer),
            "dim": int(dim), "inner": int(inner), "n": int(n), "pre_copy": {"input": 0, "output": 0}}


# ---- the benchmark configurations ---------------------------------------------------
def cfg1_step(count: int = 4096 * 4096) -> dict:
    p = Program()
    a, b, c = p.input("f32"), p.input("f32"), p.input("f32")
    y0 = p.add(p.mul(p.exp(a), b), c)
    m = p.maximum(a, b)
    y1 = p.add(m, p.mul(p.tanh(c), p.const("f32", -1.0)))
    return elementwise(p, [y0, y1], count)


def cfg2_step(rows: int = 65536, cols: int = 1024) -> dict:
    p = Program()
    x = p.input("f32")
    return reduce(p, x, ["sum", "max", "min", "argmax"], rows, cols)


def cfg3_steps(dtype: str = "f16", rows: int = 32768, cols: int = 4096) -> list:
    """Step 0: m = max(cast(x)); step 1: s = sum(exp(cast(x) + m*(-1)));
    step 2: y = cast(exp(cast(x) + m*(-1)) / s, dtype)."""
    p0 = Program()
    x0 = p0.input(dtype)
    step0 = reduce(p0, p0.cast(x0, "f32"), ["max"], rows, cols)

    p1 = Program()
    x1, m1 = p1.input(dtype), p1.input("f32", "outer")
    xf = p1.cast(x1, "f32")
    e1 = p1.exp(p1.add(xf, p1.mul(m1, p1.const("f32", -1.0))))
    step1 = reduce(p1, e1, ["sum"], rows, cols)

    p2 = Program()
    x2, m2, s2 = p2.input(dtype), p2.input("f32", "outer"), p2.input("f32", "outer")
    xf2 = p2.cast(x2, "f32")
    e2 = p2.exp(p2.add(xf2, p2.mul(m2, p2.const("f32", -1.0))))
    y = p2.cast(p2.div(e2, s2), dtype)
    step2 = elementwise(p2, [y], rows * cols, inner=cols)
    return [step0, step1, step2]


def cfg4_gather_step(rows: int = 1 << 20, dim: int = 256, n: int = 1 << 23, index_dtype: str = "i64") -> dict:
    return gather("f32", index_dtype, rows, dim, n)


def cfg4_scatter_step(rows: int = 1 << 20, dim: int = 256, n: int = 1 << 23, dtype: str = "f32",
                      index_dtype: str = "i64") -> dict:
    return scatter_add(dtype, index_dtype, rows, dim, n)


def cfg5a_step(count: int = 1 << 32, index_base: int = 0) -> dict:
    p = Program()
    x = p.input("f32")
    return reduce(p, x, ["sum", "min", "argmin"], 1, count, index_base=index_base, strategy="split")


def cfg5b_step(count: int = 1 << 31) -> dict:
    p = Program()
    x, y = p.input("i32"), p.input("i32")
    t = p.bitwise_xor(p.shift_left(x, p.const("i32", 3)), p.shift_right(x, p.const("i32", 5)))
    z = p.add(p.bitwise_and(t, p.const("i32", 0x7FFFFFFF)), y)
    return elementwise(p, [z], count)


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Leading-axis slice [begin, end) of rank `rank` among `world` ranks:
    contiguous, in rank order, sizes differing by at most one unit of 1024
    elements so every shard starts on a 4 KiB boundary."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    unit = 1024 if total >= 1024 * world else 1
    units = (total + unit - 1) // unit
    base, extra = divmod(units, world)
    begin = (rank * base + min(rank, extra)) * unit
    end = min(total, begin + (base + (1 if rank < extra else 0)) * unit)
    return min(begin, total), end
