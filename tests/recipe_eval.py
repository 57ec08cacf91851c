"""A numpy evaluator for lowered integer recipes (test helper).

The lowering adapter turns a step source into a recipe whose program reads
its inputs through index maps ("full", "scalar", "view") and may read the
iteration coordinates ("coord").  This evaluator runs such a recipe over
the whole iteration shape at once, with the same view rule as the device
interpreter (a view port reads element offset + sum((c - lo) / step * stride)
where every axis has c - lo >= 0, divisible by step, (c - lo) / step < extent,
else its pad constant), so the lowering's translation can be checked against
numpy on the CPU.  Only the integer and bool instructions that lowered index
maps and integer programs use (plus f32 add, mul, maximum and minimum, exact
on small integers) are supported; anything else raises.
"""
import numpy as np

_NP = {"i32": np.int32, "i64": np.int64, "bool": np.bool_, "i8": np.int8, "i16": np.int16, "f32": np.float32}


def _input(port, arr, shape, inner, reduce_dims=None):
    m = port.get("map", "full")
    flat = np.ascontiguousarray(arr).reshape(-1)
    if m == "scalar":
        return np.full(shape, flat[0])
    if m == "full":
        return flat.reshape(shape)
    if m in ("outer", "inner"):
        i = np.arange(int(np.prod(shape)), dtype=np.int64)
        if reduce_dims:  # a reduction's outer port holds one value per output (o, i)
            _, e, n = reduce_dims
            return flat[(i // (e * n)) * n + i % n].reshape(shape)
        return flat[i // inner if m == "outer" else i % inner].reshape(shape)
    if m != "view":
        raise NotImplementedError(m)
    v = port["view"]
    ok, off = _window(v, np.indices(shape, dtype=np.int64))
    out = np.full(shape, v["pad"], dtype=flat.dtype)
    if "inner" in v:  # off is a row-major position in the inner shape, read through the inner window
        w = v["inner"]
        pos = np.where(ok, off, 0)
        iok, ioff = _window(w, np.stack(np.unravel_index(pos, w["shape"])))
        out[ok & ~iok] = w["pad"]
        ok &= iok
        off = ioff
    out[ok] = flat[off[ok]]
    return out


def _window(v, coords):
    """(valid, offset) of a view window at coordinates [rank, ...]."""
    ok = np.ones(coords.shape[1:], dtype=bool)
    off = np.full(coords.shape[1:], v["offset"], dtype=np.int64)
    for d in range(coords.shape[0]):
        s = coords[d] - v["lo"][d]
        q = np.floor_divide(s, v["step"][d])
        ok &= (s >= 0) & (q * v["step"][d] == s) & (q < v["extent"][d])
        off += q * v["stride"][d]
    return ok, off


def _reduce(recipe, values):
    """Reductions of an integer reduce recipe: each value is viewed as
    [outer, extent, inner] and folded over the middle axis (sums wrap in the
    value's type; arg positions are the first extreme plus index_base)."""
    o, e, i = recipe["outer"], recipe["extent"], recipe["inner"]
    out = []
    for r in recipe["reductions"]:
        v = values[r["value"]].reshape(o, e, i)
        op = r["op"]
        if op == "reduce_sum":
            x = v.sum(axis=1, dtype=np.int64).astype(v.dtype)
        elif op == "reduce_prod":
            x = v.prod(axis=1, dtype=np.int64).astype(v.dtype)
        elif op in ("reduce_max", "reduce_any"):
            x = v.max(axis=1)
        elif op in ("reduce_min", "reduce_all"):
            x = v.min(axis=1)
        elif op in ("argmax", "argmin"):
            x = (np.argmax(v, axis=1) if op == "argmax" else np.argmin(v, axis=1)).astype(np.int64)
            x = x + int(recipe.get("index_base", 0))
        else:
            raise NotImplementedError(op)
        out.append(x.reshape(-1))
    return out


def evaluate(recipe, inputs):
    """Outputs (flat numpy arrays) of an integer elementwise or reduce recipe."""
    if recipe["family"] == "reduce":
        shape = tuple(recipe.get("shape") or [recipe["outer"], recipe["extent"], recipe["inner"]])
        values = _program(dict(recipe, shape=list(shape)), inputs, shape)
        return _reduce(recipe, [v.reshape(-1) for v in values])
    assert recipe["family"] == "elementwise"
    shape = tuple(recipe.get("shape") or [recipe["count"]])
    return [v.reshape(-1) for v in _program(recipe, inputs, shape)]


def _program(recipe, inputs, shape):
    """The program's result arrays over the iteration shape."""
    regs = []
    for ins in recipe["program"]:
        op = ins[0]
        if op == "const":
            t = _NP[ins[1]]
            x = np.full(shape, ins[2], dtype=t)
        elif op == "input":
            dims = (recipe["outer"], recipe["extent"], recipe["inner"]) if recipe["family"] == "reduce" else None
            x = _input(recipe["inputs"][ins[1]], inputs[ins[1]], shape, int(recipe.get("inner", 1)), dims)
        elif op == "coord":
            x = np.indices(shape, dtype=np.int64)[ins[1]]
        elif op == "select":
            x = np.where(regs[ins[1]].astype(bool), regs[ins[2]], regs[ins[3]])
        elif op == "compare":
            a, b = regs[ins[2]], regs[ins[3]]
            x = {"lt": a < b, "le": a <= b, "gt": a > b, "ge": a >= b, "eq": a == b, "ne": a != b}[ins[1]]
        elif op == "cast":
            x = regs[ins[1]].astype(_NP[ins[2]])
        elif op in ("add", "mul", "maximum", "minimum", "mod", "floordiv", "bitwise_and", "bitwise_or", "bitwise_xor"):
            a, b = regs[ins[1]], regs[ins[2]]
            with np.errstate(over="ignore"):
                x = {"add": np.add, "mul": np.multiply, "maximum": np.maximum, "minimum": np.minimum,
                     "mod": np.mod, "floordiv": np.floor_divide, "bitwise_and": np.bitwise_and,
                     "bitwise_or": np.bitwise_or, "bitwise_xor": np.bitwise_xor}[op](a, b).astype(np.result_type(a, b))
        elif op in ("abs", "bitwise_not"):
            with np.errstate(over="ignore"):
                x = {"abs": np.abs, "bitwise_not": np.invert}[op](regs[ins[1]])
        else:
            raise NotImplementedError(op)
        regs.append(x)
    return [regs[r] for r in recipe["results"]]
