"""Lowering adapter: ASK step sources (MLIR text) -> recipes -> programs.

The step sources below are written in the form the reference's partitioner
prints (lib/Frontend/Partition.cpp:178-273: one func.func per owned step, ASK
ops in MLIR generic form, ask.* attributes on ops and arguments).  Each config
of the benchmark is lowered and must select the same specialised kernel as
its hand-written recipe; a partition report with three softmax steps and one
with gather -> scatter_add become runtime programs.  The GPU tests run lowered
programs against the hand-written recipes, bit for bit.
"""
import json

import numpy as np
import pytest

import ask_b200
from ask_b200 import recipes as R
from ask_b200 import runtime as rt
import recipe_eval


def ttype(shape, dt):
    mlir = {"bool": "i1"}.get(dt, dt)
    return f"tensor<{'x'.join(str(d) for d in shape)}{'x' if shape else ''}{mlir}>"


class Step:
    """Builds one step source in the printed MLIR form."""

    def __init__(self, name="ask_kernel_0", kernel="kernel0"):
        self.name, self.kernel = name, kernel
        self.args, self.lines, self.n = [], [], 0

    def arg(self, shape, dt):
        k = len(self.args)
        self.args.append((shape, dt))
        return f"%arg{k}", shape, dt

    def op(self, name, operands, shape, dt, attrs=""):
        v = f"%{self.n}"
        self.n += 1
        a = f'{{ask.id = "{self.kernel}.op{self.n}", ask.value_id = "v{self.n}"{", " + attrs if attrs else ""}}}'
        ins = ", ".join(o[0] for o in operands)
        tys = ", ".join(ttype(o[1], o[2]) if o[1] is not None else o[2] for o in operands)
        out = ttype(shape, dt) if shape is not None else dt
        self.lines.append(f'    {v} = "ask.{name}"({ins}) {a} : ({tys}) -> {out}')
        return v, shape, dt

    def const(self, value, dt):
        v = f"%{self.n}"
        self.n += 1
        self.lines.append(f'    {v} = "ask.constant"() {{ask.id = "{self.kernel}.scalar{self.n}", value = {value} : {dt}}}'
                          f" : () -> {dt}")
        return v, None, dt

    def splat(self, c, shape):
        return self.op("splat", [c], shape, c[2], f"shape = array<i64: {', '.join(map(str, shape))}>")

    def text(self, results):
        args = ", ".join(f'%arg{k}: {ttype(s, d)} {{ask.source_value_id = "x{k}", ask.value_id = "{self.kernel}.arg{k}"}}'
                         for k, (s, d) in enumerate(self.args))
        res = ", ".join(ttype(r[1], r[2]) for r in results)
        ret = ", ".join(r[0] for r in results)
        return ("module {\n"
                f"  func.func @{self.name}({args}) -> ({res}) attributes {{ask.kernel_id = \"{self.kernel}\", "
                f"ask.kernel_kind = \"owned\", ask.source_function = \"main\"}} {{\n"
                + "\n".join(self.lines) + "\n"
                f"    return {ret} : {res}\n  }}\n}}\n")


def cfg1_source(n=4096):
    s = Step()
    a, b, c = (s.arg([n, n], "f32") for _ in range(3))
    sh = [n, n]
    y0 = s.op("add", [s.op("mul", [s.op("exp", [a], sh, "f32"), b], sh, "f32"), c], sh, "f32", 'overflow = "wrap"')
    m = s.op("maximum", [a, b], sh, "f32")
    neg = s.op("mul", [s.op("tanh", [c], sh, "f32"), s.splat(s.const("-1.000000e+00", "f32"), sh)], sh, "f32")
    y1 = s.op("add", [m, neg], sh, "f32")
    return s.text([y0, y1])


def cfg2_source(rows=65536, cols=1024):
    s = Step()
    x = s.arg([rows, cols], "f32")
    outs = [s.op(f"reduce_{k}", [x], [rows], "f32", "axes = array<i64: 1>") for k in ("sum", "max", "min")]
    outs.append(s.op("argmax", [x], [rows], "i64", "axis = 1 : i64"))
    return s.text(outs)


def cfg3_sources(dt="f16", rows=32768, cols=4096):
    sh = [rows, cols]
    s0 = Step("ask_kernel_0", "kernel0")
    x = s0.arg(sh, dt)
    m = s0.op("reduce_max", [s0.op("cast", [x], sh, "f32")], [rows], "f32", "axes = array<i64: 1>")
    src0 = s0.text([m])

    def shifted(s):
        x = s.arg(sh, dt)
        m = s.arg([rows], "f32")
        xf = s.op("cast", [x], sh, "f32")
        mb = s.op("broadcast_in_dim", [m], sh, "f32", f"dimensions = array<i64: 0>, shape = array<i64: {rows}, {cols}>")
        neg = s.op("mul", [mb, s.splat(s.const("-1.000000e+00", "f32"), sh)], sh, "f32")
        return s.op("exp", [s.op("add", [xf, neg], sh, "f32", 'overflow = "wrap"')], sh, "f32")

    s1 = Step("ask_kernel_1", "kernel1")
    e = shifted(s1)
    src1 = s1.text([s1.op("reduce_sum", [e], [rows], "f32", "axes = array<i64: 1>")])
    s2 = Step("ask_kernel_2", "kernel2")
    e = shifted(s2)
    sarg = s2.arg([rows], "f32")
    sb = s2.op("broadcast_in_dim", [sarg], sh, "f32", f"dimensions = array<i64: 0>, shape = array<i64: {rows}, {cols}>")
    y = s2.op("cast", [s2.op("div", [e, sb], sh, "f32")], sh, dt)
    return [src0, src1, s2.text([y])]


def cfg4_sources(rows=1 << 20, dim=256, n=1 << 23):
    g = Step("ask_kernel_0", "kernel0")
    t, i = g.arg([rows, dim], "f32"), g.arg([n], "i64")
    gsrc = g.text([g.op("gather", [t, i], [n, dim], "f32", "axis = 0 : i64")])
    s = Step("ask_kernel_1", "kernel1")
    base, idx, upd = s.arg([rows, dim], "f32"), s.arg([n], "i64"), s.arg([n, dim], "f32")
    ssrc = s.text([s.op("scatter_add", [base, idx, upd], [rows, dim], "f32", "axis = 0 : i64")])
    return gsrc, ssrc


def cfg5_sources(na=1 << 32, nb=1 << 31):
    a = Step()
    x = a.arg([na], "f32")
    outs = [a.op("reduce_sum", [x], [], "f32", "axes = array<i64: 0>"),
            a.op("reduce_min", [x], [], "f32", "axes = array<i64: 0>"),
            a.op("argmin", [x], [], "i64", "axis = 0 : i64")]
    b = Step()
    x, y = b.arg([nb], "i32"), b.arg([nb], "i32")
    sh = [nb]
    t = b.op("bitwise_xor", [b.op("shift_left", [x, b.splat(b.const(3, "i32"), sh)], sh, "i32"),
                             b.op("shift_right", [x, b.splat(b.const(5, "i32"), sh)], sh, "i32")], sh, "i32")
    z = b.op("add", [b.op("bitwise_and", [t, b.splat(b.const(2147483647, "i32"), sh)], sh, "i32"), y], sh, "i32",
             'overflow = "wrap"')
    return a.text(outs), b.text([z])


def kernel_of(recipe):
    return ask_b200.Plan(recipe, device=-1).describe()["kernel"]


@pytest.mark.parametrize("name,source,hand", [
    ("cfg1", lambda: cfg1_source(), lambda: R.cfg1_step()),
    ("cfg2", lambda: cfg2_source(), lambda: R.cfg2_step()),
    ("cfg5a", lambda: cfg5_sources()[0], lambda: R.cfg5a_step()),
    ("cfg5b", lambda: cfg5_sources()[1], lambda: R.cfg5b_step()),
    ("cfg4g", lambda: cfg4_sources()[0], lambda: R.cfg4_gather_step()),
    ("cfg4s", lambda: cfg4_sources()[1], lambda: R.cfg4_scatter_step()),
])
def test_configs_lower_to_the_specialised_kernels(name, source, hand):
    out = rt.lower_step(source())
    lowered, want = ask_b200.Plan(out["recipe"], -1).describe(), ask_b200.Plan(hand(), -1).describe()
    for key in ("family", "kernel", "strategy", "port_map", "scratch_bytes"):
        assert lowered.get(key) == want.get(key), key
    assert out["input_arguments"] == list(range(len(out["input_arguments"])))


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_softmax_steps_lower_to_the_specialised_kernels(dt):
    for src, hand in zip(cfg3_sources(dt), R.cfg3_steps(dt)):
        assert kernel_of(rt.lower_step(src)["recipe"]) == kernel_of(hand)


def test_constants_keep_their_exact_value():
    s = Step()
    x = s.arg([8], "f16")
    c = s.splat(s.const("0x7E00", "f16"), [8])  # a NaN printed as its bit pattern
    d = s.splat(s.const("1.000000e-01", "f16"), [8])
    y = s.op("add", [s.op("maximum", [x, c], [8], "f16"), d], [8], "f16")
    r = rt.lower_step(s.text([y]))["recipe"]
    consts = [i for i in r["program"] if i[0] == "const"]
    assert consts == [["const", "f16", "bits:0x7E00"], ["const", "f16", "1.000000e-01"]]
    ask_b200.Plan(r, -1)


def test_index_maps():
    s = Step()
    x = s.arg([4, 8], "f32")
    row = s.arg([4], "f32")
    col = s.arg([8], "f32")
    one = s.arg([], "f32")
    rb = s.op("broadcast_in_dim", [row], [4, 8], "f32", "dimensions = array<i64: 0>, shape = array<i64: 4, 8>")
    cb = s.op("broadcast_in_dim", [col], [4, 8], "f32", "dimensions = array<i64: 1>, shape = array<i64: 4, 8>")
    ob = s.op("broadcast_in_dim", [one], [4, 8], "f32", "dimensions = array<i64>, shape = array<i64: 4, 8>")
    y = s.op("add", [s.op("mul", [x, rb], [4, 8], "f32"), s.op("add", [cb, ob], [4, 8], "f32")], [4, 8], "f32")
    r = rt.lower_step(s.text([y]))["recipe"]
    assert [p["map"] for p in r["inputs"]] == ["full", "outer", "inner", "scalar"]
    assert r["inner"] == 8
    ask_b200.Plan(r, -1)


def arr(v):
    return f"array<i64: {', '.join(str(int(x)) for x in v)}>" if len(v) else "array<i64>"


def view_steps():
    """(name, step source, input arrays, numpy expectation) of index-map steps."""
    rng = np.random.default_rng(5)
    cases = []
    # transpose of an argument plus a full-shape argument
    s = Step()
    x, b = s.arg([3, 5], "i32"), s.arg([5, 3], "i32")
    y = s.op("add", [s.op("transpose", [x], [5, 3], "i32", "permutation = " + arr([1, 0])), b], [5, 3], "i32")
    xv, bv = rng.integers(-99, 99, (3, 5)).astype(np.int32), rng.integers(-99, 99, (5, 3)).astype(np.int32)
    cases.append(("transpose", s.text([y]), [xv, bv], xv.T + bv))
    # slice with a negative step and a positive one
    s = Step()
    x = s.arg([7, 9], "i32")
    sl = s.op("slice", [x], [4, 3], "i32", f"starts = {arr([6, 1])}, stops = {arr([-1, 8])}, steps = {arr([-2, 3])}")
    y = s.op("mul", [sl, s.splat(s.const(3, "i32"), [4, 3])], [4, 3], "i32")
    xv = rng.integers(-99, 99, (7, 9)).astype(np.int32)
    cases.append(("slice", s.text([y]), [xv], xv[6::-2, 1:8:3] * 3))
    # pad with low, high and interior padding, f32 (exact adds of small integers)
    s = Step()
    x = s.arg([2, 3], "f32")
    pv = s.splat(s.const("5.000000e-01", "f32"), [])
    pd = s.op("pad", [x, pv], [6, 8], "f32",
              f"pad_low = {arr([1, 0])}, pad_high = {arr([2, 1])}, interior = {arr([1, 2])}")
    y = s.op("add", [pd, s.splat(s.const("1.000000e+00", "f32"), [6, 8])], [6, 8], "f32")
    xv = rng.integers(-9, 9, (2, 3)).astype(np.float32)
    want = np.full((6, 8), 0.5, np.float32)
    want[1:1 + 2 * 2:2, 0:0 + 3 * 3:3] = xv
    cases.append(("pad", s.text([y]), [xv], want + 1))
    # concatenate of three arguments along axis 1, one of them transposed
    s = Step()
    a1, a2, a3 = s.arg([4, 2], "i32"), s.arg([4, 3], "i32"), s.arg([1, 4], "i32")
    t3 = s.op("transpose", [a3], [4, 1], "i32", "permutation = " + arr([1, 0]))
    y = s.op("concatenate", [a1, a2, t3], [4, 6], "i32", "axis = 1 : i64")
    v1, v2, v3 = (rng.integers(-99, 99, sh).astype(np.int32) for sh in ([4, 2], [4, 3], [1, 4]))
    cases.append(("concatenate", s.text([y]), [v1, v2, v3], np.concatenate([v1, v2, v3.T], axis=1)))
    # iota along axis 1 cast to f32, plus a general broadcast of a [3,1] column
    s = Step()
    col = s.arg([3, 1], "f32")
    io = s.op("iota", [], [3, 4], "f32", "dimension = 1 : i64")
    bc = s.op("broadcast_in_dim", [col], [3, 4], "f32", f"dimensions = {arr([0, 1])}, shape = {arr([3, 4])}")
    y = s.op("add", [io, bc], [3, 4], "f32")
    cv = rng.integers(-9, 9, (3, 1)).astype(np.float32)
    cases.append(("iota_broadcast", s.text([y]), [cv], np.arange(4, dtype=np.float32)[None, :] + cv))
    # reshapes no strided window expresses: of a transpose (read at the same
    # row-major position, ScalarEmitter.h:622), of a pad and of a strided slice
    s = Step()
    x = s.arg([4, 6], "i32")
    t = s.op("transpose", [x], [6, 4], "i32", "permutation = " + arr([1, 0]))
    y = s.op("add", [s.op("reshape", [t], [3, 8], "i32", f"shape = {arr([3, 8])}"),
                     s.splat(s.const(1, "i32"), [3, 8])], [3, 8], "i32")
    xv = rng.integers(-99, 99, (4, 6)).astype(np.int32)
    cases.append(("reshape_of_transpose", s.text([y]), [xv], xv.T.reshape(3, 8) + 1))
    s = Step()
    x = s.arg([2, 3], "i32")
    pd = s.op("pad", [x, s.splat(s.const(7, "i32"), [])], [3, 5], "i32",
              f"pad_low = {arr([1, 0])}, pad_high = {arr([0, 0])}, interior = {arr([0, 1])}")
    y = s.op("reshape", [pd], [5, 3], "i32", f"shape = {arr([5, 3])}")
    xv = rng.integers(-99, 99, (2, 3)).astype(np.int32)
    pw = np.full((3, 5), 7, np.int32)
    pw[1:3, 0:5:2] = xv
    cases.append(("reshape_of_pad", s.text([y]), [xv], pw.reshape(5, 3)))
    s = Step()
    x = s.arg([5, 9], "i32")
    sl = s.op("slice", [x], [3, 4], "i32", f"starts = {arr([0, 1])}, stops = {arr([5, 9])}, steps = {arr([2, 2])}")
    y = s.op("mul", [s.op("reshape", [sl], [2, 6], "i32", f"shape = {arr([2, 6])}"),
                     s.op("transpose", [s.arg([6, 2], "i32")], [2, 6], "i32", "permutation = " + arr([1, 0]))],
             [2, 6], "i32")
    xv, bv = rng.integers(-9, 9, (5, 9)).astype(np.int32), rng.integers(-9, 9, (6, 2)).astype(np.int32)
    cases.append(("reshape_of_slice", s.text([y]), [xv, bv], xv[0:5:2, 1:9:2].reshape(2, 6) * bv.T))
    return cases


@pytest.mark.parametrize("case", [c for c in view_steps() if c[0].startswith("reshape_of")], ids=lambda c: c[0])
def test_reshapes_through_an_inner_window_evaluate(case):
    name, src, ins, want = case
    out = rt.lower_step(src)
    r = out["recipe"]
    assert any("inner" in p.get("view", {}) for p in r["inputs"]), name
    got = recipe_eval.evaluate(r, [ins[a] for a in out["input_arguments"]])
    assert np.array_equal(got[0].reshape(want.shape), want), name


def test_two_stacked_reshapes_are_unsupported():
    s = Step()
    x = s.arg([4, 6], "i32")
    t = s.op("transpose", [x], [6, 4], "i32", "permutation = " + arr([1, 0]))
    r1 = s.op("reshape", [t], [3, 8], "i32", f"shape = {arr([3, 8])}")
    t2 = s.op("transpose", [r1], [8, 3], "i32", "permutation = " + arr([1, 0]))
    r2 = s.op("reshape", [t2], [24], "i32", f"shape = {arr([24])}")
    with pytest.raises(rt.CUDAError) as err:
        rt.lower_step(s.text([s.op("abs", [r2], [24], "i32")]))
    assert err.value.status == ask_b200.E_UNSUPPORTED


@pytest.mark.parametrize("case", view_steps(), ids=lambda c: c[0])
def test_index_maps_lower_to_views(case):
    name, src, ins, want = case
    out = rt.lower_step(src)
    r = out["recipe"]
    assert r["shape"] == list(want.shape)
    assert ask_b200.Plan(r, -1).describe()["kernel"] == "ew_view"
    assert len(out["input_arguments"]) == len(r["inputs"])


def reduce_view_steps():
    """(name, step source, input arrays, expected outputs) of reductions whose
    operand reads arguments through index maps."""
    rng = np.random.default_rng(9)
    cases = []
    # sum and argmax along axis 1 of a transposed argument: a column reduction of x
    s = Step()
    x = s.arg([6, 40], "i32")
    t = s.op("transpose", [x], [40, 6], "i32", "permutation = " + arr([1, 0]))
    outs = [s.op("reduce_sum", [t], [40], "i32", "axes = array<i64: 1>"), s.op("argmax", [t], [40], "i64", "axis = 1 : i64")]
    xv = rng.integers(-50, 50, (6, 40)).astype(np.int32)
    cases.append(("transpose_rows", s.text(outs), [xv], [xv.T.sum(axis=1).astype(np.int32), np.argmax(xv.T, axis=1)]))
    # max and min over axis 0 (inner > 1) of a strided slice
    s = Step()
    x = s.arg([9, 12], "f32")
    sl = s.op("slice", [x], [4, 6], "f32", f"starts = {arr([1, 0])}, stops = {arr([9, 12])}, steps = {arr([2, 2])}")
    outs = [s.op("reduce_max", [sl], [6], "f32", "axes = array<i64: 0>"), s.op("reduce_min", [sl], [6], "f32", "axes = array<i64: 0>")]
    xv = rng.standard_normal((9, 12)).astype(np.float32)
    sv = xv[1:9:2, 0:12:2]
    cases.append(("slice_columns", s.text(outs), [xv], [sv.max(axis=0), sv.min(axis=0)]))
    # weighted row sum with iota: sum_j j * x[i, j] (coordinates inside a reduction prologue)
    s = Step()
    x = s.arg([5, 33], "i64")
    io = s.op("iota", [], [5, 33], "i64", "dimension = 1 : i64")
    prod = s.op("mul", [io, x], [5, 33], "i64")
    outs = [s.op("reduce_sum", [prod], [5], "i64", "axes = array<i64: 1>")]
    xv = rng.integers(-1000, 1000, (5, 33)).astype(np.int64)
    cases.append(("iota_weights", s.text(outs), [xv], [(xv * np.arange(33)[None, :]).sum(axis=1)]))
    # a general broadcast of a middle-axis vector added before a reduction over the last two axes
    s = Step()
    x = s.arg([3, 4, 7], "i32")
    v = s.arg([4], "i32")
    bc = s.op("broadcast_in_dim", [v], [3, 4, 7], "i32", f"dimensions = {arr([1])}, shape = {arr([3, 4, 7])}")
    outs = [s.op("reduce_sum", [s.op("add", [x, bc], [3, 4, 7], "i32")], [3], "i32", "axes = array<i64: 1, 2>")]
    xv = rng.integers(-20, 20, (3, 4, 7)).astype(np.int32)
    vv = rng.integers(-20, 20, 4).astype(np.int32)
    cases.append(("broadcast_middle", s.text(outs), [xv, vv], [(xv + vv[None, :, None]).sum(axis=(1, 2)).astype(np.int32)]))
    return cases


@pytest.mark.parametrize("case", reduce_view_steps(), ids=lambda c: c[0])
def test_reductions_over_index_maps_lower_to_the_view_kernel(case):
    """Reductions read index maps through the view kernel -- except a plain
    transpose, which becomes the column reduction of the argument itself."""
    name, src, ins, want = case
    out = rt.lower_step(src)
    r = out["recipe"]
    d = ask_b200.Plan(r, -1).describe()
    if name == "transpose_rows":
        assert "shape" not in r and [p["map"] for p in r["inputs"]] == ["full"]
        assert (r["outer"], r["extent"], r["inner"]) == (1, 6, 40) and d["strategy"] == "column"
    else:
        assert r["family"] == "reduce" and "shape" in r
        assert d["kernel"] == "reduce_view" and d["strategy"] == "view"


@pytest.mark.gpu
@pytest.mark.parametrize("case", reduce_view_steps(), ids=lambda c: c[0])
def test_reductions_over_index_maps_on_gpu(device, case):
    import torch
    name, src, ins, want = case
    out = rt.lower_step(src)
    plan = ask_b200.Plan(out["recipe"], 0)
    dev_in = [torch.from_numpy(np.ascontiguousarray(ins[a])).cuda() for a in out["input_arguments"]]
    dev_out = [torch.empty(w.size, dtype=torch.from_numpy(np.ascontiguousarray(w)).dtype, device="cuda") for w in want]
    plan.launch(dev_in, dev_out, None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    for got, w in zip(dev_out, want):
        assert np.array_equal(got.cpu().numpy(), np.asarray(w).reshape(-1)), name


def computed_map_steps():
    """(name, step source, input arrays, expected outputs) of index maps of
    computed values: the maps move onto the operands."""
    rng = np.random.default_rng(13)
    cases = []
    # transpose of an elementwise expression, then an elementwise use
    s = Step()
    x, y, b = s.arg([4, 6], "i32"), s.arg([4, 6], "i32"), s.arg([6, 4], "i32")
    e = s.op("add", [s.op("mul", [x, s.splat(s.const(3, "i32"), [4, 6])], [4, 6], "i32"), y], [4, 6], "i32")
    t = s.op("transpose", [e], [6, 4], "i32", "permutation = " + arr([1, 0]))
    out = s.op("add", [t, b], [6, 4], "i32")
    xv, yv, bv = (rng.integers(-99, 99, sh).astype(np.int32) for sh in ([4, 6], [4, 6], [6, 4]))
    cases.append(("transpose_expr", s.text([out]), [xv, yv, bv], [(xv * 3 + yv).T + bv]))
    # general broadcast of abs(v) along the middle axis, then a slice of a select
    s = Step()
    x, v = s.arg([3, 5, 2], "i32"), s.arg([5], "i32")
    bc = s.op("broadcast_in_dim", [s.op("abs", [v], [5], "i32")], [3, 5, 2], "i32",
              f"dimensions = {arr([1])}, shape = {arr([3, 5, 2])}")
    zero = s.splat(s.const(0, "i32"), [3, 5, 2])
    neg = s.op("mul", [x, s.splat(s.const(-1, "i32"), [3, 5, 2])], [3, 5, 2], "i32")
    sel = s.op("select", [s.op("compare", [x, zero], [3, 5, 2], "bool", 'predicate = "lt"'), neg, x], [3, 5, 2], "i32")
    out = s.op("add", [sel, bc], [3, 5, 2], "i32")
    xv, vv = rng.integers(-9, 9, (3, 5, 2)).astype(np.int32), rng.integers(-9, 9, 5).astype(np.int32)
    cases.append(("broadcast_select", s.text([out]), [xv, vv], [np.abs(xv) + np.abs(vv)[None, :, None]]))
    # slice of a reshape of a computed value
    s = Step()
    x = s.arg([3, 8], "i64")
    r = s.op("reshape", [s.op("add", [x, x], [3, 8], "i64")], [6, 4], "i64", f"shape = {arr([6, 4])}")
    sl = s.op("slice", [r], [3, 2], "i64", f"starts = {arr([0, 1])}, stops = {arr([6, 4])}, steps = {arr([2, 2])}")
    xv = rng.integers(-1000, 1000, (3, 8)).astype(np.int64)
    cases.append(("slice_reshape", s.text([sl]), [xv], [(2 * xv).reshape(6, 4)[0:6:2, 1:4:2]]))
    # a reduction of a transposed product: column sums of x * y
    s = Step()
    x, y = s.arg([7, 5], "i32"), s.arg([7, 5], "i32")
    t = s.op("transpose", [s.op("mul", [x, y], [7, 5], "i32")], [5, 7], "i32", "permutation = " + arr([1, 0]))
    outs = [s.op("reduce_sum", [t], [5], "i32", "axes = array<i64: 1>"), s.op("argmin", [t], [5], "i64", "axis = 1 : i64")]
    xv, yv = rng.integers(-30, 30, (7, 5)).astype(np.int32), rng.integers(-30, 30, (7, 5)).astype(np.int32)
    cases.append(("reduce_transposed_product", s.text(outs), [xv, yv],
                  [(xv * yv).sum(axis=0).astype(np.int32), np.argmin((xv * yv).T, axis=1)]))
    return cases


@pytest.mark.parametrize("case", computed_map_steps(), ids=lambda c: c[0])
def test_index_maps_of_computed_values_lower(case):
    name, src, ins, want = case
    out = rt.lower_step(src)
    ask_b200.Plan(out["recipe"], -1)  # validates


@pytest.mark.gpu
@pytest.mark.parametrize("case", computed_map_steps(), ids=lambda c: c[0])
def test_index_maps_of_computed_values_on_gpu(device, case):
    import torch
    name, src, ins, want = case
    out = rt.lower_step(src)
    plan = ask_b200.Plan(out["recipe"], 0)
    dev_in = [torch.from_numpy(np.ascontiguousarray(ins[a])).cuda() for a in out["input_arguments"]]
    dev_out = [torch.empty(np.asarray(w).size, dtype=torch.from_numpy(np.ascontiguousarray(w)).dtype, device="cuda")
               for w in want]
    plan.launch(dev_in, dev_out, None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    for got, w in zip(dev_out, want):
        assert np.array_equal(got.cpu().numpy(), np.asarray(w).reshape(-1)), name


def padded_concat_steps():
    """pad and concatenate of computed values (and a pad with interior padding)."""
    rng = np.random.default_rng(21)
    cases = []
    s = Step()
    x = s.arg([3, 4], "i32")
    e = s.op("mul", [x, s.splat(s.const(5, "i32"), [3, 4])], [3, 4], "i32")
    pv = s.splat(s.const(-7, "i32"), [])
    y = s.op("pad", [e, pv], [7, 9], "i32", f"pad_low = {arr([1, 2])}, pad_high = {arr([1, 1])}, interior = {arr([1, 1])}")
    xv = rng.integers(-9, 9, (3, 4)).astype(np.int32)
    want = np.full((7, 9), -7, np.int32)
    want[1:1 + 3 * 2:2, 2:2 + 4 * 2:2] = xv * 5
    cases.append(("pad_interior", s.text([y]), [xv], [want]))
    s = Step()
    a, b = s.arg([2, 3], "i32"), s.arg([2, 5], "i32")
    ea = s.op("abs", [a], [2, 3], "i32")
    eb = s.op("add", [b, b], [2, 5], "i32")
    y = s.op("concatenate", [ea, b, eb], [2, 13], "i32", "axis = 1 : i64")
    av, bv = rng.integers(-9, 9, (2, 3)).astype(np.int32), rng.integers(-9, 9, (2, 5)).astype(np.int32)
    cases.append(("concat_computed", s.text([y]), [av, bv], [np.concatenate([np.abs(av), bv, 2 * bv], axis=1)]))
    s = Step()
    x = s.arg([4, 6], "i32")
    t = s.op("transpose", [s.op("maximum", [x, s.splat(s.const(0, "i32"), [4, 6])], [4, 6], "i32")], [6, 4], "i32",
             "permutation = " + arr([1, 0]))
    pv = s.splat(s.const(3, "i32"), [])
    y = s.op("pad", [t, pv], [8, 5], "i32", f"pad_low = {arr([2, 0])}, pad_high = {arr([0, 1])}, interior = {arr([0, 0])}")
    xv = rng.integers(-9, 9, (4, 6)).astype(np.int32)
    want = np.full((8, 5), 3, np.int32)
    want[2:8, 0:4] = np.maximum(xv, 0).T
    cases.append(("pad_of_transposed_max", s.text([y]), [xv], [want]))
    # slices of a padded argument: the slice's step meets the pad's interior step
    for k, (start, step) in enumerate([(1, 3), (0, 2), (2, 4), (3, 1)]):
        s = Step()
        x = s.arg([5, 4], "i32")
        pv = s.splat(s.const(-1, "i32"), [])
        pd = s.op("pad", [x, pv], [12, 9], "i32",
                  f"pad_low = {arr([2, 1])}, pad_high = {arr([2, 1])}, interior = {arr([1, 1])}")
        full = np.full((12, 9), -1, np.int32)
        xv = rng.integers(-9, 9, (5, 4)).astype(np.int32)
        full[2:2 + 5 * 2:2, 1:1 + 4 * 2:2] = xv
        sl = full[start::step, 1::2]
        y = s.op("slice", [pd], list(sl.shape), "i32",
                 f"starts = {arr([start, 1])}, stops = {arr([12, 9])}, steps = {arr([step, 2])}")
        out = s.op("add", [y, s.splat(s.const(0, "i32"), list(sl.shape))], list(sl.shape), "i32")
        cases.append((f"slice_of_pad_{k}", s.text([out]), [xv], [sl]))
    # slice and transpose of a padded computed value (the pad's mask composes with the map)
    s = Step()
    x = s.arg([4, 5], "i32")
    e = s.op("add", [x, x], [4, 5], "i32")
    pv = s.splat(s.const(9, "i32"), [])
    pd = s.op("pad", [e, pv], [10, 8], "i32", f"pad_low = {arr([1, 2])}, pad_high = {arr([2, 1])}, interior = {arr([1, 0])}")
    xv = rng.integers(-9, 9, (4, 5)).astype(np.int32)
    full = np.full((10, 8), 9, np.int32)
    full[1:1 + 4 * 2:2, 2:7] = 2 * xv
    sl = full[1::3, 0::2]
    y = s.op("slice", [pd], list(sl.shape), "i32", f"starts = {arr([1, 0])}, stops = {arr([10, 8])}, steps = {arr([3, 2])}")
    tr = s.op("transpose", [y], list(sl.T.shape), "i32", "permutation = " + arr([1, 0]))
    cases.append(("transposed_slice_of_padded_sum", s.text([tr]), [xv], [np.ascontiguousarray(sl.T)]))
    # a strided slice of a concatenation of arguments, read through an elementwise op
    s = Step()
    a, b = s.arg([8, 1, 5], "i32"), s.arg([8, 2, 5], "i32")
    c = s.op("concatenate", [a, b], [8, 3, 5], "i32", "axis = 1 : i64")
    ab = s.op("abs", [c], [8, 3, 5], "i32")
    y = s.op("slice", [ab], [4, 2, 5], "i32",
             f"starts = {arr([0, 1, 0])}, stops = {arr([7, 3, 5])}, steps = {arr([2, 1, 1])}")
    av, bv = rng.integers(-9, 9, (8, 1, 5)).astype(np.int32), rng.integers(-9, 9, (8, 2, 5)).astype(np.int32)
    cases.append(("slice_of_concatenated_arguments", s.text([y]), [av, bv],
                  [np.abs(np.concatenate([av, bv], axis=1))[0:7:2, 1:3, :]]))
    # a pad of a padded computed value: the inner window and mask compose with the outer
    s = Step()
    x = s.arg([3, 2], "i32")
    e = s.op("mul", [x, x], [3, 2], "i32")
    p1 = s.op("pad", [e, s.splat(s.const(4, "i32"), [])], [6, 4], "i32",
              f"pad_low = {arr([1, 0])}, pad_high = {arr([0, 1])}, interior = {arr([1, 0])}")
    p2 = s.op("pad", [p1, s.splat(s.const(-2, "i32"), [])], [13, 7], "i32",
              f"pad_low = {arr([0, 2])}, pad_high = {arr([2, 1])}, interior = {arr([1, 0])}")
    xv = rng.integers(-9, 9, (3, 2)).astype(np.int32)
    inner = np.full((6, 4), 4, np.int32)
    inner[1::2, 0:2] = xv * xv
    outer = np.full((13, 7), -2, np.int32)
    outer[0:11:2, 2:6] = inner
    cases.append(("pad_of_padded_product", s.text([p2]), [xv], [outer]))
    # a concatenation holding a concatenation of arguments and a computed value
    s = Step()
    a, b = s.arg([2, 1, 4], "i32"), s.arg([2, 2, 4], "i32")
    c = s.op("concatenate", [a, b], [2, 3, 4], "i32", "axis = 1 : i64")
    d = s.op("slice", [s.splat(s.const(6, "i32"), [4, 4, 5])], [3, 3, 4], "i32",
             f"starts = {arr([0, 0, 1])}, stops = {arr([3, 3, 5])}, steps = {arr([1, 1, 1])}")
    y = s.op("concatenate", [c, d], [5, 3, 4], "i32", "axis = 0 : i64")
    av, bv = rng.integers(-9, 9, (2, 1, 4)).astype(np.int32), rng.integers(-9, 9, (2, 2, 4)).astype(np.int32)
    cases.append(("concatenation_of_a_concatenation", s.text([y]), [av, bv],
                  [np.concatenate([np.concatenate([av, bv], axis=1), np.full((3, 3, 4), 6, np.int32)], axis=0)]))
    # a slice that reaches into a high pad of an argument
    s = Step()
    x = s.arg([4, 3], "i32")
    pd = s.op("pad", [x, s.splat(s.const(5, "i32"), [])], [4, 7], "i32",
              f"pad_low = {arr([0, 0])}, pad_high = {arr([0, 4])}, interior = {arr([0, 0])}")
    y = s.op("slice", [pd], [4, 3], "i32", f"starts = {arr([0, 1])}, stops = {arr([4, 7])}, steps = {arr([1, 2])}")
    out = s.op("add", [y, s.splat(s.const(0, "i32"), [4, 3])], [4, 3], "i32")
    xv = rng.integers(-9, 9, (4, 3)).astype(np.int32)
    full = np.full((4, 7), 5, np.int32)
    full[:, :3] = xv
    cases.append(("slice_into_a_high_pad", s.text([out]), [xv], [full[:, 1:7:2]]))
    return cases


@pytest.mark.parametrize("case", padded_concat_steps(), ids=lambda c: c[0])
def test_pad_and_concatenate_of_computed_values_lower(case):
    name, src, ins, want = case
    out = rt.lower_step(src)
    assert ask_b200.Plan(out["recipe"], -1).describe()["kernel"] == "ew_view"


@pytest.mark.parametrize("case", padded_concat_steps(), ids=lambda c: c[0])
def test_pad_and_concatenate_of_computed_values_evaluate(case):
    """The lowered recipe, evaluated on the CPU by the recipe evaluator, equals numpy."""
    name, src, ins, want = case
    out = rt.lower_step(src)
    got = recipe_eval.evaluate(out["recipe"], [ins[a] for a in out["input_arguments"]])
    assert np.array_equal(got[0].reshape(want[0].shape), want[0]), name


@pytest.mark.gpu
@pytest.mark.parametrize("case", padded_concat_steps(), ids=lambda c: c[0])
def test_pad_and_concatenate_of_computed_values_on_gpu(device, case):
    import torch
    name, src, ins, want = case
    out = rt.lower_step(src)
    plan = ask_b200.Plan(out["recipe"], 0)
    dev_in = [torch.from_numpy(np.ascontiguousarray(ins[a])).cuda() for a in out["input_arguments"]]
    y = torch.empty(want[0].size, dtype=torch.int32, device="cuda")
    plan.launch(dev_in, [y], None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().reshape(want[0].shape), want[0]), name


@pytest.mark.gpu
@pytest.mark.parametrize("case", view_steps(), ids=lambda c: c[0])
def test_index_map_steps_on_gpu(device, case):
    import torch
    name, src, ins, want = case
    out = rt.lower_step(src)
    plan = ask_b200.Plan(out["recipe"], 0)
    dev_in = [torch.from_numpy(np.ascontiguousarray(ins[a])).cuda() for a in out["input_arguments"]]
    y = torch.empty(want.size, dtype=torch.from_numpy(want).dtype, device="cuda")
    plan.launch(dev_in, [y], None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().reshape(want.shape), want)


def test_marks_lower_as_erased():
    """ask.mark pass-throughs (value and port markers, which the reference's
    prepare phase erases) leave the lowered recipe unchanged."""
    def build(marks):
        s = Step()
        x, y = s.arg([8, 16], "f32"), s.arg([16, 8], "f32")
        if marks:
            x = s.op("mark", [x], [8, 16], "f32", 'mark_id = "m0", role = "input", port_id = "x"')
        t = s.op("transpose", [y], [8, 16], "f32", "permutation = " + arr([1, 0]))
        if marks:
            t = s.op("mark", [t], [8, 16], "f32", 'mark_id = "m1", role = "value", value_id = "t"')
        z = s.op("add", [x, t], [8, 16], "f32")
        r = s.op("reduce_sum", [z], [8], "f32", "axes = " + arr([1]))
        if marks:
            r = s.op("mark", [r], [8], "f32", 'mark_id = "m2", role = "output", port_id = "r"')
        return s.text([r])
    assert rt.lower_step(build(True)) == rt.lower_step(build(False))


def test_malformed_sources_are_invalid():
    for text in ["module {}", "module { func.func @f(%arg0: tensor<?xf32>) -> tensor<?xf32> { return %arg0 : tensor<?xf32> } }"]:
        with pytest.raises(rt.CUDAError) as err:
            rt.lower_step(text)
        assert err.value.status == ask_b200.E_INVALID


def report(sources, buffers, inputs, outputs, steps):
    return {"execution_plan": {"schema_version": 1, "kind": "ask.cuda.execution_plan", "inputs": inputs,
                               "outputs": outputs, "buffers": buffers,
                               "steps": [{"id": f"kernel{k}", "kind": "owned", "function": f"ask_kernel_{k}",
                                          "inputs": i, "outputs": o, "depends_on": []} for k, (i, o) in enumerate(steps)]},
            "step_sources": {f"kernel{k}": src for k, src in enumerate(sources)}}


def softmax_report(dt, rows, cols):
    buffers = [{"id": "v_x", "shape": [rows, cols], "element_type": dt},
               {"id": "v_m", "shape": [rows], "element_type": "f32"},
               {"id": "v_s", "shape": [rows], "element_type": "f32"},
               {"id": "v_y", "shape": [rows, cols], "element_type": dt}]
    return report(cfg3_sources(dt, rows, cols), buffers, ["v_x"], ["v_y"],
                  [(["v_x"], ["v_m"]), (["v_x", "v_m"], ["v_s"]), (["v_x", "v_m", "v_s"], ["v_y"])])


def scatter_report(rows, dim, n):
    g, s = cfg4_sources(rows, dim, n)
    buffers = [{"id": "table", "shape": [rows, dim], "element_type": "f32"},
               {"id": "idx", "shape": [n], "element_type": "i64"},
               {"id": "base", "shape": [rows, dim], "element_type": "f32"},
               {"id": "g", "shape": [n, dim], "element_type": "f32"},
               {"id": "out", "shape": [rows, dim], "element_type": "f32"}]
    return report([g, s], buffers, ["table", "idx", "base"], ["out"],
                  [(["table", "idx"], ["g"]), (["base", "idx", "g"], ["out"])])


def test_report_lowers_to_a_program():
    prog = rt.lower_report(softmax_report("f16", 32768, 4096))
    assert prog["buffer_sizes"] == [2 * 32768 * 4096, 4 * 32768, 4 * 32768, 2 * 32768 * 4096]
    assert prog["inputs"] == [0] and prog["outputs"] == [3]
    assert [s["inputs"] for s in prog["steps"]] == [[0], [0, 1], [0, 1, 2]]
    assert [kernel_of(json.loads(s["recipe"])) for s in prog["steps"]] == [
        "softmax_rows_max_f16", "softmax_rows_sum_f16", "softmax_rows_norm_f16"]
    prog = rt.lower_report(scatter_report(1 << 20, 256, 1 << 23))
    assert [s["inputs"] for s in prog["steps"]] == [[0, 1], [2, 1, 3]]


def mixed_results_step(rows=6, cols=10):
    """One step returning row sums [rows], column sums [cols], a row maximum
    [rows] and two elementwise results [rows, cols] of the same argument."""
    s = Step()
    x = s.arg([rows, cols], "i32")
    y = s.op("mul", [x, s.splat(s.const(2, "i32"), [rows, cols])], [rows, cols], "i32")
    outs = [s.op("reduce_sum", [x], [rows], "i32", "axes = " + arr([1])),
            s.op("reduce_sum", [x], [cols], "i32", "axes = " + arr([0])),
            y,
            s.op("reduce_max", [x], [rows], "i32", "axes = " + arr([1])),
            s.op("abs", [x], [rows, cols], "i32")]
    return s.text(outs)


def test_steps_with_mixed_results_lower_to_one_recipe_per_group():
    """A step whose results one recipe cannot hold together (reductions over
    different axes and elementwise results) becomes one program step per
    group -- row reductions, column reductions, elementwise -- each writing
    its own outputs; every recipe evaluated on the CPU equals numpy."""
    rows, cols = 6, 10
    buffers = [{"id": "v_x", "shape": [rows, cols], "element_type": "i32"},
               {"id": "v_r", "shape": [rows], "element_type": "i32"},
               {"id": "v_c", "shape": [cols], "element_type": "i32"},
               {"id": "v_y", "shape": [rows, cols], "element_type": "i32"},
               {"id": "v_m", "shape": [rows], "element_type": "i32"},
               {"id": "v_a", "shape": [rows, cols], "element_type": "i32"}]
    rep = report([mixed_results_step(rows, cols)], buffers, ["v_x"], ["v_r", "v_c", "v_y", "v_m", "v_a"],
                 [(["v_x"], ["v_r", "v_c", "v_y", "v_m", "v_a"])])
    prog = rt.lower_report(rep)
    assert [s["id"] for s in prog["steps"]] == ["kernel0#0", "kernel0#1", "kernel0#2"]
    ok, why = rt.check_allocation({"buffer_count": len(prog["buffer_sizes"]), "public_inputs": prog["inputs"],
                                   "public_outputs": prog["outputs"],
                                   "steps": [{"inputs": s["inputs"], "outputs": s["outputs"]} for s in prog["steps"]]})
    assert ok, why
    assert [s["outputs"] for s in prog["steps"]] == [[1, 4], [2], [3, 5]]
    x = np.random.default_rng(4).integers(-50, 50, (rows, cols)).astype(np.int32)
    want = {1: x.sum(axis=1), 2: x.sum(axis=0), 3: 2 * x, 4: x.max(axis=1), 5: np.abs(x)}
    for st in prog["steps"]:
        rec = json.loads(st["recipe"])
        ask_b200.Plan(rec, -1)
        got = recipe_eval.evaluate(rec, [x for _ in st["inputs"]])
        for g, b in zip(got, st["outputs"]):
            assert np.array_equal(g, want[b].astype(np.int32).reshape(-1)), b
    # a step that one recipe holds stays one program step with its own id
    single = report([cfg1_source(64)], [{"id": f"v{k}", "shape": [64], "element_type": "f32"} for k in range(5)],
                    ["v0", "v1", "v2"], ["v3", "v4"], [(["v0", "v1", "v2"], ["v3", "v4"])])
    assert [s["id"] for s in rt.lower_report(single)["steps"]] == ["kernel0"]


def run_program_on_cpu(prog, inputs, dtypes):
    """Runs a lowered program's steps in order on the CPU (test helper):
    elementwise and reduce recipes through the recipe evaluator, gather and
    scatter_add through the oracle.  `dtypes` gives each buffer's numpy type."""
    import oracle
    bufs = {b: np.ascontiguousarray(v).reshape(-1) for b, v in zip(prog["inputs"], inputs)}
    for st in prog["steps"]:
        rec = json.loads(st["recipe"])
        ask_b200.Plan(rec, -1)
        args = [bufs[b] for b in st["inputs"]]
        if rec["family"] == "gather":
            got = [oracle.gather(args[0], args[1], rec["outer"], rec["dim"], rec["inner"])]
        elif rec["family"] == "scatter_add":
            got = [oracle.scatter_add(rec["dtype"], args[0], args[1], args[2], rec["outer"], rec["dim"], rec["inner"])]
        else:
            got = recipe_eval.evaluate(rec, args)
        for b, g in zip(st["outputs"], got):
            bufs[b] = np.asarray(g).astype(dtypes[b]).reshape(-1)
    return bufs


def test_gather_and_scatter_of_computed_operands():
    """A step gathering rows of a computed table at a computed index, and
    a step scattering computed updates, lower to elementwise steps writing
    internal buffers followed by the gather/scatter_add step; the program,
    run step by step on the CPU, equals numpy."""
    rows, dim, n = 40, 8, 300
    g = Step("ask_kernel_0", "kernel0")
    t, i = g.arg([rows, dim], "i32"), g.arg([n], "i64")
    t2 = g.op("add", [g.op("mul", [t, g.splat(g.const(2, "i32"), [rows, dim])], [rows, dim], "i32"),
                      g.splat(g.const(1, "i32"), [rows, dim])], [rows, dim], "i32")
    i2 = g.op("add", [i, g.splat(g.const(3, "i64"), [n])], [n], "i64")
    gsrc = g.text([g.op("gather", [t2, i2], [n, dim], "i32", "axis = 0 : i64")])
    s = Step("ask_kernel_1", "kernel1")
    base, idx, upd = s.arg([rows, dim], "i32"), s.arg([n], "i64"), s.arg([n, dim], "i32")
    u2 = s.op("abs", [upd], [n, dim], "i32")
    ssrc = s.text([s.op("scatter_add", [base, idx, u2], [rows, dim], "i32", "axis = 0 : i64")])
    buffers = [{"id": "table", "shape": [rows, dim], "element_type": "i32"},
               {"id": "idx", "shape": [n], "element_type": "i64"},
               {"id": "base", "shape": [rows, dim], "element_type": "i32"},
               {"id": "g", "shape": [n, dim], "element_type": "i32"},
               {"id": "out", "shape": [rows, dim], "element_type": "i32"}]
    rep = report([gsrc, ssrc], buffers, ["table", "idx", "base"], ["out"],
                 [(["table", "idx"], ["g"]), (["base", "idx", "g"], ["out"])])
    prog = rt.lower_report(rep)
    # table * 2 + 1 and idx + 3 into internal buffers 5 and 6, then the gather;
    # |g| into internal buffer 7, then the scatter_add
    assert [st["id"] for st in prog["steps"]] == ["kernel0#0", "kernel0#1", "kernel0#2", "kernel1#0", "kernel1#1"]
    assert len(prog["buffer_sizes"]) == 8 and prog["buffer_sizes"][5:] == [4 * rows * dim, 8 * n, 4 * n * dim]
    assert [st["outputs"] for st in prog["steps"]] == [[5], [6], [3], [7], [4]]
    assert prog["steps"][2]["inputs"] == [5, 6] and prog["steps"][4]["inputs"] == [2, 1, 7]
    ok, why = rt.check_allocation({"buffer_count": len(prog["buffer_sizes"]), "public_inputs": prog["inputs"],
                                   "public_outputs": prog["outputs"],
                                   "steps": [{"inputs": st["inputs"], "outputs": st["outputs"]} for st in prog["steps"]]})
    assert ok, why
    rng = np.random.default_rng(8)
    tv = rng.integers(-9, 9, (rows, dim)).astype(np.int32)
    iv = rng.integers(-6, rows, n).astype(np.int64)  # idx + 3 falls outside [0, rows) at both ends
    bv = rng.integers(-9, 9, (rows, dim)).astype(np.int32)
    dtypes = {0: np.int32, 1: np.int64, 2: np.int32, 3: np.int32, 4: np.int32, 5: np.int32, 6: np.int64, 7: np.int32}
    bufs = run_program_on_cpu(prog, [tv, iv, bv], dtypes)
    table2, idx2 = tv * 2 + 1, iv + 3
    ok_rows = (idx2 >= 0) & (idx2 < rows)
    want_g = np.zeros((n, dim), np.int32)
    want_g[ok_rows] = table2[idx2[ok_rows]]
    assert np.array_equal(bufs[3].reshape(n, dim), want_g)
    want_out = bv.copy()
    in_range = (iv >= 0) & (iv < rows)
    np.add.at(want_out, iv[in_range], np.abs(want_g[in_range]))
    assert np.array_equal(bufs[4].reshape(rows, dim), want_out)


def test_marked_and_shared_scatter_operands():
    """A scatter_add whose operands are an ask.mark of an argument (erased, as
    the reference's prepare phase erases marks) and one computed value used
    twice (base and updates of the same shape) lowers to one elementwise step
    into one internal buffer and the scatter_add step; a marked gather result
    stays a gather step."""
    rows, dim = 16, 8
    s = Step("ask_kernel_0", "kernel0")
    x, idx = s.arg([rows, dim], "i32"), s.arg([rows], "i64")
    mi = s.op("mark", [idx], [rows], "i64", 'mark_id = "m0", role = "input", port_id = "idx"')
    c = s.op("mul", [x, s.splat(s.const(3, "i32"), [rows, dim])], [rows, dim], "i32")
    out = s.op("scatter_add", [c, mi, c], [rows, dim], "i32", "axis = 0 : i64")
    out = s.op("mark", [out], [rows, dim], "i32", 'mark_id = "m1", role = "output", port_id = "out"')
    buffers = [{"id": "x", "shape": [rows, dim], "element_type": "i32"},
               {"id": "idx", "shape": [rows], "element_type": "i64"},
               {"id": "out", "shape": [rows, dim], "element_type": "i32"}]
    prog = rt.lower_report(report([s.text([out])], buffers, ["x", "idx"], ["out"], [(["x", "idx"], ["out"])]))
    assert [st["id"] for st in prog["steps"]] == ["kernel0#0", "kernel0#1"]
    assert prog["buffer_sizes"] == [4 * rows * dim, 8 * rows, 4 * rows * dim, 4 * rows * dim]  # one internal buffer
    assert [st["outputs"] for st in prog["steps"]] == [[3], [2]]
    assert prog["steps"][1]["inputs"] == [3, 1, 3]  # the mark's argument read directly
    rng = np.random.default_rng(3)
    xv = rng.integers(-9, 9, (rows, dim)).astype(np.int32)
    iv = rng.integers(-2, rows + 2, rows).astype(np.int64)
    bufs = run_program_on_cpu(prog, [xv, iv], {0: np.int32, 1: np.int64, 2: np.int32, 3: np.int32})
    want = 3 * xv
    ok = (iv >= 0) & (iv < rows)
    np.add.at(want, iv[ok], (3 * xv)[ok])
    assert np.array_equal(bufs[2].reshape(rows, dim), want)
    g = Step("ask_kernel_0", "kernel0")
    t, i = g.arg([rows, dim], "i32"), g.arg([4], "i64")
    gm = g.op("mark", [g.op("gather", [t, i], [4, dim], "i32", "axis = 0 : i64")], [4, dim], "i32",
              'mark_id = "m2", role = "output", port_id = "g"')
    step = rt.lower_step(g.text([gm]))
    assert step["recipe"]["family"] == "gather" and step["input_arguments"] == [0, 1]


def random_mixed_step(seed):
    """A rank-3 i32 argument with results: a sum and a max over random axis
    sets (scattered ones included), an elementwise value and a strided slice
    of another shape.  Returns (source, argument, [expected results], result
    shapes)."""
    rng = np.random.default_rng(seed)
    shape = [int(x) for x in rng.integers(2, 6, 3)]
    s = Step()
    x = s.arg(shape, "i32")
    xv = rng.integers(-30, 30, shape).astype(np.int32)
    results, want = [], []
    for op, f in (("reduce_sum", np.sum), ("reduce_max", np.max)):
        axes = sorted(int(a) for a in rng.choice(3, int(rng.integers(1, 3)), replace=False))
        kept = [shape[d] for d in range(3) if d not in axes]
        results.append(s.op(op, [x], kept, "i32", "axes = " + arr(axes)))
        want.append(f(xv, axis=tuple(axes)).astype(np.int32))
    results.append(s.op("mul", [x, s.splat(s.const(3, "i32"), shape)], shape, "i32"))
    want.append(xv * 3)
    sl_shape = [(d + 1) // 2 for d in shape]
    results.append(s.op("slice", [x], sl_shape, "i32", f"starts = {arr([0, 0, 0])}, stops = {arr(shape)}, "
                                                     f"steps = {arr([2, 2, 2])}"))
    want.append(xv[::2, ::2, ::2])
    return s.text(results), xv, want, [list(w.shape) for w in want]


def test_random_mixed_steps_through_reports():
    """Random steps mixing reductions over different (and scattered) axis
    sets with elementwise and sliced results lower through a partition report
    to one program step per group, pass the plan verifier, and, run step by
    step on the CPU, give numpy's results."""
    for seed in range(60):
        src, xv, want, shapes = random_mixed_step(seed)
        buffers = [{"id": "x", "shape": list(xv.shape), "element_type": "i32"}] + \
                  [{"id": f"r{k}", "shape": sh, "element_type": "i32"} for k, sh in enumerate(shapes)]
        outs = [f"r{k}" for k in range(len(shapes))]
        prog = rt.lower_report(report([src], buffers, ["x"], outs, [(["x"], outs)]))
        ok, why = rt.check_allocation({"buffer_count": len(prog["buffer_sizes"]), "public_inputs": prog["inputs"],
                                       "public_outputs": prog["outputs"],
                                       "steps": [{"inputs": st["inputs"], "outputs": st["outputs"]}
                                                 for st in prog["steps"]]})
        assert ok, (seed, why)
        bufs = run_program_on_cpu(prog, [xv], {b: np.int32 for b in range(len(prog["buffer_sizes"]))})
        for k, w in enumerate(want):
            assert np.array_equal(bufs[1 + k], w.reshape(-1)), (seed, k)


def test_non_owned_steps_stay_for_the_caller():
    """An external or library step is not lowered: it keeps its buffers and is
    listed as unresolved, for the caller to bind a loaded kernel to it; a step
    of unknown kind is invalid."""
    r = softmax_report("f16", 8, 16)
    r["execution_plan"]["steps"][1]["kind"] = "external"
    prog = rt.lower_report(r)
    assert prog["unresolved_steps"] == ["kernel1"]
    assert prog["steps"][1] == {"id": "kernel1", "unresolved": {"kind": "external", "function": "ask_kernel_1"},
                                "inputs": [0, 1], "outputs": [2]}
    r["execution_plan"]["steps"][1]["kind"] = "fused"
    with pytest.raises(rt.CUDAError) as err:
        rt.lower_report(r)
    assert err.value.status == ask_b200.E_INVALID


# ---- on the GPU: lowered programs against the hand-written recipes ------------------------
@pytest.mark.gpu
@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_lowered_softmax_program_matches_hand_recipes(device, graph, dt):
    import torch
    from gpu_util import gen_dev
    rows, cols = 256, 4096
    x = gen_dev(2 if dt == "f16" else 3, 0xA5C3, 0, rows * cols, 0.0, 2.0, torch.int16)
    session = rt.Session.create(0)
    hand = session.prepareProgram(
        [2 * rows * cols, 4 * rows, 4 * rows, 2 * rows * cols], [0], [3],
        [rt.PlanStep(s, i, o) for s, i, o in zip(R.cfg3_steps(dt, rows, cols), [[0], [0, 1], [0, 1, 2]], [[1], [2], [3]])],
        graph)
    lowered = rt.prepare_report(session, softmax_report(dt, rows, cols), graph)
    xin = session.importTensor(x, readonly=True)
    session.waitForExternalStream(torch.cuda.current_stream())
    (a,), ea = hand.run([xin])
    (b,), eb = lowered.run([xin])
    ea.wait()
    eb.wait()
    assert a.copyToHost() == b.copyToHost()


@pytest.mark.gpu
@pytest.mark.parametrize("graph", [False, True])
def test_lowered_gather_scatter_program(device, graph):
    import torch
    from gpu_util import gen_dev
    rows, dim, n = 2048, 64, 20000
    table = (gen_dev(4, 0xA5C4, 0, rows * dim, 0, 0, torch.int32) % 1000).float()  # small integers
    idx = gen_dev(5, 0xA5C4, 1, n, 1.1, rows, torch.int64)
    base = torch.zeros(rows * dim, dtype=torch.float32, device="cuda")
    session = rt.Session.create(0)
    program = rt.prepare_report(session, scatter_report(rows, dim, n), graph)
    ins = [session.importTensor(t, readonly=True) for t in (table, idx, base)]
    session.waitForExternalStream(torch.cuda.current_stream())
    (out,), ev = program.run(ins)
    ev.wait()
    got = np.frombuffer(out.copyToHost(), np.float32).reshape(rows, dim)
    t, ix = table.view(rows, dim).cpu().numpy().astype(np.float64), idx.cpu().numpy()
    want = np.zeros((rows, dim))
    np.add.at(want, ix, t[ix])
    # integer-valued f32 updates: every partial sum is exact, so the result is too
    assert np.array_equal(got, want.astype(np.float32))


# ---- random steps: elementwise ops and index maps, against numpy ---------------------------
def random_map_step(seed, depth=3):
    """A random i32 step mixing elementwise ops with transpose, slice,
    broadcast_in_dim and reshape of arguments and of computed values.
    Returns (source, argument arrays, expected result)."""
    rng = np.random.default_rng(seed)
    s = Step()
    args = []

    def leaf(shape):
        if rng.random() < 0.2:
            c = int(rng.integers(-5, 6))
            return s.splat(s.const(c, "i32"), list(shape)), np.full(shape, c, np.int32)
        v = rng.integers(-20, 21, shape).astype(np.int32)
        args.append(v)
        return s.arg(list(shape), "i32"), v

    def gen(shape, d):
        r = rng.random()
        if d == 0 or r < 0.2:
            return leaf(shape)
        if r < 0.5:
            op = ["add", "mul", "maximum", "minimum"][int(rng.integers(4))]
            (a, av), (b, bv) = gen(shape, d - 1), gen(shape, d - 1)
            f = {"add": np.add, "mul": np.multiply, "maximum": np.maximum, "minimum": np.minimum}[op]
            return s.op(op, [a, b], list(shape), "i32"), f(av, bv).astype(np.int32)
        if r < 0.6:
            a, av = gen(shape, d - 1)
            return s.op("abs", [a], list(shape), "i32"), np.abs(av).astype(np.int32)
        if r < 0.72 and len(shape) > 1:
            perm = [int(x) for x in rng.permutation(len(shape))]
            inner = [0] * len(shape)
            for dd, p in enumerate(perm):
                inner[p] = shape[dd]
            a, av = gen(inner, d - 1)
            return s.op("transpose", [a], list(shape), "i32", "permutation = " + arr(perm)), np.transpose(av, perm)
        if r < 0.84:
            starts = [int(rng.integers(0, 3)) for _ in shape]
            steps = [int(rng.integers(1, 3)) for _ in shape]
            inner = [st + (n - 1) * sp + 1 + int(rng.integers(0, 2)) for st, sp, n in zip(starts, steps, shape)]
            stops = [st + (n - 1) * sp + 1 for st, sp, n in zip(starts, steps, shape)]
            a, av = gen(inner, d - 1)
            sl = tuple(slice(st, sp_, stp) for st, sp_, stp in zip(starts, stops, steps))
            return (s.op("slice", [a], list(shape), "i32",
                         f"starts = {arr(starts)}, stops = {arr(stops)}, steps = {arr(steps)}"), av[sl])
        if r < 0.94:
            keep = [dd for dd in range(len(shape)) if rng.random() < 0.6]
            inner = [shape[dd] for dd in keep]
            a, av = gen(inner, d - 1)
            bv = np.broadcast_to(av.reshape([shape[dd] if dd in keep else 1 for dd in range(len(shape))]), shape)
            return (s.op("broadcast_in_dim", [a], list(shape), "i32",
                         f"dimensions = {arr(keep)}, shape = {arr(shape)}"), np.ascontiguousarray(bv))
        if r < 0.97:
            # from a flat vector, or from the same extents in another order
            # (whose operand may then be transposed, sliced or padded)
            n = int(np.prod(shape))
            inner = [n] if rng.random() < 0.5 else [int(x) for x in rng.permutation(shape)]
            a, av = gen(inner, d - 1)
            return s.op("reshape", [a], list(shape), "i32", f"shape = {arr(shape)}"), av.reshape(shape)
        if r < 0.985:
            low = [int(rng.integers(0, 2)) for _ in shape]
            interior = [int(rng.integers(0, 2)) if n > 1 else 0 for n in shape]
            inner = [max(1, (n - lo + it) // (it + 1)) for n, lo, it in zip(shape, low, interior)]
            high = [n - lo - (m - 1) * (it + 1) - 1 for n, lo, m, it in zip(shape, low, inner, interior)]
            a, av = gen(inner, d - 1)
            c = int(rng.integers(-5, 6))
            pv = s.splat(s.const(c, "i32"), [])
            out = np.full(shape, c, np.int32)
            out[tuple(slice(lo, lo + (m - 1) * (it + 1) + 1, it + 1) for lo, m, it in zip(low, inner, interior))] = av
            return (s.op("pad", [a, pv], list(shape), "i32",
                         f"pad_low = {arr(low)}, pad_high = {arr(high)}, interior = {arr(interior)}"), out)
        axis = int(rng.integers(0, len(shape)))
        if shape[axis] < 2:
            return leaf(shape)
        cut = int(rng.integers(1, shape[axis]))
        s1, s2 = list(shape), list(shape)
        s1[axis], s2[axis] = cut, shape[axis] - cut
        (a, av), (b, bv) = gen(s1, d - 1), gen(s2, d - 1)
        return (s.op("concatenate", [a, b], list(shape), "i32", f"axis = {axis} : i64"),
                np.concatenate([av, bv], axis=axis))

    shape = [int(x) for x in rng.integers(2, 6, int(rng.integers(2, 4)))]
    y, yv = gen(shape, depth)
    if not args:  # a step reads at least one argument
        a, av = leaf(shape)
        while not args:
            a, av = leaf(shape)
        y, yv = s.op("add", [y, a], list(shape), "i32"), (yv + av).astype(np.int32)
    return s.text([y]), args, yv


def _lower_random(seed):
    src, args, want = random_map_step(seed)
    try:
        return rt.lower_step(src), args, want
    except rt.CUDAError as e:
        assert e.status == ask_b200.E_UNSUPPORTED, str(e)
        return None, args, want


def test_random_map_steps_lower():
    lowered = 0
    for seed in range(60):
        out, args, want = _lower_random(seed)
        if out is not None:
            ask_b200.Plan(out["recipe"], -1)
            lowered += 1
    assert lowered >= 40, lowered


def test_random_map_steps_evaluate():
    """400 random steps: at least 95% lower, and every lowered recipe,
    evaluated on the CPU by the recipe evaluator, equals numpy."""
    lowered = 0
    for seed in range(400):
        out, args, want = _lower_random(seed)
        if out is None:
            continue
        ask_b200.Plan(out["recipe"], -1)
        got = recipe_eval.evaluate(out["recipe"], [args[a] for a in out["input_arguments"]])
        assert np.array_equal(got[0].astype(np.int32), want.reshape(-1)), seed
        lowered += 1
    assert lowered >= 390, lowered


@pytest.mark.gpu
def test_random_map_steps_on_gpu(device):
    import torch
    checked = 0
    for seed in range(60):
        out, args, want = _lower_random(seed)
        if out is None:
            continue
        plan = ask_b200.Plan(out["recipe"], 0)
        dev_in = [torch.from_numpy(np.ascontiguousarray(args[a])).cuda() for a in out["input_arguments"]]
        y = torch.empty(want.size, dtype=torch.int32, device="cuda")
        plan.launch(dev_in, [y], None, torch.cuda.current_stream())
        torch.cuda.synchronize()
        assert np.array_equal(y.cpu().numpy(), want.reshape(-1)), seed
        checked += 1
    assert checked >= 40


def strided_view_step(seed, dt="i32"):
    """A step over [batch..., R, C] adding transposed arguments (stored
    [batch..., C, R]), a straight strided slice, a full argument, a scalar and
    a view that moves a batch axis.  Returns (source, arrays, expected,
    number of transposed reads)."""
    rng = np.random.default_rng(seed)
    batch = [int(x) for x in rng.integers(1, 4, int(rng.integers(0, 3)))]
    R, C = int(rng.integers(1, 80)), int(rng.integers(2, 80))
    shape = batch + [R, C]
    rank = len(shape)
    npdt = {"i32": np.int32, "i64": np.int64, "f16": np.float16}[dt]
    s = Step()
    terms, arrays, values = [], [], []

    def arg(sh):
        v = rng.integers(-9, 10, sh).astype(npdt)
        arrays.append(v)
        return s.arg(list(sh), dt), v

    n_t = int(rng.integers(0, 5))
    for _ in range(n_t):  # transposed: the argument's last two axes swapped
        a, av = arg(batch + [C, R])
        perm = list(range(len(batch))) + [rank - 1, rank - 2]
        terms.append(s.op("transpose", [a], shape, dt, "permutation = " + arr(perm)))
        values.append(np.transpose(av, perm))
    if rng.random() < 0.6:  # a straight strided slice (step 1, an offset)
        a, av = arg([d + 2 for d in shape])
        terms.append(s.op("slice", [a], shape, dt, f"starts = {arr([1] * rank)}, stops = {arr([d + 1 for d in shape])}, "
                                                  f"steps = {arr([1] * rank)}"))
        values.append(av[tuple(slice(1, d + 1) for d in shape)])
    if rng.random() < 0.5:
        a, av = arg(shape)
        terms.append(a)
        values.append(av)
    if batch and rng.random() < 0.5:  # a batch axis moved past R: still contiguous along C
        a, av = arg([R] + batch + [C])
        perm = list(range(1, len(batch) + 1)) + [0, rank - 1]
        terms.append(s.op("transpose", [a], shape, dt, "permutation = " + arr(perm)))
        values.append(np.transpose(av, perm))
    if not terms:
        a, av = arg(shape)
        terms.append(a)
        values.append(av)
    y, want = terms[0], values[0].copy()
    for tm, v in zip(terms[1:], values[1:]):
        y = s.op("add", [y, tm], shape, dt)
        want = (want + v).astype(npdt)
    return s.text([y]), arrays, want, n_t


def test_strided_views_evaluate():
    """Steps adding transposed, sliced, batch-permuted, full and scalar reads
    lower (to the view kernel when a transposed read remains) and equal numpy."""
    for seed in range(150):
        src, args, want, n_t = strided_view_step(seed)
        out = rt.lower_step(src)
        kernel = ask_b200.Plan(out["recipe"], -1).describe()["kernel"]
        assert kernel in ("ew_view", "ew_generic"), (seed, kernel)
        if n_t and want.shape[-1] > 1 and want.shape[-2] > 1:
            assert kernel == "ew_view", seed
        got = recipe_eval.evaluate(out["recipe"], [args[a] for a in out["input_arguments"]])
        assert np.array_equal(got[0].reshape(want.shape), want), seed


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ["i32", "i64", "f16"])
def test_strided_views_on_gpu(device, dt):
    import torch
    from gpu_util import NUMPY
    for seed in range(60):
        src, args, want, _ = strided_view_step(seed, dt)
        out = rt.lower_step(src)
        plan = ask_b200.Plan(out["recipe"], 0)
        dev_in = [torch.from_numpy(np.ascontiguousarray(args[a]).view(NUMPY[dt])).cuda() for a in out["input_arguments"]]
        y = torch.empty(want.size, dtype=dev_in[0].dtype, device="cuda")
        plan.launch(dev_in, [y], None, torch.cuda.current_stream())
        torch.cuda.synchronize()
        assert np.array_equal(y.cpu().numpy().view(want.dtype).reshape(want.shape), want), (dt, seed)


def _factor_shape(rng, n):
    """A random shape (rank 1..4) whose extents multiply to n."""
    dims, left = [], n
    for _ in range(int(rng.integers(0, 3))):
        divs = [d for d in range(1, left + 1) if left % d == 0]
        d = int(rng.choice(divs))
        dims.append(d)
        left //= d
    dims.append(left)
    return [int(x) for x in rng.permutation(dims)]


def random_reshape_step(seed):
    """An i32 argument read through a transpose, strided slice or broadcast,
    then reshaped to a random shape of the same size, plus one.  Returns
    (source, argument arrays, expected result)."""
    rng = np.random.default_rng(seed)
    s = Step()
    shape = [int(x) for x in rng.integers(1, 6, int(rng.integers(2, 4)))]
    kind = ["transpose", "slice", "broadcast"][seed % 3]
    if kind == "transpose":
        perm = [int(x) for x in rng.permutation(len(shape))]
        src_shape = [0] * len(shape)
        for d, p_ in enumerate(perm):
            src_shape[p_] = shape[d]
        x = s.arg(src_shape, "i32")
        xv = rng.integers(-50, 50, src_shape).astype(np.int32)
        v = s.op("transpose", [x], shape, "i32", "permutation = " + arr(perm))
        vv = np.transpose(xv, perm)
    elif kind == "slice":
        steps = [int(rng.integers(1, 3)) for _ in shape]
        starts = [int(rng.integers(0, 2)) for _ in shape]
        src_shape = [st + (n - 1) * sp + 1 + int(rng.integers(0, 2)) for st, sp, n in zip(starts, steps, shape)]
        stops = [st + (n - 1) * sp + 1 for st, sp, n in zip(starts, steps, shape)]
        x = s.arg(src_shape, "i32")
        xv = rng.integers(-50, 50, src_shape).astype(np.int32)
        v = s.op("slice", [x], shape, "i32", f"starts = {arr(starts)}, stops = {arr(stops)}, steps = {arr(steps)}")
        vv = xv[tuple(slice(a, b, c) for a, b, c in zip(starts, stops, steps))]
    else:
        keep = sorted(set(int(d) for d in rng.choice(len(shape), int(rng.integers(1, len(shape))), replace=False)))
        src_shape = [shape[d] for d in keep]
        x = s.arg(src_shape, "i32")
        xv = rng.integers(-50, 50, src_shape).astype(np.int32)
        v = s.op("broadcast_in_dim", [x], shape, "i32", f"dimensions = {arr(keep)}, shape = {arr(shape)}")
        vv = np.broadcast_to(xv.reshape([shape[d] if d in keep else 1 for d in range(len(shape))]), shape)
    to = _factor_shape(rng, int(np.prod(shape)))
    r = s.op("reshape", [v], to, "i32", f"shape = {arr(to)}")
    y = s.op("add", [r, s.splat(s.const(1, "i32"), to)], to, "i32")
    nocopy = vv.view()
    try:
        nocopy.shape = to  # numpy refuses when the reshape would need a copy
    except AttributeError:
        nocopy = None
    return s.text([y]), [xv], np.ascontiguousarray(vv).reshape(to) + 1, nocopy is not None


def _lower_reshape(seed):
    src, args, want, strided = random_reshape_step(seed)
    try:
        return rt.lower_step(src), args, want, strided
    except rt.CUDAError as e:
        assert e.status == ask_b200.E_UNSUPPORTED, str(e)
        return None, args, want, strided


def test_reshapes_of_views_evaluate():
    """Every reshape of a transposed, sliced or broadcast argument lowers: to
    one strided view whenever numpy can reshape that view without a copy (the
    axes merged or split nest in memory), otherwise through an inner window at
    the same row-major position; each equals numpy."""
    inner = 0
    for seed in range(300):
        out, args, want, strided = _lower_reshape(seed)
        assert out is not None, seed
        r = out["recipe"]
        views = [p["view"] for p in r["inputs"] if p.get("map") == "view"]
        if any("inner" in v for v in views):
            assert not strided, seed  # a reshape numpy makes without a copy needs no inner window
            inner += 1
        ask_b200.Plan(r, -1)
        got = recipe_eval.evaluate(r, [args[a] for a in out["input_arguments"]])
        assert np.array_equal(got[0], want.reshape(-1)), seed
    assert inner >= 50, inner


@pytest.mark.gpu
def test_reshapes_of_views_on_gpu(device):
    import torch
    checked = 0
    for seed in range(120):
        out, args, want, _ = _lower_reshape(seed)
        if out is None:
            continue
        plan = ask_b200.Plan(out["recipe"], 0)
        dev_in = [torch.from_numpy(np.ascontiguousarray(args[a])).cuda() for a in out["input_arguments"]]
        y = torch.empty(want.size, dtype=torch.int32, device="cuda")
        plan.launch(dev_in, [y], None, torch.cuda.current_stream())
        torch.cuda.synchronize()
        assert np.array_equal(y.cpu().numpy(), want.reshape(-1)), seed
        checked += 1
    assert checked >= 45, checked


def broadcast_steps():
    """Rank-preserving broadcasts (a [rows, 1] column, a [1, cols] row, a
    [1, 1] scalar, a transposed column) added to a full argument, f32: these
    read through the fast vector maps, not the view interpreter."""
    rng = np.random.default_rng(9)
    cases = []
    for name, bshape, dims, want_map in (("column", [32, 1], [0, 1], "outer"), ("row", [1, 64], [0, 1], "inner"),
                                         ("scalar", [1, 1], [0, 1], "scalar"), ("row_rank3", [1, 1, 64], [0, 1, 2], "inner"),
                                         ("column_rank3", [2, 16, 1], [0, 1, 2], "outer")):
        shape = [32, 64] if len(bshape) == 2 else [2, 16, 64]
        s = Step()
        x, b = s.arg(shape, "f32"), s.arg(bshape, "f32")
        bc = s.op("broadcast_in_dim", [b], shape, "f32", f"dimensions = {arr(dims)}, shape = {arr(shape)}")
        y = s.op("add", [x, bc], shape, "f32")
        xv = rng.integers(-50, 50, shape).astype(np.float32)
        bv = rng.integers(-50, 50, bshape).astype(np.float32)
        cases.append((name, s.text([y]), [xv, bv], xv + bv, want_map))
    # a [64, 1] column read through a transpose as a row of the [32, 64] output
    s = Step()
    x, b = s.arg([32, 64], "f32"), s.arg([64, 1], "f32")
    t = s.op("transpose", [b], [1, 64], "f32", "permutation = " + arr([1, 0]))
    bc = s.op("broadcast_in_dim", [t], [32, 64], "f32", f"dimensions = {arr([0, 1])}, shape = {arr([32, 64])}")
    y = s.op("add", [x, bc], [32, 64], "f32")
    xv = rng.integers(-50, 50, (32, 64)).astype(np.float32)
    bv = rng.integers(-50, 50, (64, 1)).astype(np.float32)
    cases.append(("transposed_column_as_row", s.text([y]), [xv, bv], xv + bv.T, "inner"))
    return cases


@pytest.mark.parametrize("case", broadcast_steps(), ids=lambda c: c[0])
def test_rank_preserving_broadcasts_use_fast_maps(case):
    name, src, ins, want, want_map = case
    out = rt.lower_step(src)
    assert [p["map"] for p in out["recipe"]["inputs"]] == ["full", want_map]
    assert ask_b200.Plan(out["recipe"], -1).describe()["kernel"] == "ew_generic"
    got = recipe_eval.evaluate(out["recipe"], [ins[a] for a in out["input_arguments"]])
    assert np.array_equal(got[0].reshape(want.shape), want)


@pytest.mark.gpu
@pytest.mark.parametrize("case", broadcast_steps(), ids=lambda c: c[0])
def test_rank_preserving_broadcasts_on_gpu(device, case):
    import torch
    name, src, ins, want, _ = case
    out = rt.lower_step(src)
    plan = ask_b200.Plan(out["recipe"], 0)
    dev_in = [torch.from_numpy(np.ascontiguousarray(ins[a])).cuda() for a in out["input_arguments"]]
    y = torch.empty(want.size, dtype=torch.float32, device="cuda")
    plan.launch(dev_in, [y], None, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().reshape(want.shape), want), name


def permuted_reduce_step(seed):
    """An i32 argument read through a random axis permutation (plus one) and
    reduced over a random block of axes with sum, max, min and, over one axis,
    argmax.  Returns (source, [argument], expected results, whether the
    reduction maps onto the argument's own axes)."""
    rng = np.random.default_rng(seed)
    rank = int(rng.integers(2, 5))
    ashape = [int(x) for x in rng.integers(2, 7, rank)]
    perm = [int(x) for x in rng.permutation(rank)]
    tshape = [ashape[p_] for p_ in perm]
    a0 = int(rng.integers(0, rank))
    a1 = a0 + 1 if rng.random() < 0.6 else int(rng.integers(a0 + 1, rank + 1))
    axes = list(range(a0, a1))
    s = Step()
    x = s.arg(ashape, "i32")
    t = s.op("transpose", [x], tshape, "i32", "permutation = " + arr(perm))
    y = s.op("add", [t, s.splat(s.const(1, "i32"), tshape)], tshape, "i32")
    kept_shape = [d for k, d in enumerate(tshape) if k not in axes]
    ot = ttype(kept_shape, "i32")
    outs = [s.op(op, [y], kept_shape, "i32", "axes = " + arr(axes)) for op in ("reduce_sum", "reduce_max", "reduce_min")]
    xv = rng.integers(-50, 50, ashape).astype(np.int32)
    yv = np.transpose(xv, perm) + 1
    want = [yv.sum(axis=tuple(axes)).astype(np.int32), yv.max(axis=tuple(axes)), yv.min(axis=tuple(axes))]
    if len(axes) == 1:
        outs.append(s.op("argmax", [y], kept_shape, "i64", f"axis = {a0} : i64"))
        want.append(np.argmax(yv, axis=a0))
    red = sorted(perm[k] for k in axes)
    kept = [perm[k] for k in range(rank) if k not in axes]
    identity = [perm[k] for k in range(rank) if ashape[perm[k]] != 1] == sorted(perm[k] for k in range(rank) if ashape[perm[k]] != 1)
    maps = identity or (red == list(range(red[0], red[-1] + 1)) and kept == sorted(kept))
    return s.text(outs), [xv], want, maps


def test_permuted_reductions_read_the_arguments_axes():
    """A reduction of a transposed argument lowers over the argument's own
    layout (full ports, the row, split or column kernels) exactly when the
    reduced axes form one block of the argument's axes and the kept axes keep
    their order; every result equals numpy's."""
    rewritten = 0
    for seed in range(300):
        src, args, want, maps = permuted_reduce_step(seed)
        out = rt.lower_step(src)
        strategy = ask_b200.Plan(out["recipe"], -1).describe()["strategy"]
        assert (strategy != "view") == maps, seed
        rewritten += maps
        got = recipe_eval.evaluate(out["recipe"], [args[a] for a in out["input_arguments"]])
        for k, (g, w) in enumerate(zip(got, want)):
            assert np.array_equal(g, w.reshape(-1)), (seed, k)
    assert rewritten >= 60, rewritten


@pytest.mark.gpu
def test_permuted_reductions_on_gpu(device):
    import torch
    for seed in range(80):
        src, args, want, _ = permuted_reduce_step(seed)
        out = rt.lower_step(src)
        plan = ask_b200.Plan(out["recipe"], 0)
        dev_in = [torch.from_numpy(np.ascontiguousarray(args[a])).cuda() for a in out["input_arguments"]]
        kinds = {"i32": torch.int32, "i64": torch.int64}
        outs = [torch.empty(p["elements"], dtype=kinds[p["element_type"]], device="cuda")
                for p in plan.describe()["port_map"][len(dev_in):]]
        plan.launch(dev_in, outs, None, torch.cuda.current_stream())
        torch.cuda.synchronize()
        for k, (g, w) in enumerate(zip(outs, want)):
            assert np.array_equal(g.cpu().numpy(), w.reshape(-1)), (seed, k)


def scattered_axes_reduce_step(seed):
    """An i32 value (an argument times three plus a second argument) reduced
    with sum, max and min over a random non-contiguous set of axes."""
    rng = np.random.default_rng(seed)
    rank = int(rng.integers(3, 5))
    shape = [int(x) for x in rng.integers(2, 6, rank)]
    while True:
        axes = sorted(int(a) for a in rng.choice(rank, int(rng.integers(2, rank)), replace=False))
        if axes != list(range(axes[0], axes[-1] + 1)):
            break
    kept = [d for d in range(rank) if d not in axes]
    s = Step()
    x, y = s.arg(shape, "i32"), s.arg(shape, "i32")
    v = s.op("add", [s.op("mul", [x, s.splat(s.const(3, "i32"), shape)], shape, "i32"), y], shape, "i32")
    kshape = [shape[d] for d in kept]
    outs = [s.op(op, [v], kshape, "i32", "axes = " + arr(axes)) for op in ("reduce_sum", "reduce_max", "reduce_min")]
    xv, yv = (rng.integers(-40, 40, shape).astype(np.int32) for _ in range(2))
    vv = xv * 3 + yv
    want = [vv.sum(axis=tuple(axes)).astype(np.int32), vv.max(axis=tuple(axes)), vv.min(axis=tuple(axes))]
    return s.text(outs), [xv, yv], want


def test_reductions_over_scattered_axes_evaluate():
    """Reductions over axes that are not one block (axes 0 and 2 of a rank-3
    value, ...) lower through a transpose that gathers the reduced axes last;
    the outputs equal numpy's."""
    for seed in range(120):
        src, args, want = scattered_axes_reduce_step(seed)
        out = rt.lower_step(src)
        ask_b200.Plan(out["recipe"], -1)
        got = recipe_eval.evaluate(out["recipe"], [args[a] for a in out["input_arguments"]])
        for k, (g, w) in enumerate(zip(got, want)):
            assert np.array_equal(g, w.reshape(-1)), (seed, k)


@pytest.mark.gpu
def test_reductions_over_scattered_axes_on_gpu(device):
    import torch
    for seed in range(40):
        src, args, want = scattered_axes_reduce_step(seed)
        out = rt.lower_step(src)
        plan = ask_b200.Plan(out["recipe"], 0)
        dev_in = [torch.from_numpy(np.ascontiguousarray(args[a])).cuda() for a in out["input_arguments"]]
        outs = [torch.empty(w.size, dtype=torch.int32, device="cuda") for w in want]
        scratch = torch.empty(max(plan.scratch_bytes, 16), dtype=torch.uint8, device="cuda")
        plan.launch(dev_in, outs, scratch, torch.cuda.current_stream())
        torch.cuda.synchronize()
        for k, (g, w) in enumerate(zip(outs, want)):
            assert np.array_equal(g.cpu().numpy(), w.reshape(-1)), (seed, k)


def random_reduce_step(seed):
    """A random map-and-elementwise i32 operand reduced over a random block of
    contiguous axes with sum, max, min and argmax (argmax over a single axis)."""
    src, args, yv = random_map_step(seed + 1000, depth=2)
    # rebuild the step with reductions of its result
    rng = np.random.default_rng(seed)
    rank = yv.ndim
    a0 = int(rng.integers(0, rank))
    a1 = a0 + 1 if rng.random() < 0.5 else int(rng.integers(a0 + 1, rank + 1))
    axes = list(range(a0, a1))
    out_shape = [d for k, d in enumerate(yv.shape) if k not in axes]
    lines = src.rstrip().splitlines()
    ret = lines[-3].strip()  # "return %v : type"
    v, ty = ret[len("return "):].split(" : ")
    body = lines[:-3]
    ot = ttype(out_shape, "i32")
    names = []
    extra = []
    for k, op in enumerate(["reduce_sum", "reduce_max", "reduce_min"]):
        r = f"%red{k}"
        extra.append(f'    {r} = "ask.{op}"({v}) {{ask.id = "kernel0.red{k}", axes = {arr(axes)}}} : ({ty}) -> {ot}')
        names.append((r, ot))
    want = [yv.sum(axis=tuple(axes)).astype(np.int32), yv.max(axis=tuple(axes)), yv.min(axis=tuple(axes))]
    if len(axes) == 1:
        extra.append(f'    %red3 = "ask.argmax"({v}) {{ask.id = "kernel0.red3", axis = {a0} : i64}} : ({ty}) -> '
                     f'{ttype(out_shape, "i64")}')
        names.append(("%red3", ttype(out_shape, "i64")))
        want.append(np.argmax(yv, axis=a0))
    head = body[0:2]
    sig_line = body[1]
    # the function's result types follow the new returns
    res = ", ".join(t for _, t in names)
    sig_line = sig_line[:sig_line.index("-> (") + 4] + res + sig_line[sig_line.index(") attributes"):]
    text = "\n".join([body[0], sig_line] + body[2:] + extra +
                     [f"    return {', '.join(n for n, _ in names)} : {res}", "  }", "}"]) + "\n"
    return text, args, want


def _lower_random_reduce(seed):
    src, args, want = random_reduce_step(seed)
    try:
        return rt.lower_step(src), args, want
    except rt.CUDAError as e:
        assert e.status == ask_b200.E_UNSUPPORTED, str(e)
        return None, args, want


def test_random_reduce_steps_evaluate():
    """Every random reduction lowers, and its recipe, evaluated on the CPU by
    the recipe evaluator, gives numpy's sums, extremes and first arg positions."""
    for seed in range(200):
        out, args, want = _lower_random_reduce(seed)
        assert out is not None, seed
        got = recipe_eval.evaluate(out["recipe"], [args[a] for a in out["input_arguments"]])
        for k, (g, w) in enumerate(zip(got, want)):
            assert np.array_equal(g, w.reshape(-1)), (seed, k)


def test_random_reduce_steps_lower():
    lowered = 0
    for seed in range(40):
        out, args, want = _lower_random_reduce(seed)
        if out is not None:
            assert out["recipe"]["family"] == "reduce"
            ask_b200.Plan(out["recipe"], -1)
            lowered += 1
    assert lowered >= 30, lowered


@pytest.mark.gpu
def test_random_reduce_steps_on_gpu(device):
    import torch
    checked = 0
    for seed in range(40):
        out, args, want = _lower_random_reduce(seed)
        if out is None:
            continue
        plan = ask_b200.Plan(out["recipe"], 0)
        dev_in = [torch.from_numpy(np.ascontiguousarray(args[a])).cuda() for a in out["input_arguments"]]
        outs = [torch.empty(np.asarray(w).size, dtype=torch.from_numpy(np.ascontiguousarray(w)).dtype, device="cuda")
                for w in want]
        plan.launch(dev_in, outs, None, torch.cuda.current_stream())
        torch.cuda.synchronize()
        for got, w in zip(outs, want):
            assert np.array_equal(got.cpu().numpy(), np.asarray(w).reshape(-1)), seed
        checked += 1
    assert checked >= 30


# ---- the reference's own documented formats ---------------------------------------------
# The graph of docs/en/api.md:34-43, as the reference documents it: a module
# with attributes, named arguments, no ask.* attributes on ops, one result.
API_DOC_INCREMENT = """module attributes {ask.schema_version = 1 : i64} {
  func.func @increment(%x: tensor<4xi32>) -> tensor<4xi32> {
    %one = "ask.constant"() {value = 1 : i32} : () -> i32
    %ones = "ask.splat"(%one) {shape = array<i64: 4>} : (i32) -> tensor<4xi32>
    %y = "ask.add"(%x, %ones) {overflow = "wrap"} : (tensor<4xi32>, tensor<4xi32>) -> tensor<4xi32>
    return %y : tensor<4xi32>
  }
}
"""


def test_api_doc_graph_lowers():
    out = rt.lower_step(API_DOC_INCREMENT)
    assert out["input_arguments"] == [0]
    x = np.array([0, -1, 2 ** 31 - 1, 7], np.int32)
    (y,) = recipe_eval.evaluate(out["recipe"], [x])
    assert np.array_equal(y, x + np.int32(1))  # wrapping add: 2^31 - 1 + 1 = -2^31
    ask_b200.Plan(out["recipe"], -1)


def partitioning_doc_report():
    """The execution plan of docs/en/partitioning.md:21-41 (an owned step, then
    an external step), with a step source for the owned step in the form the
    reference's partitioner prints (keyed by step id, Partition.cpp:272)."""
    plan = {"schema_version": 1, "kind": "ask.cuda.execution_plan", "inputs": ["x"], "outputs": ["y"],
            "buffers": [{"id": "x", "shape": [128], "element_type": "f32"},
                        {"id": "tmp", "shape": [128], "element_type": "f32"},
                        {"id": "y", "shape": [128], "element_type": "f32"}],
            "steps": [{"id": "k0", "kind": "owned", "function": "kernel_0", "inputs": ["x"], "outputs": ["tmp"],
                       "depends_on": []},
                      {"id": "k1", "kind": "external", "function": "kernel_1", "inputs": ["tmp"], "outputs": ["y"],
                       "depends_on": ["k0"], "external_id": "graph.external0"}],
            "scheduling": {"policy": "sequential", "stream": "session"}}
    k0 = ("module attributes {ask.schema_version = 1 : i64} {\n"
          "  func.func @kernel_0(%arg0: tensor<128xf32>) -> tensor<128xf32> attributes {ask.kernel_id = \"k0\", "
          "ask.kernel_kind = \"owned\"} {\n"
          "    %0 = \"ask.exp\"(%arg0) : (tensor<128xf32>) -> tensor<128xf32>\n"
          "    return %0 : tensor<128xf32>\n  }\n}\n")
    return {"phase": "partitioned", "execution_plan": plan, "step_sources": {"k0": k0}, "external_requests": []}


def test_partitioning_doc_plan_keeps_its_external_step():
    prog = rt.lower_report(partitioning_doc_report())
    assert prog["buffer_sizes"] == [512, 512, 512] and prog["inputs"] == [0] and prog["outputs"] == [2]
    owned, ext = prog["steps"]
    assert owned["id"] == "k0" and owned["inputs"] == [0] and owned["outputs"] == [1]
    assert json.loads(owned["recipe"])["program"] == [["input", 0], ["exp", 0]]
    assert ext == {"id": "k1", "unresolved": {"kind": "external", "function": "kernel_1",
                                              "external_id": "graph.external0"}, "inputs": [1], "outputs": [2]}
    assert prog["unresolved_steps"] == ["k1"]


REPORT_FIELDS = {"statistics_stage", "kernel_count", "indexing", "warp_reduction_groups", "output_loop_count",
                 "input_load_count", "reduction_loop_count", "zero_element_outputs", "temporary_buffer_count",
                 "groups", "bool_storage", "cast_semantics"}


def test_cuda_lowering_report():
    """The fields of the reference's cuda_lowering diagnostics
    (lib/Lowering/CUDA.cpp:408-417), describing this library's kernels."""
    r1 = rt.lower_step(cfg1_source())["cuda_lowering"]
    assert REPORT_FIELDS <= set(r1) and "pre_copy" not in r1
    assert (r1["statistics_stage"], r1["indexing"], r1["warp_reduction_groups"], r1["output_loop_count"],
            r1["input_load_count"], r1["reduction_loop_count"], r1["kernel_count"]) == (
        "cuda_lowering", "linear_grid_stride", 0, 1, 3, 0, 1)
    assert r1["groups"] == [{"outputs": [0, 1], "element_count": 4096 * 4096, "threads_per_output": 1}]
    assert (r1["bool_storage"], r1["cast_semantics"]) == ("one-byte-zero-or-one", "rne-saturating-fptosi-nan-zero-v1")
    r2 = rt.lower_step(cfg2_source())["cuda_lowering"]
    assert (r2["indexing"], r2["warp_reduction_groups"], r2["reduction_loop_count"], r2["strategy"]) == (
        "cooperative_grid_stride", 1, 1, "warp_row")
    assert r2["groups"] == [{"outputs": [0, 1, 2, 3], "element_count": 65536, "threads_per_output": 32}]
    r5 = rt.lower_step(cfg5_sources()[0])["cuda_lowering"]
    assert r5["strategy"] == "split" and r5["kernel_count"] == 2 and r5["scratch_bytes"] > 0
    rs = rt.lower_step(cfg4_sources()[1])["cuda_lowering"]
    assert rs["pre_copy"] == {"input": 0, "output": 0}
    assert rs["groups"][0]["element_count"] == (1 << 23) * 256
    # every recipe step of a lowered report carries its report
    prog = rt.lower_report(softmax_report("f16", 64, 4096))
    assert all(REPORT_FIELDS <= set(s["cuda_lowering"]) for s in prog["steps"])


def pipeline_report():
    """A partition report shaped like the one the reference's partitioner
    makes of its frontend pipeline fixture (owned y = x + 1, an external
    kernel, owned + 3; tests/ir/pipeline.mlir): each step source is a module
    that also carries the graph's module-level declarations (the partitioner
    clones every non-function op into each step module, Partition.cpp:268-270)
    and the ask.mark ports around the external step."""
    decls = ('  "ask.semantics"() {\n    sym_name = "double_i32_v1",\n'
             '    function_type = (tensor<?xi32>) -> tensor<?xi32>,\n'
             '    shape_rule = "same_as", shape_operand = 0 : i64, effects = "none"\n  } : () -> ()\n'
             '  "ask.implementation"() {\n    sym_name = "ext_double", compiler = "cuda", entry = "double_it",\n'
             '    source = "extern \\22C\\22 __global__ void double_it(int* t, int* u) {\\0A}\\0A",\n'
             '    signature = {t = "*i32", u = "*i32"}, source_bindings = {t = "input:0", u = "output:0"},\n'
             '    constants = {N = 10 : i64}, options = {num_warps = 4 : i64},\n'
             '    target = {backend = "cuda", arch = 100 : i64, warp_size = 32 : i64},\n'
             '    grid = array<i64: 1, 1, 1>\n  } : () -> ()\n')

    def step(fn, kid, k, mark):
        body = (f'    %0 = "ask.constant"() {{value = {k} : i32}} : () -> i32\n'
                '    %1 = "ask.splat"(%0) {shape = array<i64: 10>} : (i32) -> tensor<10xi32>\n')
        arg = "%arg0"
        if mark == "in":  # the external step's output port, marked where it enters
            body += ('    %2 = "ask.mark"(%arg0) {mark_id = "m_F_out", value_id = "v_u", port_id = "F.out", '
                     'role = "output"} : (tensor<10xi32>) -> tensor<10xi32>\n')
            arg = "%2"
        body += (f'    %3 = "ask.add"({arg}, %1) {{ask.id = "{kid}", overflow = "wrap"}} : '
                 '(tensor<10xi32>, tensor<10xi32>) -> tensor<10xi32>\n')
        res = "%3"
        if mark == "out":
            body += ('    %4 = "ask.mark"(%3) {mark_id = "m_F_in", value_id = "v_t", port_id = "F.in", role = "input"} '
                     ': (tensor<10xi32>) -> tensor<10xi32>\n')
            res = "%4"
        return ("module attributes {ask.schema_version = 1 : i64} {\n" + decls +
                f'  func.func @{fn}(%arg0: tensor<10xi32>) -> tensor<10xi32> attributes {{ask.kernel_id = "{kid}", '
                'ask.kernel_kind = "owned"} {\n' + body + f"    return {res} : tensor<10xi32>\n  }}\n}}\n")
    plan = {"schema_version": 1, "kind": "ask.cuda.execution_plan", "inputs": ["v_x"], "outputs": ["v_y"],
            "buffers": [{"id": b, "shape": [10], "element_type": "i32"} for b in ("v_x", "v_t", "v_u", "v_y")],
            "steps": [{"id": "P", "kind": "owned", "function": "kernel_0", "inputs": ["v_x"], "outputs": ["v_t"],
                       "depends_on": []},
                      {"id": "F", "kind": "external", "function": "kernel_1", "inputs": ["v_t"], "outputs": ["v_u"],
                       "depends_on": ["P"], "external_id": "F"},
                      {"id": "Q", "kind": "owned", "function": "kernel_2", "inputs": ["v_u"], "outputs": ["v_y"],
                       "depends_on": ["F"]}],
            "scheduling": {"policy": "sequential", "stream": "session"}}
    return {"phase": "partitioned", "execution_plan": plan,
            "step_sources": {"P": step("kernel_0", "P", 1, "out"), "Q": step("kernel_2", "Q", 3, "in")}}


def test_pipeline_report_with_declarations_and_an_external_step():
    prog = rt.lower_report(pipeline_report())
    assert [s["id"] for s in prog["steps"]] == ["P", "F", "Q"] and prog["unresolved_steps"] == ["F"]
    assert prog["steps"][1]["unresolved"] == {"kind": "external", "function": "kernel_1", "external_id": "F"}
    x = np.array([0, 1, -1, 7, 2 ** 31 - 1, -(2 ** 31), 5, 6, 8, 9], np.int32)
    (t,) = recipe_eval.evaluate(json.loads(prog["steps"][0]["recipe"]), [x])
    u = (t.astype(np.int64) * 2).astype(np.int32)  # the external kernel, doubled with wrap
    (y,) = recipe_eval.evaluate(json.loads(prog["steps"][2]["recipe"]), [u])
    want = ((x.astype(np.int64) + 1) * 2 + 3).astype(np.int64)
    want = ((want + 2 ** 31) % 2 ** 32 - 2 ** 31).astype(np.int32)
    assert np.array_equal(y, want)
