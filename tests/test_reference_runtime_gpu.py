"""Kernel artifacts run by the REFERENCE's own Runtime.

oracle/_ref/libask_ref.so is the reference's lib/Runtime/CUDA.cpp (with its
PASS checker) compiled from source.  Each test compiles an ask_b200 artifact
through the worker path and hands it to that Runtime exactly as an ASK caller
would: Session::load with the artifact's entry, element types, arch 100 and
parameter widths (its cuFuncGetParamInfo layout check included), then
prepareProgram with one kernel PlanStep, run -- in stream and graph mode, with
fresh inputs per run so graph mode re-binds its node.  Results are compared
with the CPU oracle under the same bars as the library's own tests.
"""
import base64

import numpy as np
import pytest

import ask_b200
import oracle
from ask_b200 import artifact as A
from ask_b200 import recipes as R
from gpu_util import NUMPY, f16_to_f32, bf16_to_f32
from test_gpu_parity import check_cfg1, random_inputs, random_program, same_with_nan

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref(device):
    from oracle import ref as ref_mod
    if ref_mod.load() is None:
        pytest.skip("the reference Runtime is not built here (oracle/_ref; oracle/ref_build.py needs its sources)")
    return ref_mod


def run_reference(ref, recipe, inputs, graph=False, repeats=1, grid=592):
    """(outputs as numpy arrays, session stats) of the recipe's artifact run by the reference Runtime."""
    req = A.request_for(recipe, entry="ref_step", grid=(grid, 1, 1), scalars=(("n", "i32", 7), ("alpha", "fp32", 0.5)))
    art = A.build_artifact(req)
    A.validate_artifact(art, req)
    ports = ask_b200.Plan(recipe, -1).describe()["port_map"]
    n_in = len(inputs)
    arg_buffer, scalars = [], []
    for a in art["arguments"]:
        if isinstance(a, str):
            kind, k = a.split(":")
            arg_buffer.append(int(k) if kind == "input" else n_in + int(k))
            scalars.append(b"")
        else:
            arg_buffer.append(-1)
            scalars.append(A.scalar_bytes(a["type"], a["value"]))
    types = list(dict.fromkeys(art["required_element_types"] + [p["element_type"] for p in ports]))
    out_ports = ports[n_in:]
    launch = art["launch"]
    outs, stats = ref.run_step(base64.b64decode(art["payload"]), art["entry"], types, art["target"]["arch"],
                               A.parameter_widths(art), arg_buffer, scalars, launch["grid"], launch["block"],
                               launch["shared_bytes"], [np.ascontiguousarray(x).tobytes() for x in inputs],
                               [p["elements"] * p["storage_bytes"] for p in out_ports], graph=graph, repeats=repeats)
    arrays = [np.frombuffer(o, dtype=NUMPY[p["element_type"]]).copy() for o, p in zip(outs, out_ports)]
    return arrays, stats


@pytest.mark.parametrize("graph", [False, True])
def test_cfg1_through_the_reference_runtime(ref, graph):
    n = 1 << 18
    rng = np.random.default_rng(7)
    a, b, c = (rng.standard_normal(n).astype(np.float32) * 3 for _ in range(3))
    (y0, y1), stats = run_reference(ref, R.cfg1_step(n), [a, b, c], graph=graph, repeats=2)
    check_cfg1(a, b, c, y0, y1)
    assert stats["module_loads"] == 1 and stats["program_submissions"] == 2
    if graph:
        assert stats["graph_instantiations"] == 1 and stats["graph_node_updates"] >= 1


@pytest.mark.parametrize("dtype", ["f32", "bf16", "i64"])
def test_random_programs_through_the_reference_runtime(ref, dtype):
    rng = np.random.default_rng(len(dtype) * 17)
    p, outs = random_program(rng, dtype)
    n = 777
    rec = R.elementwise(p, outs, n)
    ins = [random_inputs(rng, dtype, n), random_inputs(rng, dtype, n), random_inputs(rng, dtype, 1)]
    got, _ = run_reference(ref, rec, ins, graph=True)
    want = oracle.elementwise(rec, ins)
    for k, (g, w) in enumerate(zip(got, want)):
        t = outs[k].dtype
        if t == "f32":
            assert same_with_nan(g, w), k
        elif t in ("f16", "bf16"):
            conv = f16_to_f32 if t == "f16" else bf16_to_f32
            assert same_with_nan(conv(g), conv(w)), k
        else:
            assert np.array_equal(g, w), k


def test_cfg5b_through_the_reference_runtime(ref):
    n = (1 << 20) + 3
    rng = np.random.default_rng(3)
    x = rng.integers(-(2 ** 31), 2 ** 31, n, dtype=np.int64).astype(np.int32)
    y = rng.integers(-(2 ** 31), 2 ** 31, n, dtype=np.int64).astype(np.int32)
    (z,), _ = run_reference(ref, R.cfg5b_step(n), [x, y])
    assert np.array_equal(z, oracle.cfg5b(x, y))


@pytest.mark.parametrize("graph", [False, True])
def test_row_statistics_through_the_reference_runtime(ref, graph):
    rows, cols = 300, 1000
    rng = np.random.default_rng(5)
    x = rng.standard_normal(rows * cols).astype(np.float32)
    x[::13] = 0.5
    rec = R.cfg2_step(rows, cols)
    got, _ = run_reference(ref, rec, [x], graph=graph)
    want = oracle.reduce(rec, [x])
    xx = x.reshape(rows, cols).astype(np.float64)
    assert np.all(np.abs(got[0] - xx.sum(axis=1)) <= 2.0 ** -20 * np.abs(xx).sum(axis=1) + 1e-30)
    for k in (1, 2, 3):
        assert np.array_equal(got[k], want[k]), k


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_softmax_steps_through_the_reference_runtime(ref, dt):
    """The softmax plan's three steps as artifacts, each run by the reference
    Runtime and fed the previous step's outputs; against the oracle."""
    rows, cols = 64, 4096
    rng = np.random.default_rng(12)
    xf = (rng.standard_normal(rows * cols) * 3).astype(np.float32)
    x = xf.astype(np.float16).view(np.uint16) if dt == "f16" else (xf.view(np.uint32) >> 16).astype(np.uint16)
    x[9] = 0x7E00 if dt == "f16" else 0x7FC0  # a NaN row
    steps = R.cfg3_steps(dt, rows, cols)
    (m,), _ = run_reference(ref, steps[0], [x])
    (s,), _ = run_reference(ref, steps[1], [x, m])
    (y,), _ = run_reference(ref, steps[2], [x, m, s])
    rm, rs, ry = oracle.softmax(dt, x, rows, cols)
    assert same_with_nan(m, rm)
    fin = np.isfinite(rs)
    assert np.array_equal(np.isnan(s), np.isnan(rs))
    assert np.all(np.abs(s[fin].astype(np.float64) - rs[fin]) <= 2.0 ** -20 * np.abs(rs[fin]))
    conv = f16_to_f32 if dt == "f16" else bf16_to_f32
    gyv, ryv = conv(y.view(np.uint16)), conv(ry)
    nan = np.isnan(ryv)
    assert np.array_equal(np.isnan(gyv), nan)
    step = np.spacing(np.abs(ryv[~nan]).astype(np.float16)).astype(np.float32) if dt == "f16" else \
        np.abs(bf16_to_f32(ry[~nan] + 1) - ryv[~nan])
    assert np.all(np.abs(gyv[~nan] - ryv[~nan]) <= step + 1e-45)


def test_gather_through_the_reference_runtime(ref):
    rng = np.random.default_rng(11)
    dim, inner, n = 500, 32, 3000
    table = rng.standard_normal(dim * inner).astype(np.float32)
    idx = rng.integers(-10, dim + 10, n).astype(np.int64)
    (out,), _ = run_reference(ref, R.gather("f32", "i64", dim, inner, n), [table, idx])
    assert np.array_equal(out.view(np.uint32), oracle.gather(table, idx, 1, dim, inner).view(np.uint32))


def test_view_step_through_the_reference_runtime(ref):
    from test_lowering import view_steps
    name, src, ins, want = view_steps()[0]  # a transposed argument plus a full one
    recipe, args = A._recipe_of(src)
    (got,), _ = run_reference(ref, recipe, [ins[a] for a in args], grid=4)
    assert np.array_equal(got.reshape(want.shape), want)


# ---- one program through both runtimes -----------------------------------------------
def _affine_i32(n, mul, add):
    p = R.Program()
    x = p.input("i32")
    return R.elementwise(p, [p.add(p.mul(x, p.const("i32", mul)), p.const("i32", add))], n)


def _add_i32(n):
    p = R.Program()
    a, b = p.input("i32"), p.input("i32")
    return R.elementwise(p, [p.add(a, b)], n)


def _programs(n):
    """(name, buffer count, inputs, outputs, steps as (kernel, ins, outs)) with internal buffers."""
    chain = [("affine", [i], [i + 1]) for i in range(6)]
    dag = [("affine", [0], [1]), ("affine", [0], [2]), ("add", [1, 2], [3]), ("affine", [3], [4]),
           ("add", [4, 1], [5]), ("affine", [5], [6])]
    return [("chain", 7, [0], [6], chain), ("fork_join", 7, [0], [6, 2], dag)]


def _random_program(seed):
    """A random DAG of affine/add steps over internal buffers: each step reads
    one or two earlier buffers; a random subset of the buffers is public."""
    rng = np.random.default_rng(seed)
    nsteps = int(rng.integers(3, 10))
    steps = []
    for k in range(nsteps):
        out = k + 1
        if k >= 1 and rng.random() < 0.4:
            a, b = (int(x) for x in rng.choice(out, 2, replace=False))
            steps.append(("add", [a, b], [out]))
        else:
            steps.append(("affine", [int(rng.integers(0, out))], [out]))
    extra = [int(b) for b in rng.choice(np.arange(1, nsteps), size=min(2, nsteps - 1), replace=False)]
    outs = sorted(set([nsteps] + extra))
    return f"random{seed}", nsteps + 1, [0], outs, steps


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("which", [0, 1] + [f"r{k}" for k in range(6)])
def test_programs_match_the_reference_runtime(ref, graph, which):
    """The same kernel-step program through this library's runtime and the
    reference's: identical outputs and identical slot and graph counters."""
    from ask_b200 import runtime as rt
    n = 1 << 16
    if isinstance(which, str):
        name, nbuf, ins, outs, steps = _random_program(int(which[1:]))
    else:
        name, nbuf, ins, outs, steps = _programs(n)[which]
    arts = {}
    for key, rec in (("affine", _affine_i32(n, 3, 1)), ("add", _add_i32(n))):
        req = A.request_for(rec, entry=f"k_{key}", grid=(148, 1, 1))
        arts[key] = (A.build_artifact(req), A.port_types(req))
    session = rt.Session.create(0)
    kernels = {k: A.load_artifact(session, a) for k, (a, _) in arts.items()}
    plan_steps = [A.artifact_step(arts[k][0], kernels[k], i, o, arts[k][1]) for k, i, o in steps]
    sizes = [4 * n] * nbuf
    prog = session.prepareProgram(sizes, ins, outs, plan_steps, graph=graph)
    x = np.random.default_rng(which if isinstance(which, int) else 100 + int(which[1:])).integers(-1000, 1000, n).astype(np.int32)
    xb = session.allocate(4 * n)
    xb.copyFromHost(x.tobytes())
    for _ in range(2):
        got, ev = prog.run([xb])
        ev.wait()
    ours = [np.frombuffer(b.copyToHost(), dtype=np.int32) for b in got]
    mine = session.stats()

    order = list(arts)
    program = {"buffer_sizes": sizes, "inputs": ins, "outputs": outs,
               "kernels": [{"entry": arts[k][0]["entry"], "types": ["i32"], "arch": 100,
                            "widths": A.parameter_widths(arts[k][0])} for k in order],
               "steps": [s.to_json(order.index(k)) for s, (k, _, _) in zip(plan_steps, steps)]}
    images = [base64.b64decode(arts[k][0]["payload"]) for k in order]
    theirs_raw, theirs = ref.run_program(program, images, [x.tobytes()], graph=graph, repeats=2)
    for a, b in zip(ours, theirs_raw):
        assert np.array_equal(a, np.frombuffer(b, dtype=np.int32))
    for key in ("prepared_internal_slots", "prepared_internal_bytes", "graph_nodes", "graph_edges",
                "graph_instantiations"):
        assert mine.get(key, 0) == theirs.get(key, 0), (name, graph, key, mine.get(key), theirs.get(key))
    session.close()
