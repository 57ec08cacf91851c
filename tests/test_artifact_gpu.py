"""Kernel artifacts on the GPU: compiled by the worker path, loaded with
Session::load's ABI checks (ask_b200_kernel_load), launched through
Session::submit and as kernel steps of prepared programs (stream and graph
mode), and compared with the CPU oracle -- bit-exact for elementwise programs,
integer work, extrema, arg-extrema and gather; float sums within the tolerance
of the recipe-path tests."""
import base64
import json

import numpy as np
import pytest
import torch

import ask_b200
import oracle
from ask_b200 import artifact as A
from ask_b200 import recipes as R
from ask_b200 import runtime as rt
from gpu_util import NUMPY, bf16_to_f32, f16_to_f32, from_dev, to_dev
from test_artifact import request_for
from test_gpu_parity import check_cfg1, random_inputs, random_program, same_with_nan

pytestmark = pytest.mark.gpu

_CUBINS = {}


def artifact_for(recipe, grid=592, scalars=(("n", "i32", 7),), source=None):
    """(artifact, port -> element type) of the recipe's step."""
    req = request_for(recipe, grid=(grid, 1, 1), scalars=scalars, source=source)
    key = json.dumps(req, sort_keys=True)
    if key not in _CUBINS:
        _CUBINS[key] = A.build_artifact(req)
    return _CUBINS[key], A.port_types(req)


@pytest.fixture(scope="module")
def session(device):
    s = rt.Session.create(0)
    yield s
    s.close()


def run_artifact(session, recipe, inputs, out_dtypes, grid=592, mode="submit", offset_bytes=0,
                 scalars=(("n", "i32", 7),)):
    """Build, load and launch the recipe's artifact; returns the outputs.
    offset_bytes must keep every port aligned to its element size."""
    art, types = artifact_for(recipe, grid, scalars)
    ports = ask_b200.Plan(recipe, -1).describe()["port_map"]
    kernel = A.load_artifact(session, art, [p["element_type"] for p in ports])
    assert all(offset_bytes % A.ELEMENT_BYTES[p["element_type"]] == 0 for p in ports)
    dev_in = [to_dev(a, offset_bytes) for a in inputs]
    n_out = [p["elements"] for p in ports[len(inputs):]]
    dev_out = [torch.zeros(n * np.dtype(NUMPY[dt]).itemsize + offset_bytes, dtype=torch.uint8,
                           device="cuda")[offset_bytes:] for n, dt in zip(n_out, out_dtypes)]
    torch.cuda.synchronize()
    bin_ = [session.importTensor(t, readonly=True) for t in dev_in]
    bout = [session.importTensor(t) for t in dev_out]
    if mode == "submit":
        args, aligns = A.submit_arguments(art, bin_, bout, types)
        session.submit(kernel, args, art["launch"]["grid"], art["launch"]["block"],
                       art["launch"]["shared_bytes"], aligns).wait()
    else:
        ni, no = len(bin_), len(bout)
        step = A.artifact_step(art, kernel, list(range(ni)), list(range(ni, ni + no)), types)
        prog = session.prepareProgram([b.size() for b in bin_ + bout], list(range(ni)), list(range(ni, ni + no)),
                                      [step], graph=(mode == "graph"))
        prog.submit(bin_, bout).wait()
    return [from_dev(t, NUMPY[dt]) for t, dt in zip(dev_out, out_dtypes)]


def assert_same(got, want, dtype):
    if dtype == "f32":
        assert same_with_nan(got, want)
    elif dtype in ("f16", "bf16"):
        conv = f16_to_f32 if dtype == "f16" else bf16_to_f32
        assert same_with_nan(conv(got), conv(want))
    else:
        assert np.array_equal(got, want)


# ---- elementwise ------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16", "i32", "i64"])
@pytest.mark.parametrize("seed", range(3))
def test_random_programs_match_oracle(session, dtype, seed):
    rng = np.random.default_rng(seed * 131 + len(dtype))
    p, outs = random_program(rng, dtype)
    n = 1031
    rec = R.elementwise(p, outs, n)
    ins = [random_inputs(rng, dtype, n), random_inputs(rng, dtype, n), random_inputs(rng, dtype, 1)]
    # an offset of one element: aligned ports, but not 16-byte aligned (the scalar path)
    got = run_artifact(session, rec, ins, [o.dtype for o in outs], offset_bytes=(seed % 2) * (8 if dtype == "i64" else 4))
    want = oracle.elementwise(rec, ins)
    for k, (g, w) in enumerate(zip(got, want)):
        assert_same(g, w, outs[k].dtype)


@pytest.mark.parametrize("mode", ["submit", "program", "graph"])
@pytest.mark.parametrize("n,grid", [(1, 1), (4099, 3), (1 << 20, 592)])
def test_cfg1(session, mode, n, grid):
    rng = np.random.default_rng(n)
    a, b, c = (rng.standard_normal(n).astype(np.float32) * 3 for _ in range(3))
    y0, y1 = run_artifact(session, R.cfg1_step(n), [a, b, c], ["f32", "f32"], grid=grid, mode=mode)
    check_cfg1(a, b, c, y0, y1)


@pytest.mark.parametrize("n", [7, 1 << 22])
def test_cfg5b_bit_exact(session, n):
    rng = np.random.default_rng(3)
    x = rng.integers(-(2 ** 31), 2 ** 31, n, dtype=np.int64).astype(np.int32)
    y = rng.integers(-(2 ** 31), 2 ** 31, n, dtype=np.int64).astype(np.int32)
    (got,) = run_artifact(session, R.cfg5b_step(n), [x, y], ["i32"], mode="program")
    assert np.array_equal(got, oracle.cfg5b(x, y))


def test_index_map_views(session):
    from test_lowering import view_steps
    for name, src, ins, want in view_steps():
        recipe, args = A._recipe_of(src)
        got = run_artifact(session, recipe, [ins[a] for a in args], [{np.int32: "i32", np.float32: "f32"}[want.dtype.type]],
                           grid=4)
        assert np.array_equal(got[0].reshape(want.shape), want), name


# ---- reductions -------------------------------------------------------------------------
@pytest.mark.parametrize("rows,cols,grid", [(3, 31, 592), (64, 1024, 592), (1000, 300, 20), (5, 70000, 592)])
def test_row_statistics(session, rows, cols, grid):
    rng = np.random.default_rng(rows * cols)
    x = rng.standard_normal(rows * cols).astype(np.float32)
    x[::17] = 0.75  # ties for argmax
    rec = R.cfg2_step(rows, cols)
    got = run_artifact(session, rec, [x], ["f32", "f32", "f32", "i64"], grid=grid)
    want = oracle.reduce(rec, [x])
    xx = x.reshape(rows, cols).astype(np.float64)
    assert np.all(np.abs(got[0] - xx.sum(axis=1)) <= 2.0 ** -20 * np.abs(xx).sum(axis=1) + 1e-30)
    for k in (1, 2, 3):
        assert np.array_equal(got[k], want[k]), k


@pytest.mark.parametrize("n", [1, 4097, 1 << 22])
def test_global_reduction(session, n):
    rng = np.random.default_rng(n)
    x = rng.random(n).astype(np.float32)
    if n > 10:
        x[n // 3] = 0.0
        x[n // 2] = 0.0  # duplicate minima: the lowest index wins
    s, m, a = run_artifact(session, R.cfg5a_step(n), [x], ["f32", "f32", "i64"], mode="graph")
    s64, _, mn, am = oracle.cfg5a(x)
    assert abs(float(s[0]) - s64) <= 2.0 ** -20 * s64 + 1e-30
    assert m[0] == mn and a[0] == am


def test_global_reduction_nan_wins_first(session):
    x = np.random.default_rng(0).random(100000).astype(np.float32)
    x[777] = np.nan
    x[70000] = np.nan
    s, m, a = run_artifact(session, R.cfg5a_step(x.size), [x], ["f32", "f32", "i64"])
    assert np.isnan(s[0]) and np.isnan(m[0]) and a[0] == 777


@pytest.mark.parametrize("outer,extent,inner", [(3, 5, 7), (1, 1000, 33), (2, 3, 1000)])
def test_column_reductions(session, outer, extent, inner):
    rng = np.random.default_rng(outer + extent + inner)
    x = rng.standard_normal(outer * extent * inner).astype(np.float32)
    x[::9] = 1.5
    p = R.Program()
    v = p.input("f32")
    rec = R.reduce(p, v, ["sum", "max", "min", "argmax", "argmin"], outer, extent, inner)
    got = run_artifact(session, rec, [x], ["f32", "f32", "f32", "i64", "i64"], grid=7)
    want = oracle.reduce(rec, [x])
    for k in (1, 2, 3, 4):
        assert np.array_equal(got[k], want[k]), k
    xx = x.reshape(outer, extent, inner).astype(np.float64)
    assert np.all(np.abs(got[0] - xx.sum(axis=1).reshape(-1)) <= 2.0 ** -20 * np.abs(xx).sum(axis=1).reshape(-1) + 1e-30)


@pytest.mark.parametrize("dtype,cols", [("i32", 301), ("i64", 5000), ("bool", 301), ("bool", 9000)])
def test_integer_and_bool_reductions(session, dtype, cols):
    rng = np.random.default_rng(cols)
    rows = 37
    if dtype == "bool":
        x = (rng.random(rows * cols) < 0.001).astype(np.uint8)
        ops = ["any", "all", "max", "min", "argmax", "argmin"]
    else:
        x = rng.integers(-1000, 1000, rows * cols).astype(NUMPY[dtype])
        ops = ["sum", "prod", "max", "min", "argmax", "argmin"]
    p = R.Program()
    v = p.input(dtype)
    rec = R.reduce(p, v, ops, rows, cols)
    out_types = [o["element_type"] for o in ask_b200.Plan(rec, -1).describe()["port_map"][1:]]
    got = run_artifact(session, rec, [x], out_types, grid=3)
    want = oracle.reduce(rec, [x])
    for k in range(len(ops)):
        assert np.array_equal(got[k], want[k]), ops[k]


@pytest.mark.parametrize("dt,rows,cols", [("f16", 64, 4096), ("bf16", 4096, 512)])
def test_softmax_steps(session, dt, rows, cols):
    """The three softmax steps as artifacts (row max; sum of exp(cast(x) - m[row])
    with an outer-indexed port; normalise) against the oracle, with a NaN, an
    infinity and an all -inf row among them."""
    rng = np.random.default_rng(2)
    xf = (rng.standard_normal(rows * cols) * 3).astype(np.float32)
    x = xf.astype(np.float16).view(np.uint16) if dt == "f16" else (xf.view(np.uint32) >> 16).astype(np.uint16)
    nan16, inf16, ninf16 = (0x7E00, 0x7C00, 0xFC00) if dt == "f16" else (0x7FC0, 0x7F80, 0xFF80)
    x[7] = nan16
    x[cols + 11] = inf16
    x[2 * cols:3 * cols] = ninf16
    steps = R.cfg3_steps(dt, rows, cols)
    (m,) = run_artifact(session, steps[0], [x], ["f32"])
    assert same_with_nan(m, oracle.reduce(steps[0], [x])[0])
    (s,) = run_artifact(session, steps[1], [x, m], ["f32"])
    (want,) = oracle.reduce(steps[1], [x, m])
    fin = np.isfinite(want)
    assert np.array_equal(np.isnan(s), np.isnan(want))
    assert np.all(np.abs(s[fin].astype(np.float64) - want[fin]) <= 2.0 ** -20 * np.abs(want[fin]))
    (y,) = run_artifact(session, steps[2], [x, m, s], [dt])
    (wy,) = oracle.elementwise(steps[2], [x, m, s])
    # CUDA's expf against the host libm's exp: within one unit of the output type
    conv = f16_to_f32 if dt == "f16" else bf16_to_f32
    gyv, wyv = conv(y), conv(wy)
    nan = np.isnan(wyv)
    assert np.array_equal(np.isnan(gyv), nan)
    gyv, wyv, wy = gyv[~nan], wyv[~nan], wy[~nan]
    step = np.spacing(np.abs(wyv).astype(np.float16)).astype(np.float32) if dt == "f16" else \
        np.abs(bf16_to_f32(wy + 1) - wyv)
    assert np.all(np.abs(gyv - wyv) <= step + 1e-45)


# ---- gather -----------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,inner,itype", [("f32", 64, "i64"), ("f16", 3, "i32"), ("i64", 5, "i64"),
                                               ("bool", 48, "i32")])
def test_gather_with_out_of_bounds(session, dtype, inner, itype):
    rng = np.random.default_rng(inner)
    dim, n = 300, 2000
    table = rng.integers(0, 200, dim * inner).astype(NUMPY[dtype])
    idx = rng.integers(-20, dim + 20, n).astype(NUMPY[itype])
    rec = R.gather(dtype, itype, dim, inner, n)
    (got,) = run_artifact(session, rec, [table, idx], [dtype], grid=50)
    want = oracle.gather(table, idx, 1, dim, inner)
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))


# ---- the loader's ABI checks --------------------------------------------------------------
def test_load_checks_the_declared_abi(session):
    art, _ = artifact_for(R.cfg5b_step(1000))
    image = base64.b64decode(art["payload"])
    widths = A.parameter_widths(art)  # [0, 0, 0, 4]
    k1 = session.load(image, art["entry"], ["i32"], 100, widths)
    before = session.stats()
    k2 = session.load(image, art["entry"], ["i32"], 100, widths)
    assert session.stats()["module_hits"] == before["module_hits"] + 1 and k2.entry() == art["entry"]
    assert k1.maxThreads() >= 256
    for bad_widths, msg in [([0, 0, 0, 8], "parameter layout differs"), ([0, 0, 0], "count differs"),
                            ([0, 0, 0, 4, 4], "count differs"), ([0, 0, 3, 4], "unsupported kernel parameter width")]:
        with pytest.raises(rt.CUDAError) as err:
            _fresh(session).load(image, art["entry"], ["i32"], 100, bad_widths)
        assert msg in str(err.value), (bad_widths, str(err.value))
    with pytest.raises(rt.CUDAError) as err:
        session.load(image, art["entry"], ["i32"], 90, widths)
    assert "incompatible" in str(err.value)
    with pytest.raises(rt.CUDAError) as err:
        session.load(image, art["entry"], ["f8"], 100, widths)
    assert "unsupported runtime element type" in str(err.value)
    with pytest.raises(rt.CUDAError) as err:
        session.load(image, "no_such_entry", ["i32"], 100, widths)
    with pytest.raises(rt.CUDAError) as err:
        session.load(image, art["entry"], ["i32"], 100, [0, 0, 0, 8])
    assert "cached kernel parameter contract differs" in str(err.value)


_fresh_sessions = []


def _fresh(session):
    """A new session, so a load is not answered from the cache."""
    s = rt.Session.create(0)
    _fresh_sessions.append(s)
    return s


def test_launch_and_argument_validation(session):
    art, types = artifact_for(R.cfg5b_step(1000))
    kernel = A.load_artifact(session, art)
    x = session.allocate(4000)
    y = session.allocate(4000)
    out = session.allocate(4000)
    with pytest.raises(rt.CUDAError) as err:
        session.submit(kernel, [x, y, out, b"\0\0"], [4, 1, 1], [256, 1, 1])
    assert "scalar argument byte width" in str(err.value)
    with pytest.raises(rt.CUDAError) as err:
        session.submit(kernel, [x, y, out], [4, 1, 1], [256, 1, 1])
    assert "argument count" in str(err.value)
    with pytest.raises(rt.CUDAError) as err:
        session.submit(kernel, [x, y, out, b"\0\0\0\0"], [4, 1, 1], [2048, 1, 1])
    assert "block" in str(err.value) or "thread count" in str(err.value)
    with pytest.raises(rt.CUDAError) as err:
        session.submit(kernel, [x, y, out, b"\0\0\0\0"], [4, 1, 1], [256, 1, 1], 1 << 20)
    assert "dynamic shared memory" in str(err.value)
    # an i32 port bound at an address that is not 4-byte aligned is refused on the host
    raw = session.allocate(4004)
    odd = session.importBuffer(raw.pointer() + 2, 4000)
    args, aligns = A.submit_arguments(art, [odd, y], [out], types)
    with pytest.raises(rt.CUDAError) as err:
        session.submit(kernel, args, [4, 1, 1], [256, 1, 1], 0, aligns)
    assert "not aligned to 4 bytes" in str(err.value)
    step = A.artifact_step(art, kernel, [0, 1], [2], types)
    prog = session.prepareProgram([4000] * 3, [0, 1], [2], [step])
    with pytest.raises(rt.CUDAError) as err:
        prog.submit([odd, y], [out])
    assert "not aligned to 4 bytes" in str(err.value)
    other = _fresh(session)
    with pytest.raises(rt.CUDAError) as err:
        other.submit(kernel, [None, None, None, b"\0\0\0\0"], [4, 1, 1], [256, 1, 1])
    assert "different CUDA execution session" in str(err.value)
    # a program step must bind every port to a parameter
    step = A.artifact_step(art, kernel, [0, 1], [2])
    step.arguments = list(step.arguments)
    step.arguments[1] = rt.PlanArgument(buffer=-1)
    with pytest.raises(rt.CUDAError) as err:
        session.prepareProgram([4000] * 3, [0, 1], [2], [step])
    assert "not bound to a kernel parameter" in str(err.value)


def test_graph_program_rebinds_ports(session):
    """Graph mode records the kernel step once and re-records it when a public
    address changes."""
    n = 1 << 16
    rec = R.cfg5b_step(n)
    art, types = artifact_for(rec)
    kernel = A.load_artifact(session, art)
    step = A.artifact_step(art, kernel, [0, 1], [2], types)
    prog = session.prepareProgram([4 * n] * 3, [0, 1], [2], [step], graph=True)
    rng = np.random.default_rng(9)
    for _ in range(3):
        x = rng.integers(-(2 ** 31), 2 ** 31, n, dtype=np.int64).astype(np.int32)
        y = rng.integers(-(2 ** 31), 2 ** 31, n, dtype=np.int64).astype(np.int32)
        tx, ty = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
        tout = torch.empty(n, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        prog.submit([session.importTensor(tx), session.importTensor(ty)], [session.importTensor(tout)]).wait()
        assert np.array_equal(tout.cpu().numpy(), oracle.cfg5b(x, y))
    st = session.stats()
    assert st["graph_instantiations"] >= 1 and st["graph_node_updates"] >= 1


@pytest.mark.parametrize("graph", [False, True])
def test_partition_report_with_an_external_step(session, graph):
    """The execution plan of the reference's partitioning document (an owned
    step, then an external step): the owned step is lowered to a recipe, the
    external step -- left unresolved by the lowering -- is bound to a loaded
    kernel artifact (here y = tmp + 1), and the program runs both."""
    from test_lowering import partitioning_doc_report
    prog = rt.lower_report(partitioning_doc_report())
    assert prog["unresolved_steps"] == ["k1"]
    p = R.Program()
    t = p.input("f32")
    plus_one = R.elementwise(p, [p.op("add", t, p.const("f32", 1.0))], 128)
    art, types = artifact_for(plus_one, grid=1)
    kernel = A.load_artifact(session, art, ["f32"])
    steps = []
    for s in prog["steps"]:
        if "unresolved" in s:
            steps.append(A.artifact_step(art, kernel, s["inputs"], s["outputs"], types))
        else:
            steps.append(rt.PlanStep(recipe=s["recipe"], inputs=s["inputs"], outputs=s["outputs"]))
    program = session.prepareProgram(prog["buffer_sizes"], prog["inputs"], prog["outputs"], steps, graph=graph)
    x = np.random.default_rng(7).uniform(-4, 4, 128).astype(np.float32)
    dx = to_dev(x)
    dy = torch.zeros(128, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    program.submit([session.importTensor(dx, readonly=True)], [session.importTensor(dy)]).wait()
    want = np.exp(x.astype(np.float64)) + 1.0
    got = dy.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - want) <= 4 * np.spacing(want.astype(np.float32)).astype(np.float64))
