"""Runtime layer on the GPU: sessions, buffers, prepared programs of plan steps.

Modelled on the reference's runtime contract test (tests/cpp/runtime.cpp):
public-port validation before any allocation, repeated and identity outputs,
read-only and overlapping outputs, the two-slot chain with workspace reuse,
graph replay with node updates, in-flight submissions, pre-copy steps -- plus
the hot-path programs the step kind exists for: the three-step softmax plan
with its row statistics in workspace slots, a split reduction whose scratch is
a private slot, and a gather -> scatter_add pair.  Every result is compared
bit for bit with the same plans launched directly.
"""
import numpy as np
import pytest
import torch

import ask_b200
from ask_b200 import recipes as R
from ask_b200 import runtime as rt

from gpu_util import gen_dev

pytestmark = pytest.mark.gpu


def double_i32(count):
    p = R.Program()
    x = p.input("i32")
    return R.elementwise(p, [p.add(x, x)], count)


def rejects(fn):
    with pytest.raises(rt.CUDAError):
        fn()


def i32s(buf):
    return np.frombuffer(buf.copyToHost(), dtype=np.int32)


@pytest.mark.parametrize("graph", [False, True])
def test_port_bindings(device, graph):
    session, other = rt.Session.create(0), rt.Session.create(0)
    inp, wrong, foreign = session.allocate(16), session.allocate(8), other.allocate(16)
    values = np.array([1, -2, 3, 4], np.int32)
    inp.copyFromHost(values)
    readonly = session.importBuffer(inp.pointer(), 16, True)

    identity = session.prepareProgram([16], [0], [0, 0], [], graph)
    before = session.stats()["allocations"]
    outs, ev = identity.run([readonly])
    ev.wait()
    assert outs == [readonly, readonly] and session.stats()["allocations"] == before

    step = rt.PlanStep(double_i32(4), [0], [1])
    program = session.prepareProgram([16, 16], [0], [1, 1], [step], graph)
    before = session.stats()["allocations"]
    for bad in (None, wrong, foreign):
        rejects(lambda: program.run([bad]))
    assert session.stats()["allocations"] == before, "invalid run allocated outputs before input validation"
    outs, ev = program.run([readonly])
    ev.wait()
    assert len(outs) == 2 and outs[0] == outs[1]
    assert np.array_equal(i32s(outs[0]), values * 2)
    ro_out = session.importBuffer(outs[0].pointer(), 16, True)
    rejects(lambda: program.submit([inp], [ro_out, ro_out]))
    rejects(lambda: program.submit([inp], [outs[0], ro_out]))
    rejects(lambda: program.submit([inp], [inp, inp]))
    rejects(lambda: program.submit([inp], [outs[0], inp]))
    program.submit([inp], outs).wait()


def test_early_read_is_rejected(device):
    session = rt.Session.create(0)
    early = rt.PlanStep(double_i32(4), [1], [2])
    producer = rt.PlanStep(double_i32(4), [0], [1])
    with pytest.raises(rt.CUDAError, match="ASK execution plan validation failed"):
        session.prepareProgram([16, 16, 16], [0], [2], [early, producer], False)


def chain_program(session, n, graph, count=4):
    steps = [rt.PlanStep(double_i32(count), [i], [i + 1]) for i in range(n)]
    return session.prepareProgram([4 * count] * (n + 1), [0], [n], steps, graph)


@pytest.mark.parametrize("graph", [False, True])
def test_chain_uses_two_slots_and_reuses_its_workspace(device, graph):
    session = rt.Session.create(0)
    program = chain_program(session, 4, graph)
    assert len(program.describe()["slot_capacity_bytes"]) == 2
    held = []
    for it in range(2):
        src = session.allocate(16)
        data = np.array([it + 1, 2, -3, 4], np.int32)
        src.copyFromHost(data)
        before = session.stats()["allocations"]
        outs, ev = program.run([src])
        if it == 0:
            assert session.stats()["allocations"] - before == 3  # one public output plus two internal slots
        ev.wait()
        assert np.array_equal(i32s(outs[0]), data * 16)
        held += [src, outs[0]]
    st = session.stats()
    assert st["workspace_reuses"] == 1
    if graph:
        assert st["graph_instantiations"] == 1 and st["graph_launches"] == 2 and st["graph_node_updates"] > 0
        assert st["graph_nodes"] == 4 and st["graph_edges"] == 3
    # two submissions in flight keep independent results (two workspaces)
    a, b = session.allocate(16), session.allocate(16)
    a.copyFromHost(np.array([1, 2, 3, 4], np.int32))
    b.copyFromHost(np.array([5, 6, 7, 8], np.int32))
    (ra,), ea = program.run([a])
    (rb,), eb = program.run([b])
    ea.wait()
    eb.wait()
    assert np.array_equal(i32s(ra), [16, 32, 48, 64]) and np.array_equal(i32s(rb), [80, 96, 112, 128])


@pytest.mark.parametrize("graph", [False, True])
def test_slot_free_program_keeps_one_workspace_in_flight(device, graph):
    """A program without internal buffers reuses its one workspace while
    earlier submissions still run: 40 submissions without waiting, cycling
    through four input/output pairs (so graph nodes are re-recorded while
    earlier launches of the same graph are queued), each result exact, one
    graph instantiated."""
    session = rt.Session.create(0)
    n = 1 << 20
    step = rt.PlanStep(double_i32(n), [0], [1])
    program = session.prepareProgram([4 * n, 4 * n], [0], [1], [step], graph)
    assert program.describe()["slot_capacity_bytes"] == []
    rng = np.random.default_rng(3)
    data = [rng.integers(-1000, 1000, n).astype(np.int32) for _ in range(4)]
    srcs = [session.allocate(4 * n) for _ in range(4)]
    dsts = [session.allocate(4 * n) for _ in range(4)]
    for src, d in zip(srcs, data):
        src.copyFromHost(d)
    events = [program.submit([srcs[k % 4]], [dsts[k % 4]]) for k in range(40)]
    events[-1].wait()
    for dst, d in zip(dsts, data):
        assert np.array_equal(i32s(dst), d * 2)
    st = session.stats()
    assert st["program_submissions"] == 40 and st["workspace_reuses"] == 39
    if graph:
        assert st["graph_instantiations"] == 1 and st["graph_launches"] == 40


@pytest.mark.parametrize("graph", [False, True])
def test_pre_copy(device, graph):
    session = rt.Session.create(0)
    with pytest.raises(rt.CUDAError):
        session.prepareProgram([16, 16], [0], [1], [rt.PlanStep(double_i32(4), [0], [1], preCopy=(2, 1))], graph)
    with pytest.raises(rt.CUDAError):
        session.prepareProgram([32, 16], [0], [1], [rt.PlanStep(double_i32(4), [0], [1], preCopy=(0, 1))], graph)
    program = session.prepareProgram([16, 16], [0], [1], [rt.PlanStep(double_i32(4), [0], [1], preCopy=(0, 1))], graph)
    for it in range(2):
        src = session.allocate(16)
        data = np.array([it + 3, -4, 5, 6], np.int32)
        src.copyFromHost(data)
        (out,), ev = program.run([src])
        ev.wait()
        assert np.array_equal(i32s(out), data * 2)


def test_fork_graph_runs_branches_and_counts_edges(device):
    session = rt.Session.create(0)
    n = 1000
    steps = [rt.PlanStep(double_i32(n), [0], [1])]
    outs = []
    for k in range(3):  # three branches of two steps each, reading the root
        steps.append(rt.PlanStep(double_i32(n), [1], [2 + 2 * k]))
        steps.append(rt.PlanStep(double_i32(n), [2 + 2 * k], [3 + 2 * k]))
        outs.append(3 + 2 * k)
    program = session.prepareProgram([4 * n] * 8, [0], outs, steps, True)
    d = program.describe()
    assert sum(len(x) for x in d["dependencies"]) == 6
    src = session.allocate(4 * n)
    data = np.arange(n, dtype=np.int32) - 400
    src.copyFromHost(data)
    results, ev = program.run([src])
    ev.wait()
    for r in results:
        assert np.array_equal(i32s(r), data * 8)


def direct(plan_recipe, ins, outs, scratch_bytes=0):
    p = ask_b200.Plan(plan_recipe, 0)
    scratch = torch.empty(max(p.scratch_bytes, 16), dtype=torch.uint8, device="cuda") if p.scratch_bytes else None
    p.launch(ins, outs, scratch, torch.cuda.current_stream())


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("fuse", [False, True])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_softmax_program_matches_direct_steps(device, graph, fuse, dtype):
    rows, cols = 512, 4096
    kind = 2 if dtype == "f16" else 3
    x = gen_dev(kind, 0xA5C3, 0, rows * cols, 0.0, 2.0, torch.int16)
    steps = R.cfg3_steps(dtype, rows, cols)
    m = torch.empty(rows, dtype=torch.float32, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    y_ref = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
    direct(steps[0], [x], [m])
    direct(steps[1], [x, m], [s])
    direct(steps[2], [x, m, s], [y_ref])
    torch.cuda.synchronize()

    session = rt.Session.create(0)
    program = session.prepareProgram(
        [2 * rows * cols, 4 * rows, 4 * rows, 2 * rows * cols], [0], [1, 2, 3],
        [rt.PlanStep(steps[0], [0], [1]), rt.PlanStep(steps[1], [0, 1], [2]), rt.PlanStep(steps[2], [0, 1, 2], [3])],
        graph, fuse=fuse)
    d = program.describe()
    if fuse:  # the runtime runs the three steps as one fused softmax step
        assert [k["kernel"] for k in d["steps"]] == [f"softmax_rows_{dtype}"]
        assert session.stats()["fused_softmax_steps"] == 1
    else:
        assert [k["kernel"] for k in d["steps"]] == [f"softmax_rows_max_{dtype}",
                                                     f"softmax_rows_sum_{dtype}", f"softmax_rows_norm_{dtype}"]
    xin = session.importTensor(x, readonly=True)
    outs = [torch.empty_like(m), torch.empty_like(s), torch.empty_like(y_ref)]
    bufs = [session.importTensor(t) for t in outs]
    session.waitForExternalStream(torch.cuda.current_stream())
    for _ in range(3):
        program.submit([xin], bufs).wait()
        assert torch.equal(outs[0].view(torch.int32), m.view(torch.int32))
        if fuse:  # the fused sum may round differently in the last place; y then by at most one unit
            assert torch.all((outs[1].double() - s.double()).abs() <= 2.0 ** -21 * s.double().abs())
            assert int((outs[2].int() - y_ref.int()).abs().max()) <= 1
        else:
            assert torch.equal(outs[1].view(torch.int32), s.view(torch.int32)) and torch.equal(outs[2], y_ref)
        for t in outs:
            t.zero_()
        torch.cuda.synchronize()


@pytest.mark.parametrize("graph", [False, True])
def test_split_reduction_scratch_is_a_private_slot(device, graph):
    n = (1 << 22) + 17
    x = gen_dev(0, 0xA5C5, 0, n, 0.0, 1.0, torch.float32)
    recipe = R.cfg5a_step(n)
    sref = torch.empty(1, dtype=torch.float32, device="cuda")
    mref = torch.empty(1, dtype=torch.float32, device="cuda")
    aref = torch.empty(1, dtype=torch.int64, device="cuda")
    direct(recipe, [x], [sref, mref, aref])
    torch.cuda.synchronize()
    session = rt.Session.create(0)
    program = session.prepareProgram([4 * n, 4, 4, 8], [0], [1, 2, 3], [rt.PlanStep(recipe, [0], [1, 2, 3])], graph)
    d = program.describe()
    assert d["steps"][0]["scratch"] == 4 and len(d["slot_capacity_bytes"]) == 1
    (s, m, a), ev = program.run([session.importTensor(x, readonly=True)])
    ev.wait()
    assert s.copyToHost() == sref.cpu().numpy().tobytes()
    assert m.copyToHost() == mref.cpu().numpy().tobytes()
    assert a.copyToHost() == aref.cpu().numpy().tobytes()


@pytest.mark.parametrize("graph", [False, True])
def test_gather_then_scatter_program(device, graph):
    rows, dim, n = 4096, 64, 50000
    table = gen_dev(1, 0xA5C4, 0, rows * dim, 0.0, 1.0, torch.float32)
    idx = gen_dev(5, 0xA5C4, 1, n, 1.1, rows, torch.int64)
    base = gen_dev(4, 0xA5C4, 3, rows * dim, 0, 0, torch.int32).float()
    gathered = torch.empty(n * dim, dtype=torch.float32, device="cuda")
    out_ref = torch.empty(rows * dim, dtype=torch.float32, device="cuda")
    direct(R.cfg4_gather_step(rows, dim, n), [table, idx], [gathered])
    direct(R.cfg4_scatter_step(rows, dim, n), [base, idx, gathered], [out_ref])
    torch.cuda.synchronize()
    session = rt.Session.create(0)
    steps = [rt.PlanStep(R.cfg4_gather_step(rows, dim, n), [0, 1], [3]),
             rt.PlanStep(R.cfg4_scatter_step(rows, dim, n), [2, 1, 3], [4])]
    program = session.prepareProgram([4 * rows * dim, 8 * n, 4 * rows * dim, 4 * n * dim, 4 * rows * dim], [0, 1, 2],
                                     [4], steps, graph)
    ins = [session.importTensor(t, readonly=True) for t in (table, idx, base)]
    (out,), ev = program.run(ins)
    ev.wait()
    got = np.frombuffer(out.copyToHost(), np.float32)
    ref = out_ref.cpu().numpy()
    # f32 scatter sums are order-dependent: compare against the direct launch within rounding
    assert np.allclose(got, ref, rtol=1e-5, atol=1e-4)


def test_closed_session_refuses_work(device):
    session = rt.Session.create(0)
    program = chain_program(session, 2, False)
    src = session.allocate(16)
    session.close()
    rejects(lambda: program.run([src]))
    rejects(lambda: session.allocate(16))


@pytest.mark.parametrize("graph", [False, True])
def test_bound_submissions_reuse_completion_events(device, graph):
    """PreparedProgram.bind repeats one submission; retired completion events
    return to the session's pool (event_reuses), as in the reference."""
    s = rt.Session.create(0)
    n = 1 << 12
    prog = s.prepareProgram([4 * n, 4 * n], [0], [1], [rt.PlanStep(double_i32(n), [0], [1])], graph=graph)
    x = s.allocate(4 * n)
    x.copyFromHost(np.arange(n, dtype=np.int32).tobytes())
    y = s.allocate(4 * n)
    run = prog.bind([x], [y])
    for _ in range(200):
        run()
    s.synchronize()
    assert np.array_equal(i32s(y), 2 * np.arange(n, dtype=np.int32))
    for _ in range(50):
        run()
    s.synchronize()
    st = s.stats()
    assert st["program_submissions"] == 250
    assert st["event_reuses"] > 0 and st["event_creations"] + st["event_reuses"] == 250
    s.close()


def test_concurrent_submissions_from_threads(device):
    """Sessions serialise every call (the reference's recursive session mutex):
    four threads submitting to one session each get their own results."""
    import threading
    s = rt.Session.create(0)
    n = 1 << 14
    prog = s.prepareProgram([4 * n, 4 * n, 4 * n], [0], [2],
                            [rt.PlanStep(double_i32(n), [0], [1]), rt.PlanStep(double_i32(n), [1], [2])], graph=True)
    errors = []

    def worker(t):
        try:
            x = s.allocate(4 * n)
            base = np.arange(n, dtype=np.int32) + 1000 * t
            x.copyFromHost(base.tobytes())
            for _ in range(30):
                outs, ev = prog.run([x])
                ev.wait()
                if not np.array_equal(i32s(outs[0]), 4 * base):
                    errors.append(t)
                    return
        except Exception as e:  # surfaced below
            errors.append(repr(e))

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(4)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    assert s.stats()["program_submissions"] == 120
    s.close()
