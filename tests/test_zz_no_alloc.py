"""The fixed-scratch entry point (ask_b200_plan_launch_noalloc).

Callers that cannot allocate device memory when they launch -- a runtime whose
device memory is entirely planned ahead by a pool, or a host with a fixed
device-memory budget -- launch reduce plans through this entry point, which
takes the scratch of a split reduction, or of a column reduction whose extent
is split into chunks, from a 1 MiB array built into the library instead of a
buffer the caller allocates.  Its results must equal those of the
ordinary entry point (ask_b200_plan_launch with caller-provided scratch); the
split reduction is deterministic, so the comparison is bit-exact, which is
within every tolerance the other reduction tests use.  Two calls in a row check
that leftover contents of the shared array do not leak into the next result.

This file is named so pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

import ask_b200
from ask_b200 import recipes as R

pytestmark = pytest.mark.gpu


def _ports(tensors):
    vals = [t.data_ptr() for t in tensors]
    return (ctypes.c_uint64 * len(vals))(*vals), len(vals)


def _outputs(plan):
    kinds = {"f32": torch.float32, "i64": torch.int64, "bool": torch.uint8, "i32": torch.int32}
    return [torch.full((p["elements"],), 7, dtype=kinds[p["element_type"]], device="cuda")
            for p in plan.describe()["port_map"][plan.n_inputs:]]


def _same_bits(a, b):
    """Bit-for-bit equality (NaN results compare equal to themselves)."""
    ints = {torch.float32: torch.int32, torch.float64: torch.int64}
    if a.dtype in ints:
        a, b = a.view(ints[a.dtype]), b.view(ints[b.dtype])
    return torch.equal(a, b)


def _launch_noalloc(plan, inputs, outputs):
    arr, n = _ports(list(inputs) + list(outputs))
    status = ask_b200._lib.ask_b200_plan_launch_noalloc(plan._h, arr, n, torch.cuda.current_stream().cuda_stream)
    assert status == ask_b200.OK, ask_b200._lib.ask_b200_last_error().decode()


def _launch_ordinary(plan, inputs, outputs):
    scratch = torch.empty(max(plan.scratch_bytes, 16), dtype=torch.uint8, device="cuda")
    arr, n = _ports(list(inputs) + list(outputs))
    status = ask_b200._lib.ask_b200_plan_launch(plan._h, arr, n, scratch.data_ptr(),
                                                torch.cuda.current_stream().cuda_stream)
    assert status == ask_b200.OK, ask_b200._lib.ask_b200_last_error().decode()


@pytest.mark.parametrize("recipe_fn,n", [
    (lambda n: R.cfg5a_step(n), (1 << 22) + 7),
    (lambda n: R.cfg5a_step(n, index_base=1000), 1 << 20),
    (lambda n: R.reduce(_prog_f32(), _prog_f32.value, ["sum", "max", "min", "argmax", "argmin", "prod"],
                        3, n // 3, strategy="split"), 3 * 300001),
])
def test_noalloc_matches_ordinary_launch_twice(recipe_fn, n):
    torch.cuda.set_device(0)
    rec = recipe_fn(n)
    plan = ask_b200.Plan(rec, 0)
    assert plan.describe()["strategy"] == "split"
    rng = np.random.default_rng(n)
    x = torch.from_numpy(rng.standard_normal(rec["outer"] * rec["extent"]).astype(np.float32)).cuda()
    x[x.numel() // 2] = float("-inf")
    ref = _outputs(plan)
    _launch_ordinary(plan, [x], ref)
    for _ in range(2):
        got = _outputs(plan)
        _launch_noalloc(plan, [x], got)
        torch.cuda.synchronize()
        for g, r in zip(got, ref):
            assert _same_bits(g, r)


def test_noalloc_column_chunks_match_ordinary_launch_twice():
    """A column reduction with few columns over a long extent splits the
    extent into chunks whose partial records live in scratch: through the
    fixed array they must combine to the same bits as with caller scratch."""
    torch.cuda.set_device(0)
    outer, extent, inner = 1, 32768, 8
    p = R.Program()
    v = p.input("f32")
    plan = ask_b200.Plan(R.reduce(p, v, ["sum", "max", "min", "argmax", "argmin"], outer, extent, inner), 0)
    d = plan.describe()
    assert d["kernel"] == "reduce_column_chunks_generic" and d["launch"]["grid"][1] > 1
    assert 0 < plan.scratch_bytes <= ask_b200_noalloc_limit()
    x = torch.from_numpy(np.random.default_rng(5).standard_normal(outer * extent * inner).astype(np.float32)).cuda()
    x.view(extent, inner)[20000, 1] = float("nan")
    x.view(extent, inner)[:, 2] = 3.0
    ref = _outputs(plan)
    _launch_ordinary(plan, [x], ref)
    for _ in range(2):
        got = _outputs(plan)
        _launch_noalloc(plan, [x], got)
        torch.cuda.synchronize()
        for g, r in zip(got, ref):
            assert _same_bits(g, r)


def _prog_f32():
    p = R.Program()
    _prog_f32.value = p.input("f32")
    return p


def test_noalloc_rejects_plans_beyond_the_fixed_array():
    torch.cuda.set_device(0)
    p = R.Program()
    v = p.input("f32")
    rec = R.reduce(p, v, ["sum", "max", "min", "argmax", "argmin", "prod"], 64, 1 << 24, strategy="split")
    plan = ask_b200.Plan(rec, 0)
    needed = 64 * plan.describe()["launch"]["grid"][0] * 6 * 16
    assert needed > ask_b200_noalloc_limit()
    x = torch.zeros(64 << 24, dtype=torch.float32, device="cuda")
    outs = _outputs(plan)  # typed and sized as the port map says
    arr, n = _ports([x] + outs)
    status = ask_b200._lib.ask_b200_plan_launch_noalloc(plan._h, arr, n, None)
    assert status == ask_b200.E_INVALID
    assert "fixed scratch array" in ask_b200._lib.ask_b200_last_error().decode()


def test_noalloc_serves_reduce_plans_only():
    torch.cuda.set_device(0)
    plan = ask_b200.Plan(R.cfg5b_step(16), 0)
    a = torch.zeros(16, dtype=torch.int32, device="cuda")
    arr, n = _ports([a, a, torch.empty_like(a)])
    assert ask_b200._lib.ask_b200_plan_launch_noalloc(plan._h, arr, n, None) == ask_b200.E_UNSUPPORTED


def ask_b200_noalloc_limit():
    return 1 << 20
