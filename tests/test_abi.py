"""The C-ABI library: it loads without a GPU, exports every entry point the
public header declares, and its host-side plan logic (recipe validation,
kernel selection, port map, error reporting) behaves as the reference's
lowering and runtime contracts require.  No kernel is launched here."""
import ctypes
import json
import os
import re

import pytest

import ask_b200
from ask_b200 import recipes as R

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ask_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(ask_b200_[a-z_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib_built):
    lib = ctypes.CDLL(ask_b200.LIBRARY_PATH)
    names = declared_symbols()
    assert len(names) >= 14
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/ask_b200.h but not exported"
    assert set(names) == set(ask_b200.exported_symbols())


def test_runtime_library_exports_every_declared_symbol(lib_built):
    from ask_b200 import runtime as rt
    lib = ctypes.CDLL(ask_b200.LIBRARY_PATH)
    text = open(os.path.join(ROOT, "include", "ask_b200_runtime.h")).read()
    names = sorted(set(re.findall(r"ASK_B200_API\s+int\s+(ask_b200_[a-z_0-9]+)\s*\(", text)))
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/ask_b200_runtime.h but not exported"
    assert set(names) == set(rt.RUNTIME_SIGNATURES)
    text = open(os.path.join(ROOT, "include", "ask_b200_lower.h")).read()
    lowered = sorted(set(re.findall(r"ASK_B200_API\s+int\s+(ask_b200_[a-z_0-9]+)\s*\(", text)))
    assert lowered == sorted(rt._LOWER_SIGNATURES)
    for name in lowered:
        assert hasattr(lib, name)


def test_runtime_session_without_gpu_is_an_error():
    import torch
    from ask_b200 import runtime as rt
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(rt.CUDAError) as err:
        rt.Session.create(0)
    assert err.value.status == ask_b200.E_DEVICE


def test_abi_version():
    assert ask_b200.abi_version() == 1


def host_plan(recipe):
    return ask_b200.Plan(recipe, device=-1)


@pytest.mark.parametrize("name,recipe,kernel", [
    ("cfg1", R.cfg1_step(), "ew_cfg1"),
    ("cfg2", R.cfg2_step(), "reduce_warp_row_rowstats_f32"),
    ("cfg5a", R.cfg5a_step(), "reduce_split_global_f32"),
    ("cfg5b", R.cfg5b_step(), "ew_cfg5b"),
    ("cfg4g", R.cfg4_gather_step(), "gather_rows"),
    ("cfg4s", R.cfg4_scatter_step(), "scatter_add_sorted_rows"),
])
def test_config_recipes_select_specialised_kernels(name, recipe, kernel):
    d = host_plan(recipe).describe()
    assert d["kernel"] == kernel
    assert d["target"] == {"backend": "cuda", "arch": 100}


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_softmax_partition_steps(dtype):
    kernels = [host_plan(s).describe()["kernel"] for s in R.cfg3_steps(dtype)]
    assert kernels == [f"softmax_rows_max_{dtype}", f"softmax_rows_sum_{dtype}", f"softmax_rows_norm_{dtype}"]
    # a grid cap keeps the warp-row reductions and the elementwise functor
    capped = [host_plan(dict(s, blocks_per_sm=4)).describe()["kernel"] for s in R.cfg3_steps(dtype)]
    assert capped == [f"reduce_warp_row_softmax_max_{dtype}", f"reduce_warp_row_softmax_sum_{dtype}",
                      f"ew_softmax_norm_{dtype}"]
    d = host_plan(R.cfg3_steps(dtype)[1]).describe()
    assert d["strategy"] == "row_cta" and d["launch"]["block"] == [128, 1, 1]
    # a forced strategy, or rows the row kernel does not take, keep the warp-row reduction
    forced = [dict(s, strategy="warp_row") for s in R.cfg3_steps(dtype)[:2]]
    assert [host_plan(s).describe()["kernel"] for s in forced] == [
        f"reduce_warp_row_softmax_max_{dtype}", f"reduce_warp_row_softmax_sum_{dtype}"]
    odd = [host_plan(s).describe()["kernel"] for s in R.cfg3_steps(dtype, 64, 1000)]
    assert odd == [f"reduce_warp_row_softmax_max_{dtype}", f"reduce_warp_row_softmax_sum_{dtype}",
                   f"ew_softmax_norm_{dtype}"]


def test_port_map_orders_inputs_then_outputs():
    d = host_plan(R.cfg1_step(1000)).describe()
    ports = d["port_map"]
    assert [p["logical_port"] for p in ports] == ["input:0", "input:1", "input:2", "output:0", "output:1"]
    assert [p["argument"] for p in ports] == list(range(5))
    assert all(p["elements"] == 1000 and p["element_type"] == "f32" for p in ports)
    assert d["requires_disjoint_outputs"] is True
    inv = d["invocation"]
    assert inv["version"] == 2 and inv["grid"] == d["launch"]["grid"] and inv["block"] == d["launch"]["block"]
    assert inv["arguments"] == [p["logical_port"] for p in d["port_map"]]
    assert d["required_element_types"] == sorted({p["element_type"] for p in d["port_map"]},
                                                 key=["bool", "i32", "i64", "f32", "f16", "bf16"].index)


def test_reduce_outputs_and_scratch():
    p = host_plan(R.cfg5a_step(1 << 20))
    d = p.describe()
    assert d["strategy"] == "split" and d["shardable"] is True
    assert [x["element_type"] for x in d["port_map"][1:]] == ["f32", "f32", "i64"]
    assert p.scratch_bytes > 0 and p.kernel_launches == 2
    q = host_plan(R.cfg2_step(64, 1024))
    assert q.scratch_bytes == 0 and q.kernel_launches == 1


def test_scatter_declares_pre_copy():
    d = host_plan(R.cfg4_scatter_step(16, 8, 32)).describe()
    assert d["pre_copy"] == {"input": 0, "output": 0}
    assert [x["logical_port"] for x in d["port_map"]] == ["input:0", "input:1", "input:2", "output:0"]


def test_generic_program_allocates_registers():
    p = R.Program()
    xs = [p.input("f32") for _ in range(4)]
    acc = xs[0]
    for x in xs[1:]:
        acc = p.add(acc, p.mul(x, x))
    d = host_plan(R.elementwise(p, [acc], 10)).describe()
    assert d["kernel"] == "ew_generic" and d["specialized"] is False
    assert d["registers"] < len(p.insns)


@pytest.mark.parametrize("bad,status,fragment", [
    ({"family": "elementwise", "count": 4, "inputs": [{"dtype": "i32"}], "outputs": [{"dtype": "i32"}],
      "program": [["input", 0], ["exp", 0]], "results": [1]}, ask_b200.E_INVALID, "needs f32"),
    ({"family": "elementwise", "count": 4, "inputs": [{"dtype": "f32"}], "outputs": [{"dtype": "f32"}],
      "program": [["input", 0], ["shift_left", 0, 0]], "results": [1]}, ask_b200.E_INVALID, "i32 or i64"),
    ({"family": "elementwise", "count": 4, "inputs": [{"dtype": "f32"}, {"dtype": "f16"}],
      "outputs": [{"dtype": "f32"}], "program": [["input", 0], ["input", 1], ["add", 0, 1]], "results": [2]},
     ask_b200.E_INVALID, "identical types"),
    ({"family": "elementwise", "count": 4, "inputs": [{"dtype": "f32"}], "outputs": [{"dtype": "f32"}],
      "program": [["input", 0], ["matmul", 0, 0]], "results": [1]}, ask_b200.E_UNSUPPORTED, "matmul"),
    ({"family": "elementwise", "count": 4, "inputs": [{"dtype": "f32"}], "outputs": [{"dtype": "f32"}],
      "program": [["input", 0], ["add", 0, 5]], "results": [1]}, ask_b200.E_INVALID, "earlier instruction"),
    ({"family": "elementwise", "count": 4, "inputs": [{"dtype": "f32"}], "outputs": [{"dtype": "i32"}],
      "program": [["input", 0]], "results": [0]}, ask_b200.E_INVALID, "does not match"),
    ({"family": "reduce", "outer": 2, "extent": 0, "inputs": [{"dtype": "f32"}], "program": [["input", 0]],
      "results": [0], "reductions": [{"op": "argmax"}]}, ask_b200.E_INVALID, "non-empty"),
    ({"family": "reduce", "outer": 2, "extent": 3, "inputs": [{"dtype": "f32"}], "program": [["input", 0]],
      "results": [0], "reductions": [{"op": "any"}]}, ask_b200.E_INVALID, "bool"),
    ({"family": "gather", "dtype": "f32", "index_dtype": "f32", "dim": 4, "inner": 2, "n": 3},
     ask_b200.E_INVALID, "i32 or i64"),
    ({"family": "softmax_v2"}, ask_b200.E_UNSUPPORTED, "unknown family"),
    ("{not json", ask_b200.E_INVALID, "recipe JSON"),
])
def test_invalid_recipes_are_rejected(bad, status, fragment):
    with pytest.raises(ask_b200.AskB200Error) as err:
        host_plan(bad)
    assert err.value.status == status
    assert fragment in str(err.value)


def test_port_limits():
    rec = {"family": "elementwise", "count": 4, "inputs": [{"dtype": "f32"}] * 16,
           "outputs": [{"dtype": "f32"}] * 16, "program": [["input", k] for k in range(16)],
           "results": list(range(16))}
    host_plan(rec)  # 32 ports is fine
    rec["inputs"] = [{"dtype": "f32"}] * 17
    with pytest.raises(ask_b200.AskB200Error) as err:
        host_plan(rec)
    assert err.value.status == ask_b200.E_UNSUPPORTED
    rec["inputs"] = [{"dtype": "f32"}] * 16
    rec["program"] = [["input", 0]] * 49
    with pytest.raises(ask_b200.AskB200Error) as err:
        host_plan(rec)
    assert err.value.status == ask_b200.E_UNSUPPORTED


def test_host_only_plan_refuses_to_launch():
    p = host_plan(R.cfg1_step(16))
    with pytest.raises(ask_b200.AskB200Error) as err:
        p.launch([1 << 20, 2 << 20, 3 << 20], [4 << 20, 5 << 20])
    assert err.value.status == ask_b200.E_DEVICE


def test_launch_checks_port_count_and_alignment():
    p = host_plan(R.cfg1_step(16))
    with pytest.raises(ask_b200.AskB200Error) as err:
        p.launch([1 << 20], [2 << 20])
    assert err.value.status == ask_b200.E_INVALID and "ports" in str(err.value)
    with pytest.raises(ask_b200.AskB200Error) as err:
        p.launch([1 << 20, (2 << 20) + 2, 3 << 20], [4 << 20, 5 << 20])
    assert "aligned" in str(err.value)


def test_last_error_is_cleared_on_success():
    with pytest.raises(ask_b200.AskB200Error):
        host_plan({"family": "nope"})
    host_plan(R.cfg1_step(8))
    assert ask_b200._lib.ask_b200_last_error() == b""


def test_constants_round_once_to_target_type():
    # 1 + 2^-11 + 2^-30 rounds directly to f16 1 + 2^-10 (one RNE step, docs/en/ir.md:108)
    p = R.Program()
    x = p.input("f16")
    c = p.const("f16", 1 + 2 ** -11 + 2 ** -30)
    d = host_plan(R.elementwise(p, [p.add(x, c)], 4)).describe()
    assert d["family"] == "elementwise"


def test_shard_ranges_partition_the_axis():
    for total in (1 << 32, 1 << 31, 1000, 7):
        for world in (1, 2, 3, 4, 8):
            spans = [R.shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
                assert e0 == b1
            if total >= 1024 * world:
                assert all(b % 1024 == 0 for b, _ in spans)


def test_blocks_per_sm_caps_persistent_grids():
    rec = R.cfg5b_step(1 << 28)
    full = ask_b200.Plan(rec, -1).describe()["launch"]["grid"][0]
    rec["blocks_per_sm"] = 3
    assert ask_b200.Plan(rec, -1).describe()["launch"]["grid"][0] == 3 * 148 < full
    red = R.cfg2_step(65536, 1024)
    red["blocks_per_sm"] = 2
    assert ask_b200.Plan(red, -1).describe()["launch"]["grid"][0] == 2 * 148
    for bad in (0, 33, -1):
        rec["blocks_per_sm"] = bad
        with pytest.raises(ask_b200.AskB200Error) as err:
            ask_b200.Plan(rec, -1)
        assert "blocks_per_sm" in str(err.value)
