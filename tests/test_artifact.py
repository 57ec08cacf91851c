"""Kernel artifacts (external-kernel-artifact v2) on the host: the generator's
sources compile for sm_100a, requests are validated as docs/en/compilers.md
specifies, the worker keeps the process interface, and scalar arguments are
encoded in the launch ABI.  Loading and running artifacts is in
test_artifact_gpu.py."""
import base64
import ctypes
import json
import os
import re
import subprocess
import sys

import numpy as np
import pytest

import ask_b200
from ask_b200 import artifact as A
from ask_b200 import recipes as R

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def ports_of(recipe):
    return ask_b200.Plan(recipe, -1).describe()["port_map"]


def request_for(recipe, entry="step_kernel", grid=(296, 1, 1), scalars=(("n", "i32", 7),), source=None):
    return A.request_for(recipe, entry, grid, scalars, source)


def fake_cubin(source):
    return b"\x7fELF" + b"\0" * 60


def cases():
    p = R.Program()
    x = p.input("bool")
    any_rec = R.reduce(p, x, ["any", "all"], 4, 5000)
    p = R.Program()
    a, s = p.input("i64"), p.input("i64", "scalar")
    i64_rec = R.elementwise(p, [p.op("mul", a, s), p.compare("gt", a, s)], 1001)
    p = R.Program()
    v = p.input("f32")
    col_rec = R.reduce(p, v, ["sum", "argmax"], 3, 50, 7)
    return {
        "cfg1": (R.cfg1_step(4099), "elementwise_functor"),
        "softmax_norm": (R.cfg3_steps("bf16", 64, 1024)[2], "elementwise_functor"),
        "cfg5b": (R.cfg5b_step(1 << 20), "elementwise_functor"),
        "i64_scalar": (i64_rec, "elementwise"),
        "cfg2_rows": (R.cfg2_step(65536, 1024), "reduce_rows_warp_fast"),
        "softmax_max": (R.cfg3_steps("f16", 64, 4096)[0], "reduce_rows_cta_fast"),
        "softmax_sum": (R.cfg3_steps("bf16", 4096, 512)[1], "reduce_rows_warp_fast"),
        "cfg5a_global": (R.cfg5a_step(1 << 24), "reduce_rows_cta_fast"),
        "bool_any_all": (any_rec, "reduce_rows_cta"),
        "columns": (col_rec, "reduce_columns"),
        "gather_rows": (R.cfg4_gather_step(1000, 64, 4096), "gather_rows"),
        "gather_elems": (R.gather("f16", "i32", 1000, 3, 77), "gather_elems"),
    }


@pytest.mark.parametrize("name", list(cases()))
def test_generated_sources_compile_for_sm100a(name):
    recipe, body = cases()[name]
    params = [p["logical_port"] for p in ports_of(recipe)] + ["i32", "fp64"]
    gen = A.artifact_source(recipe, "k_" + name, [592, 1, 1], params)
    assert gen["body"] == body
    assert gen["launch"] == {"grid": [592, 1, 1], "block": [256, 1, 1], "shared_bytes": 0}
    assert gen["parameter_widths"] == [0] * (len(params) - 2) + [4, 8]
    # functor entries are compiled for the functor's occupancy (the cfg1 functor keeps two units in flight)
    bounds = "askb::art::kThreads" if body != "elementwise_functor" else \
        "askb::art::kThreads, askb::art::kDeepFunctorMinBlocks" if name == "cfg1" else \
        "askb::art::kThreads, askb::art::kFunctorMinBlocks"
    assert f'extern "C" __global__ void __launch_bounds__({bounds}) k_{name}(' in gen["source"]
    cubin = A.compile_source(gen["source"])
    assert cubin[:4] == b"\x7fELF"


def test_view_steps_use_the_view_loop():
    from test_lowering import view_steps
    for name, src, ins, want in view_steps():
        out = A._recipe_of(src)[0]
        params = [p["logical_port"] for p in ports_of(out)]
        gen = A.artifact_source(out, "view_" + name, [8, 1, 1], params)
        assert gen["body"] == "elementwise_view", name
        assert "__constant__ askb::ViewSet kViews" in gen["source"]
    A.compile_source(gen["source"])


def test_generator_refuses_what_an_artifact_cannot_express():
    scat = R.cfg4_scatter_step(100, 16, 1000)
    params = [p["logical_port"] for p in ports_of(scat)]
    with pytest.raises(A.ArtifactError) as err:
        A.artifact_source(scat, "k", [1, 1, 1], params)
    assert err.value.status == ask_b200.E_UNSUPPORTED and "pre_copy" in str(err.value)
    rec = R.cfg1_step(100)
    ps = [p["logical_port"] for p in ports_of(rec)]
    for grid, params, msg in [([4, 2, 1], ps, "one-dimensional"),
                              ([0, 1, 1], ps, "grid entries"),
                              ([4, 1, 1], ps[:-1], "output:1 is bound to no parameter"),
                              ([4, 1, 1], ps + ["input:0"], "binds a port twice"),
                              ([4, 1, 1], ps + ["input:9"], "names no port"),
                              ([4, 1, 1], ps + ["f8"], "unknown scalar"),
                              ([4, 1, 1], ps + ["input:01"], "neither")]:
        with pytest.raises(A.ArtifactError) as err:
            A.artifact_source(rec, "k", grid, params)
        assert msg in str(err.value), (msg, str(err.value))
    with pytest.raises(A.ArtifactError) as err:
        A.artifact_source(rec, "9k", [4, 1, 1], ps)
    assert "entry" in str(err.value)


def test_request_to_artifact_fields():
    rec = R.cfg1_step(4099)
    req = request_for(rec, scalars=(("n", "i32", 4099), ("alpha", "fp32", 0.5), ("flag", "i1", True)))
    art = A.build_artifact(req, compile_fn=fake_cubin)
    assert list(art) == list(A.ARTIFACT_FIELDS)
    assert art["entry"] == "step_kernel" and art["format"] == "cubin"
    assert art["target"] == {"backend": "cuda", "arch": 100, "warp_size": 32}
    assert art["launch"]["grid"] == [296, 1, 1] and art["launch"]["block"] == [256, 1, 1]
    assert art["arguments"] == ["input:0", "input:1", "input:2", "output:0", "output:1",
                                {"type": "i32", "value": 4099}, {"type": "fp32", "value": 0.5},
                                {"type": "i1", "value": True}]
    assert art["required_element_types"] == ["f32"]
    assert A.parameter_widths(art) == [0, 0, 0, 0, 0, 4, 4, 1]
    A.validate_artifact(art, req)


def test_request_parameter_order_is_the_signature_order():
    rec = R.cfg1_step(64)
    req = request_for(rec, scalars=())
    keys = list(req["signature"])
    order = [keys[4], "n", keys[0], keys[3], keys[2], keys[1]]
    req["signature"] = {k: (req["signature"][k] if k != "n" else "u16") for k in order}
    req["source_bindings"] = {k: (req["source_bindings"][k] if k != "n" else 9) for k in order}
    gen_params = []
    art = A.build_artifact(req, compile_fn=lambda src: gen_params.append(src) or fake_cubin(src))
    assert art["arguments"] == ["output:1", {"type": "u16", "value": 9}, "input:0", "output:0", "input:2", "input:1"]
    assert re.search(r"k\(void\* __restrict__ p0, uint16_t p1, const void\* __restrict__ p2", gen_params[0].replace(
        "step_kernel", "k"))


@pytest.mark.parametrize("mutate,msg", [
    (lambda r: r.update(protocol_version=1), "protocol version 2"),
    (lambda r: r["target"].update(arch=90), "sm_100a"),
    (lambda r: r["target"].update(backend="rocm"), "backend"),
    (lambda r: r.update(grid=[1, 1]), "grid"),
    (lambda r: r.update(grid=[2, 2, 1]), "one-dimensional"),
    (lambda r: r.update(extra=1), "unknown request fields"),
    (lambda r: r.pop("port_shapes"), "missing request fields"),
    (lambda r: r.update(fixed_options={"format": "ptx"}), "fixed_options"),
    (lambda r: r.update(entry="bad name"), "identifier"),
    (lambda r: r["signature"].update(input_0="*fp16"), "holds f32"),
    (lambda r: r["source_bindings"].update(n=1 << 40), "outside"),
    (lambda r: r["source_bindings"].update(n=1.5), "integers"),
    (lambda r: r["source_bindings"].update(input_0="output:0"), "binds a port twice"),
    (lambda r: r["port_shapes"].update({"input:0": [4, 1001]}), "elements"),
    (lambda r: r["port_shapes"].pop("output:1"), "no shape"),
    (lambda r: r.update(source="{not json"), "recipe JSON"),
    (lambda r: r.update(source='{"a": 1}'), "not an ask_b200 recipe"),
    (lambda r: r.update(source="module {}"), "supported ASK step"),
])
def test_malformed_requests_are_refused(mutate, msg):
    req = request_for(R.cfg1_step(4000))
    mutate(req)
    with pytest.raises(A.ArtifactError) as err:
        A.build_artifact(req, compile_fn=fake_cubin)
    assert msg in str(err.value), str(err.value)


def test_routing_fields_are_ignored():
    req = request_for(R.cfg5b_step(100))
    req.update(compiler="ask_b200", op_id=3, function="main", implementation="impl0")
    A.build_artifact(req, compile_fn=fake_cubin)


def test_step_module_sources_bind_function_arguments():
    from test_lowering import view_steps
    name, src, ins, want = view_steps()[3]  # concatenate of three arguments, one transposed
    lowered = A._recipe_of(src)
    recipe, args = lowered
    shapes = {f"input:{k}": list(a.shape) for k, a in enumerate(ins)}
    shapes["output:0"] = list(want.shape)
    sig = {f"a{k}": "*i32" for k in range(len(ins))}
    sig["out"] = "*i32"
    bind = {f"a{k}": f"input:{k}" for k in range(len(ins))}
    bind["out"] = "output:0"
    req = {"protocol_version": 2, "source": src, "entry": "concat3", "signature": sig, "source_bindings": bind,
           "constants": {}, "fixed_options": {}, "target": {"backend": "cuda", "arch": 100}, "grid": [4, 1, 1],
           "port_shapes": shapes}
    art = A.build_artifact(req, compile_fn=fake_cubin)
    assert art["arguments"] == ["input:0", "input:1", "input:2", "output:0"]


def test_validate_artifact_catches_mismatches():
    req = request_for(R.cfg5b_step(100))
    art = A.build_artifact(req, compile_fn=fake_cubin)
    for mutate, msg in [(lambda a: a.update(extra=1), "exactly the fields"),
                        (lambda a: a["launch"].update(grid=[1, 1, 1]), "grid differs"),
                        (lambda a: a["arguments"].append("input:0"), "exactly once"),
                        (lambda a: a.update(payload=base64.b64encode(b"abcd").decode()), "ELF"),
                        (lambda a: a["arguments"].__setitem__(-1, {"type": "i32", "value": 8}), "bindings")]:
        bad = json.loads(json.dumps(art))
        mutate(bad)
        with pytest.raises(A.ArtifactError) as err:
            A.validate_artifact(bad, req)
        assert msg in str(err.value)


def test_scalar_abi_bytes():
    assert A.scalar_bytes("i1", True) == b"\x01" and A.scalar_bytes("i1", False) == b"\x00"
    assert A.scalar_bytes("i8", -2) == b"\xfe"
    assert A.scalar_bytes("u16", 0xBEEF) == b"\xef\xbe"
    assert A.scalar_bytes("i32", -1) == b"\xff\xff\xff\xff"
    assert A.scalar_bytes("u64", 2**64 - 1) == b"\xff" * 8
    assert A.scalar_bytes("i64", -(2**63)) == b"\0" * 7 + b"\x80"
    assert A.scalar_bytes("fp32", 0.1) == np.float32(0.1).tobytes()
    assert A.scalar_bytes("fp64", 0.1) == np.float64(0.1).tobytes()
    assert A.scalar_bytes("fp16", 1 / 3) == np.float16(1 / 3).tobytes()
    # bf16: round to nearest even of the f32 value
    for v in [1.0, 1 / 3, -2.5e-3, 3.0e38, 1.00390625, 1.01171875]:
        f = np.float32(v).view(np.uint32)
        want = ((int(f) + 0x7FFF + ((int(f) >> 16) & 1)) >> 16) & 0xFFFF
        assert A.scalar_bytes("bf16", v) == int(want).to_bytes(2, "little")
    assert A.scalar_bytes("bf16", 1.00390625) == (0x3F80).to_bytes(2, "little")  # tie to even
    with pytest.raises(A.ArtifactError):
        A.scalar_bytes("u8", 256)
    with pytest.raises(A.ArtifactError):
        A.scalar_bytes("fp32", float("inf"))


def test_artifact_step_binds_logical_buffers():
    req = request_for(R.cfg5b_step(100), scalars=(("n", "i32", 100),))
    art = A.build_artifact(req, compile_fn=fake_cubin)
    step = A.artifact_step(art, kernel=object(), inputs=[4, 7], outputs=[9])
    d = step.to_json(kernel_index=0)
    assert d["kernel"] == 0 and d["inputs"] == [4, 7] and d["outputs"] == [9]
    assert d["arguments"] == [{"buffer": 4}, {"buffer": 7}, {"buffer": 9}, {"scalar": "64000000"}]
    assert d["grid"] == [296, 1, 1] and d["block"] == [256, 1, 1] and d["shared_bytes"] == 0


def run_worker(*args, cwd=ROOT):
    return subprocess.run([sys.executable, "-m", "ask_b200.worker", *args], capture_output=True, text=True, cwd=cwd)


def test_worker_process_interface(tmp_path):
    req = request_for(R.cfg5b_step(1 << 12), scalars=(("n", "i32", 4096),))
    rpath, apath = tmp_path / "req.json", tmp_path / "art.json"
    rpath.write_text(json.dumps(req))
    pr = run_worker("--probe", "--request", str(rpath))
    assert pr.returncode == 0, pr.stderr
    fp = json.loads(pr.stdout)
    assert fp["producer"] == {"name": "ask_b200", "version": f"abi-{ask_b200.abi_version()}"}
    assert fp["adapter_version"].startswith("ask_b200-") and len(fp["adapter_version"]) > 20
    # the fingerprint follows the source
    req2 = dict(req, source=json.dumps(R.cfg5b_step(1 << 13)))
    rpath2 = tmp_path / "req2.json"
    rpath2.write_text(json.dumps(req2))
    assert json.loads(run_worker("--probe", "--request", str(rpath2)).stdout)["adapter_version"] != fp["adapter_version"]
    r = run_worker("--request", str(rpath), "--output", str(apath))
    assert r.returncode == 0, r.stderr
    art = json.loads(apath.read_text())
    A.validate_artifact(art, req)
    assert base64.b64decode(art["payload"])[:4] == b"\x7fELF"
    assert [p.name for p in tmp_path.iterdir() if p.name.startswith(".artifact-")] == []


def test_worker_failure_leaves_no_output(tmp_path):
    req = request_for(R.cfg4_scatter_step(100, 16, 1000), scalars=())
    rpath, apath = tmp_path / "req.json", tmp_path / "art.json"
    rpath.write_text(json.dumps(req))
    r = run_worker("--request", str(rpath), "--output", str(apath))
    assert r.returncode == 1 and "pre_copy" in r.stderr
    assert not apath.exists() and list(tmp_path.iterdir()) == [rpath]
    rpath.write_text("{broken")
    r = run_worker("--request", str(rpath), "--output", str(apath))
    assert r.returncode == 1 and "cannot read the request" in r.stderr


def test_artifact_header_exports(lib_built):
    lib = ctypes.CDLL(ask_b200.LIBRARY_PATH)
    text = open(os.path.join(ROOT, "include", "ask_b200_artifact.h")).read()
    names = sorted(set(re.findall(r"ASK_B200_API\s+int\s+(ask_b200_[a-z_0-9]+)\s*\(", text)))
    assert names == sorted(A.ARTIFACT_SIGNATURES)
    for name in names:
        assert hasattr(lib, name)
