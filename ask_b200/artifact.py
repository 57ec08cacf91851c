"""Kernel artifacts for ASK's external-worker path.

ASK hands an external compiler worker a request (protocol v2,
schemas/external-compiler-request-v2.schema.json) and loads what it returns --
an "external-kernel-artifact v2" (schemas/external-kernel-artifact-v2.schema.json)
-- through Session::load with the entry's parameter widths
(include/ask/Runtime/CUDA.h:75-78).  docs/en/compilers.md specifies both.

This module is the ask_b200 side of that contract:

* :func:`artifact_source` -- the C ABI generator (include/ask_b200_artifact.h):
  a recipe step -> CUDA source of one ``extern "C"`` kernel whose parameters
  are port pointers and ignored scalars, every size compiled in;
* :func:`compile_source` -- nvcc to an sm_100a cubin;
* :func:`build_artifact` / :func:`probe` -- a request in, an artifact (or the
  dependency fingerprint) out; ``python -m ask_b200.worker`` wraps them in the
  worker's process interface;
* :func:`scalar_bytes`, :func:`load_artifact`, :func:`artifact_step` -- what a
  caller does with an artifact: load it on a :class:`~ask_b200.runtime.Session`
  and bind it as a program step.

A request's ``source`` is an ask_b200 recipe (JSON text with a ``family``) or
an ASK step module (the partitioner's MLIR text, lowered with
:func:`ask_b200.runtime.lower_step`).  ``signature`` lists the kernel's
parameters in order: ``*T`` pointers bound to ``input:N``/``output:N`` ports
(every port of the step exactly once, T the port's element type) and scalars,
which the kernel accepts and ignores.  ``target`` must be CUDA arch 100; the
grid must be one-dimensional.
"""
from __future__ import annotations

import base64
import ctypes
import hashlib
import json
import math
import os
import shutil
import struct
import subprocess
import tempfile
from typing import Optional, Sequence

from . import OK, AskB200Error, _lib, abi_version

_sz = ctypes.c_size_t
# Every entry point declared in include/ask_b200_artifact.h, with its ctypes signature.
ARTIFACT_SIGNATURES = {
    "ask_b200_artifact_source": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _sz,
                                                ctypes.POINTER(_sz)]),
}
for _name, (_res, _args) in ARTIFACT_SIGNATURES.items():
    getattr(_lib, _name).restype = _res
    getattr(_lib, _name).argtypes = _args

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
PRODUCER = {"name": "ask_b200", "version": f"abi-{abi_version()}"}
ARCH = 100
# The library's device flags (ask_b200/build.py): no multiply-add contraction.
NVCC_FLAGS = ["-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-fmad=false",
              "--expt-relaxed-constexpr", "-Xptxas", "-O3", f"-I{CSRC}", f"-I{INCLUDE}"]
# Headers the generated source includes (directly or through one another).
SOURCE_HEADERS = ["artifact_bodies.cuh", "ew_body.cuh", "reduce_acc.cuh", "ask_numerics.cuh", "vec_io.cuh",
                  "kernels.h", "ask_types.h"]

# Request pointer types (docs/en/compilers.md, "Request Protocol v2") -> ASK element types.
POINTER_TYPES = {"*i1": "bool", "*i32": "i32", "*i64": "i64", "*fp32": "f32", "*fp16": "f16", "*bf16": "bf16"}
SCALAR_TYPES = ("i1", "i8", "i16", "i32", "i64", "u8", "u16", "u32", "u64", "fp16", "bf16", "fp32", "fp64")
REQUEST_FIELDS = {"protocol_version", "source", "entry", "signature", "source_bindings", "constants", "fixed_options",
                  "target", "grid", "port_shapes"}
# Routing fields a caller may leave in a request; the worker ignores them.
ROUTING_FIELDS = {"compiler", "op_id", "function", "implementation"}


class ArtifactError(AskB200Error):
    """A request the worker cannot serve, or a malformed artifact."""

    def __init__(self, message: str, status: int = -2):
        super().__init__(status, message)


def artifact_source(recipe, entry: str, grid: Sequence[int], parameters: Sequence[str]) -> dict:
    """The generator (ask_b200_artifact_source): source, launch, widths, types."""
    rj = recipe if isinstance(recipe, str) else json.dumps(recipe)
    opt = json.dumps({"entry": entry, "grid": [int(g) for g in grid], "parameters": list(parameters)})
    need = _sz()
    rc = _lib.ask_b200_artifact_source(rj.encode(), opt.encode(), None, 0, ctypes.byref(need))
    if rc != OK:
        raise ArtifactError(_lib.ask_b200_last_error().decode(), rc)
    buf = ctypes.create_string_buffer(need.value)
    rc = _lib.ask_b200_artifact_source(rj.encode(), opt.encode(), buf, need.value, ctypes.byref(need))
    if rc != OK:
        raise ArtifactError(_lib.ask_b200_last_error().decode(), rc)
    return json.loads(buf.value.decode())


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise ArtifactError("nvcc not found; compiling kernel artifacts needs the CUDA 12.9 toolkit")
    return path


def compile_source(source: str) -> bytes:
    """CUDA source -> sm_100a cubin bytes."""
    with tempfile.TemporaryDirectory(prefix="ask_b200_artifact_") as tmp:
        src = os.path.join(tmp, "artifact.cu")
        out = os.path.join(tmp, "artifact.cubin")
        with open(src, "w") as f:
            f.write(source)
        proc = subprocess.run([nvcc()] + NVCC_FLAGS + [src, "-o", out], capture_output=True, text=True)
        if proc.returncode != 0:
            raise ArtifactError("nvcc failed:\n" + proc.stderr[-4000:])
        with open(out, "rb") as f:
            return f.read()


def _digest(h, path: str) -> None:
    with open(path, "rb") as f:
        h.update(hashlib.sha256(f.read()).digest())


def probe(request: dict) -> dict:
    """The worker's dependency fingerprint (docs/en/compilers.md, "Process
    Interface"): the request's source and options, this worker's code, the
    headers the generated source includes, the generator library and nvcc."""
    h = hashlib.sha256()
    h.update(json.dumps({k: request.get(k) for k in ("source", "entry", "fixed_options", "constants")},
                        sort_keys=True).encode())
    for path in [os.path.abspath(__file__), os.path.join(HERE, "worker.py"), os.path.join(HERE, "libask_b200.so")] + \
            [os.path.join(CSRC, f) for f in SOURCE_HEADERS]:
        _digest(h, path)
    try:
        version = subprocess.run([nvcc(), "--version"], capture_output=True, text=True).stdout
    except ArtifactError:
        version = "nvcc missing"
    h.update(version.encode())
    h.update(" ".join(NVCC_FLAGS[:-2]).encode())  # flags without this machine's include paths
    return {"producer": dict(PRODUCER), "adapter_version": "ask_b200-" + h.hexdigest()[:32]}


def _require(ok: bool, message: str) -> None:
    if not ok:
        raise ArtifactError(message)


def _recipe_of(source: str):
    """(recipe, input_arguments) from a request source: recipe JSON or an ASK step module."""
    text = source.strip()
    if text.startswith("{"):
        try:
            recipe = json.loads(text)
        except json.JSONDecodeError as e:
            raise ArtifactError(f"request source is not valid recipe JSON: {e}")
        _require(isinstance(recipe, dict) and "family" in recipe, "request source JSON is not an ask_b200 recipe")
        return recipe, None
    from .runtime import lower_step  # the lowering adapter (include/ask_b200_lower.h)
    try:
        lowered = lower_step(source)
    except AskB200Error as e:
        raise ArtifactError(f"request source is not a supported ASK step: {e}")
    return json.loads(lowered["recipe"]) if isinstance(lowered["recipe"], str) else lowered["recipe"], \
        lowered["input_arguments"]


def _check_scalar(t: str, v) -> None:
    if t == "i1":
        _require(isinstance(v, bool), "i1 scalars bind booleans")
        return
    if t in ("fp16", "bf16", "fp32", "fp64"):
        _require(isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(v),
                 f"{t} scalars bind finite numbers")
        return
    _require(isinstance(v, int) and not isinstance(v, bool), f"{t} scalars bind integers")
    bits = int(t[1:])
    lo, hi = (-(1 << (bits - 1)), (1 << (bits - 1)) - 1) if t[0] == "i" else (0, (1 << bits) - 1)
    _require(lo <= v <= hi, f"{t} scalar {v} is outside [{lo}, {hi}]")


def build_artifact(request: dict, compile_fn=compile_source) -> dict:
    """A request (protocol v2) -> an artifact (v2).  Raises ArtifactError."""
    _require(isinstance(request, dict), "request must be a JSON object")
    unknown = set(request) - REQUEST_FIELDS - ROUTING_FIELDS
    _require(not unknown, f"unknown request fields: {sorted(unknown)}")
    missing = REQUEST_FIELDS - set(request)
    _require(not missing, f"missing request fields: {sorted(missing)}")
    _require(request["protocol_version"] == 2, "only request protocol version 2 is supported")
    source, entry = request["source"], request["entry"]
    _require(isinstance(source, str) and source, "source must be a non-empty string")
    _require(isinstance(entry, str) and entry.isidentifier() and entry.isascii(), "entry must be an identifier")
    target = request["target"]
    _require(isinstance(target, dict) and target.get("backend") == "cuda", "target backend must be cuda")
    _require(set(target) <= {"backend", "arch", "warp_size"}, "unknown target fields")
    _require(target.get("arch") == ARCH, f"ask_b200 produces sm_100a code only (target arch {ARCH})")
    _require(target.get("warp_size", 32) == 32, "warp_size must be 32")
    grid = request["grid"]
    _require(isinstance(grid, list) and len(grid) == 3 and all(isinstance(g, int) and 1 <= g <= 2**31 - 1 for g in grid),
             "grid must be three integers in [1, 2^31-1]")
    options = request["fixed_options"]
    _require(isinstance(options, dict), "fixed_options must be an object")
    _require(set(options) <= {"format"} and options.get("format", "cubin") == "cubin",
             "fixed_options supports only {\"format\": \"cubin\"}")
    _require(isinstance(request["constants"], dict), "constants must be an object")
    signature, bindings = request["signature"], request["source_bindings"]
    _require(isinstance(signature, dict) and signature, "signature must be a non-empty object")
    _require(isinstance(bindings, dict) and set(bindings) == set(signature),
             "source_bindings must share the signature's keys")
    _require(len(signature) <= 64, "at most 64 kernel parameters")

    recipe, input_arguments = _recipe_of(source)
    parameters, arguments = [], []
    for name, t in signature.items():
        b = bindings[name]
        if t in POINTER_TYPES:
            _require(isinstance(b, str) and (b.startswith("input:") or b.startswith("output:")),
                     f"pointer parameter {name} must bind input:N or output:N")
            parameters.append(b)
            arguments.append(b)
        else:
            _require(t in SCALAR_TYPES, f"parameter {name} has unknown type {t!r}")
            _check_scalar(t, b)
            parameters.append(t)
            arguments.append({"type": t, "value": b})
    if input_arguments is not None:
        # recipe input port i reads step argument input_arguments[i]: request
        # port input:A is recipe port i with input_arguments[i] == A
        remap = {f"input:{a}": f"input:{i}" for i, a in enumerate(input_arguments)}
        for b in parameters:
            _require(not b.startswith("input:") or b in remap, f"{b} is not an argument the step reads")
        parameters = [remap.get(p, p) for p in parameters]
    gen = artifact_source(recipe, entry, grid, parameters)

    # Port types and shapes against the step's ports.
    ports = {p["logical_port"]: p for p in gen["port_map"]}
    shapes = request["port_shapes"]
    _require(isinstance(shapes, dict), "port_shapes must be an object")
    for name, t in signature.items():
        if t in POINTER_TYPES:
            port = ports[parameters[list(signature).index(name)]]
            _require(POINTER_TYPES[t] == port["element_type"],
                     f"parameter {name} is {t} but {bindings[name]} holds {port['element_type']}")
    for port_name, shape in shapes.items():
        _require(isinstance(shape, list) and all(isinstance(d, int) and d >= 0 for d in shape),
                 f"port_shapes[{port_name}] must be a list of non-negative integers")
    for b in set(bindings[n] for n, t in signature.items() if t in POINTER_TYPES):
        _require(b in shapes, f"port_shapes has no shape for {b}")
        recipe_port = ports[parameters[[bindings[n] for n in signature].index(b)]]
        _require(math.prod(shapes[b]) == recipe_port["elements"],
                 f"{b} has shape {shapes[b]} ({math.prod(shapes[b])} elements); the step's port holds "
                 f"{recipe_port['elements']}")

    cubin = compile_fn(gen["source"])
    return {"protocol_version": 2, "format": "cubin", "payload": base64.b64encode(cubin).decode(), "entry": entry,
            "target": {"backend": "cuda", "arch": ARCH, "warp_size": 32}, "producer": dict(PRODUCER),
            "launch": gen["launch"], "arguments": arguments, "required_element_types": gen["required_element_types"]}


def request_for(recipe, entry: str = "step_kernel", grid: Sequence[int] = (592, 1, 1), scalars=(),
                source: Optional[str] = None) -> dict:
    """A protocol-v2 request for a recipe step: one pointer parameter per port
    in port-map order (named input_N / output_N), then the given
    (name, type, value) scalars."""
    from . import Plan
    ptype = {v: k for k, v in POINTER_TYPES.items()}
    sig, bind, shapes = {}, {}, {}
    for p in Plan(recipe, -1).describe()["port_map"]:
        name = p["logical_port"].replace(":", "_")
        sig[name] = ptype[p["element_type"]]
        bind[name] = p["logical_port"]
        shapes[p["logical_port"]] = [p["elements"]]
    for name, t, v in scalars:
        sig[name] = t
        bind[name] = v
    return {"protocol_version": 2, "source": source if source is not None else json.dumps(recipe), "entry": entry,
            "signature": sig, "source_bindings": bind, "constants": {}, "fixed_options": {},
            "target": {"backend": "cuda", "arch": ARCH}, "grid": [int(g) for g in grid], "port_shapes": shapes}


ARTIFACT_FIELDS = ("protocol_version", "format", "payload", "entry", "target", "producer", "launch", "arguments",
                   "required_element_types")


def validate_artifact(artifact: dict, request: Optional[dict] = None) -> None:
    """The caller-side checks of docs/en/compilers.md "Minimal Response": exact
    fields, target and grid matching the request, each port bound once, scalars
    matching the request's bindings."""
    _require(isinstance(artifact, dict) and set(artifact) == set(ARTIFACT_FIELDS),
             f"an artifact has exactly the fields {list(ARTIFACT_FIELDS)}")
    _require(artifact["protocol_version"] == 2 and artifact["format"] in ("cubin", "ptx"), "not an artifact v2")
    try:
        payload = base64.b64decode(artifact["payload"], validate=True) if artifact["format"] == "cubin" else b""
    except ValueError:
        raise ArtifactError("payload is not base64")
    _require(artifact["format"] != "cubin" or payload[:4] == b"\x7fELF", "cubin payload is not an ELF image")
    launch = artifact["launch"]
    _require(set(launch) == {"grid", "block", "shared_bytes"}, "launch has grid, block and shared_bytes")
    ports = [a for a in artifact["arguments"] if isinstance(a, str) and a != "null"]
    _require(len(ports) == len(set(ports)), "each tensor port appears exactly once")
    if request is not None:
        _require(artifact["target"]["arch"] == request["target"]["arch"], "artifact target differs from the request")
        _require(list(launch["grid"]) == list(request["grid"]), "artifact grid differs from the request")
        expected = [b if t in POINTER_TYPES else {"type": t, "value": b}
                    for t, b in ((request["signature"][k], request["source_bindings"][k]) for k in request["signature"])]
        _require(artifact["arguments"] == expected, "artifact arguments differ from the request's bindings")


def _bf16_bits(x: float) -> int:
    """Round-to-nearest-even f64 -> bf16 through f32 (both roundings RNE)."""
    f = struct.unpack("<I", struct.pack("<f", x))[0]
    return ((f + 0x7FFF + ((f >> 16) & 1)) >> 16) & 0xFFFF


def scalar_bytes(t: str, value) -> bytes:
    """The launch ABI bytes of a scalar argument (little-endian; floats RNE)."""
    _check_scalar(t, value)
    if t == "i1":
        return bytes([1 if value else 0])
    if t == "fp16":
        return struct.pack("<e", float(value))
    if t == "bf16":
        return struct.pack("<H", _bf16_bits(float(value)))
    if t == "fp32":
        return struct.pack("<f", float(value))
    if t == "fp64":
        return struct.pack("<d", float(value))
    bits = int(t[1:])
    return int(value).to_bytes(bits // 8, "little", signed=t[0] == "i")


def parameter_widths(artifact: dict):
    """Session::load's parameterWidths for an artifact: 0 per pointer, the scalar's bytes otherwise."""
    return [0 if isinstance(a, str) else len(scalar_bytes(a["type"], a["value"])) for a in artifact["arguments"]]


def submit_arguments(artifact: dict, inputs: Sequence, outputs: Sequence, types: Optional[dict] = None):
    """(arguments, alignments) for Session.submit: DeviceBuffers for ports,
    ABI bytes for scalars, and each pointer's element size as its alignment."""
    args, aligns = [], []
    for a in artifact["arguments"]:
        if isinstance(a, str):
            if a == "null":
                args.append(None)
                aligns.append(1)
            else:
                kind, n = a.split(":")
                args.append((inputs if kind == "input" else outputs)[int(n)])
                aligns.append(ELEMENT_BYTES[types[a]] if types and a in types else 1)
        else:
            args.append(scalar_bytes(a["type"], a["value"]))
            aligns.append(1)
    return args, aligns


def load_artifact(session, artifact: dict, element_types: Optional[Sequence[str]] = None):
    """Load an artifact on a runtime Session (Session::load with its declared
    widths and required element types merged with the port types)."""
    validate_artifact(artifact)
    payload = base64.b64decode(artifact["payload"]) if artifact["format"] == "cubin" else artifact["payload"].encode()
    types = list(dict.fromkeys(list(artifact["required_element_types"]) + list(element_types or [])))
    return session.load(payload, artifact["entry"], types, artifact["target"]["arch"], parameter_widths(artifact))


def request_parameters(request: dict) -> list:
    """The generator's parameter list of a request whose source is a recipe:
    each signature entry's port binding, or its scalar type."""
    return [request["source_bindings"][k] if t in POINTER_TYPES else t for k, t in request["signature"].items()]


ELEMENT_BYTES = {"bool": 1, "i32": 4, "i64": 8, "f32": 4, "f16": 2, "bf16": 2}


def port_types(request: dict) -> dict:
    """{"input:N" / "output:N": element type} from a request's pointer signature."""
    return {request["source_bindings"][k]: POINTER_TYPES[t] for k, t in request["signature"].items()
            if t in POINTER_TYPES}


def artifact_step(artifact: dict, kernel, inputs: Sequence[int], outputs: Sequence[int],
                  types: Optional[dict] = None):
    """A program step launching a loaded artifact: input:N / output:N bind the
    logical buffers inputs[N] / outputs[N]; scalars carry their ABI bytes.
    With ``types`` (port -> element type, :func:`port_types`) each pointer
    carries its element size as the alignment the runtime checks."""
    from .runtime import PlanArgument, PlanStep
    args = []
    for a in artifact["arguments"]:
        if isinstance(a, str):
            if a == "null":
                args.append(PlanArgument(buffer=-1))
            else:
                kind, n = a.split(":")
                align = ELEMENT_BYTES[types[a]] if types and a in types else 1
                args.append(PlanArgument(buffer=int((inputs if kind == "input" else outputs)[int(n)]), align=align))
        else:
            args.append(PlanArgument(scalar=scalar_bytes(a["type"], a["value"])))
    launch = artifact["launch"]
    return PlanStep(kernel=kernel, inputs=list(inputs), outputs=list(outputs), arguments=args, grid=launch["grid"],
                    block=launch["block"], sharedBytes=launch["shared_bytes"])
