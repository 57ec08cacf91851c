"""Runtime layer: sessions, device buffers, prepared programs and events.

Python binding of include/ask_b200_runtime.h.  The names follow the reference
Runtime's C++ API (include/ask/Runtime/CUDA.h:66-175) so code written against
``ask::runtime`` reads the same: ``Session.create``, ``allocate``,
``importBuffer``, ``prepareProgram(sizes, inputs, outputs, steps, graph)``,
``PreparedProgram.submit/run``, ``DeviceBuffer.pointer/size/readonly/
copyFromHost/copyToHost``, ``Event.query/wait``, ``Session.load/submit`` and
``Session.stats``.  A :class:`PlanStep` holds an ask_b200 recipe (one owned
step, see :mod:`ask_b200.recipes`) or, as in the reference, a loaded
:class:`Kernel` with its arguments and launch (kernel artifacts:
:mod:`ask_b200.artifact`).

``check_allocation`` and ``assign_slots`` expose the plan verifier and the
slot assigners on the host (no GPU needed).
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass, field
from typing import Optional, Sequence

from . import AskB200Error, OK, _lib

_p = ctypes.c_void_p
_sz = ctypes.c_size_t
_u64 = ctypes.c_uint64
_TEXT = [ctypes.c_char_p, _sz, ctypes.POINTER(_sz)]

# Every entry point declared in include/ask_b200_runtime.h, with its ctypes signature.
RUNTIME_SIGNATURES = {
    "ask_b200_session_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(_p)]),
    "ask_b200_session_release": (ctypes.c_int, [_p]),
    "ask_b200_session_synchronize": (ctypes.c_int, [_p]),
    "ask_b200_session_reap": (ctypes.c_int, [_p]),
    "ask_b200_session_stream": (ctypes.c_int, [_p, ctypes.POINTER(_p)]),
    "ask_b200_session_wait_stream": (ctypes.c_int, [_p, _p]),
    "ask_b200_session_stats": (ctypes.c_int, [_p] + _TEXT),
    "ask_b200_buffer_allocate": (ctypes.c_int, [_p, _sz, ctypes.POINTER(_p)]),
    "ask_b200_buffer_import": (ctypes.c_int, [_p, _u64, _sz, ctypes.c_int, ctypes.POINTER(_p)]),
    "ask_b200_buffer_info": (ctypes.c_int, [_p, ctypes.POINTER(_u64), ctypes.POINTER(_sz), ctypes.POINTER(ctypes.c_int)]),
    "ask_b200_buffer_copy_from_host": (ctypes.c_int, [_p, _p, _sz]),
    "ask_b200_buffer_copy_to_host": (ctypes.c_int, [_p, _p, _sz]),
    "ask_b200_buffer_release": (ctypes.c_int, [_p]),
    "ask_b200_program_prepare": (ctypes.c_int, [_p, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(_p)]),
    "ask_b200_program_describe": (ctypes.c_int, [_p] + _TEXT),
    "ask_b200_program_submit": (ctypes.c_int, [_p, ctypes.POINTER(_p), _sz, ctypes.POINTER(_p), _sz,
                                               ctypes.POINTER(_p)]),
    "ask_b200_program_run": (ctypes.c_int, [_p, ctypes.POINTER(_p), _sz, ctypes.POINTER(_p), _sz, ctypes.POINTER(_p)]),
    "ask_b200_program_release": (ctypes.c_int, [_p]),
    "ask_b200_event_query": (ctypes.c_int, [_p, ctypes.POINTER(ctypes.c_int)]),
    "ask_b200_event_wait": (ctypes.c_int, [_p]),
    "ask_b200_event_release": (ctypes.c_int, [_p]),
    "ask_b200_program_prepare_kernels": (ctypes.c_int, [_p, ctypes.c_char_p, ctypes.POINTER(_p), _sz, ctypes.c_int,
                                                        ctypes.POINTER(_p)]),
    "ask_b200_kernel_load": (ctypes.c_int, [_p, ctypes.c_void_p, _sz, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p),
                                            _sz, ctypes.c_int, ctypes.POINTER(ctypes.c_uint), _sz, ctypes.POINTER(_p)]),
    "ask_b200_kernel_info": (ctypes.c_int, [_p] + _TEXT + [ctypes.POINTER(ctypes.c_uint)]),
    "ask_b200_kernel_release": (ctypes.c_int, [_p]),
    "ask_b200_kernel_submit": (ctypes.c_int, [_p, _p, ctypes.c_void_p, _sz, ctypes.POINTER(ctypes.c_uint),
                                              ctypes.POINTER(ctypes.c_uint), ctypes.c_uint, ctypes.POINTER(_p)]),
    "ask_b200_allocation_check": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)] + _TEXT),
    "ask_b200_allocation_assign": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int] + _TEXT),
}

for _name, (_res, _args) in RUNTIME_SIGNATURES.items():
    _fn = getattr(_lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class CUDAError(AskB200Error):
    """A failed runtime call (the reference's ask::runtime::CUDAError)."""


def _check(status: int) -> None:
    if status != OK:
        raise CUDAError(status, _lib.ask_b200_last_error().decode())


def _text(fn, *args) -> str:
    need = _sz()
    _check(fn(*args, None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    _check(fn(*args, buf, need.value, ctypes.byref(need)))
    return buf.value.decode()


@dataclass
class PlanArgument:
    """One kernel-step argument (the reference's PlanArgument): a logical
    buffer for a pointer parameter (-1 = null) or the scalar's ABI bytes."""
    buffer: int = -1
    scalar: bytes = b""
    align: int = 1  # address alignment the kernel needs for this pointer (its element size)

    def to_json(self) -> dict:
        if self.scalar:
            return {"scalar": self.scalar.hex()}
        d = {"buffer": int(self.buffer)}
        if self.align > 1:
            d["align"] = int(self.align)
        return d


@dataclass
class PlanStep:
    """One program step bound to logical buffers: an ask_b200 recipe, or a
    loaded :class:`Kernel` with ``arguments`` (PlanArgument or int buffer
    indices), ``grid``, ``block`` and ``sharedBytes``.

    A recipe's ``inputs``/``outputs`` bind its ports in port-map order;
    ``preCopy`` = (source, destination) is the reference's PlanStep::preCopy.
    """
    recipe: Optional[dict] = None
    inputs: Sequence[int] = ()
    outputs: Sequence[int] = ()
    preCopy: Optional[tuple] = None
    kernel: Optional["Kernel"] = None
    arguments: Sequence = ()
    grid: Sequence[int] = (1, 1, 1)
    block: Sequence[int] = (1, 1, 1)
    sharedBytes: int = 0

    def to_json(self, kernel_index: Optional[int] = None) -> dict:
        d = {"inputs": [int(i) for i in self.inputs], "outputs": [int(o) for o in self.outputs]}
        if self.kernel is not None:
            d.update({"kernel": kernel_index, "grid": [int(x) for x in self.grid], "block": [int(x) for x in self.block],
                      "shared_bytes": int(self.sharedBytes),
                      "arguments": [(a if isinstance(a, PlanArgument) else PlanArgument(buffer=int(a))).to_json()
                                    for a in self.arguments]})
        else:
            d["recipe"] = self.recipe if isinstance(self.recipe, str) else json.dumps(self.recipe)
        if self.preCopy is not None:
            d["pre_copy"] = {"source": int(self.preCopy[0]), "destination": int(self.preCopy[1])}
        return d


class Kernel:
    """A loaded kernel entry (ask::runtime::Kernel)."""

    def __init__(self, handle: _p, session: "Session"):
        self._h = handle
        self.session = session

    def entry(self) -> str:
        need = _sz()
        _check(_lib.ask_b200_kernel_info(self._h, None, 0, ctypes.byref(need), None))
        buf = ctypes.create_string_buffer(need.value)
        _check(_lib.ask_b200_kernel_info(self._h, buf, need.value, ctypes.byref(need), None))
        return buf.value.decode()

    def maxThreads(self) -> int:
        n = ctypes.c_uint()
        _check(_lib.ask_b200_kernel_info(self._h, None, 0, None, ctypes.byref(n)))
        return n.value

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.ask_b200_kernel_release(self._h)
            self._h = None


class DeviceBuffer:
    def __init__(self, handle: _p, session: "Session"):
        self._h = handle
        self.session = session
        ptr, size, ro = _u64(), _sz(), ctypes.c_int()
        _check(_lib.ask_b200_buffer_info(handle, ctypes.byref(ptr), ctypes.byref(size), ctypes.byref(ro)))
        self._ptr, self._size, self._ro = ptr.value, size.value, bool(ro.value)

    def pointer(self) -> int:
        return self._ptr

    def size(self) -> int:
        return self._size

    def readonly(self) -> bool:
        return self._ro

    def copyFromHost(self, data) -> None:
        mv = memoryview(data).cast("B")
        buf = (ctypes.c_char * len(mv)).from_buffer_copy(mv) if len(mv) else None
        _check(_lib.ask_b200_buffer_copy_from_host(self._h, buf, len(mv)))

    def copyToHost(self) -> bytes:
        buf = ctypes.create_string_buffer(self._size)
        _check(_lib.ask_b200_buffer_copy_to_host(self._h, buf, self._size))
        return buf.raw[:self._size]

    def __eq__(self, other) -> bool:  # same storage (the reference compares shared_ptr identity)
        return isinstance(other, DeviceBuffer) and other._ptr == self._ptr and other._size == self._size

    def __hash__(self) -> int:
        return hash((self._ptr, self._size))

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.ask_b200_buffer_release(self._h)
            self._h = None


class Event:
    def __init__(self, handle: _p):
        self._h = handle

    def query(self) -> bool:
        done = ctypes.c_int()
        _check(_lib.ask_b200_event_query(self._h, ctypes.byref(done)))
        return bool(done.value)

    def wait(self) -> None:
        _check(_lib.ask_b200_event_wait(self._h))

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.ask_b200_event_release(self._h)
            self._h = None


class _KernelArg(ctypes.Structure):
    _fields_ = [("buffer", _p), ("scalar", ctypes.c_void_p), ("scalar_bytes", _sz), ("align", _sz)]


def _handles(buffers) -> ctypes.Array:
    arr = (_p * max(len(buffers), 1))()
    for i, b in enumerate(buffers):
        arr[i] = b._h if b is not None else None
    return arr


class PreparedProgram:
    def __init__(self, handle: _p, session: "Session", n_outputs: int):
        self._h = handle
        self.session = session
        self._n_outputs = n_outputs

    def describe(self) -> dict:
        return json.loads(_text(_lib.ask_b200_program_describe, self._h))

    def submit(self, inputs: Sequence[DeviceBuffer], outputs: Sequence[DeviceBuffer]) -> Event:
        ev = _p()
        _check(_lib.ask_b200_program_submit(self._h, _handles(inputs), len(inputs), _handles(outputs), len(outputs),
                                            ctypes.byref(ev)))
        return Event(ev)

    def bind(self, inputs: Sequence[DeviceBuffer], outputs: Sequence[DeviceBuffer]):
        """A pre-marshalled ``submit(inputs, outputs)`` for repeated submissions
        of the same buffers: each call enqueues the program and drops its
        completion handle (the session keeps the submission alive until the
        GPU is done; ``Session.synchronize`` waits for it)."""
        ins, outs = _handles(inputs), _handles(outputs)
        ni, no = len(inputs), len(outputs)
        ev = _p()
        ref = ctypes.byref(ev)
        h, submit, release = self._h, _lib.ask_b200_program_submit, _lib.ask_b200_event_release
        keep = (self, list(inputs), list(outputs))

        def run():
            status = submit(h, ins, ni, outs, no, ref)
            if status != OK:
                _check(status)
            release(ev)
        run.keep = keep
        return run

    def run(self, inputs: Sequence[DeviceBuffer]):
        outs = (_p * max(self._n_outputs, 1))()
        ev = _p()
        _check(_lib.ask_b200_program_run(self._h, _handles(inputs), len(inputs), outs, self._n_outputs,
                                         ctypes.byref(ev)))
        return [DeviceBuffer(_p(outs[i]), self.session) for i in range(self._n_outputs)], Event(ev)

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.ask_b200_program_release(self._h)
            self._h = None


class Session:
    """One device and its non-blocking stream (ask::runtime::Session)."""

    def __init__(self, handle: _p, device: int):
        self._h = handle
        self._device = device

    @staticmethod
    def create(device: int = 0) -> "Session":
        h = _p()
        _check(_lib.ask_b200_session_create(int(device), ctypes.byref(h)))
        return Session(h, device)

    def device(self) -> int:
        return self._device

    def allocate(self, nbytes: int) -> DeviceBuffer:
        h = _p()
        _check(_lib.ask_b200_buffer_allocate(self._h, int(nbytes), ctypes.byref(h)))
        return DeviceBuffer(h, self)

    def importBuffer(self, pointer: int, nbytes: int, readonly: bool = False) -> DeviceBuffer:
        h = _p()
        _check(_lib.ask_b200_buffer_import(self._h, int(pointer), int(nbytes), 1 if readonly else 0, ctypes.byref(h)))
        return DeviceBuffer(h, self)

    def importTensor(self, tensor, readonly: bool = False) -> DeviceBuffer:
        """A torch tensor's storage as a buffer (the tensor must stay alive)."""
        return self.importBuffer(int(tensor.data_ptr()), tensor.numel() * tensor.element_size(), readonly)

    def prepareProgram(self, sizes: Sequence[int], inputs: Sequence[int], outputs: Sequence[int],
                       steps: Sequence[PlanStep], graph: bool = False, fuse: bool = True) -> PreparedProgram:
        """``fuse=False`` keeps a three-step softmax as three steps (by default
        the runtime runs it as one fused step that writes the same buffers)."""
        kernels = []
        step_json = []
        for s in steps:
            index = None
            if s.kernel is not None:
                index = next((i for i, k in enumerate(kernels) if k is s.kernel), None)
                if index is None:
                    kernels.append(s.kernel)
                    index = len(kernels) - 1
            step_json.append(s.to_json(index))
        text = json.dumps({"buffer_sizes": [int(s) for s in sizes], "inputs": [int(i) for i in inputs],
                           "outputs": [int(o) for o in outputs], "steps": step_json, "fuse": bool(fuse)})
        h = _p()
        if kernels:
            arr = (_p * len(kernels))(*[k._h for k in kernels])
            _check(_lib.ask_b200_program_prepare_kernels(self._h, text.encode(), arr, len(kernels), 1 if graph else 0,
                                                         ctypes.byref(h)))
        else:
            _check(_lib.ask_b200_program_prepare(self._h, text.encode(), 1 if graph else 0, ctypes.byref(h)))
        program = PreparedProgram(h, self, len(outputs))
        program._kernels = kernels
        return program

    def load(self, image: bytes, entry: str, requiredTypes: Sequence[str], arch: int,
             parameterWidths: Sequence[int]) -> Kernel:
        """Session::load: a cubin (or PTX text) entry with its declared ABI
        (0 = device pointer, 1/2/4/8 = scalar bytes)."""
        data = image.encode() if isinstance(image, str) else bytes(image)
        types = (ctypes.c_char_p * max(len(requiredTypes), 1))(*[t.encode() for t in requiredTypes])
        widths = (ctypes.c_uint * max(len(parameterWidths), 1))(*[int(w) for w in parameterWidths])
        h = _p()
        _check(_lib.ask_b200_kernel_load(self._h, data, len(data), entry.encode(), types, len(requiredTypes), int(arch),
                                         widths, len(parameterWidths), ctypes.byref(h)))
        return Kernel(h, self)

    def submit(self, kernel: Kernel, arguments: Sequence, grid: Sequence[int], block: Sequence[int],
               sharedBytes: int = 0, alignments: Optional[Sequence[int]] = None) -> Event:
        """Session::submit: arguments are DeviceBuffer, None (null pointer) or
        bytes (a scalar's ABI bytes); ``alignments[i]`` (optional) is the
        address alignment pointer argument i needs."""
        n = len(arguments)
        args = (_KernelArg * max(n, 1))()
        keep = []
        for i, a in enumerate(arguments):
            if isinstance(a, (bytes, bytearray)):
                buf = ctypes.create_string_buffer(bytes(a), len(a))
                keep.append(buf)
                args[i].scalar = ctypes.cast(buf, ctypes.c_void_p)
                args[i].scalar_bytes = len(a)
            elif a is not None:
                args[i].buffer = a._h
            if alignments is not None:
                args[i].align = int(alignments[i])
        g = (ctypes.c_uint * 3)(*[int(x) for x in grid])
        b = (ctypes.c_uint * 3)(*[int(x) for x in block])
        ev = _p()
        _check(_lib.ask_b200_kernel_submit(self._h, kernel._h, args, n, g, b, int(sharedBytes), ctypes.byref(ev)))
        return Event(ev)

    def stream(self) -> int:
        s = _p()
        _check(_lib.ask_b200_session_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    def waitForExternalStream(self, stream) -> None:
        handle = stream if isinstance(stream, int) else int(stream.cuda_stream)
        _check(_lib.ask_b200_session_wait_stream(self._h, handle))

    def synchronize(self) -> None:
        _check(_lib.ask_b200_session_synchronize(self._h))

    def reap(self) -> None:
        _check(_lib.ask_b200_session_reap(self._h))

    def stats(self) -> dict:
        return json.loads(_text(_lib.ask_b200_session_stats, self._h))

    def close(self) -> None:
        if self._h:
            _check(_lib.ask_b200_session_release(self._h))
            self._h = None

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.ask_b200_session_release(self._h)
            self._h = None


def check_allocation(allocation: dict):
    """The plan verifier: returns (passed, explanation)."""
    ok = ctypes.c_int()
    need = _sz()
    text = json.dumps(allocation).encode()
    _check(_lib.ask_b200_allocation_check(text, ctypes.byref(ok), None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    _check(_lib.ask_b200_allocation_check(text, ctypes.byref(ok), buf, need.value, ctypes.byref(need)))
    return bool(ok.value), buf.value.decode()


def assign_slots(plan: dict, graph: bool = False) -> dict:
    """Slot assignment for a plan with buffer_sizes; returns the allocation fields."""
    return json.loads(_text(_lib.ask_b200_allocation_assign, json.dumps(plan).encode(), 1 if graph else 0))


# ---- lowering adapter (include/ask_b200_lower.h) --------------------------------------
_LOWER_SIGNATURES = {
    "ask_b200_lower_step": (ctypes.c_int, [ctypes.c_char_p] + _TEXT),
    "ask_b200_lower_report": (ctypes.c_int, [ctypes.c_char_p] + _TEXT),
}
for _name, (_res, _args) in _LOWER_SIGNATURES.items():
    _fn = getattr(_lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def lower_step(step_source: str) -> dict:
    """One ASK step source (MLIR text) -> {"recipe": ..., "input_arguments": [...]}."""
    return json.loads(_text(_lib.ask_b200_lower_step, step_source.encode()))


def lower_report(report) -> dict:
    """A partition report (execution_plan + step_sources) -> a runtime program."""
    text = report if isinstance(report, str) else json.dumps(report)
    return json.loads(_text(_lib.ask_b200_lower_report, text.encode()))


def prepare_report(session: Session, report, graph: bool = False) -> PreparedProgram:
    """Lower a partition report and prepare it as a program on `session`."""
    program = lower_report(report)
    h = _p()
    _check(_lib.ask_b200_program_prepare(session._h, json.dumps(program).encode(), 1 if graph else 0, ctypes.byref(h)))
    return PreparedProgram(h, session, len(program["outputs"]))
