"""ask_b200: B200-native (sm_100a) kernels for ASK's data-parallel hot path.

Python binding of the C ABI in include/ask_b200.h (libask_b200.so, built
in-tree by ``python ask_b200/build.py``).  A :class:`Plan` is one owned ASK
execution-plan step -- the unit ask::lowerToCUDALLVM compiles and the Runtime's
step launcher runs (lib/Lowering/CUDA.cpp:152-419, lib/Runtime/CUDA.cpp:360-371)
-- described by a recipe (see :mod:`ask_b200.recipes`).  Ports are device
addresses ordered inputs first, then outputs, as in the reference's kernel ABI.

There is no CPU fallback: importing this package without the built library
raises, and every compute call goes through the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import json
import os
from typing import Iterable, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(_HERE, "libask_b200.so")

OK = 0
E_INVALID = -1
E_UNSUPPORTED = -2
E_CUDA = -3
E_NCCL = -4
E_DEVICE = -5
E_TIMEOUT = -6

# Generator kinds of ask_b200_generate.
GEN_UNIFORM_F32, GEN_NORMAL_F32, GEN_NORMAL_F16, GEN_NORMAL_BF16, GEN_I32, GEN_ZIPF_I64, GEN_ZIPF_I32 = range(7)

# Every entry point declared in include/ask_b200.h, with its ctypes signature.
_u64 = ctypes.c_uint64
_p = ctypes.c_void_p
_SIGNATURES = {
    "ask_b200_abi_version": (ctypes.c_int, []),
    "ask_b200_last_error": (ctypes.c_char_p, []),
    "ask_b200_plan_create": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(_p)]),
    "ask_b200_plan_destroy": (ctypes.c_int, [_p]),
    "ask_b200_plan_ports": (ctypes.c_int, [_p, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
    "ask_b200_plan_scratch_bytes": (ctypes.c_int, [_p, ctypes.POINTER(ctypes.c_size_t)]),
    "ask_b200_plan_describe": (ctypes.c_int, [_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "ask_b200_plan_kernel_launches": (ctypes.c_int, [_p, ctypes.POINTER(ctypes.c_int)]),
    "ask_b200_plan_launch": (ctypes.c_int, [_p, ctypes.POINTER(_u64), ctypes.c_size_t, _u64, _p]),
    "ask_b200_plan_launch_noalloc": (ctypes.c_int, [_p, ctypes.POINTER(_u64), ctypes.c_size_t, _p]),
    "ask_b200_comm_status": (ctypes.c_int, [_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "ask_b200_comm_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
    "ask_b200_comm_create": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(_p)]),
    "ask_b200_comm_destroy": (ctypes.c_int, [_p]),
    "ask_b200_plan_launch_sharded": (ctypes.c_int, [_p, _p, ctypes.POINTER(_u64), ctypes.c_size_t, _u64, _p]),
    "ask_b200_generate": (ctypes.c_int, [ctypes.c_int, _u64, ctypes.c_uint32, _u64, _u64, ctypes.c_double,
                                         ctypes.c_double, _u64, _p]),
}


class AskB200Error(RuntimeError):
    """A non-zero status from the C ABI (the reference raises CUDAError,
    lib/Runtime/CUDA.cpp:156-162)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"ask_b200 error {status}: {message}")
        self.status = status


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIBRARY_PATH):
        raise ImportError(
            f"{LIBRARY_PATH} is missing: build it with `python ask_b200/build.py` "
            "(there is no CPU fallback for the ask_b200 kernels)")
    lib = ctypes.CDLL(LIBRARY_PATH)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = _load()


def _check(status: int) -> None:
    if status != OK:
        raise AskB200Error(status, _lib.ask_b200_last_error().decode())


def abi_version() -> int:
    return _lib.ask_b200_abi_version()


def _ptr(x) -> int:
    """Device address of a port: an int, or an object with data_ptr() (torch)."""
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream_handle(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


class Plan:
    """One owned step: build from a recipe (dict or JSON), launch on ports.

    ``device=-1`` builds a host-only plan (validation/describe; no GPU needed).
    """

    def __init__(self, recipe, device: int = 0):
        text = recipe if isinstance(recipe, str) else json.dumps(recipe)
        handle = _p()
        _check(_lib.ask_b200_plan_create(text.encode(), int(device), ctypes.byref(handle)))
        self._h = handle
        self.device = device
        ni, no = ctypes.c_size_t(), ctypes.c_size_t()
        _check(_lib.ask_b200_plan_ports(self._h, ctypes.byref(ni), ctypes.byref(no)))
        self.n_inputs, self.n_outputs = ni.value, no.value
        sb = ctypes.c_size_t()
        _check(_lib.ask_b200_plan_scratch_bytes(self._h, ctypes.byref(sb)))
        self.scratch_bytes = sb.value
        kl = ctypes.c_int()
        _check(_lib.ask_b200_plan_kernel_launches(self._h, ctypes.byref(kl)))
        self.kernel_launches = kl.value

    def describe(self) -> dict:
        need = ctypes.c_size_t()
        _check(_lib.ask_b200_plan_describe(self._h, None, 0, ctypes.byref(need)))
        buf = ctypes.create_string_buffer(need.value)
        _check(_lib.ask_b200_plan_describe(self._h, buf, need.value, ctypes.byref(need)))
        return json.loads(buf.value.decode())

    def _ports(self, inputs: Sequence, outputs: Sequence):
        ports = [_ptr(x) for x in list(inputs) + list(outputs)]
        return (_u64 * max(1, len(ports)))(*ports), len(ports)

    def launch(self, inputs: Sequence, outputs: Sequence, scratch=None, stream=None) -> None:
        """Enqueue the step on `stream` (a torch.cuda.Stream, a raw handle, or
        None for the legacy default stream)."""
        arr, n = self._ports(inputs, outputs)
        _check(_lib.ask_b200_plan_launch(self._h, arr, n, _ptr(scratch), _stream_handle(stream)))

    def bind(self, inputs: Sequence, outputs: Sequence, scratch=None, stream=None):
        """A zero-argument callable that enqueues the step on fixed ports: the
        port array and handles are marshalled once, so a loop of launches pays
        only the C call (the tensors must outlive the callable)."""
        arr, n = self._ports(inputs, outputs)
        fn, h, sc, st = _lib.ask_b200_plan_launch, self._h, _ptr(scratch), _stream_handle(stream)

        def launch() -> None:
            status = fn(h, arr, n, sc, st)
            if status != OK:
                _check(status)
        return launch

    def launch_noalloc(self, inputs: Sequence, outputs: Sequence, stream=None) -> None:
        """Reduce plans only: scratch comes from the library's fixed device
        array (see ask_b200_plan_launch_noalloc in include/ask_b200.h)."""
        arr, n = self._ports(inputs, outputs)
        _check(_lib.ask_b200_plan_launch_noalloc(self._h, arr, n, _stream_handle(stream)))

    def launch_sharded(self, comm: "Comm", inputs: Sequence, outputs: Sequence, scratch, stream=None) -> None:
        arr, n = self._ports(inputs, outputs)
        _check(_lib.ask_b200_plan_launch_sharded(self._h, comm._h, arr, n, _ptr(scratch), _stream_handle(stream)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.ask_b200_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def comm_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _check(_lib.ask_b200_comm_unique_id(buf))
    return buf.raw


class Comm:
    """NCCL communicator for sharded plans (one rank per process and GPU)."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int, device: int):
        if len(unique_id) != 128:
            raise ValueError("unique id must be 128 bytes")
        handle = _p()
        _check(_lib.ask_b200_comm_create(unique_id, nranks, rank, device, ctypes.byref(handle)))
        self._h = handle
        self.nranks, self.rank, self.device = nranks, rank, device

    def status(self) -> tuple:
        """(status, peer_exchange): status is OK or E_TIMEOUT (a bounded wait for
        the other ranks ran out; the communicator must then be closed);
        peer_exchange tells whether records cross GPUs by peer memory (else
        by the NCCL all-gather).  Synchronous."""
        st, pe = ctypes.c_int(), ctypes.c_int()
        _check(_lib.ask_b200_comm_status(self._h, ctypes.byref(st), ctypes.byref(pe)))
        return st.value, bool(pe.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _check(_lib.ask_b200_comm_destroy(self._h))
            self._h = None


def generate(kind: int, seed: int, stream_id: int, offset: int, count: int, p0: float, p1: float, dst,
             stream=None) -> None:
    """Fill `dst` (device memory) with seeded synthetic values on the GPU."""
    _check(_lib.ask_b200_generate(int(kind), int(seed), int(stream_id), int(offset), int(count), float(p0),
                                  float(p1), _ptr(dst), _stream_handle(stream)))


def exported_symbols() -> Iterable[str]:
    return list(_SIGNATURES)
