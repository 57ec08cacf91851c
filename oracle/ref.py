"""ctypes binding of oracle/_ref/libask_ref.so: the reference's own Runtime
and PASS checker built from its sources (oracle/ref_build.py).  Test
infrastructure: the tests compare the runtime layer's verifier with
``pass_check`` and run kernel artifacts through the reference's
Session::load with ``run_step``."""
from __future__ import annotations

import ctypes
import json
import os

from . import ref_build

_lib = None


def load():
    """The library, or None when it is neither built nor buildable here."""
    global _lib
    if _lib is None:
        path = ref_build.build()
        if path is None or not os.path.exists(path):
            return None
        lib = ctypes.CDLL(path)
        lib.askref_pass_check.restype = ctypes.c_int
        lib.askref_pass_check.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p,
                                          ctypes.c_size_t]
        lib.askref_run_step.restype = ctypes.c_int
        u = ctypes.c_uint
        lib.askref_run_step.argtypes = [
            ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int,
            ctypes.POINTER(u), ctypes.c_size_t, ctypes.POINTER(ctypes.c_int64), ctypes.c_char_p,
            ctypes.POINTER(u), ctypes.POINTER(u), u, ctypes.POINTER(ctypes.c_size_t), ctypes.c_size_t,
            ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
            ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
        lib.askref_run_program.restype = ctypes.c_int
        lib.askref_run_program.argtypes = [
            ctypes.c_int, ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_size_t),
            ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
            ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
        _lib = lib
    return _lib


def pass_check(allocation: dict):
    """ask::pass::checkPlan / checkAllocationPlan: (passed, explanation)."""
    lib = load()
    ok = ctypes.c_int()
    buf = ctypes.create_string_buffer(1 << 16)
    if lib.askref_pass_check(json.dumps(allocation).encode(), ctypes.byref(ok), buf, len(buf)) != 0:
        raise RuntimeError(buf.value.decode())
    return bool(ok.value), buf.value.decode()


def run_step(image: bytes, entry: str, types, arch: int, widths, arg_buffer, scalars, grid, block, shared: int,
             inputs, output_sizes, graph: bool = False, repeats: int = 1, device: int = 0):
    """One kernel step through the reference Runtime (Session::load +
    prepareProgram + run).  inputs: bytes-like host data of buffers 0..n_in-1;
    arg_buffer[i]: logical buffer of pointer parameter i (-1 = null);
    scalars[i]: ABI bytes of scalar parameter i.  Returns (outputs as bytes,
    session stats)."""
    lib = load()
    n = len(widths)
    u3 = lambda v: (ctypes.c_uint * 3)(*[int(x) for x in v])
    sc = bytearray(8 * n)
    for i, b in enumerate(scalars):
        if b:
            sc[8 * i:8 * i + len(b)] = b
    keep = [ctypes.create_string_buffer(bytes(x), max(len(x), 1)) for x in inputs]
    outs = [ctypes.create_string_buffer(max(int(s), 1)) for s in output_sizes]
    sizes = (ctypes.c_size_t * (len(inputs) + len(outs)))(*([len(x) for x in inputs] + [int(s) for s in output_sizes]))
    stats = ctypes.create_string_buffer(1 << 14)
    err = ctypes.create_string_buffer(1 << 12)
    rc = lib.askref_run_step(
        int(device), bytes(image), len(image), entry.encode(), ",".join(types).encode(), int(arch),
        (ctypes.c_uint * n)(*widths), n, (ctypes.c_int64 * n)(*arg_buffer), bytes(sc), u3(grid), u3(block),
        int(shared), sizes, len(inputs), len(outs),
        (ctypes.c_void_p * max(len(keep), 1))(*[ctypes.cast(k, ctypes.c_void_p) for k in keep]),
        (ctypes.c_void_p * max(len(outs), 1))(*[ctypes.cast(o, ctypes.c_void_p) for o in outs]),
        1 if graph else 0, int(repeats), stats, len(stats), err, len(err))
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return [o.raw[:int(s)] for o, s in zip(outs, output_sizes)], json.loads(stats.value.decode())


def run_program(program: dict, images, inputs, graph: bool = False, repeats: int = 1, device: int = 0):
    """A program of kernel steps (the JSON of ask_b200_program_prepare_kernels
    plus a "kernels" list of {"entry", "types", "arch", "widths"}) through the
    reference Runtime; images[k] is kernels[k]'s cubin, inputs the host data of
    the program inputs.  Returns (outputs as bytes, session stats)."""
    lib = load()
    sizes = program["buffer_sizes"]
    out_sizes = [sizes[o] for o in program["outputs"]]
    imgs = [ctypes.create_string_buffer(bytes(i), len(i)) for i in images]
    keep = [ctypes.create_string_buffer(bytes(x), max(len(x), 1)) for x in inputs]
    outs = [ctypes.create_string_buffer(max(int(s), 1)) for s in out_sizes]
    vp = lambda bufs: (ctypes.c_void_p * max(len(bufs), 1))(*[ctypes.cast(b, ctypes.c_void_p) for b in bufs])
    stats = ctypes.create_string_buffer(1 << 14)
    err = ctypes.create_string_buffer(1 << 12)
    rc = lib.askref_run_program(int(device), json.dumps(program).encode(), vp(imgs),
                                (ctypes.c_size_t * max(len(images), 1))(*[len(i) for i in images]), vp(keep), vp(outs),
                                1 if graph else 0, int(repeats), stats, len(stats), err, len(err))
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return [o.raw[:int(s)] for o, s in zip(outs, out_sizes)], json.loads(stats.value.decode())
