"""Helpers for the GPU parity tests: device buffers through torch (plumbing
only), launches through the ask_b200 C ABI, comparisons against the oracle."""
import numpy as np
import torch

import ask_b200

TORCH = {np.dtype(np.float32): torch.float32, np.dtype(np.int32): torch.int32, np.dtype(np.int64): torch.int64,
         np.dtype(np.uint8): torch.uint8, np.dtype(np.uint16): torch.int16, np.dtype(np.uint32): torch.int32,
         np.dtype(np.float64): torch.float64}
NUMPY = {"bool": np.uint8, "i32": np.int32, "i64": np.int64, "f32": np.float32, "f16": np.uint16,
         "bf16": np.uint16}


def to_dev(a: np.ndarray, offset_bytes: int = 0) -> torch.Tensor:
    """Copy to the GPU; with offset_bytes > 0 the data starts that many bytes
    into a larger allocation (to exercise unaligned ports)."""
    a = np.ascontiguousarray(a)
    raw = a.view(np.uint8).reshape(-1)
    buf = torch.empty(raw.size + offset_bytes + 16, dtype=torch.uint8, device="cuda")
    buf[offset_bytes:offset_bytes + raw.size].copy_(torch.from_numpy(raw.copy()))
    return buf[offset_bytes:offset_bytes + raw.size]


def empty_dev(n: int, dtype: str, offset_bytes: int = 0) -> torch.Tensor:
    nbytes = n * np.dtype(NUMPY[dtype]).itemsize
    buf = torch.empty(nbytes + offset_bytes + 16, dtype=torch.uint8, device="cuda")
    return buf[offset_bytes:offset_bytes + nbytes]


def from_dev(t: torch.Tensor, dtype) -> np.ndarray:
    return t.cpu().numpy().view(np.uint8).view(np.dtype(dtype))


def run_plan(recipe: dict, inputs: list, out_dtypes: list, offset_bytes: int = 0, scratch_fill: int | None = None):
    plan = ask_b200.Plan(recipe, device=0)
    dev_in = [to_dev(a, offset_bytes) for a in inputs]
    n_out = [p["elements"] for p in plan.describe()["port_map"][len(inputs):]]
    dev_out = [empty_dev(n, dt, offset_bytes) for n, dt in zip(n_out, out_dtypes)]
    scratch = None
    if plan.scratch_bytes:
        scratch = torch.empty(plan.scratch_bytes, dtype=torch.uint8, device="cuda")
        if scratch_fill is not None:
            scratch.fill_(scratch_fill)
    plan.launch(dev_in, dev_out, scratch, torch.cuda.current_stream())
    torch.cuda.synchronize()
    return [from_dev(t, NUMPY[dt]) for t, dt in zip(dev_out, out_dtypes)]


def gen_dev(kind: int, seed: int, stream: int, count: int, p0: float, p1: float, dtype: torch.dtype,
            offset: int = 0) -> torch.Tensor:
    t = torch.empty(count, dtype=dtype, device="cuda")
    ask_b200.generate(kind, seed, stream, offset, count, p0, p1, t, torch.cuda.current_stream())
    return t


def ulp_f32(x: np.ndarray) -> np.ndarray:
    x = np.abs(x.astype(np.float32))
    return np.spacing(np.maximum(x, np.float32(1.1754944e-38)))


def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)
