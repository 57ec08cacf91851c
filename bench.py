"""Benchmark: achieved HBM GB/s per plan on B200, next to ASK's host CPU path.

Default workload (BASELINE.json's "at 1/2/4/8 B200" plan): cfg5, the sharded
large plan -- part one a global sum/min/argmin over 2^32 f32, part two the i32
chain ((x<<3) ^ (x>>5)) & 0x7fffffff + y over 2^31 elements -- split along the
leading axis across N GPUs (strong scaling), with one NCCL all-gather of the
reduction partials per step.  One step = both parts of the plan.
Other workloads (cfg1, cfg2, cfg3, cfg3bf, cfg4g, cfg4s) run one GPU each.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg5|...]

Rank 0 prints one JSON line.  Inputs are seeded synthetic data generated on
the device (Philox4x32-10) and are larger than L2, so no flush is needed
between steps.  The CPU baseline and the reference arm run the oracle
(a restatement of ASK's single-threaded host code path; the reference's own
host compiler needs an LLVM 23 SDK that is not available) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEED = {"cfg1": 0xA5C1, "cfg2": 0xA5C2, "cfg3": 0xA5C3, "cfg4": 0xA5C4, "cfg5": 0xA5C5}
METRIC = "achieved HBM GB/s per plan (% of ~8 TB/s) at 1/2/4/8 B200 vs ASK host CPU"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
class Workload:
    """A benchmark plan: device inputs/outputs, the plans, and per-kernel
    algorithmic bytes.  `kernels` lists (name, bytes per launch, launch fn)."""

    name = ""
    scaling = "weak"
    dtype = "f32"

    def bytes_per_step(self) -> int:
        return sum(b for _, b, _ in self.kernels)

    def launches_per_step(self) -> int:
        return sum(p.kernel_launches for p in self.plans)


def static_config(name, world, small=False):
    """The `config` object of a workload's bench line (both arms print it)."""
    if name == "cfg5":
        return {"workload": "cfg5: sum/min/argmin over 2^32 f32 U[0,1) + i32 chain over 2^31, "
                            "leading-axis shards" + (" (SMALL profiling case)" if small else ""),
                "elements_f32": (1 << 28) if small else (1 << 32), "elements_i32": (1 << 27) if small else (1 << 31),
                "parallelism": f"shard{world}", "l2": "inputs 40 GB >> 126 MB L2, no flush needed"}
    if name == "cfg1":
        return {"workload": "cfg1: y0=exp(a)*b+c, y1=max(a,b)-tanh(c), f32 [4096,4096]",
                "l2": "320 MB per step > 126 MB L2"}
    if name == "cfg2":
        return {"workload": "cfg2: row sum/max/min/argmax, f32 [65536,1024]", "l2": "256 MB > L2"}
    if name in ("cfg3", "cfg3bf"):
        dt = "f16" if name == "cfg3" else "bf16"
        return {"workload": f"cfg3: 3-step softmax plan, {dt} [32768,4096]", "l2": "256 MB input > L2"}
    if name == "cfg4g":
        return {"workload": "cfg4 gather: table f32 [2^20,256], idx i64 Zipf(1.1) [2^23]", "l2": "8 GiB output > L2"}
    if name == "cfg4s":
        return {"workload": "cfg4 scatter_add: grad f32 [2^23,256] into zeros [2^20,256], idx Zipf(1.1)",
                "l2": "8 GiB updates > L2"}
    if name in ARTIFACT_WORKLOADS:
        base = static_config(ARTIFACT_WORKLOADS[name], world, small)
        return dict(base, workload=base["workload"] + ", as an external-kernel artifact v2 (cubin) run by the "
                                                      "runtime's Session::load kernel step, CUDA graph")
    raise SystemExit(f"unknown workload {name}")


# Kernel-artifact variants of single-GPU workloads: the same step compiled by
# the artifact worker into a flat-parameter cubin and run as a loaded-kernel
# program step (ask_b200.artifact).
ARTIFACT_WORKLOADS = {"cfg1a": "cfg1", "cfg2a": "cfg2"}


class _ArtifactLaunches:
    """Launch accounting of an artifact step (one kernel per step)."""
    kernel_launches = 1

    def __init__(self, grid):
        self._grid = grid

    def describe(self):
        return {"launch": {"grid": [self._grid, 1, 1]}}


def artifact_step_runner(recipe, ins, outs, grid):
    """Compile the recipe's artifact, load it on a runtime session and return
    (session, submit function, kernel name)."""
    from ask_b200 import artifact as A
    from ask_b200 import runtime as rt
    req = A.request_for(recipe, entry="bench_step", grid=(grid, 1, 1))
    art = A.build_artifact(req)
    session = rt.Session.create(rank_device())
    kernel = A.load_artifact(session, art)
    ni, no = len(ins), len(outs)
    step = A.artifact_step(art, kernel, list(range(ni)), list(range(ni, ni + no)), A.port_types(req))
    sizes = [t.numel() * t.element_size() for t in ins + outs]
    prog = session.prepareProgram(sizes, list(range(ni)), list(range(ni, ni + no)), [step], graph=True)
    bin_ = [session.importTensor(t, readonly=True) for t in ins]
    bout = [session.importTensor(t) for t in outs]
    body = A.artifact_source(recipe, "bench_step", [grid, 1, 1], A.request_parameters(req))["body"]
    return session, prog, prog.bind(bin_, bout), f"artifact_{body}"


def make_workload(name, rank, world, torch, ask_b200, R, comm, small=False):
    st = torch.cuda.current_stream()
    dev = torch.device("cuda", torch.cuda.current_device())

    def gen(kind, seed, sid, count, p0, p1, dt, offset=0):
        t = torch.empty(count, dtype=dt, device=dev)
        ask_b200.generate(kind, seed, sid, offset, count, p0, p1, t, st)
        return t

    w = Workload()
    w.name = name
    if name == "cfg5":
        w.scaling = "strong"
        w.dtype = "f32+i32"
        na, nb = (1 << 28, 1 << 27) if small else (1 << 32, 1 << 31)
        a0, a1 = R.shard_range(na, world, rank)
        b0, b1 = R.shard_range(nb, world, rank)
        x = gen(0, SEED["cfg5"], 0, a1 - a0, 0.0, 1.0, torch.float32, a0)
        xi = gen(4, SEED["cfg5"], 1, b1 - b0, 0, 0, torch.int32, b0)
        yi = gen(4, SEED["cfg5"], 2, b1 - b0, 0, 0, torch.int32, b0)
        pa = ask_b200.Plan(R.cfg5a_step(a1 - a0, index_base=a0), rank_device())
        pb = ask_b200.Plan(R.cfg5b_step(b1 - b0), rank_device())
        outs = [torch.empty(1, dtype=torch.float32, device=dev), torch.empty(1, dtype=torch.float32, device=dev),
                torch.empty(1, dtype=torch.int64, device=dev)]
        z = torch.empty_like(xi)
        scratch = torch.empty(max(pa.scratch_bytes, 16), dtype=torch.uint8, device=dev)

        w.plans = [pa, pb]
        run_b = pb.bind([xi, yi], [z], None, st)
        if world > 1:
            # The sharded reduction ends in an all-gather that waits for every
            # rank; it runs on a side stream beside the i32 chain so that wait
            # (and the exchange) hides behind the chain's streaming.  The two
            # plans share no data; the step joins both streams.
            side = torch.cuda.Stream(priority=-1)
            fork, join = torch.cuda.Event(), torch.cuda.Event()

            def run_step():
                fork.record(st)
                side.wait_event(fork)
                pa.launch_sharded(comm, [x], outs, scratch, side)
                join.record(side)
                run_b()
                st.wait_event(join)
            w.kernels = [("reduce_split_global_f32+ew_cfg5b", 4 * (a1 - a0) + 12 * (b1 - b0), run_step)]
        else:
            w.kernels = [("reduce_split_global_f32", 4 * (a1 - a0), pa.bind([x], outs, scratch, st)),
                         ("ew_cfg5b", 12 * (b1 - b0), run_b)]
        w.global_bytes = 4 * na + 12 * nb
        w.config = static_config(name, world, small)
        w.tensors = {"x": x, "xi": xi, "yi": yi, "z": z, "outs": outs, "scratch": scratch}
        w.e2e = {"inputs": [x, xi, yi], "results": outs + [z]}

        def launch_a(stream):
            if world > 1:
                pa.launch_sharded(comm, [x], outs, scratch, stream)
            else:
                pa.launch([x], outs, scratch, stream)
        # e2e: the two independent plans on their own streams, so one plan's
        # device->host copy overlaps the other's host->device copies
        w.e2e_groups = [([xi, yi], lambda stream: pb.launch([xi, yi], [z], None, stream), [z]),
                        ([x], launch_a, outs)]
        return w
    if world > 1:
        raise SystemExit(f"workload {name} is single-GPU (replicas only)")
    if name in ARTIFACT_WORKLOADS:
        w = make_workload(ARTIFACT_WORKLOADS[name], rank, world, torch, ask_b200, R, comm, small)
        w.name = name
        recipe = R.cfg1_step(4096 * 4096) if name == "cfg1a" else R.cfg2_step(65536, 1024)
        ins, outs = w.e2e["inputs"], w.e2e["results"]
        grid = w.plans[0].describe()["launch"]["grid"][0]  # the request asks for the recipe path's grid
        session, prog, run, kname = artifact_step_runner(recipe, ins, outs, grid)
        (_, nbytes, _), = w.kernels
        w.kernels = [(kname, nbytes, run)]
        w.plans = [_ArtifactLaunches(grid)]
        w.session, w.program, w.stream_handle = session, prog, session.stream()
        w.config = static_config(name, world)
        return w
    if name == "cfg1":
        n = 4096 * 4096
        a, b, c = (gen(0, SEED["cfg1"], s, n, -4.0, 4.0, torch.float32) for s in range(3))
        y0, y1 = torch.empty_like(a), torch.empty_like(a)
        p = ask_b200.Plan(R.cfg1_step(n), rank_device())
        w.plans = [p]
        w.kernels = [("ew_cfg1", 20 * n, p.bind([a, b, c], [y0, y1], None, st))]
        w.config = static_config(name, world)
        w.e2e = {"inputs": [a, b, c], "results": [y0, y1]}
    elif name == "cfg2":
        rows, cols = 65536, 1024
        x = gen(1, SEED["cfg2"], 0, rows * cols, 0.0, 1.0, torch.float32)
        outs = [torch.empty(rows, dtype=torch.float32, device=dev) for _ in range(3)] + \
               [torch.empty(rows, dtype=torch.int64, device=dev)]
        p = ask_b200.Plan(R.cfg2_step(rows, cols), rank_device())
        w.plans = [p]
        w.kernels = [("reduce_warp_row_rowstats_f32", 4 * rows * cols + rows * 20,
                      p.bind([x], outs, None, st))]
        w.config = static_config(name, world)
        w.e2e = {"inputs": [x], "results": outs}
    elif name in ("cfg3", "cfg3bf"):
        dt = "f16" if name == "cfg3" else "bf16"
        rows, cols = 32768, 4096
        x = gen(2 if dt == "f16" else 3, SEED["cfg3"], 0, rows * cols, 0.0, 2.0, torch.int16)
        m = torch.empty(rows, dtype=torch.float32, device=dev)
        s = torch.empty(rows, dtype=torch.float32, device=dev)
        y = torch.empty_like(x)
        # The reference's plan: three owned steps over x, m, s, y.  The runtime
        # layer runs them as one fused softmax step (graph mode); the graded bytes
        # stay the plan's port bytes (x read by all three steps).
        from ask_b200 import runtime as rt
        n = rows * cols
        session = rt.Session.create(rank_device())
        steps = R.cfg3_steps(dt, rows, cols)
        prog = session.prepareProgram([2 * n, 4 * rows, 4 * rows, 2 * n], [0], [1, 2, 3],
                                      [rt.PlanStep(steps[0], [0], [1]), rt.PlanStep(steps[1], [0, 1], [2]),
                                       rt.PlanStep(steps[2], [0, 1, 2], [3])], graph=True)
        kernel = prog.describe()["steps"][0]["kernel"]
        run = prog.bind([session.importTensor(x, readonly=True)], [session.importTensor(t) for t in (m, s, y)])
        w.plans = [ask_b200.Plan({"family": "softmax", "dtype": dt, "rows": rows, "cols": cols}, rank_device())]
        w.kernels = [(kernel, 4 * n + 8 * rows, run)]
        w.global_bytes = 4 * 2 * n + 6 * 4 * rows
        w.session, w.program, w.stream_handle = session, prog, session.stream()
        w.config = dict(static_config(name, world),
                        plan=f"3 owned steps (max, sum of exp, normalise) run by the runtime as one {kernel} step, "
                             "CUDA graph", graded_bytes="plan port bytes 4*2n + 6*4*rows")
        w.dtype = dt
        w.e2e = {"inputs": [x], "results": [y]}
    elif name in ("cfg4g", "cfg4s"):
        rows, dim, n = 1 << 20, 256, (1 << 21) if small else (1 << 23)
        idx = gen(5, SEED["cfg4"], 1, n, 1.1, rows, torch.int64)
        if name == "cfg4g":
            table = gen(1, SEED["cfg4"], 0, rows * dim, 0.0, 0.02, torch.float32)
            out = torch.empty(n * dim, dtype=torch.float32, device=dev)
            p = ask_b200.Plan(R.cfg4_gather_step(rows, dim, n), rank_device())
            distinct = int(torch.unique(idx).numel())
            w.kernels = [("gather_rows", 8 * n + 4 * n * dim + 4 * dim * distinct,
                          p.bind([table, idx], [out], None, st))]
            w.config = dict(static_config(name, world), distinct_rows=distinct,
                            graded_bytes="compulsory 8N + 4ND + 4D*distinct",
                            logical_bytes=8 * n + 8 * n * dim)
            w.e2e = {"inputs": [table, idx], "results": [out]}
        else:
            grad = gen(1, SEED["cfg4"], 2, n * dim, 0.0, 1.0, torch.float32)
            base = torch.zeros(rows * dim, dtype=torch.float32, device=dev)
            out = torch.empty_like(base)
            p = ask_b200.Plan(R.cfg4_scatter_step(rows, dim, n), rank_device())
            scratch = torch.empty(max(p.scratch_bytes, 16), dtype=torch.uint8, device=dev)
            w.kernels = [("scatter_add_sorted_rows", 8 * n + 4 * n * dim + 8 * rows * dim,
                          p.bind([base, idx, grad], [out], scratch, st))]
            w.config = static_config(name, world)
            w.e2e = {"inputs": [base, idx, grad], "results": [out]}
        w.plans = [p]
    else:
        raise SystemExit(f"unknown workload {name}")
    if not hasattr(w, "global_bytes"):
        w.global_bytes = w.bytes_per_step()
    return w


def rank_device() -> int:
    import torch
    return torch.cuda.current_device()


# ---------------------------------------------------------------------------
def cpu_sample(name: str, threads: int, budget_s: float = 12.0):
    """Time the oracle (ASK host-path restatement) on a bounded sample of the
    workload.  Returns (bytes_per_second, seconds, description)."""
    import numpy as np
    import oracle
    name = ARTIFACT_WORKLOADS.get(name, name)
    if name == "cfg5":
        na = 1 << 26
        nb = 1 << 25
        x = oracle.generate(0, SEED["cfg5"], 0, 0, na, 0.0, 1.0, threads=max(threads, 8))
        xi = oracle.generate(4, SEED["cfg5"], 1, 0, nb, 0, 0, threads=max(threads, 8))
        yi = oracle.generate(4, SEED["cfg5"], 2, 0, nb, 0, 0, threads=max(threads, 8))
        bytes_one = 4 * na + 12 * nb

        def run():
            oracle.cfg5a(x, threads=threads)
            oracle.cfg5b(xi, yi, threads=threads)
        desc = f"cfg5 prefix: sum/min/argmin over 2^26 f32 + i32 chain over 2^25, {threads} thread(s)"
    elif name == "cfg1":
        n = 1 << 22
        a, b, c = (oracle.generate(0, SEED["cfg1"], s, 0, n, -4.0, 4.0, threads=8) for s in range(3))
        bytes_one = 20 * n

        def run():
            oracle.cfg1(a, b, c, threads=threads)
        desc = f"cfg1 first 2^22 elements, {threads} thread(s)"
    elif name == "cfg2":
        rows, cols = 8192, 1024
        x = oracle.generate(1, SEED["cfg2"], 0, 0, rows * cols, 0.0, 1.0, threads=8)
        bytes_one = 4 * rows * cols + 20 * rows

        def run():
            oracle.rowstats(x, rows, cols, threads=threads)
        desc = f"cfg2 first 8192 rows, {threads} thread(s)"
    elif name in ("cfg3", "cfg3bf"):
        dt = "f16" if name == "cfg3" else "bf16"
        rows, cols = 1024, 4096
        x = oracle.generate(2 if dt == "f16" else 3, SEED["cfg3"], 0, 0, rows * cols, 0.0, 2.0, threads=8)
        bytes_one = 8 * rows * cols

        def run():
            oracle.softmax(dt, x, rows, cols, threads=threads)
        desc = f"cfg3 ({dt}) first 1024 rows, 3-step plan, {threads} thread(s)"
    else:
        rows, dim, n = 1 << 20, 256, 1 << 18
        idx = oracle.generate(5, SEED["cfg4"], 1, 0, n, 1.1, rows, threads=8)
        if name == "cfg4g":
            table = np.zeros(rows * dim, np.float32)
            # the GPU arm's compulsory bytes: indices, output rows, each distinct table row once
            bytes_one = 8 * n + 4 * n * dim + 4 * dim * int(np.unique(idx).size)

            def run():
                oracle.gather(table, idx, 1, rows, dim, threads=threads)
            desc = f"cfg4 gather of the first 2^18 indices, {threads} thread(s)"
        else:
            base = np.zeros(rows * dim, np.float32)
            upd = oracle.generate(1, SEED["cfg4"], 2, 0, n * dim, 0.0, 1.0, threads=8)
            bytes_one = 8 * n + 4 * n * dim + 8 * rows * dim

            def run():
                oracle.scatter_add("f32", base, idx, upd, 1, rows, dim)
            desc = f"cfg4 scatter_add of the first 2^18 updates (single-threaded reference order)"
    run()  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        run()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 50:
            break
    return bytes_one * reps / el, el, desc


# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser(description="ask_b200 benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg5")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--small", action="store_true", help="cfg5 at 1/16 size, cfg4 with 2^21 update rows (profiling captures only)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, world, rank)

    import torch
    import ask_b200
    from ask_b200 import recipes as R

    torch.cuda.set_device(local)
    dist = None
    comm = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        uid = [ask_b200.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = ask_b200.Comm(uid[0], world, rank, local)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    w = make_workload(args.workload, rank, world, torch, ask_b200, R, comm, small=args.small)
    torch.cuda.synchronize()
    if getattr(w, "stream_handle", None):  # a runtime session's stream: time and copy on it
        torch.cuda.set_stream(torch.cuda.ExternalStream(w.stream_handle))
    st = torch.cuda.current_stream()

    # warm-up
    for _ in range(max(args.warmup, 3)):
        for _, _, fn in w.kernels:
            fn()
    barrier()

    # timed region: per-kernel events on the launching stream
    nk = len(w.kernels)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)] for _ in range(args.steps)]
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.25)
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    # A step of one plan is timed by the region's two events alone (its launches
    # follow one another without event records in between); a step of several
    # plans also records an event after each plan for the per-plan times.
    start.record(st)
    for s in range(args.steps):
        if nk > 1:
            ev[s][0].record(st)
        for k, (_, _, fn) in enumerate(w.kernels):
            fn()
            if nk > 1:
                ev[s][k + 1].record(st)
    end.record(st)
    barrier()
    clocks = sampler.stop()
    total_ms = start.elapsed_time(end)
    if nk > 1:
        per_kernel_ms = [sum(ev[s][k].elapsed_time(ev[s][k + 1]) for s in range(args.steps)) / args.steps
                         for k in range(nk)]
    else:
        per_kernel_ms = [total_ms / args.steps]
    t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_per_step = max_ms / args.steps
    value = w.global_bytes / (ms_per_step * 1e-3) / 1e9

    peak, peak_kind = peaks()
    kernels = []
    grids = [pl.describe()["launch"]["grid"][0] for pl in w.plans]
    for (name, nbytes, _), ms in zip(w.kernels, per_kernel_ms):
        gbs = nbytes / (ms * 1e-3) / 1e9
        kernels.append({"kernel": name, "bytes_per_launch": nbytes, "ms": round(ms, 4), "gbs": round(gbs, 1),
                        "frac": round(gbs / peak, 4)})
    dom = max(range(nk), key=lambda k: per_kernel_ms[k])
    traffic = load_traffic(w.kernels[dom][0], w.kernels[dom][1])
    roofline = {"bound": "hbm", "achieved": kernels[dom]["gbs"], "peak": peak, "unit": "GB/s",
                "frac": kernels[dom]["frac"], "traffic": traffic, "kernel": kernels[dom]["kernel"],
                "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                else "fallback 6.65 TB/s"}

    # end-to-end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(w, args, torch, barrier, dist)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        bps, secs, desc = cpu_sample(args.workload, 1)
        cpu = {"value": round(bps / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": desc + f", {secs:.1f} s timed", "cpu": cpu_model()}

    w.config["grids"] = grids
    line = {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": w.scaling, "vs_baseline": None, "dtype": w.dtype, "data": "synthetic (seeded Philox4x32-10)",
            "config": w.config, "roofline": roofline, "kernels": kernels, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": w.launches_per_step() * args.steps, "clocks": clocks,
            "pct_of_8tbs": round(100.0 * value / world / 8000.0, 2)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def load_traffic(kernel: str, algorithmic_bytes: int):
    """Per-launch DRAM traffic of `kernel` scaled from the committed ncu
    summary (profiles/traffic.json: bytes per algorithmic byte), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            ratios = json.load(f)
        r = ratios.get(kernel)
        return None if r is None else int(r["dram_bytes_per_algorithmic_byte"] * algorithmic_bytes)
    except Exception:
        return None


def run_e2e(w, args, torch, barrier, dist):
    """Same plan, host buffers: H2D of every input from pinned memory and D2H
    of every result inside the timed region, through the public Plan API.
    Independent plans of a step (w.e2e_groups) each run on their own stream,
    so their copies overlap in both PCIe directions."""
    ins, outs = w.e2e["inputs"], w.e2e["results"]
    need = sum(t.numel() * t.element_size() for t in ins + outs)
    avail = host_memory_available()
    if need * 1.3 > avail:
        return {"value": None, "unit": "GB/s", "skipped": f"needs {need / 2**30:.1f} GiB pinned host memory, "
                                                          f"{avail / 2**30:.1f} GiB available"}
    st = torch.cuda.current_stream()
    h_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in ins]
    h_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in outs]
    for h, d in zip(h_in, ins):
        h.copy_(d)
    torch.cuda.synchronize()

    host_of = {id(d): h for d, h in zip(ins + outs, h_in + h_out)}
    groups = getattr(w, "e2e_groups", None)
    streams = [torch.cuda.Stream() for _ in groups] if groups else []
    forks = [torch.cuda.Event() for _ in streams]

    def step():
        if not groups:
            for h, d in zip(h_in, ins):
                d.copy_(h, non_blocking=True)
            for _, _, fn in w.kernels:
                fn()
            for h, d in zip(h_out, outs):
                h.copy_(d, non_blocking=True)
            return
        main = torch.cuda.current_stream()
        for (g_in, launch, g_out), s, ev in zip(groups, streams, forks):
            s.wait_stream(main)
            with torch.cuda.stream(s):
                for d in g_in:
                    d.copy_(host_of[id(d)], non_blocking=True)
                launch(s)
                for d in g_out:
                    host_of[id(d)].copy_(d, non_blocking=True)
            ev.record(s)
        for ev in forks:
            main.wait_event(ev)

    step()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(args.e2e_steps):
        step()
    b.record(st)
    barrier()
    t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.e2e_steps
    h2d = sum(t.numel() * t.element_size() for t in ins)
    d2h = sum(t.numel() * t.element_size() for t in outs)
    if dist is not None:
        sums = torch.tensor([h2d, d2h], dtype=torch.float64, device="cuda")
        dist.all_reduce(sums)
        h2d, d2h = int(sums[0].item()), int(sums[1].item())
    return {"value": round(w.global_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 3),
            "path": "pinned host -> device copies, Plan.launch, device -> pinned host" +
                    (f", {len(groups)} independent plans on their own streams" if groups else ", one stream")}


def host_memory_available() -> int:
    """Available host memory, bounded by the container's cgroup limit."""
    import psutil
    avail = psutil.virtual_memory().available
    for path, used in (("/sys/fs/cgroup/memory.max", "/sys/fs/cgroup/memory.current"),
                       ("/sys/fs/cgroup/memory/memory.limit_in_bytes", "/sys/fs/cgroup/memory/memory.usage_in_bytes")):
        try:
            with open(path) as f:
                lim = f.read().strip()
            if lim == "max":
                continue
            with open(used) as f:
                cur = int(f.read().strip())
            avail = min(avail, int(lim) - cur)
        except Exception:
            continue
    return avail


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip() + f" ({os.cpu_count()} logical CPUs)"
    except Exception:
        pass
    return f"{os.cpu_count()} logical CPUs"


def reference_arm(args, world, rank):
    """ASK's host code path restated (oracle), all host threads, bounded samples."""
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    vals = []
    desc = ""
    for _ in range(max(args.warmup, 0)):
        cpu_sample(args.workload, threads, budget_s=0.5)
    for _ in range(args.steps):
        bps, secs, desc = cpu_sample(args.workload, threads, budget_s=2.0)
        vals.append(bps / 1e9)
    value = statistics.median(vals)
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "impl": "reference", "vs_baseline": None,
            "data": "synthetic (seeded Philox4x32-10)", "config": static_config(args.workload, world),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc, "cpu": cpu_model()},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "ASK's host path needs an LLVM/MLIR 23.1 SDK to build; its semantics are restated in "
                    "oracle/ask_oracle.cpp and run here on all host threads (rows/elements split across threads)"}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
