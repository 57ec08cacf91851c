"""Benchmark: achieved HBM GB/s per plan on B200, next to ASK's host CPU path.

Headline workload (BASELINE.json's "at 1/2/4/8 B200" plan): cfg5, the sharded
large plan -- part one a global sum/min/argmin over 2^32 f32, part two the i32
chain ((x<<3) ^ (x>>5)) & 0x7fffffff + y over 2^31 elements -- split along the
leading axis across N GPUs (strong scaling), with one NCCL all-gather of the
reduction partials per step.  One step = both parts of the plan.  At N=1 the
line also carries `per_config`: cfg1, cfg2, cfg3, cfg3bf, cfg4g and cfg4s at
full size, each with its own value, roofline, CPU baseline, end-to-end figure
and output check (those configs are single-GPU: replicas only at N>1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg5|cfg1|...] [--no-per-config] [--no-check]

Rank 0 prints one JSON line.  Inputs are seeded synthetic data generated on
the device (Philox4x32-10) and are larger than L2, so no flush is needed
between steps.  After the timed region every output is checked on the device
(`check`).  The CPU baseline (a bounded sample, one thread) and the reference
arm (the full config, all host threads, plus a single-thread figure) run the
oracle: a restatement of ASK's host code path, whose own host compiler needs an
LLVM 23 SDK that is not available here.
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
# measured beside the headline cfg5 at N=1 (single-GPU configs: replicas only at N>1)
PER_CONFIG = ["cfg1", "cfg2", "cfg3", "cfg3bf", "cfg3u", "cfg4g", "cfg4s"]


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
    if name in ("cfg3u", "cfg3ubf"):
        dt = "f16" if name == "cfg3u" else "bf16"
        return {"workload": f"cfg3: 3-step softmax plan, {dt} [32768,4096], each owned step its own plan launch "
                            "(no runtime fusion)", "l2": "256 MB input > L2"}
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
        w.tensors = {"x": x, "xi": xi, "yi": yi, "z": z, "outs": outs, "scratch": scratch, "a0": a0}
        w.parts = (pa, x, outs, scratch, comm)
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
        w.tensors = {"abc": (a, b, c), "y": (y0, y1)}
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
        w.tensors = {"x": x, "outs": outs, "rows": rows, "cols": cols}
    elif name in ("cfg3u", "cfg3ubf"):
        # The same plan launched step by step through ask_b200_plan_launch, as
        # a Runtime that binds each owned step to its own kernel does: three
        # kernels, x read by each.
        dt = "f16" if name == "cfg3u" else "bf16"
        rows, cols = 32768, 4096
        n = rows * cols
        x = gen(2 if dt == "f16" else 3, SEED["cfg3"], 0, n, 0.0, 2.0, torch.int16)
        m = torch.empty(rows, dtype=torch.float32, device=dev)
        s = torch.empty(rows, dtype=torch.float32, device=dev)
        y = torch.empty_like(x)
        w.plans = [ask_b200.Plan(r, rank_device()) for r in R.cfg3_steps(dt, rows, cols)]
        pm, ps, py = w.plans
        w.kernels = [(pm.describe()["kernel"], 2 * n + 4 * rows, pm.bind([x], [m], None, st)),
                     (ps.describe()["kernel"], 2 * n + 8 * rows, ps.bind([x, m], [s], None, st)),
                     (py.describe()["kernel"], 4 * n + 8 * rows, py.bind([x, m, s], [y], None, st))]
        w.config = dict(static_config(name, world),
                        graded_bytes="each step's port bytes: max 2n + 4*rows, sum 2n + 8*rows, "
                                     "normalise 4n + 8*rows")
        w.dtype = dt
        w.e2e = {"inputs": [x], "results": [y]}
        w.tensors = {"x": x, "m": m, "s": s, "y": y, "rows": rows, "cols": cols}
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
        # value and roofline count the fused step's own bytes (x read once, y, m, s written);
        # plan_port_gbs counts the reference plan's port bytes (x read by all three steps)
        w.plan_port_bytes = 4 * 2 * n + 6 * 4 * rows
        w.session, w.program, w.stream_handle = session, prog, session.stream()
        w.config = dict(static_config(name, world),
                        plan=f"3 owned steps (max, sum of exp, normalise) run by the runtime as one {kernel} step, "
                             "CUDA graph", graded_bytes="the fused step's own bytes 2n (x) + 2n (y) + 8*rows (m, s); "
                                                        "plan_port_gbs: the 3-step plan's port bytes 8n + 24*rows")
        w.dtype = dt
        w.e2e = {"inputs": [x], "results": [y]}
        w.tensors = {"x": x, "m": m, "s": s, "y": y, "rows": rows, "cols": cols}
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
            w.tensors = {"table": table, "idx": idx, "out": out, "dim": dim}
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
            w.tensors = {"base": base, "idx": idx, "grad": grad, "out": out, "dim": dim}
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
# Output checks: run after the timed region (and outside it) on the bench's own
# inputs and outputs, with torch on the device as the checker.  Tolerances are
# the parity bars of the tests: bit-exact for integer, index, extreme and
# gather results; 2^-20 of the magnitude sum for float sums.
SUM_TOL = 2.0 ** -20
CHUNK = 1 << 28


def check_outputs(w, torch, dist, world):
    """Returns {"ok", "failures", "checked", ...} for the workload's outputs;
    every rank takes part (cfg5 combines its figures over the ranks)."""
    t = w.tensors
    fails, notes = 0, {}
    if w.name == "cfg5":
        x, xi, yi, z, outs = t["x"], t["xi"], t["yi"], t["z"], t["outs"]
        s64 = torch.zeros((), dtype=torch.float64, device=x.device)
        sabs = torch.zeros_like(s64)
        for i in range(0, x.numel(), CHUNK):
            c = x[i:i + CHUNK].double()
            s64 += c.sum()
            sabs += c.abs().sum()
        mn = torch.min(x)
        am = torch.argmin(x)  # first (lowest-index) minimum
        rec = torch.stack([s64, sabs, mn.double(), (am + t["a0"]).double()])
        if dist is not None:
            allrec = [torch.empty_like(rec) for _ in range(world)]
            dist.all_gather(allrec, rec)
        else:
            allrec = [rec]
        allrec = [r.cpu().tolist() for r in allrec]
        gsum = sum(r[0] for r in allrec)
        gabs = sum(r[1] for r in allrec)
        gmin, gidx = min((r[2], r[3]) for r in allrec)
        got = [outs[0].item(), outs[1].item(), int(outs[2].item())]
        sum_err = abs(got[0] - gsum)
        fails += int(sum_err > SUM_TOL * gabs) + int(got[1] != gmin) + int(got[2] != int(gidx))
        bad = torch.zeros((), dtype=torch.int64, device=x.device)
        for i in range(0, xi.numel(), CHUNK):
            a, b = xi[i:i + CHUNK], yi[i:i + CHUNK]
            ref = torch.bitwise_and(torch.bitwise_xor(a << 3, a >> 5), 0x7FFFFFFF) + b
            bad += (ref != z[i:i + CHUNK]).sum()
        if dist is not None:
            dist.all_reduce(bad)
        fails += int(bad.item())
        notes = {"sum_abs_err": sum_err, "sum_tol": SUM_TOL * gabs, "min": got[1], "argmin": got[2],
                 "i32_mismatches": int(bad.item()),
                 "checked": "global sum vs an f64 device sum over every rank's slice (tol 2^-20*sum|x|); min and "
                            "argmin vs torch min/argmin per slice combined lowest-index-first over the ranks; every "
                            "element of the i32 chain vs a torch int32 restatement"}
    elif w.name in ("cfg1", "cfg1a"):
        a, b, c = (v.double() for v in t["abc"])
        y0, y1 = t["y"]
        ea = a.exp()
        r0 = ea * b + c
        mx = torch.maximum(a, b)
        th = torch.tanh(c)
        r1 = mx - th
        tol0 = SUM_TOL * torch.maximum((ea * b).abs(), c.abs())
        tol1 = SUM_TOL * torch.maximum(mx.abs(), th.abs())
        fails += int(((y0.double() - r0).abs() > tol0).sum()) + int(((y1.double() - r1).abs() > tol1).sum())
        notes = {"checked": "every element of y0, y1 vs an f64 evaluation, within 2^-20 of the largest term "
                            "(about 8 f32 ulps)"}
    elif w.name in ("cfg2", "cfg2a"):
        x = t["x"].view(t["rows"], t["cols"])
        s, mx, mn, am = t["outs"]
        x64 = x.double()
        ref = x64.sum(1)
        tol = SUM_TOL * x64.abs().sum(1)
        del x64
        fails += int(((s.double() - ref).abs() > tol).sum())
        fails += int((mx != x.amax(1)).sum()) + int((mn != x.amin(1)).sum()) + int((am != x.argmax(1)).sum())
        notes = {"checked": "every row: sum vs f64 (tol 2^-20*sum|x|), max/min/argmax (first index) bit-exact vs torch"}
    elif w.name in ("cfg3", "cfg3bf", "cfg3u", "cfg3ubf"):
        tdt = torch.float16 if w.name in ("cfg3", "cfg3u") else torch.bfloat16
        x = t["x"].view(tdt).view(t["rows"], t["cols"]).float()
        m, s, y = t["m"], t["s"], t["y"]
        mref = x.amax(1)
        e = torch.exp(x - mref[:, None])
        sref = e.sum(1)
        yref = e / sref[:, None]
        del e, x
        # one unit in the last place of the 16-bit output type at yref
        mant = 10 if tdt == torch.float16 else 7
        tiny = 2.0 ** (-14 if tdt == torch.float16 else -126)
        ulp = torch.exp2(torch.floor(torch.log2(torch.clamp(yref.abs(), min=tiny))) - mant)
        yg = y.view(tdt).view(t["rows"], t["cols"]).float()
        fails += int(((yg - yref).abs() > ulp).sum())
        fails += int((m != mref).sum()) + int(((s - sref).abs() > 2.0 ** -16 * sref).sum())
        notes = {"checked": "all rows: m bit-exact vs torch amax, s within 2^-16 relative, every y within one "
                            "16-bit ulp of the f32 quotient"}
    elif w.name == "cfg4g":
        table, idx, out = t["table"], t["idx"], t["out"]
        dim = t["dim"]
        tv = table.view(-1, dim)
        ov = out.view(-1, dim)
        step = 1 << 20
        for i in range(0, idx.numel(), step):
            ref = tv.index_select(0, idx[i:i + step])
            fails += int((ov[i:i + step].view(torch.int32) != ref.view(torch.int32)).any(1).sum())
        notes = {"checked": "every gathered row bit-exact vs torch index_select"}
    elif w.name == "cfg4s":
        base, idx, grad, out = t["base"], t["idx"], t["grad"], t["out"]
        dim = t["dim"]
        ref = base.view(-1, dim).double().clone()
        mag = base.view(-1, dim).double().abs()
        gv = grad.view(-1, dim)
        step = 1 << 20
        for i in range(0, idx.numel(), step):
            g = gv[i:i + step].double()
            ref.index_add_(0, idx[i:i + step], g)
            mag.index_add_(0, idx[i:i + step], g.abs())
        fails += int(((out.view(-1, dim).double() - ref).abs() > SUM_TOL * mag).sum())
        notes = {"checked": "every table element vs an f64 segment sum (torch index_add_), tol 2^-20*sum|upd|"}
    else:
        return None
    return dict({"ok": fails == 0, "failures": fails}, **notes)


# ---------------------------------------------------------------------------
def measure(w, args, torch, barrier, dist, local):
    """Warm up, then time exactly args.steps steps between barriers; the max
    over ranks is the step time.  Returns the figures of a bench line."""
    st = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 3)):
        for _, _, fn in w.kernels:
            fn()
    barrier()
    nk = len(w.kernels)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.25)
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    # The timed region holds the steps alone, launched back to back as a user
    # runs them: an event between two plans would stop the next kernel from
    # starting early (programmatic dependent launch) and add its own gap.
    start.record(st)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        for _, _, fn in w.kernels:
            fn()
    h1 = time.perf_counter()
    end.record(st)
    barrier()
    clocks = sampler.stop()
    total_ms = start.elapsed_time(end)
    if nk > 1:
        # per-plan times for the rooflines: a second pass of as many steps,
        # after the timed region, with an event after each plan
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)] for _ in range(args.steps)]
        for s in range(args.steps):
            ev[s][0].record(st)
            for k, (_, _, fn) in enumerate(w.kernels):
                fn()
                ev[s][k + 1].record(st)
        barrier()
        per_kernel_ms = [sum(ev[s][k].elapsed_time(ev[s][k + 1]) for s in range(args.steps)) / args.steps
                         for k in range(nk)]
    else:
        per_kernel_ms = [total_ms / args.steps]
    t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    peak, peak_kind = peaks()
    kernels = []
    for (name, nbytes, _), ms in zip(w.kernels, per_kernel_ms):
        gbs = nbytes / (ms * 1e-3) / 1e9
        kernels.append({"kernel": name, "bytes_per_launch": nbytes, "ms": round(ms, 4), "gbs": round(gbs, 1),
                        "frac": round(gbs / peak, 4)})
    dom = max(range(nk), key=lambda k: per_kernel_ms[k])
    roofline = {"bound": "hbm", "achieved": kernels[dom]["gbs"], "peak": peak, "unit": "GB/s",
                "frac": kernels[dom]["frac"], "traffic": load_traffic(w.kernels[dom][0], w.kernels[dom][1]),
                "kernel": kernels[dom]["kernel"],
                "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                else "fallback 6.65 TB/s"}
    # host time to enqueue one step through the public API (Python -> C ABI
    # launch, or a runtime program's graph launch); the GPU runs behind it
    host_us = 1e6 * (h1 - h0) / args.steps
    return {"value": round(w.global_bytes / (ms_per_step * 1e-3) / 1e9, 1), "ms_per_step": round(ms_per_step, 4),
            "roofline": roofline, "kernels": kernels, "clocks": clocks,
            "gpu_launches": w.launches_per_step() * args.steps,
            "host_enqueue_us_per_step": round(host_us, 1),
            "kernel_timing": "the step's time" if nk == 1 else
            "a second pass of the same steps after the timed region, an event after each plan"}


def exchange_timing(w, args, torch, barrier, dist):
    """cfg5 at N>1: the cost of combining the ranks' reduction partials, as
    the time of the sharded reduction (split kernel, all-gather of the partial
    records, combine) minus the same plan combined locally, per step, max over
    ranks.  Leaves the outputs holding the sharded (global) result."""
    pa, x, outs, scratch, comm = w.parts
    st = torch.cuda.current_stream()
    k = max(args.steps, 10)

    def timed(fn):
        for _ in range(3):
            fn()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(k):
            fn()
        b.record(st)
        barrier()
        v = torch.tensor([a.elapsed_time(b) / k], dtype=torch.float64, device="cuda")
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return float(v.item())
    local = timed(lambda: pa.launch([x], outs, scratch, st))
    sharded = timed(lambda: pa.launch_sharded(comm, [x], outs, scratch, st))
    st_code, peer = comm.status()
    return {"reduce_local_ms": round(local, 4), "reduce_sharded_ms": round(sharded, 4),
            "exchange_us": round(1000.0 * (sharded - local), 1),
            "transport": "peer stores over NVLink" if peer else "NCCL all-gather", "status": st_code,
            "how": "sharded reduce (split kernel, records exchanged between the ranks, combine) minus the same plan "
                   "combined locally, back-to-back launches, CUDA events, max over ranks: the exchange plus each "
                   "launch's wait for the slowest rank; in a bench step it runs on a side stream beside the i32 chain"}


def pcie_bandwidth(torch, barrier, dist, nbytes=1 << 30):
    """Plain pinned-memory copy bandwidth of this rank (all ranks copying at
    once), host->device and device->host, GB/s."""
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream()
    out = {}
    for name, fn in (("h2d_gbs", lambda: d.copy_(h, non_blocking=True)),
                     ("d2h_gbs", lambda: h.copy_(d, non_blocking=True))):
        fn()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(4):
            fn()
        b.record(st)
        barrier()
        out[name] = round(4 * nbytes / (a.elapsed_time(b) * 1e-3) / 1e9, 2)
    del h, d
    return out


def bind_numa_local(torch, local):
    """Run this rank on the CPUs of its GPU's NUMA node, so that the pinned
    host buffers of the end-to-end run are allocated in that node's memory.
    Returns {"node": n, "cpus": k} or {"node": None, "why": reason}."""
    try:
        p = torch.cuda.get_device_properties(local)
        dev = f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        if not os.path.exists(dev):
            return {"node": None, "why": f"{dev} not visible"}
        with open(os.path.join(dev, "numa_node")) as f:
            node = int(f.read().strip())
        if node < 0:
            return {"node": None, "why": "the GPU reports no NUMA node"}
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = set()
            for part in f.read().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return {"node": node, "why": "none of the node's CPUs is available to this process"}
        os.sched_setaffinity(0, cpus)
        return {"node": node, "cpus": len(cpus)}
    except Exception as e:  # the topology is informational: never fail the bench on it
        return {"node": None, "why": f"{type(e).__name__}: {e}"}


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
    h2d_rank = sum(t.numel() * t.element_size() for t in ins)
    d2h_rank = sum(t.numel() * t.element_size() for t in outs)
    h2d, d2h = h2d_rank, d2h_rank
    if dist is not None:
        sums = torch.tensor([h2d, d2h], dtype=torch.float64, device="cuda")
        dist.all_reduce(sums)
        h2d, d2h = int(sums[0].item()), int(sums[1].item())
    del h_in, h_out
    bw = pcie_bandwidth(torch, barrier, dist)
    if dist is not None:
        v = torch.tensor([bw["h2d_gbs"], bw["d2h_gbs"]], dtype=torch.float64, device="cuda")
        dist.all_reduce(v, op=dist.ReduceOp.MIN)
        bw = {"h2d_gbs": round(float(v[0].item()), 2), "d2h_gbs": round(float(v[1].item()), 2)}
    # the time each direction needs at the measured copy rate, against the step
    t_h2d = h2d_rank / (bw["h2d_gbs"] * 1e9) if bw["h2d_gbs"] else 0.0
    t_d2h = d2h_rank / (bw["d2h_gbs"] * 1e9) if bw["d2h_gbs"] else 0.0
    step_s = ms * 1e-3
    frac = max(t_h2d, t_d2h) / step_s
    serial = (t_h2d + t_d2h) / step_s
    kernels = 100.0 * w.device_ms / ms if getattr(w, "device_ms", None) else None
    if frac > 0.85:
        limiter = f"the host<->device link: the busier direction ({'H2D' if t_h2d >= t_d2h else 'D2H'}) alone needs " \
                  f"{100 * frac:.0f}% of the step at the measured copy rate"
    elif serial > 0.85:
        limiter = (f"the host<->device copies: at the rates measured with every rank copying at once, H2D and D2H "
                   f"together need {100 * serial:.0f}% of the step ("
                   + ("one stream orders them" if not groups else
                      "the plans' streams overlap them, but both directions draw on the same host memory") + ")")
    else:
        limiter = f"neither link direction (busier {100 * frac:.0f}%, both {100 * serial:.0f}% of the step)"
    if kernels is not None:
        limiter += f"; the kernels take {kernels:.1f}% of the step"
    return {"value": round(w.global_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 3),
            "path": "pinned host -> device copies, Plan.launch, device -> pinned host" +
                    (f", {len(groups)} independent plans on their own streams" if groups else ", one stream"),
            "pcie": dict(bw, e2e_h2d_gbs_per_gpu=round(h2d_rank / step_s / 1e9, 2),
                         e2e_d2h_gbs_per_gpu=round(d2h_rank / step_s / 1e9, 2), numa=getattr(w, "numa_node", None),
                         copy_probe="1 GiB pinned copies, all ranks at once, min over ranks"),
            "pcie_frac": round(frac, 4), "serial_copy_frac": round(serial, 4), "limiter": limiter}


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


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


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
    ap.add_argument("--no-check", action="store_true")
    ap.add_argument("--no-per-config", action="store_true",
                    help="headline workload only (at N=1 the other configs are measured too by default)")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU baseline per config")
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
    numa = bind_numa_local(torch, local)
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

    def run_one(name, cpu_budget):
        """Build, time, check and (optionally) run end to end one workload."""
        w = make_workload(name, rank, world, torch, ask_b200, R, comm, small=args.small)
        w.numa_node = numa
        torch.cuda.synchronize()
        default_stream = torch.cuda.current_stream()
        if getattr(w, "stream_handle", None):  # a runtime session's stream: time and copy on it
            torch.cuda.set_stream(torch.cuda.ExternalStream(w.stream_handle))
        m = measure(w, args, torch, barrier, dist, local)
        w.device_ms = m["ms_per_step"]
        part = dict(m)
        if hasattr(w, "plan_port_bytes"):
            part["plan_port_gbs"] = round(w.plan_port_bytes / (m["ms_per_step"] * 1e-3) / 1e9, 1)
        if not args.no_check:
            part["check"] = check_outputs(w, torch, dist, world)
        if name == "cfg5" and world > 1:
            part["exchange"] = exchange_timing(w, args, torch, barrier, dist)
        if not args.no_e2e:
            part["e2e"] = run_e2e(w, args, torch, barrier, dist)
        if rank == 0 and world == 1 and not args.no_cpu:
            bps, secs, desc = cpu_sample(name, 1, budget_s=cpu_budget)
            part["cpu_baseline"] = {"value": round(bps / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                                    "sample": desc + f", {secs:.1f} s timed", "cpu": cpu_model()}
        w.config["grids"] = [pl.describe()["launch"]["grid"][0] for pl in w.plans]
        part["config"] = w.config
        part["dtype"] = w.dtype
        part["scaling"] = w.scaling
        part.update(getattr(w, "extra", {}))
        torch.cuda.set_stream(default_stream)
        torch.cuda.synchronize()
        for attr in ("session", "program"):
            if hasattr(w, attr):
                setattr(w, attr, None)
        del w
        torch.cuda.empty_cache()
        if hasattr(torch._C, "_host_emptyCache"):  # give the pinned e2e buffers back before the next config
            torch._C._host_emptyCache()
        return part

    head = run_one(args.workload, args.cpu_budget)
    per_config = None
    if world == 1 and not args.no_per_config and args.workload == "cfg5" and not args.small:
        per_config = {}
        for name in PER_CONFIG:
            try:
                per_config[name] = run_one(name, min(args.cpu_budget, 5.0))
            except Exception as e:  # one config failing must not take the headline line with it
                torch.cuda.synchronize()
                torch.cuda.empty_cache()
                per_config[name] = {"error": f"{type(e).__name__}: {e}"[:500]}

    line = {"metric": METRIC, "value": head["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": head["scaling"], "vs_baseline": None, "dtype": head["dtype"],
            "data": "synthetic (seeded Philox4x32-10)", "config": head["config"], "roofline": head["roofline"],
            "kernels": head["kernels"], "cpu_baseline": head.get("cpu_baseline"), "e2e": head.get("e2e"),
            "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
            "pct_of_8tbs": round(100.0 * head["value"] / world / 8000.0, 2)}
    for key in ("check", "exchange", "plan_port_gbs", "host_enqueue_us_per_step"):
        if key in head:
            line[key] = head[key]
    if per_config is not None:
        line["per_config"] = per_config
        line["gpu_launches"] += sum(p.get("gpu_launches", 0) for p in per_config.values())
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


# ---------------------------------------------------------------------------
# The CPU side: ASK's host code path restated (oracle/), test infrastructure
# used here only as the timed CPU baseline and the reference arm.
def cpu_case(name: str, threads: int, full: bool):
    """Inputs and a run function for the oracle on config `name`: the full
    config when `full` (host memory permitting), else a bounded sample.
    Returns (run, bytes per run, description)."""
    import numpy as np
    import oracle
    name = ARTIFACT_WORKLOADS.get(name, name)
    by_steps = name in ("cfg3u", "cfg3ubf")  # counted at the three steps' port bytes
    name = {"cfg3u": "cfg3", "cfg3ubf": "cfg3bf"}.get(name, name)
    gt = max(threads, host_threads())
    avail = host_memory_available()

    def fits(nbytes):
        return nbytes * 1.25 < avail

    if name == "cfg5":
        na, nb = 1 << 32, 1 << 31
        if not full or not fits(4 * na + 12 * nb):
            na, nb = (1 << 26, 1 << 25) if not full else (1 << 30, 1 << 29)
        x = oracle.generate(0, SEED["cfg5"], 0, 0, na, 0.0, 1.0, threads=gt)
        xi = oracle.generate(4, SEED["cfg5"], 1, 0, nb, 0, 0, threads=gt)
        yi = oracle.generate(4, SEED["cfg5"], 2, 0, nb, 0, 0, threads=gt)
        z = np.empty_like(xi)

        def run(th):
            oracle.cfg5a(x, threads=th)
            oracle.cfg5b(xi, yi, threads=th, out=z)
        what = "full config" if na == 1 << 32 else f"prefix of the config"
        return run, 4 * na + 12 * nb, f"cfg5 {what}: sum/min/argmin over {na} f32 + i32 chain over {nb}"
    if name == "cfg1":
        n = 4096 * 4096 if full else 1 << 22
        a, b, c = (oracle.generate(0, SEED["cfg1"], s, 0, n, -4.0, 4.0, threads=gt) for s in range(3))
        out = (np.empty_like(a), np.empty_like(a))
        return (lambda th: oracle.cfg1(a, b, c, threads=th, out=out)), 20 * n, f"cfg1 over {n} elements"
    if name == "cfg2":
        rows, cols = (65536 if full else 8192), 1024
        x = oracle.generate(1, SEED["cfg2"], 0, 0, rows * cols, 0.0, 1.0, threads=gt)
        return ((lambda th: oracle.rowstats(x, rows, cols, threads=th)), 4 * rows * cols + 20 * rows,
                f"cfg2 over {rows} rows")
    if name in ("cfg3", "cfg3bf"):
        dt = "f16" if name == "cfg3" else "bf16"
        rows, cols = (32768 if full else 1024), 4096
        x = oracle.generate(2 if dt == "f16" else 3, SEED["cfg3"], 0, 0, rows * cols, 0.0, 2.0, threads=gt)
        y = np.empty(rows * cols, np.uint16)
        # the oracle runs the 3-step plan (x read three times); counted at the bytes the GPU arm's
        # value counts: the fused step's own (4 per element) or, for cfg3u, the three steps' ports
        nbytes = 8 * rows * cols + 20 * rows if by_steps else 4 * rows * cols + 8 * rows
        return ((lambda th: oracle.softmax(dt, x, rows, cols, threads=th, out=y)), nbytes,
                f"cfg3 ({dt}) over {rows} rows, 3-step plan, counted at "
                + ("the three steps' port bytes" if by_steps else "the fused step's bytes"))
    rows, dim = 1 << 20, 256
    n = (1 << 23) if full else (1 << 18)
    idx = oracle.generate(5, SEED["cfg4"], 1, 0, n, 1.1, rows, threads=gt)
    if name == "cfg4g":
        if full and not fits(4 * rows * dim + 4 * n * dim):
            n = 1 << 21
            idx = idx[:n]
        table = oracle.generate(1, SEED["cfg4"], 0, 0, rows * dim, 0.0, 0.02, threads=gt)
        out = np.empty(n * dim, np.float32)
        nbytes = 8 * n + 4 * n * dim + 4 * dim * int(np.unique(idx).size)
        return ((lambda th: oracle.gather(table, idx, 1, rows, dim, threads=th, out=out)), nbytes,
                f"cfg4 gather of {n} indices")
    base = np.zeros(rows * dim, np.float32)
    upd = oracle.generate(1, SEED["cfg4"], 2, 0, n * dim, 0.0, 1.0, threads=gt)
    out = np.empty_like(base)
    return ((lambda th: oracle.scatter_add("f32", base, idx, upd, 1, rows, dim, out=out)),
            8 * n + 4 * n * dim + 8 * rows * dim, f"cfg4 scatter_add of {n} updates (single-threaded reference order)")


def cpu_sample(name: str, threads: int, budget_s: float = 12.0):
    """Time the oracle on a bounded sample of the workload.  Returns
    (bytes_per_second, seconds, description)."""
    run, nbytes, desc = cpu_case(name, threads, full=False)
    run(threads)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        run(threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 50:
            break
    return nbytes * reps / el, el, desc + f", {threads} thread(s)"


def reference_arm(args, world, rank):
    """ASK's host code path (restated in oracle/; the reference's own host
    compiler needs an LLVM 23 SDK that is not available) on the full config:
    `value` uses every host thread (rows/elements split across threads), and
    `single_thread` is the reference's own behaviour (its generated host
    function is single-threaded, lib/Lowering/Host.cpp:850-877)."""
    if rank != 0:
        return
    threads = host_threads()
    run, nbytes, desc = cpu_case(args.workload, threads, full=True)

    def timed(th):
        t0 = time.perf_counter()
        run(th)
        return nbytes / (time.perf_counter() - t0) / 1e9
    for _ in range(max(args.warmup, 0)):
        timed(threads)
    vals = [timed(threads) for _ in range(args.steps)]
    single = [timed(1) for _ in range(min(args.steps, 2))]
    value = statistics.median(vals)
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "impl": "reference", "vs_baseline": None,
            "data": "synthetic (seeded Philox4x32-10)", "config": static_config(args.workload, world),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc + f", one step = one run over it, {threads} threads", "cpu": cpu_model()},
            "single_thread": {"value": round(statistics.median(single), 3), "unit": "GB/s", "cores": 1,
                              "runs": len(single), "note": "the reference's own behaviour: one host thread"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "ASK's host path needs an LLVM/MLIR 23.1 SDK to build; its semantics are restated in "
                    "oracle/ask_oracle.cpp and run here on all host threads (value) and on one (single_thread)"}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
