"""The output checks `bench.py` runs after its timed region (host only).

`bench.check_outputs` is the evidence a bench line carries that the outputs it
timed are right (`"check": {"ok": ...}`).  Here it runs on CPU tensors: for
every workload a correct set of outputs must pass and one planted mistake must
be caught; cfg5's global sum/min/argmin check runs on two gloo ranks, each
holding its own slice, as it does under torchrun.
"""
import os
import socket
import types

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _work(name, **tensors):
    return types.SimpleNamespace(name=name, tensors=tensors)


def _cfg5_tensors(n, nb, a0, rng):
    x = torch.from_numpy(rng.random(n, dtype=np.float32))
    xi = torch.from_numpy(rng.integers(-2 ** 31, 2 ** 31, nb, dtype=np.int64).astype(np.int32))
    yi = torch.from_numpy(rng.integers(-2 ** 31, 2 ** 31, nb, dtype=np.int64).astype(np.int32))
    z = torch.bitwise_and(torch.bitwise_xor(xi << 3, xi >> 5), 0x7FFFFFFF) + yi
    return x, xi, yi, z


def test_cfg5_single_rank():
    rng = np.random.default_rng(1)
    x, xi, yi, z = _cfg5_tensors(4099, 1000, 0, rng)
    x[77] = 0.0
    x[3000] = 0.0  # a tie: the lowest index wins
    outs = [torch.tensor([float(x.double().sum())], dtype=torch.float32), torch.tensor([0.0]),
            torch.tensor([77], dtype=torch.int64)]
    w = _work("cfg5", x=x, xi=xi, yi=yi, z=z, outs=outs, a0=0)
    assert bench.check_outputs(w, torch, None, 1)["ok"]
    outs[2][0] = 3000
    assert bench.check_outputs(w, torch, None, 1)["failures"] == 1
    outs[2][0] = 77
    z[5] += 1
    r = bench.check_outputs(w, torch, None, 1)
    assert not r["ok"] and r["i32_mismatches"] == 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, plant, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, nb = 5000, 1200
        rng = np.random.default_rng(10 + rank)
        x, xi, yi, z = _cfg5_tensors(n, nb, rank * n, rng)
        x[123] = 0.0  # every rank holds a zero minimum; rank 0's is the global first
        # every rank holds the global answer, as after the record exchange
        all_sum = torch.zeros(1, dtype=torch.float64)
        all_sum[0] = x.double().sum()
        dist.all_reduce(all_sum)
        outs = [all_sum.float(), torch.tensor([0.0]), torch.tensor([123], dtype=torch.int64)]
        if plant and rank == 1:
            z[7] ^= 1
        w = _work("cfg5", x=x, xi=xi, yi=yi, z=z, outs=outs, a0=rank * n)
        r = bench.check_outputs(w, torch, dist, world)
        queue.put((rank, r["ok"], r["failures"], r["argmin"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("plant", [False, True])
def test_cfg5_two_gloo_ranks(plant):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, plant, queue)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (ok, f, am)) for r, ok, f, am in (queue.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        ok, failures, argmin = got[r]
        assert argmin == 123
        # the i32 mismatch on rank 1 is summed over the ranks: both report it
        assert (ok, failures) == ((False, 1) if plant else (True, 0))


def test_cfg1():
    rng = np.random.default_rng(2)
    a, b, c = (torch.from_numpy(rng.uniform(-4, 4, 1000).astype(np.float32)) for _ in range(3))
    y0 = torch.exp(a) * b + c
    y1 = torch.maximum(a, b) - torch.tanh(c)
    w = _work("cfg1", abc=(a, b, c), y=(y0, y1))
    assert bench.check_outputs(w, torch, None, 1)["ok"]
    y1[9] = torch.nextafter(y1[9], torch.tensor(1e9)) * 1.001
    assert bench.check_outputs(w, torch, None, 1)["failures"] == 1


def test_cfg2():
    rng = np.random.default_rng(3)
    rows, cols = 64, 256
    x = torch.from_numpy(rng.standard_normal(rows * cols).astype(np.float32))
    x2 = x.view(rows, cols)
    x2[5, 7] = x2[5].max()  # a tie: argmax keeps the first
    outs = [x2.double().sum(1).float(), x2.amax(1), x2.amin(1), x2.argmax(1)]
    w = _work("cfg2", x=x, outs=outs, rows=rows, cols=cols)
    assert bench.check_outputs(w, torch, None, 1)["ok"]
    outs[3][5] = cols - 1
    assert bench.check_outputs(w, torch, None, 1)["failures"] == 1


@pytest.mark.parametrize("name,tdt", [("cfg3", torch.float16), ("cfg3bf", torch.bfloat16), ("cfg3u", torch.float16)])
def test_cfg3(name, tdt):
    rng = np.random.default_rng(4)
    rows, cols = 16, 512
    xv = torch.from_numpy(rng.normal(0, 2, rows * cols).astype(np.float32)).to(tdt)
    xf = xv.float().view(rows, cols)
    m = xf.amax(1)
    e = torch.exp(xf - m[:, None])
    s = e.sum(1)
    y = (e / s[:, None]).to(tdt).reshape(-1)
    w = _work(name, x=xv.view(torch.int16), m=m, s=s, y=y.view(torch.int16), rows=rows, cols=cols)
    assert bench.check_outputs(w, torch, None, 1)["ok"]
    yb = y.view(torch.int16)
    yb[100] += 3  # three units in the last place
    assert bench.check_outputs(w, torch, None, 1)["failures"] == 1


def test_cfg4_gather_and_scatter():
    rng = np.random.default_rng(5)
    rows, dim, n = 40, 8, 300
    table = torch.from_numpy(rng.standard_normal(rows * dim).astype(np.float32))
    idx = torch.from_numpy(rng.integers(0, rows, n).astype(np.int64))
    out = table.view(rows, dim)[idx].reshape(-1).clone()
    w = _work("cfg4g", table=table, idx=idx, out=out, dim=dim)
    assert bench.check_outputs(w, torch, None, 1)["ok"]
    out[dim * 11 + 3] += 1.0
    assert bench.check_outputs(w, torch, None, 1)["failures"] == 1
    grad = torch.from_numpy(rng.standard_normal(n * dim).astype(np.float32))
    base = torch.zeros(rows * dim)
    res = base.view(rows, dim).double().index_add(0, idx, grad.view(n, dim).double()).float().reshape(-1)
    w = _work("cfg4s", base=base, idx=idx, grad=grad, out=res, dim=dim)
    assert bench.check_outputs(w, torch, None, 1)["ok"]
    res[5] += 0.25
    assert bench.check_outputs(w, torch, None, 1)["failures"] == 1
