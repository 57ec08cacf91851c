"""Multi-rank host logic of sharded plans, on CPU with gloo (world size 2 and 3).

Every rank builds the plan for its own slice (ask_b200.recipes.shard_range,
"index_base" = the slice's global offset), folds its slice into one partial
record per reduction (the CPU oracle stands in for the device here), the
records are exchanged with an all-gather, and every rank combines them in rank
order with the reference's rule (first NaN wins, else the smallest value,
ties to the lowest index; lib/Lowering/ScalarEmitter.h:506-517).  The result
must equal the single-process answer and be identical on all ranks.
"""
import math
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

N = 1_000_003
SEED = 0xA5C5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _combine(records):
    total = sum(r[0] for r in records)
    best = None
    for s64, mn, am in records:  # rank order
        if am < 0:
            continue
        if best is None:
            best = (mn, am)
            continue
        bn, cn = math.isnan(best[0]), math.isnan(mn)
        if (cn and not bn) or (not cn and not bn and mn < best[0]) or \
                ((cn == bn) and (cn or mn == best[0]) and am < best[1]):
            best = (mn, am)
    return total, best[0], best[1]


CASES = ["plain", "nan", "ties"]


def _input(case):
    import oracle
    x = oracle.generate(0, SEED, 0, 0, N, 0.0, 1.0)
    if case == "nan":
        x[N - 10] = np.nan       # in the last shard
        x[N // 2 + 7] = np.nan   # an earlier NaN in a middle shard wins
    if case == "ties":
        x[:] = np.maximum(x, np.float32(0.25))
        x[N - 3] = 0.125          # the minimum only in the last shard
        x[N // 3] = 0.125         # and an earlier equal one
    return x


def _rank(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import ask_b200
        import oracle
        from ask_b200 import recipes as R
        b, e = R.shard_range(N, world, rank)
        plan = ask_b200.Plan(R.cfg5a_step(e - b, index_base=b), device=-1)
        d = plan.describe()
        assert d["index_base"] == b and d["extent"] == e - b and d["shardable"]
        out = {}
        for case in CASES:
            x = _input(case)
            s64, _, mn, am = oracle.cfg5a(x[b:e], index_base=b)
            records = [None] * world
            dist.all_gather_object(records, (s64, mn, am))
            out[case] = _combine(records)
        queue.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_combine_matches_single_process(world):
    import oracle
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for case in CASES:
        s64, _, mn, am = oracle.cfg5a(_input(case))
        for rank in range(world):
            total, gmin, gidx = results[rank][case]
            assert gidx == am, case
            assert (math.isnan(gmin) and math.isnan(mn)) or gmin == mn, case
            assert (math.isnan(total) and math.isnan(s64)) or abs(total - s64) <= 1e-6 * abs(s64), case
        assert len({str(results[r][case]) for r in range(world)}) == 1  # identical on every rank
