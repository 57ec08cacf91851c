"""Sharded cfg5 on several GPUs (one process per GPU): the record exchange of
ask_b200_plan_launch_sharded -- over peer memory, or by the NCCL all-gather
when the peer exchange is switched off -- must give every rank the single-GPU
answer, and the i32 shards (no collective) must equal the corresponding slice.
A rank that skips a launch makes the others' bounded wait run out: they report
ASK_B200_E_TIMEOUT instead of hanging.  Skipped when fewer than two GPUs are
visible.  NVLS is off in every child (NCCL_NVLS_ENABLE=0)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
N = (1 << 26) + 12345
SEED = 0xA5C5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, queue, peer=True):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    if not peer:
        os.environ["ASK_B200_NO_PEER_EXCHANGE"] = "1"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = None
    try:
        import ask_b200
        from ask_b200 import recipes as R
        uid = [ask_b200.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = ask_b200.Comm(uid[0], world, rank, rank)
        st = torch.cuda.current_stream()
        b, e = R.shard_range(N, world, rank)
        x = torch.empty(e - b, dtype=torch.float32, device="cuda")
        ask_b200.generate(0, SEED, 0, b, e - b, 0.0, 1.0, x, st)
        if rank == world - 1:
            x[-5] = 0.0   # a minimum in the last shard ...
        if rank == 0:
            x[7] = 0.0    # ... and an earlier one in the first
        plan = ask_b200.Plan(R.cfg5a_step(e - b, index_base=b), rank)
        outs = [torch.empty(1, device="cuda"), torch.empty(1, device="cuda"),
                torch.empty(1, dtype=torch.int64, device="cuda")]
        scratch = torch.empty(plan.scratch_bytes, dtype=torch.uint8, device="cuda")
        for _ in range(5):  # repeated launches reuse scratch, records and the inboxes' two parities
            plan.launch_sharded(comm, [x], outs, scratch, st)
        torch.cuda.synchronize()
        status, used_peer = comm.status()
        assert status == ask_b200.OK and used_peer == peer, (status, used_peer)
        # the i32 chain on this rank's slice
        nb = (1 << 24) + 7
        bb, be = R.shard_range(nb, world, rank)
        xi = torch.empty(be - bb, dtype=torch.int32, device="cuda")
        yi = torch.empty_like(xi)
        ask_b200.generate(4, SEED, 1, bb, be - bb, 0, 0, xi, st)
        ask_b200.generate(4, SEED, 2, bb, be - bb, 0, 0, yi, st)
        z = torch.empty_like(xi)
        ask_b200.Plan(R.cfg5b_step(be - bb), rank).launch([xi, yi], [z], None, st)
        torch.cuda.synchronize()
        queue.put((rank, (float(outs[0].item()), float(outs[1].item()), int(outs[2].item())),
                   (bb, z.cpu().numpy())))
        dist.barrier()  # every rank's launches are done before any communicator goes
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("peer", [True, False], ids=["peer_exchange", "nccl_all_gather"])
def test_sharded_cfg5_matches_single_gpu(device, peer):
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    import ask_b200
    import oracle
    from ask_b200 import recipes as R
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue, peer)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, red, ew = queue.get(timeout=300)
        got[r] = (red, ew)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # single-GPU reference on device 0
    x = torch.empty(N, dtype=torch.float32, device="cuda:0")
    ask_b200.generate(0, SEED, 0, 0, N, 0.0, 1.0, x, torch.cuda.current_stream())
    b_last, _ = R.shard_range(N, world, world - 1)
    x[N - 5] = 0.0
    x[7] = 0.0
    plan = ask_b200.Plan(R.cfg5a_step(N), 0)
    outs = [torch.empty(1, device="cuda"), torch.empty(1, device="cuda"), torch.empty(1, dtype=torch.int64, device="cuda")]
    plan.launch([x], outs, torch.empty(plan.scratch_bytes, dtype=torch.uint8, device="cuda"), torch.cuda.current_stream())
    torch.cuda.synchronize()
    ref = (float(outs[0].item()), float(outs[1].item()), int(outs[2].item()))
    assert ref[1] == 0.0 and ref[2] == 7
    for r in range(world):
        s, m, a = got[r][0]
        assert m == ref[1] and a == ref[2]
        assert abs(s - ref[0]) <= 2.0 ** -20 * ref[0]
    assert len({got[r][0] for r in range(world)}) == 1  # identical on all ranks
    nb = (1 << 24) + 7
    xi = oracle.generate(4, SEED, 1, 0, nb, 0, 0)
    yi = oracle.generate(4, SEED, 2, 0, nb, 0, 0)
    z = oracle.cfg5b(xi, yi)
    for r in range(world):
        bb, zz = got[r][1]
        assert np.array_equal(zz, z[bb:bb + zz.size])


def _timeout_rank(rank, world, port, queue):
    """Rank 1 skips the second launch: rank 0 waits for its flag, gives up
    after ASK_B200_EXCHANGE_TIMEOUT_MS and reports it.  Both ranks stay alive
    (and keep their buffers mapped) until rank 0's kernel has returned."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      ASK_B200_EXCHANGE_TIMEOUT_MS="200")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = None
    try:
        import ask_b200
        from ask_b200 import recipes as R
        uid = [ask_b200.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = ask_b200.Comm(uid[0], world, rank, rank)
        st = torch.cuda.current_stream()
        n = 1 << 20
        x = torch.rand(n, device="cuda")
        plan = ask_b200.Plan(R.cfg5a_step(n, index_base=rank * n), rank)
        outs = [torch.full((1,), -1.0, device="cuda"), torch.full((1,), -1.0, device="cuda"),
                torch.full((1,), -1, dtype=torch.int64, device="cuda")]
        scratch = torch.empty(plan.scratch_bytes, dtype=torch.uint8, device="cuda")
        plan.launch_sharded(comm, [x], outs, scratch, st)  # both ranks: completes
        torch.cuda.synchronize()
        first = comm.status()
        dist.barrier()
        if rank == 0:
            outs[0].fill_(-7.0)
            plan.launch_sharded(comm, [x], outs, scratch, st)  # nobody answers
            torch.cuda.synchronize()
        dist.barrier()  # rank 0's kernel has returned before anyone's buffers could go
        queue.put((rank, first, comm.status(), float(outs[0].item())))
        dist.barrier()
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_peer_exchange_wait_is_bounded(device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    import ask_b200
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, first, after, sum0 = queue.get(timeout=300)
        got[r] = (first, after, sum0)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    if not got[0][0][1]:
        pytest.skip("the peer exchange is not available between these GPUs (NCCL all-gather path)")
    assert got[0][0] == (ask_b200.OK, True) and got[1][0] == (ask_b200.OK, True)
    assert got[0][1] == (ask_b200.E_TIMEOUT, True)   # rank 0's wait ran out
    assert got[0][2] == -7.0                          # ... and left its outputs as they were
    assert got[1][1] == (ask_b200.OK, True)


def _graph_rank(rank, world, port, queue):
    """Sharded launches captured once in a CUDA graph and replayed: the
    exchange's epoch advances on the device, so every replay matches the
    eagerly launched result."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = None
    try:
        import ask_b200
        from ask_b200 import recipes as R
        uid = [ask_b200.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = ask_b200.Comm(uid[0], world, rank, rank)
        n = (1 << 22) + 3 * rank
        b = sum((1 << 22) + 3 * r for r in range(rank))
        x = torch.empty(n, dtype=torch.float32, device="cuda")
        ask_b200.generate(0, SEED, 0, b, n, 0.0, 1.0, x, torch.cuda.current_stream())
        plan = ask_b200.Plan(R.cfg5a_step(n, index_base=b), rank)
        scratch = torch.empty(plan.scratch_bytes, dtype=torch.uint8, device="cuda")
        eager = [torch.empty(1, device="cuda"), torch.empty(1, device="cuda"), torch.empty(1, dtype=torch.int64, device="cuda")]
        plan.launch_sharded(comm, [x], eager, scratch, torch.cuda.current_stream())
        torch.cuda.synchronize()
        outs = [torch.empty(1, device="cuda"), torch.empty(1, device="cuda"), torch.empty(1, dtype=torch.int64, device="cuda")]
        side = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        dist.barrier()
        with torch.cuda.graph(g, stream=side):
            plan.launch_sharded(comm, [x], outs, scratch, side)
        results = []
        for _ in range(3):
            for t in outs:
                t.fill_(-1)
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            results.append([float(outs[0].item()), float(outs[1].item()), int(outs[2].item())])
        dist.barrier()
        del g
        queue.put((rank, [float(eager[0].item()), float(eager[1].item()), int(eager[2].item())], results,
                   comm.status()))
        dist.barrier()
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_sharded_launch_replays_in_a_cuda_graph(device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    import ask_b200
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_graph_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, eager, replays, status = queue.get(timeout=300)
        got[r] = (eager, replays, status)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        eager, replays, status = got[r]
        assert status[0] == ask_b200.OK
        assert all(rep == eager for rep in replays), (eager, replays)
    assert got[0][0] == got[1][0]


def test_single_rank_sharded_launch_matches_plain_launch(device):
    """A communicator of one rank takes the peer-exchange path (its own inbox
    only): repeated sharded launches equal the plan's plain launch bit for bit
    and report no timeout.  Runs on one GPU."""
    import ask_b200
    from ask_b200 import recipes as R
    torch.cuda.set_device(0)
    comm = ask_b200.Comm(ask_b200.comm_unique_id(), 1, 0, 0)
    try:
        n = (1 << 24) + 5
        x = torch.empty(n, dtype=torch.float32, device="cuda")
        ask_b200.generate(0, SEED, 0, 0, n, 0.0, 1.0, x, torch.cuda.current_stream())
        x[12345] = 0.0
        plan = ask_b200.Plan(R.cfg5a_step(n), 0)
        scratch = torch.empty(plan.scratch_bytes, dtype=torch.uint8, device="cuda")
        mk = lambda: [torch.empty(1, device="cuda"), torch.empty(1, device="cuda"),
                      torch.empty(1, dtype=torch.int64, device="cuda")]
        plain = mk()
        plan.launch([x], plain, scratch, torch.cuda.current_stream())
        for _ in range(3):
            got = mk()
            plan.launch_sharded(comm, [x], got, scratch, torch.cuda.current_stream())
            torch.cuda.synchronize()
            assert [g.item() for g in got] == [p.item() for p in plain]
        assert int(plain[2].item()) == 12345 and float(plain[1].item()) == 0.0
        assert comm.status() == (ask_b200.OK, True)
    finally:
        comm.close()
