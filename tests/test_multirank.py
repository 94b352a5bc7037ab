"""The N > 1 path of bench.py on CPU: world_size-2 gloo ranks (no GPU).  Each rank owns an
independent pack (its own keys and tokens); the only collectives are the set-up broadcast of
rank 0's calibration, the barrier and the max-over-ranks reduction of the timed region, and
rank 0 reports the aggregate."""
import os
import socket
import sys

import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, ws, port, q):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        bench.barrier(ws)
        ms = 1000.0 + 250.0 * rank            # rank 1 is the slow one
        ms_max = bench.max_over_ranks(ms, ws)
        # calibration results travel from rank 0 (the other ranks pass None)
        seeds = bench.broadcast_object({"L0.tm": (1.5, -0.25, 3), "gain:L0.u": 0.5} if rank == 0 else None, ws)
        q.put((rank, ms_max, bench.pack_seeds(rank), bench.aggregate_tokens_per_s(64, ws, 2, ms_max), seeds))
        bench.barrier(ws)
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_reduction_and_packs():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    assert [g[1] for g in got] == [1250.0, 1250.0]          # every rank sees the slowest time
    assert got[0][2] != got[1][2]                            # distinct packs
    assert abs(got[0][3] - 64 * 2 * 2 / 1.25) < 1e-9         # 64 conversations x 2 ranks x 2 steps / 1.25 s
    assert got[0][4] == got[1][4] == {"L0.tm": (1.5, -0.25, 3), "gain:L0.u": 0.5}   # rank 0's seeds everywhere
