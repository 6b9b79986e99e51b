"""Host logic of the N > 1 bench path on CPU: two gloo ranks.

bench.py reports whole-job throughput from the maximum device time over
ranks; these tests run that reduction and the rank bookkeeping as two real
processes (torch.distributed, gloo, 127.0.0.1) without a GPU."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      LOCAL_RANK=str(rank), WORLD_SIZE=str(world))
    import datetime
    import bench
    try:
        w, r, local = bench.dist_setup(world)
        torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
        # each rank "timed" a different duration; everyone must see the max
        got = bench.max_over_ranks(10.0 + 5.0 * r, w, torch.device("cpu"))
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        q.put((r, w, local, got))
    except BaseException as e:  # report, do not hang the parent
        q.put((rank, "error", repr(e), None))


@pytest.mark.timeout(120)
def test_max_over_ranks_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=100) for _ in procs]
    for p in procs:
        p.join(timeout=30)
    results.sort()
    assert [r[1] for r in results] == [2, 2], results
    assert [r[2] for r in results] == [0, 1]
    assert all(r[3] == 15.0 for r in results)


def test_dist_setup_rejects_mismatched_world(monkeypatch):
    import bench
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("LOCAL_RANK", "1")
    with pytest.raises(SystemExit):
        bench.dist_setup(4)
    assert bench.dist_setup(2) == (2, 1, 1)
    monkeypatch.setenv("WORLD_SIZE", "1")
    assert bench.max_over_ranks(3.5, 1, None) == 3.5
