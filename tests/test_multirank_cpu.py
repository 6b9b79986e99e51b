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


# ---- tensor-parallel shard plan (host logic of the N > 1 serving path) ----

def _plans(cfg, size):
    import qwen35
    return [qwen35.tp_plan(cfg, r, size) for r in range(size)]


def _assert_partition(ranges, total):
    pos = 0
    for a, b in ranges:
        assert a == pos and b > a, ranges
        pos = b
    assert pos == total, ranges


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_tp_plan_partitions_config1(size):
    import qwen35
    c = qwen35.CONFIG1
    plans = _plans(c, size)
    _assert_partition([p["query_heads"] for p in plans], c.heads)
    _assert_partition([p["gdn_heads"] for p in plans], c.ssm_values)
    _assert_partition([p["ffn_blocks"] for p in plans], c.ffn // 256)
    _assert_partition([p["vocab_rows"] for p in plans], c.vocab)
    _assert_partition([p["hidden_rows"] for p in plans], c.hidden)
    group = c.heads // c.kv_heads
    for p in plans:
        q0, q1 = p["query_heads"]
        # the KV heads a rank keeps are exactly those its query heads read
        assert p["kv_heads"] == (q0 // group, (q1 - 1) // group + 1)
        assert ((q1 - q0) * c.head_dim) % 256 == 0
        v0, v1 = p["vocab_rows"]
        assert v0 % 128 == 0
    if size == 8:   # two ranks share each KV head
        assert [p["kv_heads"] for p in plans] == [(i // 2, i // 2 + 1) for i in range(8)]


def test_tp_plan_rejects_unsplittable_geometry():
    from dataclasses import replace
    import prism_b200 as pb
    import qwen35
    c = qwen35.CONFIG1
    with pytest.raises(pb.PrismB200Error) as e:
        qwen35.tp_plan(c, 0, 3)            # 16 heads do not split 3 ways
    assert e.value.code == pb.E_UNSUPPORTED
    with pytest.raises(pb.PrismB200Error) as e:
        qwen35.tp_plan(qwen35.SMALL, 0, 2)  # key heads != value heads
    assert e.value.code == pb.E_UNSUPPORTED
    with pytest.raises(pb.PrismB200Error) as e:
        qwen35.tp_plan(c, 2, 2)            # rank outside the group
    assert e.value.code == pb.E_INVALID
    with pytest.raises(pb.PrismB200Error) as e:
        qwen35.tp_plan(c, 0, 16)           # more ranks than the exchange supports
    assert e.value.code == pb.E_INVALID
    assert qwen35.tp_plan(replace(qwen35.SMALL, ssm_groups=4), 1, 2)["gdn_heads"] == (2, 4)
    # one rank owns everything, whatever the geometry
    assert qwen35.tp_plan(qwen35.SMALL, 0, 1)["gdn_heads"] == (0, qwen35.SMALL.ssm_values)


def _plan_rank(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "prism-inference_b200")):
        sys.path.insert(0, p)
    try:
        import datetime
        import qwen35
        torch.distributed.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port,
                                             rank=rank, world_size=world,
                                             timeout=datetime.timedelta(seconds=60))
        mine = qwen35.tp_plan(qwen35.CONFIG1, rank, world)
        plans = [None] * world
        torch.distributed.all_gather_object(plans, mine)
        torch.distributed.destroy_process_group()
        q.put((rank, plans))
    except BaseException as e:
        q.put((rank, repr(e)))


@pytest.mark.timeout(120)
def test_tp_plan_two_gloo_ranks_agree():
    """Each rank derives only its own slice; gathered, the slices tile every
    axis, as the serving processes rely on without exchanging the plan."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_plan_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert not isinstance(res[0], str), res[0]
    assert res[0] == res[1]
    import qwen35
    c = qwen35.CONFIG1
    _assert_partition([p["query_heads"] for p in res[0]], c.heads)
    _assert_partition([p["vocab_rows"] for p in res[0]], c.vocab)
