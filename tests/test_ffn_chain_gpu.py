"""The FFN chain over token tiles (prism_b200_ffn_*, the reference's
project_f32_ffn_chain_tokens, src/kernels/projection.rs:261-350).

One GPU: every token's output is the CPU oracle's chain bit for bit --
Q8_K of x, the gate and up projections, SwiGLU in binary32 (silu(v) =
v / (1 + exp(-v)), the exponential evaluated in binary64 and rounded once,
as the kernels and the oracle's model do), Q8_K of the product, the down
projection and the residual added last.

Tensor-parallel on 2 GPUs (one process each): the down projection's partial
sums are all-reduced in rank order, so each output is within a stated
tolerance of the one-GPU chain -- |tp - one| <= 1e-5 * max|one| over the
tile (each row sums 2 x F/512 block terms in two chains instead of one) --
and the ranks agree bit for bit.
"""
import os
import socket

import numpy as np
import pytest

import prism_b200 as pb

pytestmark = pytest.mark.gpu
TP_TOL = 1e-5


def _silu(v):
    e = np.exp(-v.astype(np.float64)).astype(np.float32)
    return (v / (np.float32(1.0) + e)).astype(np.float32)


def _oracle_chain(kind, gate, up, down, H, F, x, residual):
    from oracle import oracle
    out = np.zeros_like(x)
    for m in range(x.shape[0]):
        q = oracle.q8k_quantize(x[m])
        g = oracle.matvec(kind, gate, F, H, q, threads=8)
        u = oracle.matvec(kind, up, F, H, q, threads=8)
        h = (u * _silu(g)).astype(np.float32)
        y = oracle.matvec(kind, down, H, F, oracle.q8k_quantize(h), threads=8)
        out[m] = y if residual is None else (residual[m] + y).astype(np.float32)
    return out


def _weights(kind, H, F, seed):
    return (pb.synth_weights(kind, F, H, seed, 1), pb.synth_weights(kind, F, H, seed, 2),
            pb.synth_weights(kind, H, F, seed, 3))


def _inputs(M, H, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((M, H)).astype(np.float32),
            rng.standard_normal((M, H)).astype(np.float32))


@pytest.mark.parametrize("kind", [pb.KIND_TQ2_0, pb.KIND_Q2_K])
@pytest.mark.parametrize("residual", [False, True])
def test_one_gpu_chain_matches_oracle(kind, residual):
    H, F, M = 512, 1024, 37
    gate, up, down = _weights(kind, H, F, 11)
    x, r = _inputs(M, H, 12)
    r = r if residual else None
    with pb.ProjectionExecutor(0) as ex:
        tens = [pb.Tensor(kind, H, F, gate), pb.Tensor(kind, H, F, up),
                pb.Tensor(kind, F, H, down)]
        f = pb.FfnChain(ex, *tens, max_tokens=64)
        got = f(x, r)
        got2 = f(x[:5], None if r is None else r[:5])  # a smaller second call
        f.close()
    want = _oracle_chain(kind, gate, up, down, H, F, x, r)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(got2.view(np.uint32), want[:5].view(np.uint32))


def test_chain_rejects_bad_geometry():
    H, F = 512, 1024
    gate, up, down = _weights(pb.KIND_TQ2_0, H, F, 13)
    with pb.ProjectionExecutor(0) as ex:
        g = pb.Tensor(pb.KIND_TQ2_0, H, F, gate)
        u = pb.Tensor(pb.KIND_TQ2_0, H, F, up)
        d = pb.Tensor(pb.KIND_TQ2_0, F, H, down)
        with pytest.raises(pb.PrismB200Error):
            pb.FfnChain(ex, g, u, g, max_tokens=8)          # down is not [H][F]
        with pytest.raises(pb.PrismB200Error):
            pb.FfnChain(ex, g, u, d, max_tokens=8, tp_rank=0, tp_size=3)  # F % (256*3)
        with pytest.raises(pb.PrismB200Error):
            pb.FfnChain(ex, g, u, d, max_tokens=8, tp_rank=2, tp_size=2)
        f = pb.FfnChain(ex, g, u, d, max_tokens=8)
        with pytest.raises(pb.PrismB200Error):
            f(np.zeros((9, H), np.float32))                  # more tokens than prepared
        f.close()


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, kind, H, F, M, q):
    try:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=180))
        gate, up, down = _weights(kind, H, F, 21)
        x, r = _inputs(M, H, 22)
        res = {}
        with pb.ProjectionExecutor(rank) as ex:
            tens = [pb.Tensor(kind, H, F, gate), pb.Tensor(kind, H, F, up),
                    pb.Tensor(kind, F, H, down)]
            f = pb.FfnChain(ex, *tens, max_tokens=M, tp_rank=rank, tp_size=world)
            handles = [None] * world
            dist.all_gather_object(handles, f.exchange_handle())
            f.connect(handles)
            dist.barrier()
            res["tp"] = [f(x, r), f(x[: M // 2], None), f(x, r)]
            dist.barrier()
            f.close()
            if rank == 0:
                one = pb.FfnChain(ex, *tens, max_tokens=M)
                res["one"] = [one(x, r), one(x[: M // 2], None)]
                one.close()
        dist.destroy_process_group()
        q.put((rank, res))
    except BaseException as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))


@pytest.mark.timeout(600)
@pytest.mark.skipif(_gpus() < 2, reason="tensor parallelism needs 2 GPUs (one per rank)")
def test_tp2_chain_allreduce_within_tolerance():
    import torch.multiprocessing as mp
    world, kind, H, F, M = 2, pb.KIND_TQ2_0, 2560, 9216, 300
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, kind, H, F, M, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in procs:
            r, res = q.get(timeout=500)
            out[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(out[r], str), "rank %d: %s" % (r, out[r])
    t0 = out[0]["tp"]
    for r in range(1, world):
        for a, b in zip(out[r]["tp"], t0):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), "ranks differ"
    one = out[0]["one"]
    for got, want in ((t0[0], one[0]), (t0[1], one[1]), (t0[2], one[0])):
        err = np.abs(got.astype(np.float64) - want)
        assert err.max() <= TP_TOL * np.abs(want).max(), err.max() / np.abs(want).max()
