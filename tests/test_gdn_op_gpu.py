"""The reference's batched gated-delta op with snapshots and replay
(src/backend/gdn.rs:24-300) on the device, bit for bit against the oracle:
cache rows and snapshot slots, per-column and raw gates, broadcast q/k heads
and sequences, and replay with records (including a round trip of the
records the op itself writes); invalid rows or control are device-side
E_INVALID errors."""
import numpy as np
import pytest

import prism_b200 as pb

pytestmark = pytest.mark.gpu


def mkop(cls, **kw):
    o = cls()
    for f, _ in cls._fields_:
        setattr(o, f, kw.get(f, 0))
    return o


def run(ex, kw, arrays):
    import torch
    from oracle import oracle
    want = oracle.gdn_delta_values(mkop(oracle.GdnOp, **kw), **arrays)
    dev = {}
    for name, a in arrays.items():
        if a is None:
            dev[name] = None
            continue
        dt = torch.int32 if a.dtype == np.int32 else torch.float32
        dev[name] = torch.from_numpy(np.ascontiguousarray(a)).to(dtype=dt).cuda()
    op = mkop(pb.GdnOp, **kw)
    out = torch.full((pb.gdn_delta_values_outputs(op),), float("nan"), device="cuda")
    # slots past the tokens keep the caller's contents: seed both sides alike
    ptr = lambda n: None if dev.get(n) is None else dev[n].data_ptr()
    pb.gdn_delta_values_device(ex, op, ptr("q"), ptr("k"), ptr("v"), ptr("gate"), ptr("beta"),
                               ptr("table"), out.data_ptr(), rows=ptr("rows"), bias=ptr("bias"),
                               weight=ptr("weight"), records=ptr("records"),
                               control=ptr("control"),
                               stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ex.sync()
    got = out.cpu().numpy()
    n = min(got.size, want.size)
    return got[:n], want[:n]


def inputs(W, H, T, S, gw=1, seed=0, rows=None, qh=None, qs=None):
    rng = np.random.default_rng(seed)
    qh, qs = qh or H, qs or S
    f = lambda *sh: rng.standard_normal(sh).astype(np.float32)
    return dict(q=f(qs, T, qh, W) * 0.2, k=f(qs, T, qh, W) * 0.2, v=f(S, T, H, W),
                gate=-np.abs(f(S, T, H, gw)) * 0.05, beta=rng.uniform(0.1, 0.9, (S, T, H))
                .astype(np.float32), table=f(rows or S, H, W, W) * 0.1)


@pytest.fixture(scope="module")
def ex():
    with pb.ProjectionExecutor(0) as e:
        yield e


@pytest.mark.parametrize("W,H,T,S,gw,snaps", [(128, 4, 9, 3, 1, 3), (128, 2, 5, 2, 128, 6),
                                              (8, 3, 4, 4, 8, 1), (64, 4, 1, 2, 1, 2)])
def test_plain_op_with_rows_and_snapshots(ex, W, H, T, S, gw, snaps):
    a = inputs(W, H, T, S, gw, seed=W + T, rows=S + 2)
    a["rows"] = np.random.default_rng(S).permutation(S + 2)[:S].astype(np.int32)
    kw = dict(width=W, heads=H, tokens=T, sequences=S, q_heads=H, k_heads=H, q_sequences=S,
              k_sequences=S, gate_width=gw, snapshots=snaps, state_rows=S + 2)
    got, want = run(ex, kw, a)
    written = ~np.isnan(got)
    assert np.array_equal(got[written].view(np.uint32), want[written].view(np.uint32))
    assert written[:W * H * T * S].all()


def test_raw_gates_and_broadcast_heads(ex):
    W, H, T, S = 128, 4, 6, 4
    a = inputs(W, H, T, S, seed=11, qh=2, qs=2)
    a["bias"] = np.array([0.5, -1.0, 30.0, 0.0], np.float32)
    a["weight"] = np.array([-0.2, 0.0, -0.1, -1.0], np.float32)
    kw = dict(width=W, heads=H, tokens=T, sequences=S, q_heads=2, k_heads=2, q_sequences=2,
              k_sequences=2, gate_width=1, snapshots=1, raw=1, state_rows=S)
    got, want = run(ex, kw, a)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_replay_with_records(ex):
    W, H, T, S, snaps = 128, 2, 5, 3, 4
    rw = (2 * W + 1) * H
    a = inputs(W, H, T, S, seed=13)
    rng = np.random.default_rng(14)
    recs = np.zeros((S, 2, snaps - 1, rw), np.float32)
    recs[..., :H * W] = rng.standard_normal((S, 2, snaps - 1, H * W)) * 0.1   # deltas
    recs[..., H * W:2 * H * W] = rng.standard_normal((S, 2, snaps - 1, H * W)) * 0.1  # keys
    recs[..., 2 * H * W:] = rng.uniform(0.8, 1.0, (S, 2, snaps - 1, H))       # decays
    a["records"] = recs
    a["control"] = np.array([3, 1, 0, 0, 2, 1], np.int32)
    kw = dict(width=W, heads=H, tokens=T, sequences=S, q_heads=H, k_heads=H, q_sequences=S,
              k_sequences=S, gate_width=1, snapshots=snaps, replay=1, state_rows=S,
              record_banks=2, record_bank_elems=(snaps - 1) * rw, records_len=recs.size)
    got, want = run(ex, kw, a)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_invalid_rows_and_control_are_device_errors(ex):
    import torch
    W, H, T, S = 8, 1, 2, 2
    a = {k: torch.from_numpy(v).cuda() for k, v in inputs(W, H, T, S, seed=15).items()}
    kw = dict(width=W, heads=H, tokens=T, sequences=S, q_heads=H, k_heads=H, q_sequences=S,
              k_sequences=S, gate_width=1, snapshots=1, state_rows=S)
    op = mkop(pb.GdnOp, **kw)
    out = torch.zeros(pb.gdn_delta_values_outputs(op), device="cuda")
    ptrs = [a[n].data_ptr() for n in ("q", "k", "v", "gate", "beta", "table")]
    stream = torch.cuda.current_stream().cuda_stream
    rows = torch.tensor([1, 1], dtype=torch.int32, device="cuda")   # not distinct
    pb.gdn_delta_values_device(ex, op, *ptrs, out.data_ptr(), rows=rows.data_ptr(),
                               stream=stream)
    torch.cuda.synchronize()
    with pytest.raises(pb.PrismB200Error) as e:
        ex.sync()
    assert e.value.code == pb.E_INVALID
    ex.reset()
    rop = mkop(pb.GdnOp, **dict(kw, snapshots=2, replay=1, record_banks=2,
                                record_bank_elems=(2 * W + 1) * H, records_len=4 * (2 * W + 1)))
    recs = torch.zeros(4 * (2 * W + 1), device="cuda")
    ctl = torch.tensor([2, 0, 0, 0], dtype=torch.int32, device="cuda")  # count >= snapshots
    rout = torch.zeros(pb.gdn_delta_values_outputs(rop), device="cuda")
    pb.gdn_delta_values_device(ex, rop, *ptrs, rout.data_ptr(), records=recs.data_ptr(),
                               control=ctl.data_ptr(), stream=stream)
    torch.cuda.synchronize()
    with pytest.raises(pb.PrismB200Error) as e:
        ex.sync()
    assert e.value.code == pb.E_INVALID
    ex.reset()
    bad = mkop(pb.GdnOp, **dict(kw, snapshots=0))
    with pytest.raises(pb.PrismB200Error) as e:   # argument errors leave it open
        pb.gdn_delta_values_device(ex, bad, *ptrs, out.data_ptr(), stream=stream)
    assert e.value.code == pb.E_INVALID
    pb.gdn_delta_values_device(ex, op, *ptrs, out.data_ptr(), stream=stream)
    torch.cuda.synchronize()
    ex.sync()
