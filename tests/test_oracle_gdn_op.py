"""The oracle's batched gated-delta op with snapshots and replay (the
reference's CpuBackend::delta_values, src/backend/gdn.rs:24-300): an
independent numpy restatement of the recurrence, the snapshot slots, the
cache-row mapping, raw gates, per-column gates, and the replay property
(records of the last tokens, re-applied to the replay state, give the state
that running those tokens gives -- the reference's rollback contract)."""
import numpy as np
import pytest


def op(oracle, **kw):
    o = oracle.GdnOp()
    for f, _ in oracle.GdnOp._fields_:
        setattr(o, f, kw.get(f, 0))
    return o


def inputs(W, H, T, S, gw=1, seed=0, rows=None):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((S, T, H, W)).astype(np.float32) * 0.3
    k = rng.standard_normal((S, T, H, W)).astype(np.float32) * 0.3
    v = rng.standard_normal((S, T, H, W)).astype(np.float32)
    g = -np.abs(rng.standard_normal((S, T, H, gw))).astype(np.float32) * 0.1
    b = rng.uniform(0.1, 0.9, (S, T, H)).astype(np.float32)
    nrow = rows if rows is not None else S
    table = rng.standard_normal((nrow, H, W, W)).astype(np.float32) * 0.1
    return q, k, v, g, b, table


def numpy_op(q, k, v, g, b, table, rows, gw):
    S, T, H, W = v.shape
    st = table[rows].astype(np.float64).copy()
    out = np.zeros((S, T, H, W))
    states = []
    for t in range(T):
        dec = np.exp(g[:, t].astype(np.float64))  # (S, H, gw)
        st *= dec[:, :, None, :] if gw == W else dec[:, :, :, None]
        dk = np.einsum("shrc,shc->shr", st, k[:, t])
        delta = (v[:, t] - dk) * b[:, t, :, None]
        st += delta[..., None] * k[:, t][:, :, None, :]
        out[:, t] = np.einsum("shrc,shc->shr", st, q[:, t]) / np.sqrt(W)
        states.append(st.copy())
    return out, states


@pytest.mark.parametrize("gw", [1, 8])
def test_recurrence_and_snapshots(oracle, gw):
    W, H, T, S, snaps = 8, 2, 5, 3, 3
    q, k, v, g, b, table = inputs(W, H, T, S, gw, rows=5)
    rows = np.array([4, 0, 2], np.int32)
    o = op(oracle, width=W, heads=H, tokens=T, sequences=S, q_heads=H, k_heads=H,
           q_sequences=S, k_sequences=S, gate_width=gw, snapshots=snaps, state_rows=5)
    got = oracle.gdn_delta_values(o, q, k, v, g, b, table, rows=rows)
    want, states = numpy_op(q, k, v, g, b, table, rows, gw)
    attn = got[:S * T * H * W].reshape(S, T, H, W)
    assert np.allclose(attn, want, rtol=1e-5, atol=1e-6)
    snap = got[S * T * H * W:].reshape(snaps, S, H, W, W)
    for slot in range(snaps):
        assert np.allclose(snap[slot], states[T - 1 - slot], rtol=1e-5, atol=1e-6)
    bad = rows.copy()
    bad[1] = 4  # rows must be distinct
    with pytest.raises(oracle.OracleError):
        oracle.gdn_delta_values(o, q, k, v, g, b, table, rows=bad)


def test_raw_gates(oracle):
    W, H, T, S = 8, 2, 3, 1
    q, k, v, g, b, table = inputs(W, H, T, S, seed=3)
    bias = np.array([0.5, -1.0], np.float32)
    weight = np.array([-0.2, 0.0], np.float32)
    o = op(oracle, width=W, heads=H, tokens=T, sequences=S, q_heads=H, k_heads=H,
           q_sequences=S, k_sequences=S, gate_width=1, snapshots=1, raw=1, state_rows=1)
    got = oracle.gdn_delta_values(o, q, k, v, g, b, table, bias=bias, weight=weight)
    bs = 1 / (1 + np.exp(-b.astype(np.float64)))
    gg = g[..., 0].astype(np.float64) + bias
    gg = weight * np.where(gg > 20, gg, np.log1p(np.exp(gg)))
    gg[:, :, 1] = 0.0  # weight 0 with finite inputs: no decay
    want, _ = numpy_op(q, k, v, gg[..., None].astype(np.float32), bs.astype(np.float32),
                       table, np.array([0]), 1)
    assert np.allclose(got[:S * T * H * W].reshape(S, T, H, W), want, rtol=1e-5, atol=1e-6)


def test_replay_records_reproduce_the_rolled_state(oracle):
    W, H, T, S, snaps = 8, 2, 6, 2, 3
    q, k, v, g, b, table = inputs(W, H, T, S, seed=5)
    base = dict(width=W, heads=H, sequences=S, q_heads=H, k_heads=H, q_sequences=S,
                k_sequences=S, gate_width=1, state_rows=S)
    # the states after every token, from the plain op over all T tokens
    full = oracle.gdn_delta_values(op(oracle, tokens=T, snapshots=T, **base),
                                   q, k, v, g, b, table)
    states = full[S * T * H * W:].reshape(T, S, H, W, W)  # slot 0 = after token T-1
    # replay over the first 5 tokens: the state after token 2 and records of 3, 4
    r = op(oracle, tokens=5, snapshots=snaps, replay=1, record_banks=2,
           record_bank_elems=(snaps - 1) * (2 * W + 1) * H,
           records_len=S * 2 * (snaps - 1) * (2 * W + 1) * H, **base)
    zero_ctl = np.zeros(2 * S, np.int32)
    rec_buf = np.zeros(S * 2 * (snaps - 1) * (2 * W + 1) * H, np.float32)
    out = oracle.gdn_delta_values(r, q[:, :5], k[:, :5], v[:, :5], g[:, :5], b[:, :5], table,
                                  records=rec_buf, control=zero_ctl)
    attn_n = S * 5 * H * W
    bstate = out[attn_n:attn_n + S * H * W * W].reshape(S, H, W, W)
    assert np.array_equal(bstate, states[T - 1 - 2])
    recs = out[attn_n + S * H * W * W:].reshape(S, snaps - 1, -1)
    # bank 1 holds the two records; replaying them then token 5 gives the
    # plain op's state after token 5, bit for bit
    banks = np.zeros((S, 2, snaps - 1, (2 * W + 1) * H), np.float32)
    banks[:, 1] = recs
    ctl = np.array([2, 1] * S, np.int32)
    r1 = op(oracle, tokens=1, snapshots=snaps, replay=1, record_banks=2,
            record_bank_elems=(snaps - 1) * (2 * W + 1) * H, records_len=banks.size, **base)
    out1 = oracle.gdn_delta_values(r1, q[:, 5:], k[:, 5:], v[:, 5:], g[:, 5:], b[:, 5:],
                                   bstate, records=banks, control=ctl)
    st1 = out1[S * H * W:S * H * W + S * H * W * W].reshape(S, H, W, W)
    assert np.array_equal(st1, states[0])
    assert np.array_equal(out1[:S * H * W], full[:S * T * H * W].reshape(S, T, H, W)[:, 5].reshape(-1))
    bad = np.array([3, 0] * S, np.int32)  # count must be below snapshots
    with pytest.raises(oracle.OracleError):
        oracle.gdn_delta_values(r1, q[:, 5:], k[:, 5:], v[:, 5:], g[:, 5:], b[:, 5:], bstate,
                                records=banks, control=bad)
