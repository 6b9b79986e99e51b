"""GDN prefill through the no-allocation entry point.

prism_b200_gdn_prefill_device_noalloc must give what
prism_b200_gdn_prefill_device gives on the same inputs, bit for bit (the same
kernels run over the same scratch layout), on consecutive calls
that reuse its fixed scratch, must refuse a call whose scratch would not fit
before anything is enqueued, and must leave a fresh executor's device free
memory unchanged.  The file name sorts last so that the test
also runs after every other test in one process.
"""
import numpy as np
import pytest
import torch

import prism_b200 as pb

pytestmark = pytest.mark.gpu

D = 128
CHUNK_SCRATCH_BYTES = (2 * 64 * 68 + 128) * 4   # M, CQ in 68-float rows, cum, P[C-1]


def inputs(batch, T, heads, key_heads, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((batch, T, key_heads, D)).astype(np.float32)
    k = rng.standard_normal((batch, T, key_heads, D)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((batch, T, heads, D)).astype(np.float32)
    decay = np.exp(-np.log1p(np.exp(rng.standard_normal((batch, T, heads))))).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((batch, T, heads))))).astype(np.float32)
    return [torch.from_numpy(a).cuda() for a in (q, k, v, decay, beta)]


def same(got, ref):
    return torch.equal(got.view(torch.int32), ref.view(torch.int32))


@pytest.fixture(scope="module")
def ex():
    e = pb.ProjectionExecutor(0)
    yield e
    e.close()


def run(ex, fn, batch, T, heads, key_heads, chunk, state, ins):
    q, k, v, decay, beta = ins
    out = torch.zeros((batch, T, heads, D), device="cuda")
    fn(ex, batch, T, heads, key_heads, chunk, state.data_ptr(), q.data_ptr(), k.data_ptr(),
       v.data_ptr(), decay.data_ptr(), beta.data_ptr(), out.data_ptr())
    ex.sync()
    torch.cuda.synchronize()
    return out


def test_consecutive_calls_match_allocating_entry_point(ex):
    # two consecutive calls of different geometry: the second reuses the
    # fixed scratch the first left behind and continues from its state
    calls = [(2, 200, 4, 4, 64, 11), (2, 300, 4, 2, 37, 12)]
    g = torch.Generator().manual_seed(5)
    s_ref = (torch.randn((2, 4, D, D), generator=g) * 0.1).cuda()
    s_fix = s_ref.clone()
    for batch, T, heads, key_heads, chunk, seed in calls:
        ins = inputs(batch, T, heads, key_heads, seed)
        o_ref = run(ex, pb.gdn_prefill_device, batch, T, heads, key_heads, chunk, s_ref, ins)
        o_fix = run(ex, pb.gdn_prefill_device_noalloc, batch, T, heads, key_heads, chunk, s_fix,
                    ins)
        assert torch.isfinite(o_fix).all()
        assert same(o_fix, o_ref), (T, chunk)
        assert same(s_fix, s_ref), (T, chunk)


def test_largest_fitting_call_and_refusal_beyond(ex):
    units = pb.GDN_STATIC_SCRATCH_BYTES // CHUNK_SCRATCH_BYTES   # (sequence, head, chunk) units
    assert units == 1009
    # exactly at the limit: one 64-token chunk for `units` heads
    heads, T = units, 64
    ins = inputs(1, T, heads, 1, 21)
    s_ref = (torch.randn((1, heads, D, D), generator=torch.Generator().manual_seed(6)) * 0.1).cuda()
    s_fix = s_ref.clone()
    o_ref = run(ex, pb.gdn_prefill_device, 1, T, heads, 1, 64, s_ref, ins)
    o_fix = run(ex, pb.gdn_prefill_device_noalloc, 1, T, heads, 1, 64, s_fix, ins)
    assert same(o_fix, o_ref) and same(s_fix, s_ref)
    del ins, s_ref, o_ref
    # one head more does not fit: refused on the host, nothing enqueued, the
    # buffers are sized for the call all the same
    heads += 1
    ins = inputs(1, T, heads, 1, 22)
    state = torch.zeros((1, heads, D, D), device="cuda")
    before = state.clone()
    with pytest.raises(pb.PrismB200Error) as err:
        run(ex, pb.gdn_prefill_device_noalloc, 1, T, heads, 1, 64, state, ins)
    assert err.value.code == pb.E_INVALID
    assert "scratch" in str(err.value)
    assert torch.equal(state, before)
    # the executor stays usable after the refusal
    ins = inputs(2, 100, 4, 4, 23)
    s_ref = torch.zeros((2, 4, D, D), device="cuda")
    s_fix = s_ref.clone()
    o_ref = run(ex, pb.gdn_prefill_device, 2, 100, 4, 4, 64, s_ref, ins)
    o_fix = run(ex, pb.gdn_prefill_device_noalloc, 2, 100, 4, 4, 64, s_fix, ins)
    assert same(o_fix, o_ref) and same(s_fix, s_ref)


def test_fresh_executor_allocates_no_device_memory(ex):
    """On a fresh executor the no-allocation prefill leaves the device's free
    memory unchanged, while the allocating entry point on the same executor
    then grows its scratch by at least the same chunk scratch -- the control
    showing that the measure sees an allocation of this size."""
    heads, T = 1009, 64                      # the largest fitting call
    ins = inputs(1, T, heads, 1, 31)
    state = torch.zeros((1, heads, D, D), device="cuda")
    out = torch.zeros((1, T, heads, D), device="cuda")
    q, k, v, decay, beta = ins

    def call(e, fn):
        fn(e, 1, T, heads, 1, 64, state.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
           decay.data_ptr(), beta.data_ptr(), out.data_ptr())
        e.sync()
        torch.cuda.synchronize()

    # the module holding the fixed scratch and both kernels are loaded on
    # this device by a first call from another executor
    call(ex, pb.gdn_prefill_device_noalloc)
    fresh = pb.ProjectionExecutor(0)
    try:
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        call(fresh, pb.gdn_prefill_device_noalloc)
        call(fresh, pb.gdn_prefill_device_noalloc)
        free1 = torch.cuda.mem_get_info()[0]
        assert free1 == free0, free0 - free1
        call(fresh, pb.gdn_prefill_device)
        free2 = torch.cuda.mem_get_info()[0]
        assert free1 - free2 >= heads * CHUNK_SCRATCH_BYTES, free1 - free2
    finally:
        fresh.close()
