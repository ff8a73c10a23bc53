"""Sequence-sharded decode step (tt_engine_step_sharded_*) on one GPU.

Several ranks of one sharded step are emulated in one process on one GPU:
each rank is its own set of engines with the same configuration and the same
inputs, and the two all-gathers between the three calls are concatenations
in rank order (what an NCCL all-gather produces).  Nothing waits across
ranks, so this runs on any single GPU.  Checked against an unsharded set of
engines fed the same inputs:

* every rank's attention output is bit-identical to every other rank's, and
  within the attention tolerance of the unsharded engines' output;
* the score feedback every rank applies is bit-identical across ranks and
  within tolerance of the unsharded feedback;
* counters stay identical.

Tier routing depends on float scores, so, as in the engine parity tests, the
unsharded engines' scores are copied into every rank's engines after each step
(score sync); without that the sets could route one token differently after
accumulated rounding differences.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-4, 1e-5
COUNTERS = ["s_count", "rw_count", "rw_head_index", "hh_count", "wr_count", "pbs_count", "pbs_blocks_used",
            "total_processed_tokens", "total_evictions"]


@pytest.fixture(scope="module")
def C_():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tritiercache_b200 import _C
    return _C


def _close(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    err = (a - b).abs()
    return bool((err <= ATOL + RTOL * b.abs()).all()), float(err.max())


def _engines(C_, n, cfg):
    return [C_.TriTierCacheEngine(*cfg) for _ in range(n)]


@pytest.mark.parametrize("world,meta,nkv,layers", [(2, "fp16", 8, 2), (3, "fp16", 8, 2), (2, "fp32", 8, 1),
                                                   (4, "fp16", 4, 3)])
def test_sharded_step_matches_unsharded(C_, world, meta, nkv, layers):
    nq, hd, msl, S, R = 32, 128, 4096, 4, 256
    cfg = (nq, nkv, hd, msl, S, R, 0.05, 0.999, 32, 16, meta)
    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + world * 10 + layers)
    ref = _engines(C_, layers, cfg)
    ranks = [_engines(C_, layers, cfg) for _ in range(world)]
    q_len = 2100
    for li in range(layers):
        K = torch.randn(q_len, nkv, hd, device="cuda", generator=g)
        V = torch.randn(q_len, nkv, hd, device="cuda", generator=g)
        ref[li].prefill(K.data_ptr(), V.data_ptr(), q_len)
        for r in range(world):
            ranks[r][li].prefill(K.data_ptr(), V.data_ptr(), q_len)
    steps = [C_.ShardedStep(ranks[r], r, world) for r in range(world)]
    for step in range(48):
        Q = [torch.randn(nq * hd, device="cuda", generator=g) for _ in range(layers)]
        Kn = [torch.randn(nkv * hd, device="cuda", generator=g) for _ in range(layers)]
        Vn = [torch.randn(nkv * hd, device="cuda", generator=g) for _ in range(layers)]
        out_ref = [torch.empty(nq * hd, device="cuda") for _ in range(layers)]
        C_.engine_step_batched(ref, Q, Kn, Vn, out_ref)
        slot = steps[0].slot_cap()
        assert all(s.slot_cap() == slot for s in steps)
        xs = [torch.full((steps[0].xch_floats,), float("nan"), device="cuda") for _ in range(world)]
        for r in range(world):
            steps[r].begin(Q, Kn, Vn, xs[r], slot)
        xa = torch.cat(xs)
        outs = [[torch.full((nq * hd,), float("nan"), device="cuda") for _ in range(layers)] for _ in range(world)]
        ms = [torch.full((layers * slot,), float("nan"), device="cuda") for _ in range(world)]
        for r in range(world):
            steps[r].merge(xa, outs[r], ms[r], slot)
        ma = torch.cat(ms)
        for r in range(world):
            steps[r].end(ma, slot)
        torch.cuda.synchronize()
        for li in range(layers):
            for r in range(1, world):
                assert torch.equal(outs[r][li], outs[0][li]), (step, li, r, "outputs differ across ranks")
            ok, err = _close(outs[0][li], out_ref[li])
            assert ok, (step, li, "output vs unsharded", err)
            gs = [ranks[r][li].get_global_attn_scores() for r in range(world)]
            for r in range(1, world):
                assert torch.equal(gs[r], gs[0]), (step, li, r, "scores differ across ranks")
            ok, err = _close(gs[0], ref[li].get_global_attn_scores())
            assert ok, (step, li, "score feedback vs unsharded", err)
            for k in COUNTERS:
                want = getattr(ref[li], k)
                for r in range(world):
                    assert getattr(ranks[r][li], k) == want, (step, li, r, k)
            # score sync
            for r in range(world):
                ranks[r][li].get_global_attn_scores().copy_(ref[li].get_global_attn_scores())
                ranks[r][li].get_HH_scores().copy_(ref[li].get_HH_scores())
    from tritiercache_b200 import _lib
    import ctypes
    e = ctypes.c_int(-1)
    assert _lib.lib().tt_device_error(1, ctypes.byref(e)) == 0 and e.value == 0


def test_sharded_step_argument_errors(C_):
    from tritiercache_b200 import _lib
    cfg = (8, 2, 64, 1024, 4, 64, 0.1, 0.999, 16, 16, "fp16")
    eng = _engines(C_, 1, cfg)
    st = C_.ShardedStep(eng, 0, 2)
    slot = st.slot_cap()
    x = torch.empty(st.xch_floats, device="cuda")
    q = [torch.zeros(8 * 64, device="cuda")]
    kv = [torch.zeros(2 * 64, device="cuda")]
    with pytest.raises(ValueError):
        st.begin(q, kv, kv, x, slot - 1)          # slot below this step's need
    bad = C_.ShardedStep(eng, 2, 2)               # rank out of range
    with pytest.raises(ValueError):
        bad.begin(q, kv, kv, x, slot)
    # the exchange rows are read as (m, l) pairs: an xch_all that is not
    # 8-byte aligned is refused before any launch
    xa = torch.zeros(2 * st.xch_floats + 1, device="cuda")
    out = [torch.zeros(8 * 64, device="cuda")]
    mw = torch.zeros(slot, device="cuda")
    with pytest.raises(ValueError):
        st.merge(xa[1:], out, mw, slot)
