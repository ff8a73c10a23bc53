"""Sequence-sharded decode step (tt_engine_step_sharded_*) on one GPU.

Several ranks of one sharded step are emulated in one process on one GPU:
each rank is its own set of engines with the same configuration and the same
inputs; the all-gathers are concatenations in rank order (what an NCCL
all-gather produces) and the score all-reduce is a sum of the ranks' packed
buffers.  Nothing waits across ranks, so this runs on any single GPU.

Each rank attends and scores only the tokens it owns; routing decisions come
from the ranks' routing rows, and the scores are synchronised only before the
steps that recompute the heavy-hitter threshold.  Checked every step against
an unsharded set of engines fed the same inputs, with no score copied from
them into the ranks:

* every rank's attention output is bit-identical to every other rank's, and
  within the attention tolerance of the unsharded output;
* every token's score, assembled from the ranks' owned scores, is within
  tolerance of the unsharded engine's score;
* counters, heavy-hitter ids, waiting-room ids, packed ids and packed words
  are identical to the unsharded engines' on every rank (routing follows the
  unsharded engine token by token).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-4, 1e-5
S_ATOL, S_RTOL = 1e-6, 1e-4  # accumulated scores: sums of about 50 decayed weights
COUNTERS = ["s_count", "rw_count", "rw_head_index", "hh_count", "wr_count", "pbs_count", "pbs_blocks_used",
            "total_processed_tokens", "total_evictions", "last_calc_pos"]


@pytest.fixture(scope="module")
def C_():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tritiercache_b200 import _C
    return _C


def _close(a, b, atol=ATOL, rtol=RTOL):
    a = a.double().cpu()
    b = b.double().cpu()
    err = (a - b).abs()
    return bool((err <= atol + rtol * b.abs()).all()), float(err.max())


def _engines(C_, n, cfg):
    return [C_.TriTierCacheEngine(*cfg) for _ in range(n)]


def _state(e):
    c = e.counters()
    nb = c["pbs_blocks_used"]
    return (e.get_HH_token_ids()[:c["hh_count"]].cpu(), e.get_WR_token_ids()[:c["wr_count"]].cpu(),
            e.get_PBS_token_ids()[:nb * 16].cpu(), e.get_PBS_K_Packed()[:nb].cpu(), e.get_PBS_V_Packed()[:nb * 16].cpu())


def run_emulated(C_, world, cfg, layers, steps, q_len, seed):
    nq, nkv, hd = cfg[0], cfg[1], cfg[2]
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    ref = _engines(C_, layers, cfg)
    ranks = [_engines(C_, layers, cfg) for _ in range(world)]
    for li in range(layers):
        K = torch.randn(q_len, nkv, hd, device="cuda", generator=g)
        V = torch.randn(q_len, nkv, hd, device="cuda", generator=g)
        ref[li].prefill(K.data_ptr(), V.data_ptr(), q_len)
        for r in range(world):
            ranks[r][li].prefill(K.data_ptr(), V.data_ptr(), q_len)
    st = [C_.ShardedStep(ranks[r], r, world) for r in range(world)]
    nf = st[0].scores_floats()
    route = None
    syncs = replaced = 0
    for step in range(steps):
        Q = [torch.randn(nq * hd, device="cuda", generator=g) for _ in range(layers)]
        Kn = [torch.randn(nkv * hd, device="cuda", generator=g) for _ in range(layers)]
        Vn = [torch.randn(nkv * hd, device="cuda", generator=g) for _ in range(layers)]
        out_ref = [torch.empty(nq * hd, device="cuda") for _ in range(layers)]
        hh_before = [e.hh_count for e in ref]
        ev_before = [e.total_evictions for e in ref]
        C_.engine_step_batched(ref, Q, Kn, Vn, out_ref)
        need = [s.sync_needed() for s in st]
        assert all(x == need[0] for x in need)
        if world > 1 and need[0]:
            bufs = [torch.full((nf,), float("nan"), device="cuda") for _ in range(world)]
            for r in range(world):
                st[r].scores_pack(bufs[r])
            total = torch.stack(bufs).sum(0)
            for r in range(world):
                st[r].scores_unpack(total)
            route = None
            syncs += 1
        xs = [torch.full((st[0].xch_floats,), float("nan"), device="cuda") for _ in range(world)]
        for r in range(world):
            st[r].begin(Q, Kn, Vn, xs[r], route)
        xa = torch.cat(xs)
        outs = [[torch.full((nq * hd,), float("nan"), device="cuda") for _ in range(layers)] for _ in range(world)]
        rs = [torch.full((st[0].route_floats,), float("nan"), device="cuda") for _ in range(world)]
        for r in range(world):
            st[r].merge(xa, outs[r], rs[r])
        route = torch.cat(rs)
        torch.cuda.synchronize()
        bufs = [torch.zeros(nf, device="cuda") for _ in range(world)]
        for r in range(world):
            st[r].scores_pack(bufs[r])
        assembled = torch.stack(bufs).sum(0)
        off = 0
        for li in range(layers):
            for r in range(1, world):
                assert torch.equal(outs[r][li], outs[0][li]), (step, li, r, "outputs differ across ranks")
            ok, err = _close(outs[0][li], out_ref[li])
            assert ok, (step, li, "output vs unsharded", err)
            msl = ref[li].max_seq_len
            ok, err = _close(assembled[off:off + msl], ref[li].get_global_attn_scores(), S_ATOL, S_RTOL)
            assert ok, (step, li, "assembled scores vs unsharded", err)
            off += msl
            want = ref[li].counters()
            sref = _state(ref[li])
            for r in range(world):
                got = ranks[r][li].counters()
                for k in COUNTERS:
                    assert got[k] == want[k], (step, li, r, k, got[k], want[k])
                for a, b in zip(_state(ranks[r][li]), sref):
                    assert torch.equal(a, b), (step, li, r, "tier contents differ")
            if ref[li].total_evictions > ev_before[li] and ref[li].hh_count == hh_before[li] == ref[li].max_hh:
                replaced += 1
    from tritiercache_b200 import _lib
    import ctypes
    e = ctypes.c_int(-1)
    assert _lib.lib().tt_device_error(1, ctypes.byref(e)) == 0 and e.value == 0
    return syncs, replaced


@pytest.mark.parametrize("world,meta,nkv,layers,h_ratio", [(2, "fp16", 8, 2, 0.05), (3, "fp16", 8, 2, 0.005),
                                                           (2, "fp32", 8, 1, 0.005), (4, "fp16", 4, 3, 0.05),
                                                           (1, "fp16", 8, 1, 0.005)])
def test_sharded_step_matches_unsharded(C_, world, meta, nkv, layers, h_ratio):
    cfg = (32, nkv, 128, 4096, 4, 256, h_ratio, 0.999, 32, 16, meta)
    syncs, replaced = run_emulated(C_, world, cfg, layers, steps=72, q_len=2100, seed=1000 + world * 10 + layers)
    if world > 1:
        assert syncs >= 2  # the first step and every update_interval tokens after it
    if h_ratio < 0.01:
        assert replaced > 0  # heavy-hitter replacement routed from the ranks' minima


def test_sharded_step_argument_errors(C_):
    cfg = (8, 2, 64, 1024, 4, 64, 0.1, 0.999, 16, 16, "fp16")
    eng = _engines(C_, 1, cfg)
    K = torch.randn(300, 2, 64, device="cuda")
    eng[0].prefill(K.data_ptr(), K.data_ptr(), 300)
    st = C_.ShardedStep(eng, 0, 2)
    x = torch.empty(st.xch_floats, device="cuda")
    q = [torch.zeros(8 * 64, device="cuda")]
    kv = [torch.zeros(2 * 64, device="cuda")]
    ra = torch.zeros(2 * st.route_floats, device="cuda")
    assert st.sync_needed()  # the first eviction computes the threshold
    with pytest.raises(ValueError):
        st.begin(q, kv, kv, x, ra)                # routing rows on a threshold step
    bad = C_.ShardedStep(eng, 2, 2)               # rank out of range
    with pytest.raises(ValueError):
        bad.begin(q, kv, kv, x, None)
    with pytest.raises(ValueError):
        st.begin(q, kv, kv, x, ra[1:])            # routing rows not 16-byte aligned
    # the exchange rows are read as (m, l) pairs: an xch_all that is not
    # 8-byte aligned is refused before any launch
    xa = torch.zeros(2 * st.xch_floats + 1, device="cuda")
    out = [torch.zeros(8 * 64, device="cuda")]
    rs = torch.zeros(st.route_floats, device="cuda")
    with pytest.raises(ValueError):
        st.merge(xa[1:], out, rs)
    with pytest.raises(ValueError):
        st.merge(xa[:-1], out, rs[1:])            # routing rows not 16-byte aligned
    assert eng[0].total_processed_tokens == 300  # nothing ran


def test_sharded_step_many_chunks(C_):
    """One layer at 60k tokens over 2 ranks: a rank's launch has more than 128
    chunk slots (56 dense + 117 packed), so its rows come from the separate
    local-merge kernel instead of the attention kernels' last CTA."""
    cfg = (32, 8, 128, 65536, 4, 256, 0.05, 0.999, 32, 16, "fp16")
    syncs, _ = run_emulated(C_, 2, cfg, 1, steps=6, q_len=60000, seed=4242)
    assert syncs >= 1
