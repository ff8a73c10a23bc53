"""Sequence-sharded decode step across GPUs: one process per GPU, NCCL.

Each rank holds the same engines, gets the same inputs and runs
a ShardedEngineStep (begin / all-gather of the exchange rows / merge /
all-gather of the routing rows, and the score all-reduce before threshold
steps; or, with the peer exchange, begin / merge with the rows written into
every rank's memory over NVLink); it also keeps an unsharded copy of the
engines on its own GPU.  No
score is copied from the unsharded copy.  Checked every step: the output is
bit-identical on all ranks and within the attention tolerance of the
unsharded copy; every token's score, assembled from the ranks' owned scores
(an all-reduce of the packed scores), within tolerance; counters and
heavy-hitter / packed ids equal.  Runs only where at least two GPUs are
visible, with NVLS off; processes are bounded by a short process-group
timeout and a join timeout.
"""
import multiprocessing as pymp
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-4, 1e-5


def _worker(rank, world, port, exchange, q):
    try:
        import os
        from datetime import timedelta
        import torch.distributed as dist
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
        from tritiercache_b200 import _C
        nq, nkv, hd, layers = 32, 8, 128, 2
        cfg = (nq, nkv, hd, 4096, 4, 256, 0.005, 0.999, 32, 16, "fp16")  # 21 heavy-hitter slots: replacements
        ref = [_C.TriTierCacheEngine(*cfg) for _ in range(layers)]
        shd = [_C.TriTierCacheEngine(*cfg) for _ in range(layers)]
        g = torch.Generator(device="cuda")
        g.manual_seed(77)
        for li in range(layers):
            K = torch.randn(2500, nkv, hd, device="cuda", generator=g)
            V = torch.randn(2500, nkv, hd, device="cuda", generator=g)
            ref[li].prefill(K.data_ptr(), V.data_ptr(), 2500)
            shd[li].prefill(K.data_ptr(), V.data_ptr(), 2500)
        worst = 0.0
        drv = _C.ShardedEngineStep(shd, exchange=exchange)
        failure = None

        def check(step, o_ref, o_shd):
            # the collectives first (every rank makes them every step), then the checks
            allo = [torch.empty(layers * nq * hd, device="cuda") for _ in range(world)]
            dist.all_gather(allo, torch.cat(o_shd))
            buf = torch.zeros(drv.step.scores_floats(), device="cuda")
            drv.step.scores_pack(buf)
            dist.all_reduce(buf)
            for r in range(1, world):
                assert torch.equal(allo[r], allo[0]), (step, "outputs differ across ranks")
            off = 0
            w = 0.0
            for li in range(layers):
                err = (o_shd[li].double() - o_ref[li].double()).abs()
                assert bool((err <= ATOL + RTOL * o_ref[li].double().abs()).all()), (step, li, float(err.max()))
                w = max(w, float(err.max()))
                gs = buf[off:off + ref[li].max_seq_len].double()
                gr = ref[li].get_global_attn_scores().double()
                assert bool(((gs - gr).abs() <= 1e-6 + 1e-4 * gr.abs()).all()), (step, li, "scores")
                off += ref[li].max_seq_len
                c, cs = ref[li].counters(), shd[li].counters()  # shd raises if a bounded wait ran out
                for k in ("total_processed_tokens", "hh_count", "pbs_blocks_used", "wr_count", "rw_head_index",
                          "last_calc_pos", "total_evictions"):
                    assert cs[k] == c[k], (step, li, k)
                assert torch.equal(shd[li].get_HH_token_ids()[:c["hh_count"]],
                                   ref[li].get_HH_token_ids()[:c["hh_count"]])
                nt = c["pbs_blocks_used"] * 16
                assert torch.equal(shd[li].get_PBS_token_ids()[:nt], ref[li].get_PBS_token_ids()[:nt])
            return w

        # Every rank runs every step whatever a check finds (a failure is kept
        # for the end): with the peer exchange no rank may stop, and free the
        # memory the others write into, while they still run steps.
        for step in range(48):
            Q = [torch.randn(nq * hd, device="cuda", generator=g) for _ in range(layers)]
            Kn = [torch.randn(nkv * hd, device="cuda", generator=g) for _ in range(layers)]
            Vn = [torch.randn(nkv * hd, device="cuda", generator=g) for _ in range(layers)]
            o_ref = [torch.empty(nq * hd, device="cuda") for _ in range(layers)]
            o_shd = [torch.full((nq * hd,), float("nan"), device="cuda") for _ in range(layers)]
            _C.engine_step_batched(ref, Q, Kn, Vn, o_ref)
            drv(shd, Q, Kn, Vn, o_shd)
            try:
                worst = max(worst, check(step, o_ref, o_shd))
            except Exception as exc:
                if failure is None:
                    failure = repr(exc)
        syncs = drv.syncs
        drv.close()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        if failure is not None:
            raise AssertionError(failure)
        assert syncs >= 1, "no score synchronisation ran"
        q.put((rank, None, worst))
    except Exception as exc:
        q.put((rank, repr(exc), None))


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_sharded_step_over_nccl(exchange):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    world = 2
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = pymp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            rank, err, worst = q.get(timeout=300)
            res[rank] = (err, worst)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert res[r][0] is None, (r, res[r][0])
