"""The exchange protocol of the sequence-sharded decode step, on CPU ranks.

tt_engine_step_sharded_* (include/tritier_b200.h) splits every engine's
tokens over `world` ranks (dense positions [D*r/w, D*(r+1)/w), packed blocks
[B*r/w, B*(r+1)/w)), has each rank reduce its share to one (max, sum,
weighted sum) row per query head, all-gathers those rows in rank order, merges
them in that order, and all-gathers each rank's mean attention weights in
[rank][slot] layout.  This test runs that protocol with world = 2 and 3 gloo
ranks (separate processes, 127.0.0.1) in float64 numpy on oracle-dequantized
tiers, and checks the merged output and the reassembled mean weights against
the oracle's unsharded fused attention.  The CUDA kernels of the same protocol
are checked on a GPU by tests/test_gpu_sharded.py.
"""
import multiprocessing as pymp
import socket

import numpy as np
import pytest

ATOL, RTOL = 1e-4, 1e-5
NQ, NKV, HD, GRP = 8, 2, 64, 16


def _shard_range(D, nblk, grp, rank, world):
    return (D * rank // world, D * (rank + 1) // world, nblk * rank // world * grp, nblk * (rank + 1) // world * grp)


def _inputs(seed, dc, nb):
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((NQ, HD)).astype(np.float32)
    dK = rng.standard_normal((dc, NKV, HD)).astype(np.float32)
    dV = rng.standard_normal((dc, NKV, HD)).astype(np.float32)
    ntok = nb * GRP
    Kf = rng.standard_normal((ntok, NKV, HD)).astype(np.float32)
    Vf = rng.standard_normal((ntok, NKV, HD)).astype(np.float32)
    kp = np.zeros((nb * GRP // 16, NKV, HD), np.int32)
    ks = np.zeros((nb, NKV, HD), np.uint16)
    kz = np.zeros((nb, NKV, HD), np.uint16)
    vp = np.zeros((ntok, NKV, HD // 16), np.int32)
    vs = np.zeros((ntok, NKV), np.uint16)
    vz = np.zeros((ntok, NKV), np.uint16)
    for b in range(nb):
        O.quantize_k_block(Kf[b * GRP:(b + 1) * GRP], kp[b * GRP // 16:(b + 1) * GRP // 16], ks[b], kz[b], NKV, HD, GRP)
        O.quantize_v_block(Vf[b * GRP:(b + 1) * GRP], vp[b * GRP:(b + 1) * GRP], vs[b * GRP:(b + 1) * GRP],
                           vz[b * GRP:(b + 1) * GRP], NKV, HD, GRP)
    ids = np.arange(ntok, dtype=np.int64) + 1000
    ids[3::7] = -1
    Kd = np.zeros((ntok, NKV, HD), np.float32)
    Vd = np.zeros((ntok, NKV, HD), np.float32)
    O.dequantize_k(kp, ks, kz, Kd, nb, NKV, HD, GRP)
    O.dequantize_v(vp, vs, vz, Vd, ntok, NKV, HD)
    return dict(Q=Q, dK=dK, dV=dV, kp=kp, ks=ks, kz=kz, vp=vp, vs=vs, vz=vz, ids=ids, Kd=Kd, Vd=Vd)


def _rank_main(rank, world, port, dc, nb, q):
    try:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        d = _inputs(7, dc, nb)
        G = NQ // NKV
        K = np.concatenate([d["dK"], d["Kd"]]).astype(np.float64)
        V = np.concatenate([d["dV"], d["Vd"]]).astype(np.float64)
        live = np.concatenate([np.ones(dc, bool), d["ids"] != -1])
        dlo, dhi, plo, phi = _shard_range(dc, nb, GRP, rank, world)
        pos = np.concatenate([np.arange(dlo, dhi), dc + np.arange(plo, phi)]).astype(np.int64)
        # local (m, l, acc) rows
        rows = np.zeros((NQ, HD + 2))
        logits = np.full((NQ, len(pos)), -np.inf)
        for h in range(NQ):
            kh = h // G
            s = K[pos, kh, :] @ d["Q"][h].astype(np.float64) / np.sqrt(HD)
            s[~live[pos]] = -np.inf
            logits[h] = s
            m = s.max() if len(s) and np.isfinite(s).any() else -np.inf
            w = np.exp(s - m) if np.isfinite(m) else np.zeros_like(s)
            rows[h, 0], rows[h, 1] = m, w.sum()
            rows[h, 2:] = w @ V[pos, kh, :] if len(pos) else 0.0
        send = torch.from_numpy(rows.ravel().copy())
        recv = [torch.empty_like(send) for _ in range(world)]
        dist.all_gather(recv, send)
        allrows = torch.stack(recv).numpy().reshape(world, NQ, HD + 2)
        # merge in rank order
        out = np.zeros((NQ, HD))
        M = allrows[:, :, 0].max(axis=0)
        L = np.zeros(NQ)
        for p in range(world):
            f = np.where(np.isfinite(allrows[p, :, 0]), np.exp(allrows[p, :, 0] - M), 0.0)
            L += allrows[p, :, 1] * f
            out += allrows[p, :, 2:] * f[:, None]
        out /= np.where(L > 0, L, 1.0)[:, None]
        # this rank's mean weights, [rank][slot] layout
        slot = -(-dc // world) + -(-nb // world) * GRP
        mw = np.zeros(slot)
        mw[:len(pos)] = (np.exp(logits - M[:, None]) / L[:, None]).sum(axis=0) / NQ
        mrecv = [torch.empty(slot, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(mrecv, torch.from_numpy(mw))
        full_mw = np.zeros(dc + nb * GRP)
        for p in range(world):
            a, b, c, e = _shard_range(dc, nb, GRP, p, world)
            pp = np.concatenate([np.arange(a, b), dc + np.arange(c, e)])
            full_mw[pp] = mrecv[p].numpy()[:len(pp)]
        dist.destroy_process_group()
        q.put((rank, out, full_mw, None))
    except Exception as exc:  # reported to the parent
        q.put((rank, None, None, repr(exc)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("world,dc,nb", [(2, 37, 9), (3, 20, 4), (2, 5, 1)])
def test_sharded_exchange_protocol_matches_unsharded_attention(world, dc, nb):
    from oracle import oracle as O
    ctx = pymp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, dc, nb, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, out, mw, err = q.get(timeout=120)
            assert err is None, (rank, err)
            results[rank] = (out, mw)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in range(1, world):
        assert np.array_equal(results[r][0], results[0][0]), "ranks merged to different outputs"
    d = _inputs(7, dc, nb)
    out = np.zeros((NQ, HD), np.float32)
    mw = np.zeros(dc + nb * GRP, np.float32)
    O.fused_attention_decode(d["Q"], d["dK"], d["dV"], dc, d["kp"], d["ks"], d["kz"], d["vp"], d["vs"], d["vz"],
                             d["ids"], nb, NQ, NKV, HD, out, mw, GRP)
    got_out, got_mw = results[0]
    assert np.all(np.abs(got_out - out) <= ATOL + RTOL * np.abs(out)), np.abs(got_out - out).max()
    assert np.all(np.abs(got_mw - mw) <= ATOL + RTOL * np.abs(mw)), np.abs(got_mw - mw).max()
