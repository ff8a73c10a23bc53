"""The protocol of the sequence-sharded decode step, on CPU ranks (gloo).

tt_engine_step_sharded_* (include/tritier_b200.h) gives every token one owner
rank while it stays in a tier slot: sink, heavy-hitter and ring slot j belong
to rank j % world, packed tokens to ranks in 256-token granules round-robin.
A rank attends and scores only what it owns; the next step's routing comes
from the ranks' routing rows (the score of the token to evict, from the owner
of its ring slot, and each rank's smallest heavy-hitter (score, slot)); the
maintenance writes the routed scores on every rank; before a step that
recomputes the heavy-hitter threshold an all-reduce of the owner-masked
scores makes every score current everywhere.  The CUDA kernels of that
protocol are checked on a GPU by tests/test_gpu_sharded.py.

Here world = 2 and 3 gloo ranks (separate processes, 127.0.0.1) run the
protocol's bookkeeping beside the oracle engine (the reference's algorithm,
unsharded), which every rank steps with the same inputs:

* the exchange rows of each rank's owned positions, all-gathered and merged
  in rank order, reproduce the oracle's attention output (float64 model);
* each rank keeps its own copy of the scores, updated only for the tokens it
  owns (with the oracle's post-step values) and by the maintenance writes;
  after every step the all-reduced owner-masked copies equal the oracle's
  scores bit for bit;
* before every eviction the routing rows give exactly the oracle's inputs to
  its routing decision: the evicted token's score and the strict argmin of
  the heavy-hitter scores.

Two more tests run ShardedEngineStep (the Python driver of the sharded step)
on gloo ranks with a recording stand-in for the device calls and check its
sequence of calls and collectives: with the NCCL-style exchange (two
all-gathers per step) and with the peer exchange (the IPC handles gathered
once, then no collective per step but the score all-reduce).
"""
import multiprocessing as pymp
import socket

import numpy as np
import pytest

NQ, NKV, HD, GRP = 8, 2, 64, 16
MSL, S, R, H_RATIO, DECAY, UI = 1024, 4, 64, 0.02, 0.999, 16
PRE, STEPS = 600, 90
GRAN = 256
ATOL, RTOL = 1e-4, 1e-5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run_ranks(target, world, args, timeout=240):
    ctx = pymp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, res, err = q.get(timeout=timeout)
            assert err is None, (rank, err)
            results[rank] = res
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


def _owned_positions(c, rank, world):
    """(tier, slot) of every position rank owns, in the CUDA kernels' local order:
    sinks, heavy hitters, ring slots, then packed tokens by granule."""
    out = [(0, j) for j in range(rank, c["s_count"], world)]
    out += [(1, j) for j in range(rank, c["hh_count"], world)]
    out += [(2, j) for j in range(rank, c["rw_count"], world)]
    P = c["pbs_blocks_used"] * GRP
    out += [(3, p) for p in range(P) if (p // GRAN) % world == rank]
    return out


def _ring_id(c, slot):
    q = (slot - c["rw_head_index"]) % R
    return c["total_processed_tokens"] - c["rw_count"] + q


def _token_id(eng, c, tier, slot):
    if tier == 0:
        return slot
    if tier == 1:
        return int(eng.buffer("HH_token_ids")[slot])
    if tier == 2:
        return _ring_id(c, slot)
    return int(eng.buffer("PBS_token_ids")[slot])


def _pack(eng, c, g_r, rank, world):
    """Owner-masked scores (k_scores_pack): owned slots, the waiting room on rank 0."""
    buf = np.zeros(MSL, np.float32)
    for tier, slot in _owned_positions(c, rank, world):
        i = _token_id(eng, c, tier, slot)
        if 0 <= i < MSL:
            buf[i] = g_r[i]
    if rank == 0:
        for i in eng.buffer("WR_token_ids")[:c["wr_count"]]:
            if 0 <= i < MSL:
                buf[i] = g_r[i]
    return buf


def _dense_rows(eng, c, slots):
    """K, V float64 rows of dense (tier, slot) positions."""
    K = {0: eng.buffer("S_K"), 1: eng.buffer("HH_K"), 2: eng.buffer("RW_K")}
    V = {0: eng.buffer("S_V"), 1: eng.buffer("HH_V"), 2: eng.buffer("RW_V")}
    kv = NKV * HD
    k = np.array([K[t][s * kv:(s + 1) * kv] for t, s in slots], np.float64).reshape(len(slots), NKV, HD)
    v = np.array([V[t][s * kv:(s + 1) * kv] for t, s in slots], np.float64).reshape(len(slots), NKV, HD)
    return k, v


def _packed_rows(eng, c):
    """Dequantized K, V of the packed tier (oracle dequantization)."""
    from oracle import oracle as O
    nb = c["pbs_blocks_used"]
    P = nb * GRP
    Kd = np.zeros((P, NKV, HD), np.float32)
    Vd = np.zeros((P, NKV, HD), np.float32)
    if nb:
        O.dequantize_k(eng.buffer("PBS_K_Packed").reshape(-1, NKV, HD)[:nb], eng.buffer("PBS_K_Scales").reshape(-1, NKV, HD)[:nb],
                       eng.buffer("PBS_K_Zeroes").reshape(-1, NKV, HD)[:nb], Kd, nb, NKV, HD, GRP)
        O.dequantize_v(eng.buffer("PBS_V_Packed").reshape(-1, NKV, HD // 16)[:P], eng.buffer("PBS_V_Scales").reshape(-1, NKV)[:P],
                       eng.buffer("PBS_V_Zeroes").reshape(-1, NKV)[:P], Vd, P, NKV, HD)
    return Kd.astype(np.float64), Vd.astype(np.float64)


def _protocol_rank(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        from oracle import oracle as O
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        rng = np.random.default_rng(5)  # the same inputs on every rank
        eng = O.Engine(NQ, NKV, HD, MSL, S, R, H_RATIO, DECAY, UI, GRP, "fp16")
        K = rng.standard_normal((PRE, NKV, HD)).astype(np.float32)
        V = rng.standard_normal((PRE, NKV, HD)).astype(np.float32)
        eng.prefill(K, V, PRE)
        max_hh = int(np.ceil(MSL * H_RATIO))
        g_r = eng.buffer("global_attn_scores").copy()  # current everywhere after prefill
        hs_r = eng.buffer("HH_scores").copy()
        rows = None
        stats = dict(syncs=0, routed=0, replaced=0, worst_out=0.0)
        G = NQ // NKV
        for step in range(STEPS):
            c = eng.counters()
            total = c["total_processed_tokens"]
            evicts = c["s_count"] == S and c["rw_count"] == R
            recompute = evicts and total - R > S and (c["last_calc_pos"] == -1 or total - c["last_calc_pos"] >= UI)
            g_true = eng.buffer("global_attn_scores").copy()
            hs_true = eng.buffer("HH_scores").copy()
            hh_ids = eng.buffer("HH_token_ids").copy()
            if recompute:
                buf = torch.from_numpy(_pack(eng, c, g_r, rank, world))
                dist.all_reduce(buf)
                g_r = buf.numpy().copy()
                assert np.array_equal(g_r, g_true), (step, "synchronised scores differ")
                hs_r[:c["hh_count"]] = g_r[hh_ids[:c["hh_count"]]]
                rows = None
                stats["syncs"] += 1
            if evicts:
                ev_id = total - R
                if rows is not None:
                    score = rows[c["rw_head_index"] % world, 0]
                    assert score == (g_true[ev_id] if ev_id < MSL else 0.0), (step, "evicted token's score")
                    g_r[ev_id] = score
                    stats["routed"] += 1
                    if c["hh_count"] == max_hh:
                        cand = [(rows[p, 1], int(rows[p, 2])) for p in range(world) if rows[p, 2] >= 0]
                        v0, i0 = min(cand)
                        j = int(np.argmin(hs_true[:c["hh_count"]]))  # first index of the minimum
                        assert (v0, i0) == (hs_true[j], j), (step, "heavy-hitter argmin")
                        if score > v0:
                            g_r[hh_ids[i0]] = v0  # the demoted token's current score
                            stats["replaced"] += 1
            Q = rng.standard_normal(NQ * HD).astype(np.float32)
            Kn = rng.standard_normal(NKV * HD).astype(np.float32)
            Vn = rng.standard_normal(NKV * HD).astype(np.float32)
            out = np.zeros(NQ * HD, np.float32)
            eng.step(Q, Kn, Vn, out)
            c = eng.counters()
            # the heavy-hitter slot a routed token entered takes its score on every rank
            hs_post = eng.buffer("HH_scores")
            new_hh = np.nonzero(eng.buffer("HH_token_ids")[:c["hh_count"]] == (c["total_processed_tokens"] - 1 - R))[0]
            for j in new_hh:
                hs_r[j] = g_r[c["total_processed_tokens"] - 1 - R]
            # attention over the owned positions: (m, l, acc) rows, merged in rank order
            own = _owned_positions(c, rank, world)
            dense = [(t, s) for t, s in own if t < 3]
            pk = np.array([s for t, s in own if t == 3], np.int64)
            kd, vd = _dense_rows(eng, c, dense)
            Kp, Vp = _packed_rows(eng, c)
            ids = np.concatenate([[_token_id(eng, c, t, s) for t, s in dense],
                                  eng.buffer("PBS_token_ids")[pk] if len(pk) else []]).astype(np.int64)
            Kall = np.concatenate([kd, Kp[pk]]) if len(pk) else kd
            Vall = np.concatenate([vd, Vp[pk]]) if len(pk) else vd
            live = np.ones(len(ids), bool)
            live[len(dense):] = ids[len(dense):] >= 0
            xr = np.zeros((NQ, HD + 2))
            for h in range(NQ):
                s = Kall[:, h // G, :] @ Q[h * HD:(h + 1) * HD].astype(np.float64) / np.sqrt(HD)
                s[~live] = -np.inf
                m = s.max() if len(s) else -np.inf
                w = np.exp(s - m) if np.isfinite(m) else np.zeros_like(s)
                xr[h, 0], xr[h, 1] = m, w.sum()
                xr[h, 2:] = w @ Vall[:, h // G, :]
            xs = torch.from_numpy(xr.ravel().copy())
            xa = torch.empty(world * xs.numel(), dtype=torch.float64)
            dist.all_gather_into_tensor(xa, xs)
            allr = xa.numpy().reshape(world, NQ, HD + 2)
            M = allr[:, :, 0].max(axis=0)
            f = np.where(np.isfinite(allr[:, :, 0]), np.exp(allr[:, :, 0] - M), 0.0)
            Lh = (allr[:, :, 1] * f).sum(0)
            o = (allr[:, :, 2:] * f[:, :, None]).sum(0) / Lh[:, None]
            err = np.abs(o.ravel() - out)
            assert np.all(err <= ATOL + RTOL * np.abs(out)), (step, float(err.max()))
            stats["worst_out"] = max(stats["worst_out"], float(err.max()))
            # owner feedback: the owned tokens take their post-step scores
            g_post = eng.buffer("global_attn_scores")
            for (t, s), i in zip(own, ids):
                if 0 <= i < MSL:
                    g_r[i] = g_post[i]
                    if t == 1:
                        hs_r[s] = hs_post[s]
            # every token's score, assembled from the owners, is the oracle's
            buf = torch.from_numpy(_pack(eng, c, g_r, rank, world))
            dist.all_reduce(buf)
            assert np.array_equal(buf.numpy(), g_post), (step, "assembled scores differ",
                                                          int(np.argmax(buf.numpy() != g_post)))
            # routing row for the next step
            row = np.array([0.0, 0.0, -1.0, 0.0], np.float64)
            if c["rw_count"] == R and c["rw_head_index"] % world == rank:
                i = c["total_processed_tokens"] - R
                row[0] = g_r[i] if 0 <= i < MSL else 0.0
            mine = [(hs_r[j], j) for j in range(rank, c["hh_count"], world)]
            if mine:
                v, j = min(mine)
                row[1], row[2] = v, j
            rs = torch.from_numpy(row)
            ra = torch.empty(world * 4, dtype=torch.float64)
            dist.all_gather_into_tensor(ra, rs)
            rows = ra.numpy().reshape(world, 4)
        dist.destroy_process_group()
        q.put((rank, stats, None))
    except Exception as exc:  # reported to the parent
        import traceback
        q.put((rank, None, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_ownership_protocol_matches_unsharded_engine(world):
    res = _run_ranks(_protocol_rank, world, ())
    for r in range(world):
        st = res[r]
        assert st["syncs"] >= 4 and st["routed"] > 20 and st["replaced"] > 0, st


class _FakeStep:
    """Stands in for ShardedStep: records the calls and writes rank-tagged rows."""

    ROUTE_FLOATS = 4

    def __init__(self, engines, rank, world):
        self.rank, self.world, self.n = rank, world, len(engines)
        self.xch_floats = self.n * 6
        self.route_floats = self.n * 4
        self.calls = []
        self.step_no = 0

    def sync_needed(self):
        return self.step_no % 3 == 0  # every third step, as a threshold schedule would

    def scores_floats(self):
        return 5

    def scores_pack(self, buf):
        import torch
        buf.copy_(torch.arange(5, dtype=buf.dtype) * (self.rank + 1))
        self.calls.append("pack")

    def scores_unpack(self, buf):
        self.calls.append(("unpack", buf.tolist()))

    def begin(self, Qs, Ks, Vs, xs, route):
        self.calls.append(("begin", None if route is None else route.tolist()))
        xs.fill_(100 * self.step_no + self.rank)

    def merge(self, xa, outs, rs):
        self.calls.append(("merge", xa.tolist()))
        rs.fill_(10 * self.step_no + self.rank)
        self.step_no += 1

    # peer exchange
    def xch_create(self):
        self.calls.append("xch_create")
        self._x = True
        return bytes([self.rank]) * 64

    def xch_open(self, handles):
        self.calls.append(("xch_open", handles))

    def xch_destroy(self):
        self.calls.append("xch_destroy")
        self._x = None

    def begin_xch(self, Qs, Ks, Vs, route_valid):
        self.calls.append(("begin_xch", route_valid))

    def merge_xch(self, outs):
        self.calls.append("merge_xch")
        self.step_no += 1


class _FakeEngine:
    def __init__(self):
        import torch
        self.device = torch.device("cpu")


def _driver_rank(rank, world, port, q, exchange="nccl"):
    try:
        import torch.distributed as dist
        from datetime import timedelta
        from tritiercache_b200 import _C
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        _C.ShardedStep = _FakeStep
        engines = [_FakeEngine(), _FakeEngine()]
        drv = _C.ShardedEngineStep(engines, exchange=exchange)
        for _ in range(5):
            drv(engines, [None] * 2, [None] * 2, [None] * 2, [None] * 2)
        drv.close()
        calls = drv.step.calls
        dist.destroy_process_group()
        q.put((rank, (calls, drv.syncs), None))
    except Exception:
        import traceback
        q.put((rank, None, traceback.format_exc()))


def test_sharded_driver_collective_sequence():
    world = 2
    res = _run_ranks(_driver_rank, world, ())
    for r in range(world):
        calls, syncs = res[r]
        assert syncs == 2  # steps 0 and 3
        it = iter(calls)
        for step in range(5):
            if step % 3 == 0:
                assert next(it) == "pack"
                op, buf = next(it)
                assert op == "unpack" and buf == [float(i * 3) for i in range(5)]  # sum over ranks 1x + 2x
            op, route = next(it)
            assert op == "begin"
            if step % 3 == 0:
                assert route is None  # threshold steps route from the synchronised scores
            else:  # the previous step's routing rows, all-gathered in rank order
                assert route == [10.0 * (step - 1) + p for p in range(world) for _ in range(8)]
            op, xa = next(it)
            assert op == "merge"
            assert xa == [100.0 * step + p for p in range(world) for _ in range(12)]


def _driver_rank_peer(rank, world, port, q):
    _driver_rank(rank, world, port, q, exchange="peer")


def test_sharded_driver_peer_exchange_sequence():
    world = 2
    res = _run_ranks(_driver_rank_peer, world, ())
    for r in range(world):
        calls, syncs = res[r]
        assert syncs == 2
        it = iter(calls)
        assert next(it) == "xch_create"
        op, handles = next(it)  # every rank's handle, in rank order
        assert op == "xch_open" and handles == b"".join(bytes([p]) * 64 for p in range(world))
        for step in range(5):
            if step % 3 == 0:
                assert next(it) == "pack"
                op, buf = next(it)
                assert op == "unpack" and buf == [float(i * 3) for i in range(5)]
            # routing rows from the last step, except on the first step and after a synchronisation
            assert next(it) == ("begin_xch", step % 3 != 0)
            assert next(it) == "merge_xch"
        assert next(it) == "xch_destroy"
        assert next(it, None) is None
