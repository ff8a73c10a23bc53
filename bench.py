"""Benchmark of the fused tiered-KV decode step on B200 (one JSON line on stdout).

Headline workload (config 2, the configuration the metric is quoted on): Llama-3-8B
shaped decode, 32 layers, 32 query / 8 KV heads (GQA 4:1), head_dim 128,
context 32768, batch 1, fp16 PBS metadata, group 16.  Per layer the tiers are:
4 sinks, the last 256 tokens in the ring, the top 5% of the middle tokens by
seeded Exp(1) accumulated score as FP32 heavy hitters (1626), the rest 2-bit
packed in id order (1930 blocks) plus 2 tokens in the waiting room.  K/V are
seeded N(0,1) with 4 per-layer outlier channels (x8) and rotate-half RoPE
(theta 500000) at positions 0..32767; Q sits at position 32768.

Synthetic data (the reference measures its kernels on synthetic tensors too),
generated with numpy so that both arms read the same numbers: four seeded
base K/V sets; layer l starts from set l mod 4 and draws its own outlier
channels and its own Exp(1) scores (so its own heavy-hitter set and packed
blocks).

A "step" is one decode step of all 32 layers through the engine: ingest the
new token (ring insert / evict / route / waiting-room flush), fused attention
over every tier, decayed score feedback.  The per-step inputs are 1.3 GB of KV
tiers, far larger than the 126 MB L2, so no flush is needed.

  value : device time per step (CUDA events, inputs resident in HBM), max over ranks.
  e2e   : the same step through the public API with host buffers: pinned
          Q/K_new/V_new copied in and the attention outputs copied out inside
          the timed region.
  roofline: the attention kernels, algorithmic bytes per step / their summed
          duration per step (CUDA events on their launch stream) against
          MEASURED_PEAKS.json hbm_gbs.
  cpu_baseline: the reference's own _C.fused_attention_decode (compiled from
          its sources into oracle/_ref) on this host's cores, on the same
          per-layer arrays built by the reference's own quantizers.
  config3: the maintenance run (1 layer, prefill 4096, then decode steps
          through engine.step), GPU and the reference's own engine.step.
  parity (N > 1): after the timed region the sharded outputs are compared
          across ranks (bit-identical) and with an unsharded engine on rank 0.

--impl reference times the reference CPU path alone (rank 0 only) on the
same config, without importing this repository's package.
--config 5 makes the Qwen2-7B 128k-context workload the
headline instead; --config 1 the single-layer 8k MHA case.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused decode-attn us/step & KV HBM GB/s (% of peak) at 32k ctx"
UNIT = "us/step"
SEED = 1234
NBASE = 4  # distinct base K/V sets; layer l starts from set l % NBASE

CONFIGS = {
    1: dict(key="config1", name="config1: single layer, 32q/32kv, hd128, ctx 8192, fp16 meta, group 16",
            layers=1, nq=32, nkv=32, hd=128, ctx=8192, sink=4, rw=256, h_ratio=0.05, meta="fp16", grp=16,
            rope_theta=None),
    2: dict(key="config2", name="config2: Llama-3-8B decode, 32 layers, 32q/8kv, hd128, ctx 32768, fp16 meta, "
                                "group 16", layers=32, nq=32, nkv=8, hd=128, ctx=32768, sink=4, rw=256,
            h_ratio=0.05, meta="fp16", grp=16, rope_theta=500000.0),
    5: dict(key="config5", name="config5: Qwen2-7B decode, 28 layers, 28q/4kv, hd128, ctx 131072, fp16 meta, "
                                "group 16", layers=28, nq=28, nkv=4, hd=128, ctx=131072, sink=4, rw=256,
            h_ratio=0.05, meta="fp16", grp=16, rope_theta=None),
}
CFG3 = dict(name="config3: maintenance run, 1 layer, 32q/8kv, hd128, max_seq_len 8192, prefill 4096 then decode "
                 "steps, update_interval 32, decay 0.999, fp16 meta, group 16",
            nq=32, nkv=8, hd=128, msl=8192, sink=4, rw=256, h_ratio=0.05, decay=0.999, ui=32, grp=16,
            meta="fp16", prefill=4096, steps=4096, sample=512)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# synthetic workload (shared by both arms and by the full-size parity tests)
# ---------------------------------------------------------------------------
def tier_plan(cfg):
    """(middle tokens, heavy hitters, packed blocks, waiting-room tokens) of one layer."""
    ctx, S, R, grp = cfg["ctx"], cfg["sink"], cfg["rw"], cfg["grp"]
    n_mid = ctx - S - R
    n_hh = int(np.ceil(cfg["h_ratio"] * n_mid))
    n_rest = n_mid - n_hh
    nblk = n_rest // grp
    return n_mid, n_hh, nblk, n_rest - nblk * grp


def layer_bytes(cfg, n_dense, nblk):
    """Algorithmic bytes one layer's attention reads (tiers + ids) and the Q/output bytes."""
    nkv, hd, nq, grp = cfg["nkv"], cfg["hd"], cfg["nq"], cfg["grp"]
    m = 2 if cfg["meta"] == "fp16" else 4
    dq = (hd + 15) // 16
    kv = 2 * n_dense * nkv * hd * 4
    pbs = nblk * (grp // 16) * nkv * hd * 4 + nblk * nkv * hd * 2 * m + nblk * grp * nkv * dq * 4 \
        + nblk * grp * nkv * 2 * m + nblk * grp * 8
    q_out = 2 * nq * hd * 4
    return kv + pbs, q_out


def base_kv(cfg, b, seed=SEED):
    rng = np.random.default_rng([seed, 7919, b])
    shape = (cfg["ctx"], cfg["nkv"], cfg["hd"])
    return rng.standard_normal(shape, dtype=np.float32), rng.standard_normal(shape, dtype=np.float32)


def bases(cfg, n=NBASE, threads=None):
    with ThreadPoolExecutor(threads or min(2 * n, host_cores())) as ex:
        return list(ex.map(lambda b: base_kv(cfg, b), range(n)))


_ROPE = {}


def apply_rope(K, theta):
    """rotate-half RoPE at positions 0..ctx-1 (float32)."""
    ctx, _, hd = K.shape
    key = (ctx, hd, theta)
    if key not in _ROPE:
        inv = theta ** (-np.arange(0, hd, 2, dtype=np.float64) / hd)
        ang = np.arange(ctx, dtype=np.float64)[:, None] * inv[None, :]
        c = np.cos(ang).astype(np.float32)
        s = np.sin(ang).astype(np.float32)
        _ROPE[key] = (np.concatenate([c, c], -1)[:, None, :], np.concatenate([s, s], -1)[:, None, :])
    cos, sin = _ROPE[key]
    half = hd // 2
    out = K * cos
    out[..., :half] -= K[..., half:] * sin[..., :half]
    out[..., half:] += K[..., :half] * sin[..., half:]
    return out


def synth_layer(cfg, layer, base, seed=SEED):
    """One layer's synthetic state: K/V of every token, heavy hitters, packed order."""
    rng = np.random.default_rng([seed, layer])
    ctx, S, R, hd = cfg["ctx"], cfg["sink"], cfg["rw"], cfg["hd"]
    K0, V = base
    outl = rng.choice(hd, 4, replace=False)
    K = K0.copy()
    K[:, :, outl] *= np.float32(8.0)
    if cfg.get("rope_theta"):
        K = apply_rope(K, cfg["rope_theta"])
    scores = rng.standard_exponential(ctx, dtype=np.float32)
    n_mid, n_hh, nblk, n_wr = tier_plan(cfg)
    mid = np.arange(S, ctx - R)
    top = np.argpartition(scores[mid], n_mid - n_hh)[n_mid - n_hh:]
    hh_ids = np.sort(mid[top])
    keep = np.ones(ctx, dtype=bool)
    keep[hh_ids] = False
    keep[:S] = False
    keep[ctx - R:] = False
    rest_ids = np.nonzero(keep)[0]
    order = np.concatenate([np.arange(S), rest_ids, np.arange(ctx - R, ctx)])
    # the threshold the reference would cache for these scores (cache_engine.cpp:126-143)
    k = int(np.float32(1.0 - cfg["h_ratio"]) * np.float32(n_mid - 1))
    thr = float(np.partition(scores[mid], k)[k])
    return dict(K=K, V=V, scores=scores, hh_ids=hh_ids, rest_ids=rest_ids, order=order, n_mid=n_mid,
                n_hh=n_hh, nblk=nblk, n_wr=n_wr, thr=thr)


def layer_stream(cfg, layers, threads=None):
    """Yields (layer, synth) for the given layers, generated ahead on a thread pool."""
    bs = bases(cfg)
    with ThreadPoolExecutor(threads or min(8, host_cores())) as ex:
        futs = {}
        layers = list(layers)
        ahead = 4
        for i, l in enumerate(layers[:ahead]):
            futs[i] = ex.submit(synth_layer, cfg, l, bs[l % NBASE])
        for i, l in enumerate(layers):
            syn = futs.pop(i).result()
            if i + ahead < len(layers):
                futs[i + ahead] = ex.submit(synth_layer, cfg, layers[i + ahead], bs[layers[i + ahead] % NBASE])
            yield l, syn


def imported_counters(cfg, syn):
    ctx = cfg["ctx"]
    return dict(hh_count=syn["n_hh"], total_processed_tokens=ctx, total_evictions=syn["n_mid"],
                last_calc_pos=ctx - 16, cached_threshold=syn["thr"])


def engine_args(cfg, msl):
    return (cfg["nq"], cfg["nkv"], cfg["hd"], msl, cfg["sink"], cfg["rw"], cfg["h_ratio"], 0.999, 32, cfg["grp"],
            cfg["meta"])


def gpu_engine(C_, torch, cfg, syn, msl):
    """A GPU engine holding the synthetic state: prefill of [sinks | packed-order
    tokens | ring] builds S, PBS, WR and RW; the heavy hitters, real token ids,
    scores and counters are written through the engine's writable views."""
    S, R, grp, ctx = cfg["sink"], cfg["rw"], cfg["grp"], cfg["ctx"]
    e = C_.TriTierCacheEngine(*engine_args(cfg, msl))
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    order = syn["order"]
    e.prefill(d(syn["K"][order]), d(syn["V"][order]), int(order.size))
    nb, nw, nh = syn["nblk"], syn["n_wr"], syn["n_hh"]
    rest, hh = syn["rest_ids"], syn["hh_ids"]
    e.get_PBS_token_ids()[: nb * grp].copy_(d(rest[: nb * grp]))
    e.get_WR_token_ids()[:nw].copy_(d(rest[nb * grp:]))
    e.get_HH_K()[:nh].copy_(d(syn["K"][hh]))
    e.get_HH_V()[:nh].copy_(d(syn["V"][hh]))
    e.get_HH_token_ids()[:nh].copy_(d(hh))
    e.get_HH_scores()[:nh].copy_(d(syn["scores"][hh]))
    g = e.get_global_attn_scores()
    g.zero_()
    g[S:ctx - R].copy_(d(syn["scores"][S:ctx - R]))
    e.set_counters(**imported_counters(cfg, syn))
    return e


def oracle_engine(O, cfg, syn, msl):
    """The same state in the CPU oracle engine (test infrastructure)."""
    S, R, grp, ctx = cfg["sink"], cfg["rw"], cfg["grp"], cfg["ctx"]
    eo = O.Engine(*engine_args(cfg, msl))
    order = syn["order"]
    eo.prefill(np.ascontiguousarray(syn["K"][order]), np.ascontiguousarray(syn["V"][order]), int(order.size))
    nb, nw, nh = syn["nblk"], syn["n_wr"], syn["n_hh"]
    rest, hh = syn["rest_ids"], syn["hh_ids"]
    kvs = cfg["nkv"] * cfg["hd"]
    eo.buffer("PBS_token_ids")[: nb * grp] = rest[: nb * grp]
    eo.buffer("WR_token_ids")[:nw] = rest[nb * grp:]
    eo.buffer("HH_K")[: nh * kvs] = syn["K"][hh].ravel()
    eo.buffer("HH_V")[: nh * kvs] = syn["V"][hh].ravel()
    eo.buffer("HH_token_ids")[:nh] = hh
    eo.buffer("HH_scores")[:nh] = syn["scores"][hh]
    g = eo.buffer("global_attn_scores")
    g[:] = 0
    g[S:ctx - R] = syn["scores"][S:ctx - R]
    eo.set_counters(**imported_counters(cfg, syn))
    return eo


def ref_layer_arrays(Q_, cfg, syn):
    """The layer's tiers as the reference's fused_attention_decode arguments,
    quantized by `Q_` (the reference's own _C, or the oracle port):
    dense [sinks | heavy hitters | ring] and the packed blocks in id order."""
    S, R, grp, ctx, nkv, hd = cfg["sink"], cfg["rw"], cfg["grp"], cfg["ctx"], cfg["nkv"], cfg["hd"]
    K, V = syn["K"], syn["V"]
    dense = np.concatenate([np.arange(S), syn["hh_ids"], np.arange(ctx - R, ctx)])
    nb = syn["nblk"]
    ids = syn["rest_ids"][: nb * grp].astype(np.int64)
    meta = cfg["meta"]
    mnp = np.uint16 if meta == "fp16" else np.float32
    kp = np.zeros((nb * grp // 16, nkv, hd), np.int32)
    ks = np.zeros((nb, nkv, hd), mnp)
    kz = np.zeros((nb, nkv, hd), mnp)
    Kp = np.ascontiguousarray(K[ids])
    Vp = np.ascontiguousarray(V[ids])
    w = grp // 16
    for b in range(nb):
        Q_.quantize_k_block(Kp[b * grp:(b + 1) * grp], kp[b * w:(b + 1) * w], ks[b], kz[b], nkv, hd, grp, meta)
    vq = np.zeros((nb * grp, nkv, hd // 16), np.int32)
    vs = np.zeros((nb * grp, nkv), mnp)
    vz = np.zeros((nb * grp, nkv), mnp)
    Q_.quantize_v_block(Vp, vq, vs, vz, nkv, hd, nb * grp, meta)
    return dict(dK=np.ascontiguousarray(K[dense]), dV=np.ascontiguousarray(V[dense]), dc=int(dense.size), nb=nb,
                kp=kp, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, ids=ids)


def step_inputs(cfg, nset=4, seed=99):
    """Per-step decode inputs: nset sets of [layer][Q | K_new | V_new] (float32)."""
    rng = np.random.default_rng([seed, cfg["layers"]])
    w = cfg["nq"] * cfg["hd"] + 2 * cfg["nkv"] * cfg["hd"]
    return [rng.standard_normal((cfg["layers"], w), dtype=np.float32) for _ in range(nset)]


def config3_inputs():
    c = CFG3
    rng = np.random.default_rng([SEED, 3])
    kvs = c["nkv"] * c["hd"]
    Kp = rng.standard_normal((c["prefill"], c["nkv"], c["hd"]), dtype=np.float32)
    Vp = rng.standard_normal((c["prefill"], c["nkv"], c["hd"]), dtype=np.float32)
    X = rng.standard_normal((c["steps"], c["nq"] * c["hd"] + 2 * kvs), dtype=np.float32)
    return Kp, Vp, X


# ---------------------------------------------------------------------------
# the reference CPU implementation (oracle/_ref, else the oracle port)
# ---------------------------------------------------------------------------
def reference_module():
    """(module, kind): the reference's own _C built from its sources, or the port."""
    from oracle import oracle as O
    R = O.load_reference()
    if R is not None:
        return R, "reference"
    return _PortAdapter(O), "port"


class _PortAdapter:
    """The oracle port behind the reference binding's call signatures."""

    def __init__(self, O):
        self.O = O

    def quantize_k_block(self, K, p, s, z, H, D, grp, meta):
        self.O.quantize_k_block(K, p, s, z, H, D, grp)

    def quantize_v_block(self, V, p, s, z, H, D, n, meta):
        self.O.quantize_v_block(V, p, s, z, H, D, n)

    def fused_attention_decode(self, q, dK, dV, dc, kp, ks, kz, vq, vs, vz, ids, nb, nq, nkv, hd, out, mw, grp, meta):
        self.O.fused_attention_decode(q, dK, dV, dc, kp, ks, kz, vq, vs, vz, ids, nb, nq, nkv, hd, out, mw, grp)

    def TriTierCacheEngine(self, *a):
        return _PortEngine(self.O, *a)


class _PortEngine:
    def __init__(self, O, *a):
        self.e = O.Engine(*a)

    def prefill(self, K, V, n):
        self.e.prefill(K, V, n)

    def step(self, q, k, v, out):
        self.e.step(q, k, v, out)


def time_reference_attention(R, cfg, arrays, qset, calls):
    """Seconds for `calls` reference fused_attention_decode calls over the layers' arrays."""
    nq, nkv, hd, grp = cfg["nq"], cfg["nkv"], cfg["hd"], cfg["grp"]
    out = np.zeros((nq, hd), np.float32)
    mws = [np.zeros(a["dc"] + a["nb"] * grp, np.float32) for a in arrays]
    qs = [np.ascontiguousarray(qset[l % qset.shape[0], : nq * hd].reshape(nq, hd)) for l in range(len(arrays))]

    def call(i):
        a = arrays[i % len(arrays)]
        R.fused_attention_decode(qs[i % len(arrays)], a["dK"], a["dV"], a["dc"], a["kp"], a["ks"], a["kz"], a["vq"],
                                 a["vs"], a["vz"], a["ids"], a["nb"], nq, nkv, hd, out, mws[i % len(arrays)], grp,
                                 cfg["meta"])

    call(0)  # warm-up (thread pool, page faults)
    t0 = time.perf_counter()
    for i in range(calls):
        call(i)
    return time.perf_counter() - t0


def time_reference_config3(R):
    """Seconds per reference engine.step over the config-3 sample (after prefill 4096)."""
    c = CFG3
    Kp, Vp, X = config3_inputs()
    e = R.TriTierCacheEngine(c["nq"], c["nkv"], c["hd"], c["msl"], c["sink"], c["rw"], c["h_ratio"], c["decay"],
                             c["ui"], c["grp"], c["meta"])
    e.prefill(Kp, Vp, c["prefill"])
    qn, kvs = c["nq"] * c["hd"], c["nkv"] * c["hd"]
    out = np.zeros(qn, np.float32)
    rows = [(np.ascontiguousarray(x[:qn]), np.ascontiguousarray(x[qn:qn + kvs]), np.ascontiguousarray(x[qn + kvs:]))
            for x in X[: c["sample"]]]
    t0 = time.perf_counter()
    for q, k, v in rows:
        e.step(q, k, v, out)
    return (time.perf_counter() - t0) / len(rows)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def wait_first(self, timeout=10.0):
        """Block until nvidia-smi has printed a sample (it takes a moment to start)."""
        t_end = time.monotonic() + timeout
        while self.proc and not self.lines and time.monotonic() < t_end:
            time.sleep(0.02)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0=None, t1=None):
        """Median SM clock, max clock and active throttle reasons of the samples
        taken in [t0, t1] (monotonic seconds; all samples when not given)."""
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, ln in self.lines:
            if t0 is not None and not (t0 <= ts <= t1):
                continue
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
def config_dict(cfg, world, dense_per_layer, blocks_per_layer, step_bytes):
    """The `config` object; identical in both arms for the same workload."""
    return {"workload": cfg["name"], "layers": cfg["layers"], "num_q_heads": cfg["nq"],
            "num_kv_heads": cfg["nkv"], "head_dim": cfg["hd"], "ctx": cfg["ctx"], "batch": 1,
            "dense_tokens_per_layer": dense_per_layer, "pbs_blocks_per_layer": blocks_per_layer,
            "step_bytes": step_bytes,
            "data": f"numpy-seeded: {NBASE} base K/V sets, per-layer outlier channels and Exp(1) scores",
            "l2": f"per-step inputs ({step_bytes / 1e9:.2f} GB) larger than the 126 MB L2; no flush needed"
                  if step_bytes > 126e6 else "per-step inputs smaller than L2",
            "parallelism": "single sequence" if world == 1 else f"sequence-sharded x{world}"}


def workload_shape(cfg):
    n_mid, n_hh, nblk, _ = tier_plan(cfg)
    dense = cfg["sink"] + n_hh + cfg["rw"]
    kvb, qo = layer_bytes(cfg, dense, nblk)
    return dense, nblk, (kvb + qo) * cfg["layers"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 5])
    ap.add_argument("--exchange", default="nccl", choices=["nccl", "peer"],
                    help="N>1: the per-step exchanges as NCCL all-gathers or over NVLink peer memory")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config3", action="store_true")
    ap.add_argument("--layers", type=int, default=None,
                    help="fewer layers (profiling cases only; the metric is quoted on the full count)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg["layers"] = args.layers
        cfg["name"] = cfg["name"].replace(f"{CONFIGS[args.config]['layers']} layers", f"{args.layers} layers")
    cores = host_cores()
    if args.impl == "reference" or world == 1:
        # the CPU legs use every host core, also under torchrun (which sets 1);
        # set before the reference's OpenMP runtime is loaded
        os.environ["OMP_NUM_THREADS"] = str(cores)
    if args.impl == "reference":
        return reference_arm(args, cfg, rank, world, cores)
    return ours_arm(args, cfg, rank, world, local, cores)


def ours_arm(args, cfg, rank, world, local, cores):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))
    from tritiercache_b200 import _C, _lib

    L = cfg["layers"]
    msl = cfg["ctx"] + 4096
    engines = [None] * L
    for l, syn in layer_stream(cfg, range(L)):
        engines[l] = gpu_engine(_C, torch, cfg, syn, msl)
        del syn
    torch.cuda.synchronize()
    nq, nkv, hd = cfg["nq"], cfg["nkv"], cfg["hd"]
    wq, wk = nq * hd, nkv * hd
    sets = [torch.from_numpy(x).cuda() for x in step_inputs(cfg)]  # same inputs on every rank
    NSET = len(sets)
    out = torch.empty((L, nq * hd), device="cuda")
    # one 2-D tensor per input, a row per layer (the API's pointer arrays are built without a Python loop)
    views = [(s[:, :wq], s[:, wq:wq + wk], s[:, wq + wk:]) for s in sets]
    history = []  # input set of every step the engines take (replayed by the parity check)

    if world > 1:
        sharded = _C.ShardedEngineStep(engines, rank, world, exchange=args.exchange)
        step_fn = sharded
    else:
        step_fn = _C.engine_step_batched

    def step(i):
        j = i % NSET
        history.append(j)
        step_fn(engines, *views[j], out)

    def barrier():
        if world > 1:
            dist.barrier()

    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        barrier()
        # Clocks are sampled every 50 ms; the timed steps sit inside one
        # continuous burst of the same steps (about 0.25 s of untimed steps on
        # either side, the same count on every rank), and the clock record is
        # the samples taken during that burst.  The events bracket only the
        # timed steps.
        e0.record(st)
        step(args.warmup)
        e1.record(st)
        torch.cuda.synchronize()
        one = torch.tensor([e0.elapsed_time(e1)], device="cuda")
        if world > 1:
            dist.all_reduce(one, op=dist.ReduceOp.MAX)
        n_roll = int(min(600, max(10, math.ceil(250.0 / max(float(one.item()), 1e-3)))))
        clk.wait_first()
        barrier()
        k = args.warmup + 1
        tb0 = time.monotonic()
        for i in range(n_roll):
            step(k + i)
        k += n_roll
        # ---- timed region: device time, inputs resident ----
        e0.record(st)
        for i in range(args.steps):
            step(k + i)
        e1.record(st)
        k += args.steps
        for i in range(n_roll):
            step(k + i)
        torch.cuda.synchronize()
        tb1 = time.monotonic()
        barrier()
    clocks = clk.summary(tb0, tb1)
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # ---- per-kernel timing pass (events on the launch stream) ----
    Lb = _lib.lib()
    Lb.tt_profile_enable(1)
    if world > 1:
        sharded.phase_timing(True)
    for i in range(args.steps):
        step(i)
    kt = _lib.KernelTimes()
    _lib.check(Lb.tt_profile_collect(__import__("ctypes").byref(kt)), "profile")
    Lb.tt_profile_enable(0)
    phases = None
    if world > 1:
        phases = sharded.phase_times(args.steps)
        sharded.phase_timing(False)
    launches_per_step = (kt.maintain_launches + kt.partial_launches + kt.finalize_launches) / args.steps

    # ---- e2e through the public API with host buffers ----
    # one pinned host buffer per direction: [layer][Q | K_new | V_new] goes up in
    # one copy, attn_output comes back in one
    hIn = torch.empty((L, wq + 2 * wk), pin_memory=True)
    hO = torch.empty((L, nq * hd), pin_memory=True)
    hIn.copy_(sets[0].cpu())
    dIn = torch.empty((L, wq + 2 * wk), device="cuda")
    dQ, dK, dV = dIn[:, :wq], dIn[:, wq:wq + wk], dIn[:, wq + wk:]
    out_rows = out

    def e2e_step():
        history.append(0)
        dIn.copy_(hIn, non_blocking=True)
        step_fn(engines, dQ, dK, dV, out_rows)
        hO.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0.record(st)
    for _ in range(args.steps):
        e2e_step()
    e1.record(st)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms_e2e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())

    # ---- algorithmic bytes of the attention kernels ----
    kv_bytes = q_out = dense_tokens = pbs_blocks = 0
    for e in engines:
        c = e.counters()
        dcount = c["s_count"] + c["hh_count"] + c["rw_count"]
        kvb, qo = layer_bytes(cfg, dcount, c["pbs_blocks_used"])
        kv_bytes += kvb
        q_out += qo
        dense_tokens += dcount
        pbs_blocks += c["pbs_blocks_used"]
    part_ms = kt.partial_ms / args.steps  # summed attention-kernel time per step
    # reads every tier once + Q; with N ranks each rank reads its 1/N share
    part_bytes = kv_bytes // world + q_out // 2
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    achieved = part_bytes / (part_ms * 1e-3) / 1e9
    # scratch written and re-read by the attention path (not algorithmic bytes):
    # the logits kept for the mean weights, nq x (this rank's positions) floats
    # per layer, written once and read once
    scratch = 2 * 4 * nq * (dense_tokens + pbs_blocks * cfg["grp"]) // world

    dense_l, blocks_l, step_bytes_cfg = workload_shape(cfg)
    step_bytes = kv_bytes + q_out
    line = {
        "metric": METRIC if cfg["key"] == "config2" else METRIC.replace("32k", f"{cfg['ctx'] // 1024}k"),
        "value": round(ms * 1000.0, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": config_dict(cfg, world, dense_l, blocks_l, step_bytes_cfg),
        "step_GBps": round(step_bytes / (ms * 1e-3) / 1e9, 1),
        "roofline": {"kernel": "k_attn_dense + k_attn_packed (concurrent, fork to join)", "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak, "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": None, "bytes_per_step": part_bytes, "scratch_bytes_per_step": scratch,
                     "attention_ms_per_step": round(part_ms, 5),
                     "kernel_ms_per_step": {"maintain": round(kt.maintain_ms / args.steps, 5),
                                            "attention": round(kt.partial_ms / args.steps, 5),
                                            "finalize": round(kt.finalize_ms / args.steps, 5)}},
        "e2e": {"value": round(ms_e2e * 1000.0, 2), "unit": UNIT,
                "h2d_bytes_per_step": int(hIn.numel() * 4),
                "d2h_bytes_per_step": int(hO.numel() * 4)},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "clocks": clocks,
    }
    if phases is not None:
        line["phase_ms_per_step"] = phases

    if world > 1:
        line["parity"] = sharded_parity(torch, dist, _C, cfg, engines, sharded, views, history, rank, world, msl)
        line["exchange"] = sharded.exchange  # outside `config`, which both arms share
        sharded.close()
        del sharded
    del engines
    torch.cuda.synchronize()

    if world == 1 and not args.no_config3:
        line["config3"] = config3_gpu(torch, _C)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        R, kind = reference_module()
        t0 = time.perf_counter()
        arrays = []
        for l, syn in layer_stream(cfg, range(min(L, 8))):
            arrays.append(ref_layer_arrays(R, cfg, syn))
            del syn
        calls = len(arrays)
        dt = time_reference_attention(R, cfg, arrays, step_inputs(cfg)[0], calls)
        line["cpu_baseline"] = {"value": round(dt / calls * L * 1e6, 1), "unit": UNIT, "cores": cores, "kind": kind,
                                "sample": f"{calls} of the step's {L} fused_attention_decode calls (layers 0..{calls - 1},"
                                          f" same arrays as the GPU step), scaled to {L} layers; "
                                          f"OMP_NUM_THREADS={cores}"}
        if "config3" in line:
            line["config3"]["cpu_baseline"] = {"value": round(time_reference_config3(R) * 1e6, 1),
                                               "unit": UNIT, "cores": cores, "kind": kind,
                                               "sample": f"first {CFG3['sample']} engine.step calls after prefill"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def config3_gpu(torch, C_):
    """Config 3 on the GPU: engine.step per decode step (CUDA events around the
    first `sample` steps, the same steps the reference arm times, and around
    the whole run)."""
    c = CFG3
    Kp, Vp, X = config3_inputs()
    e = C_.TriTierCacheEngine(c["nq"], c["nkv"], c["hd"], c["msl"], c["sink"], c["rw"], c["h_ratio"], c["decay"],
                              c["ui"], c["grp"], c["meta"])
    e.prefill(torch.from_numpy(Kp).cuda(), torch.from_numpy(Vp).cuda(), c["prefill"])
    qn, kvs = c["nq"] * c["hd"], c["nkv"] * c["hd"]
    Xd = torch.from_numpy(X).cuda()
    rows = [(Xd[i, :qn], Xd[i, qn:qn + kvs], Xd[i, qn + kvs:]) for i in range(c["steps"])]
    out = torch.empty(qn, device="cuda")
    st = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    torch.cuda.synchronize()
    ev[0].record(st)
    for i, (q, k, v) in enumerate(rows):
        if i == c["sample"]:
            ev[1].record(st)
        e.step(q, k, v, out)
    ev[2].record(st)
    torch.cuda.synchronize()
    cnt = e.counters()
    return {"workload": c["name"], "value": round(ev[0].elapsed_time(ev[1]) * 1000.0 / c["sample"], 2),
            "unit": UNIT, "sample": f"first {c['sample']} steps after prefill {c['prefill']}",
            "full_run_us_per_step": round(ev[0].elapsed_time(ev[2]) * 1000.0 / c["steps"], 2),
            "full_run_steps": c["steps"],
            "end_state": {k_: cnt[k_] for k_ in ("hh_count", "pbs_blocks_used", "wr_count", "total_evictions")}}


def sharded_parity(torch, dist, C_, cfg, engines, sharded, views, history, rank, world, msl, steps=3):
    """After timing: a few more sharded steps, compared across ranks (bit-identical)
    and, on rank 0, with an unsharded engine of layer 0 that replays every step the
    sharded engines took (same inputs) through the single-GPU path."""
    nq, hd = cfg["nq"], cfg["hd"]
    L = cfg["layers"]
    out = torch.empty((L, nq * hd), device="cuda")
    outs = []
    for s in range(steps):
        j = (len(history) + s) % len(views)
        sharded(engines, *views[j], out)
        outs.append(out.clone())
    got = torch.stack(outs)
    allg = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(allg, got)
    same = all(torch.equal(allg[0], a) for a in allg[1:])
    res = {"ranks_bit_identical": bool(same), "steps_checked": steps}
    ok_ref = None
    err = None
    if rank == 0:
        for l, syn in layer_stream(cfg, [0]):
            ref = gpu_engine(C_, torch, cfg, syn, msl)
        o1 = torch.empty((1, nq * hd), device="cuda")
        for j in history:
            C_.engine_step_batched([ref], views[j][0][:1], views[j][1][:1], views[j][2][:1], o1)
        errs = []
        for s in range(steps):
            j = (len(history) + s) % len(views)
            C_.engine_step_batched([ref], views[j][0][:1], views[j][1][:1], views[j][2][:1], o1)
            a, b = got[s, 0].double(), o1[0].double()
            errs.append(bool(((a - b).abs() <= 1e-4 + 1e-5 * b.abs()).all()))
            err = max(err or 0.0, float((a - b).abs().max()))
        ok_ref = all(errs)
        del ref
    flag = torch.tensor([1 if (ok_ref is None or ok_ref) else 0], device="cuda")
    dist.broadcast(flag, 0)
    res["layer0_vs_unsharded"] = bool(flag.item())
    if err is not None:
        res["layer0_max_abs_err"] = err
    res["ok"] = bool(same and flag.item())
    return res


def reference_arm(args, cfg, rank, world, cores):
    """The reference CPU implementation alone (rank 0); other ranks exit.
    Imports nothing from this repository's package: the tier arrays are built
    from the same numpy data with the reference's own quantizers."""
    if rank != 0:
        return
    R, kind = reference_module()
    L = cfg["layers"]
    arrays = []
    for l, syn in layer_stream(cfg, range(L)):
        arrays.append(ref_layer_arrays(R, cfg, syn))
        del syn
    qset = step_inputs(cfg)[0]
    time_reference_attention(R, cfg, arrays, qset, 1)
    times = []
    for i in range(args.warmup + args.steps):
        dt = time_reference_attention(R, cfg, arrays, qset, L)
        if i >= args.warmup:
            times.append(dt)
    us = float(np.mean(times)) * 1e6
    dense_l, blocks_l, step_bytes = workload_shape(cfg)
    line = {"metric": METRIC if cfg["key"] == "config2" else METRIC.replace("32k", f"{cfg['ctx'] // 1024}k"),
            "value": round(us, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(us / 1000, 3), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": config_dict(cfg, world, dense_l, blocks_l, step_bytes),
            "cpu_baseline": {"value": round(us, 1), "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": f"each step = the {L} layers' fused_attention_decode calls "
                                       f"(the whole step), OMP_NUM_THREADS={cores}"},
            "e2e": {"value": round(us, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not args.no_config3:
        line["config3"] = {"workload": CFG3["name"], "value": round(time_reference_config3(R) * 1e6, 1),
                           "unit": UNIT, "sample": f"first {CFG3['sample']} engine.step calls after prefill "
                                                   f"{CFG3['prefill']}", "cores": cores, "kind": kind}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
