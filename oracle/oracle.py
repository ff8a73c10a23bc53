"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the CPU oracle.

`liboracle.so` (built from ``tt_oracle.c`` by ``oracle/Makefile``) is a
plain-C restatement of TriTierCache's reference algorithms for the decode hot
path.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
cpu_baseline leg load this module; the product library never does.

``load_reference()`` loads the reference's own ``_C`` extension compiled from
its sources into ``oracle/_ref/`` (``make -C oracle ref``), when present.
"""
from __future__ import annotations

import ctypes as C
import glob
import importlib.util
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (and the reference build when its sources exist)."""
    cmd = ["make", "-C", HERE]
    subprocess.run(cmd + (["-s"] if quiet else []), check=True)
    ref = reference_root()
    if os.path.isdir(os.path.join(ref, "csrc")):
        subprocess.run(cmd + ["ref", f"REF_ROOT={ref}"] + (["-s"] if quiet else []), check=True)


def reference_root() -> str:
    """The reference checkout: $REF_ROOT, else a directory named `reference`
    beside this repository's root (absent on machines that only run tests)."""
    return os.environ.get("REF_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _LIB = C.CDLL(path)
        _declare(_LIB)
    return _LIB


class EngineParams(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("num_q_heads", "num_kv_heads", "head_dim", "max_seq_len",
                                        "sink_size", "rw_size")] + \
               [("h_ratio", C.c_float), ("score_decay", C.c_float)] + \
               [(n, C.c_int) for n in ("update_interval", "k_group_size", "meta_fp16")]


class EngineCounters(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "s_count", "rw_count", "rw_head_index", "hh_count", "wr_count", "pbs_allocated_blocks",
        "pbs_blocks_used", "pbs_count", "total_processed_tokens", "total_evictions",
        "last_calc_pos", "max_hh", "chunk_size")] + [("cached_threshold", C.c_float)]


def _declare(L):
    vp, i = C.c_void_p, C.c_int
    L.orc_quantize_k_block.argtypes = [vp, vp, vp, vp, i, i, i, i]
    L.orc_quantize_v_block.argtypes = [vp, vp, vp, vp, i, i, i, i]
    L.orc_dequantize_k.argtypes = [vp, vp, vp, vp, i, i, i, i, i]
    L.orc_dequantize_v.argtypes = [vp, vp, vp, vp, i, i, i, i]
    L.orc_fused_attention_decode.argtypes = [vp, vp, vp, i, vp, vp, vp, vp, vp, vp, vp,
                                             i, i, i, i, vp, vp, i, i]
    L.orc_fused_attention_decode_logits.argtypes = [vp, vp, vp, i, vp, vp, vp, vp, vp, vp, vp,
                                                    i, i, i, i, vp, vp, i, i, vp]
    L.orc_engine_create.restype = vp
    L.orc_engine_create.argtypes = [C.POINTER(EngineParams)]
    L.orc_engine_destroy.argtypes = [vp]
    L.orc_engine_step.argtypes = [vp, vp, vp, vp, vp]
    L.orc_engine_prefill.argtypes = [vp, vp, vp, i]
    L.orc_engine_buffer_bytes.restype = C.c_size_t
    L.orc_engine_buffer_bytes.argtypes = [vp]
    L.orc_engine_counters_get.argtypes = [vp, C.POINTER(EngineCounters)]
    L.orc_engine_counters_set.argtypes = [vp, C.POINTER(EngineCounters)]
    L.orc_engine_buffer.restype = vp
    L.orc_engine_buffer.argtypes = [vp, i, C.POINTER(C.c_size_t), C.POINTER(C.c_int)]
    L.orc_f32_to_f16.restype = C.c_uint16
    L.orc_f32_to_f16.argtypes = [C.c_float]


def _p(a):
    return None if a is None else a.ctypes.data


def _meta_fp16(scale):
    return 1 if scale.dtype in (np.uint16, np.float16) else 0


def quantize_k_block(K, packed, scale, zero, num_heads, head_dim, k_group_size=16):
    lib().orc_quantize_k_block(_p(K), _p(packed), _p(scale), _p(zero), _meta_fp16(scale),
                               num_heads, head_dim, k_group_size)


def quantize_v_block(V, packed, scale, zero, num_heads, head_dim, chunk_size=16):
    lib().orc_quantize_v_block(_p(V), _p(packed), _p(scale), _p(zero), _meta_fp16(scale),
                               num_heads, head_dim, chunk_size)


def dequantize_k(packed, scale, zero, out, num_blocks, num_heads, head_dim, k_group_size=16):
    lib().orc_dequantize_k(_p(packed), _p(scale), _p(zero), _p(out), _meta_fp16(scale),
                           num_blocks, num_heads, head_dim, k_group_size)


def dequantize_v(packed, scale, zero, out, total_tokens, num_heads, head_dim):
    lib().orc_dequantize_v(_p(packed), _p(scale), _p(zero), _p(out), _meta_fp16(scale),
                           total_tokens, num_heads, head_dim)


def fused_attention_decode(Q, dense_K, dense_V, dense_count, kp, ks, kz, vp_, vs, vz, ids,
                           num_blocks, nq, nkv, hd, out, mw=None, k_group_size=16):
    meta16 = _meta_fp16(ks) if ks is not None else 0
    lib().orc_fused_attention_decode(_p(Q), _p(dense_K), _p(dense_V), dense_count, _p(kp), _p(ks),
                                     _p(kz), _p(vp_), _p(vs), _p(vz), _p(ids), num_blocks, nq, nkv,
                                     hd, _p(out), _p(mw), k_group_size, meta16)


def fused_attention_logits(Q, dense_K, dense_V, dense_count, kp, ks, kz, vp_, vs, vz, ids,
                           num_blocks, nq, nkv, hd, out, mw=None, k_group_size=16):
    """fused_attention_decode that also returns the per-head logits [nq][T]."""
    meta16 = _meta_fp16(ks) if ks is not None else 0
    T = dense_count + num_blocks * k_group_size
    logits = np.zeros((nq, max(T, 1)), np.float32)
    lib().orc_fused_attention_decode_logits(_p(Q), _p(dense_K), _p(dense_V), dense_count, _p(kp), _p(ks),
                                            _p(kz), _p(vp_), _p(vs), _p(vz), _p(ids), num_blocks, nq, nkv,
                                            hd, _p(out), _p(mw), k_group_size, meta16, _p(logits))
    return logits[:, :T]


def mean_weights_f64(logits):
    """The reference's head-mean softmax weights (fused_attn_avx2.cpp:286-300)
    evaluated in double precision from its float32 logits."""
    l = logits.astype(np.float64)
    mx = np.max(l, axis=1, keepdims=True)
    e = np.where(np.isfinite(l), np.exp(l - mx), 0.0)
    return (e / e.sum(axis=1, keepdims=True)).mean(axis=0)


_BUF_NAMES = ["S_K", "S_V", "RW_K", "RW_V", "HH_K", "HH_V", "HH_token_ids", "HH_scores", "WR_K",
              "WR_V", "WR_token_ids", "PBS_K_Packed", "PBS_K_Scales", "PBS_K_Zeroes",
              "PBS_V_Packed", "PBS_V_Scales", "PBS_V_Zeroes", "PBS_token_ids",
              "global_attn_scores", "mean_attn_weights"]
_BUF_DTYPES = {"HH_token_ids": np.int64, "WR_token_ids": np.int64, "PBS_token_ids": np.int64,
               "PBS_K_Packed": np.int32, "PBS_V_Packed": np.int32}


class Engine:
    """Oracle engine (cache_engine.cpp restated); buffers are writable numpy views."""

    def __init__(self, num_q_heads, num_kv_heads, head_dim, max_seq_len, sink_size=4, rw_size=64,
                 h_ratio=0.1, score_decay=0.999, update_interval=16, k_group_size=16,
                 pbs_metadata_dtype="fp16"):
        self.params = EngineParams(num_q_heads, num_kv_heads, head_dim, max_seq_len, sink_size,
                                   rw_size, h_ratio, score_decay, update_interval, k_group_size,
                                   1 if pbs_metadata_dtype == "fp16" else 0)
        self.h = lib().orc_engine_create(C.byref(self.params))
        self.num_q_heads, self.num_kv_heads, self.head_dim = num_q_heads, num_kv_heads, head_dim

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_engine_destroy(self.h)
            self.h = None

    def step(self, Q, K, V, out):
        lib().orc_engine_step(self.h, _p(Q), _p(K), _p(V), _p(out))

    def prefill(self, K, V, q_len):
        lib().orc_engine_prefill(self.h, _p(K), _p(V), q_len)

    def counters(self) -> dict:
        c = EngineCounters()
        lib().orc_engine_counters_get(self.h, C.byref(c))
        return {n: getattr(c, n) for n, _ in EngineCounters._fields_}

    def set_counters(self, **kw) -> None:
        """Overwrite integer state (test set-up of synthetic tier layouts)."""
        c = EngineCounters()
        lib().orc_engine_counters_get(self.h, C.byref(c))
        for k, v in kw.items():
            setattr(c, k, v)
        lib().orc_engine_counters_set(self.h, C.byref(c))

    def get_buffer_bytes(self):
        return lib().orc_engine_buffer_bytes(self.h)

    def buffer(self, name):
        n, es = C.c_size_t(), C.c_int()
        ptr = lib().orc_engine_buffer(self.h, _BUF_NAMES.index(name), C.byref(n), C.byref(es))
        if n.value == 0 or not ptr:
            dt = _BUF_DTYPES.get(name, np.float32)
            return np.zeros(0, dtype=dt)
        if name in _BUF_DTYPES:
            dt = _BUF_DTYPES[name]
        elif es.value == 2:
            dt = np.uint16
        else:
            dt = np.float32
        arr = (C.c_byte * (n.value * es.value)).from_address(ptr)
        return np.frombuffer(arr, dtype=dt, count=n.value)


def _meta_f32(a, meta16):
    a = np.asarray(a)
    return a.view(np.float16).astype(np.float32) if meta16 else a.astype(np.float32)


def reconstruct_full_cache(st: dict):
    """src/tri_tier/cache.py:326-372 restated in numpy over an engine state
    dump `st` (tier buffers in the engine layouts plus the counters):
    [sinks | heavy hitters and live packed tokens sorted by id | ring in
    logical order]; packed tokens dequantized as code * scale + zero with two
    float32 roundings (the reference's torch expression).  Group 16 or 32."""
    S, hh, rw, head = st["s_count"], st["hh_count"], st["rw_count"], st["rw_head_index"]
    R, grp, nkv, hd, m16 = st["rw_size"], st["grp"], st["nkv"], st["hd"], st["meta16"]
    total, nb = st["total"], st["pbs_blocks_used"]
    kvs = nkv * hd
    sK = st["S_K"].reshape(-1, nkv, hd)[:S]
    sV = st["S_V"].reshape(-1, nkv, hd)[:S]
    sid = np.arange(S, dtype=np.int64)
    n = nb * grp
    kp = st["PBS_K_Packed"].reshape(-1, kvs)[: nb * (grp // 16)].view(np.uint32).reshape(nb, grp // 16, nkv, hd)
    t = np.arange(grp)
    codes = (kp[:, t // 16, :, :] >> (2 * (t % 16)).astype(np.uint32)[None, :, None, None]) & 3  # [nb][grp][nkv][hd]
    ks = _meta_f32(st["PBS_K_Scales"], m16).reshape(-1, nkv, hd)[:nb]
    kz = _meta_f32(st["PBS_K_Zeroes"], m16).reshape(-1, nkv, hd)[:nb]
    pK = (codes.astype(np.float32) * ks[:, None]) + kz[:, None]
    pK = pK.reshape(n, nkv, hd)
    qhd = (hd + 15) // 16
    vp = st["PBS_V_Packed"].reshape(-1, nkv, qhd)[:n].view(np.uint32)
    c = np.arange(hd)
    vcodes = (vp[:, :, c // 16] >> (2 * (c % 16)).astype(np.uint32)[None, None, :]) & 3  # [n][nkv][hd]
    vs = _meta_f32(st["PBS_V_Scales"], m16).reshape(-1, nkv)[:n]
    vz = _meta_f32(st["PBS_V_Zeroes"], m16).reshape(-1, nkv)[:n]
    pV = (vcodes.astype(np.float32) * vs[:, :, None]) + vz[:, :, None]
    pid = st["PBS_token_ids"][:n]
    live = pid != -1
    mK = np.concatenate([st["HH_K"].reshape(-1, nkv, hd)[:hh], pK[live]])
    mV = np.concatenate([st["HH_V"].reshape(-1, nkv, hd)[:hh], pV[live]])
    mid = np.concatenate([st["HH_token_ids"][:hh], pid[live]])
    perm = np.argsort(mid, kind="stable")
    mK, mV, mid = mK[perm], mV[perm], mid[perm]
    rK = st["RW_K"].reshape(-1, nkv, hd)
    rV = st["RW_V"].reshape(-1, nkv, hd)
    if rw < R:
        rK, rV = rK[:rw], rV[:rw]
        rid = np.arange(S, S + rw, dtype=np.int64)
    else:
        rK, rV = np.roll(rK, -head, axis=0), np.roll(rV, -head, axis=0)
        rid = np.arange(total - R, total, dtype=np.int64)
    return (np.concatenate([sK, mK, rK]).astype(np.float32), np.concatenate([sV, mV, rV]).astype(np.float32),
            np.concatenate([sid, mid, rid]).astype(np.int64))


def accumulate_attn_scrs(g, weights, ids):
    """src/tri_tier/cache.py:164-187: g[ids] += weights.mean(heads), skipping -1."""
    mean = np.asarray(weights, np.float32).mean(axis=0, dtype=np.float32)
    ok = ids != -1
    np.add.at(g, ids[ok], mean[ok])


def load_reference():
    """The reference `_C` compiled from its own sources into oracle/_ref/, or None."""
    cands = glob.glob(os.path.join(HERE, "_ref", "_C*.so"))
    if not cands:
        return None
    spec = importlib.util.spec_from_file_location("_C", cands[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod
