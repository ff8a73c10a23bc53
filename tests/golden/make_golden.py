"""Generate the golden fixtures under tests/golden/ (run in the build container).

Two sources, both from the reference project (its checkout is given by the
REF_ROOT environment variable, or else is a directory named `reference` beside
this repository's root):

1. Known-answer vectors of the reference's own C++ tests, read as text:
   tests/test_quantize_v.cpp (16 tokens x 2 heads x head_dim 32 V block with
   expected per-token min, scale and 64 packed words) and tests/tie_test_v.cpp
   (round-half-to-even ties).  -> kat_quantize_v.npz, kat_tie_v.npz
2. Outputs of the reference's own C++ kernels and engine, compiled from its
   sources by `make -C oracle ref` (oracle/_ref/_C*.so), on seeded inputs.
   -> ref_quant.npz, ref_attn.npz, ref_engine.npz

The GPU tests and the oracle tests only read the .npz files; nothing at test
time touches the reference tree.  Usage:
    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
REF_ROOT = os.environ.get("REF_ROOT") or os.path.join(os.path.dirname(ROOT), "reference")


def _cpp_array(src: str, name: str, kind: str):
    m = re.search(r"std::vector<[^>]+>\s+" + name + r"\s*=\s*\{(.*?)\};", src, re.S)
    if not m:
        raise RuntimeError(f"array {name} not found")
    body = m.group(1)
    if kind == "f32":
        vals = [float(x.strip().rstrip("f")) for x in body.split(",") if x.strip()]
        return np.array(vals, dtype=np.float32)
    vals = re.findall(r"0x([0-9a-fA-F]+)u", body)
    return np.array([int(v, 16) for v in vals], dtype=np.uint32).view(np.int32)


def kat_fixtures():
    src = open(os.path.join(REF_ROOT, "tests", "test_quantize_v.cpp")).read()
    heads = int(re.search(r"num_heads\s*=\s*(\d+)", src).group(1))
    hd = int(re.search(r"head_dim\s*=\s*(\d+)", src).group(1))
    V = _cpp_array(src, "V", "f32")
    exp_min = _cpp_array(src, "expected_min", "f32")
    exp_scale = _cpp_array(src, "expected_scale", "f32")
    exp_packed = _cpp_array(src, "expected_packed", "hex")
    tokens = V.size // (heads * hd)
    np.savez_compressed(os.path.join(HERE, "kat_quantize_v.npz"), V=V.reshape(tokens, heads, hd),
                        expected_min=exp_min, expected_scale=exp_scale,
                        expected_packed=exp_packed, num_heads=heads, head_dim=hd,
                        tolerance=np.float32(1e-4))
    # tie_test_v.cpp: one head, head_dim 16, all 3.0 except token-0 channels
    # 0 (min 0), 1 (max 6 -> scale 2), 2 (1.0 -> 0.5 -> 0), 3 (3.0 -> 1.5 -> 2),
    # 10 (5.0 -> 2.5 -> 2).
    tsrc = open(os.path.join(REF_ROOT, "tests", "tie_test_v.cpp")).read()
    assigns = {int(c): float(v) for c, v in re.findall(r"row\[(\d+)\]\s*=\s*([0-9.]+)f", tsrc)}
    want = {int(c): int(v) for c, v in re.findall(r"ch(\d+)=%d\(want (\d+)\)", tsrc)}
    fill = float(re.search(r"std::vector<float> V\(16 \* head_dim, ([0-9.]+)f\)", tsrc).group(1))
    Vt = np.full((16, 1, 16), fill, dtype=np.float32)
    for c, v in assigns.items():
        Vt[0, 0, c] = v
    np.savez_compressed(os.path.join(HERE, "kat_tie_v.npz"), V=Vt,
                        check_channels=np.array(sorted(want), dtype=np.int32),
                        expected_codes=np.array([want[c] for c in sorted(want)], dtype=np.int32))


def _meta(meta):
    return np.uint16 if meta == "fp16" else np.float32


def ref_quant(R, rng):
    out = {}
    cases = [(16, "fp32", 2, 32), (16, "fp16", 8, 128), (32, "fp32", 4, 64), (32, "fp16", 2, 128),
             (16, "fp16", 3, 48)]
    for ci, (grp, meta, H, D) in enumerate(cases):
        K = rng.standard_normal((grp, H, D)).astype(np.float32) * 1.7
        K[:, :, 3] *= 8.0                      # outlier channel
        K[:, 0, 1] = 0.25                      # constant channel -> scale 1e-9
        K[:5, H - 1, 2] = -0.0
        K[5:, H - 1, 2] = 0.0                  # signed zeros
        V = rng.standard_normal((grp, H, D)).astype(np.float32)
        V[1, 0, :] = -2.0                      # constant token
        V[2, H - 1, ::2] = 1.0
        V[2, H - 1, 1::2] = 4.0                # exact ties after scaling
        kp = np.zeros((grp // 16, H, D), np.int32)
        ks = np.zeros((H, D), _meta(meta))
        kz = np.zeros((H, D), _meta(meta))
        R.quantize_k_block(K, kp, ks, kz, H, D, grp, meta)
        vq = np.zeros((grp, H, D // 16), np.int32)
        vs = np.zeros((grp, H), _meta(meta))
        vz = np.zeros((grp, H), _meta(meta))
        R.quantize_v_block(V, vq, vs, vz, H, D, grp, meta)
        kd = np.zeros((grp, H, D), np.float32)
        R.dequantize_k(kp, ks, kz, kd, 1, H, D, grp, meta)
        vd = np.zeros((grp, H, D), np.float32)
        R.dequantize_v(vq, vs, vz, vd, grp, H, D, meta)
        for k, v in dict(K=K, V=V, kp=kp, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, kd=kd, vd=vd,
                         cfg=np.array([grp, 1 if meta == "fp16" else 0, H, D])).items():
            out[f"c{ci}_{k}"] = v
    out["ncases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "ref_quant.npz"), **out)


def _pbs_from_tokens(R, K, V, meta, grp):
    """Quantize [nblk*grp, H, D] token data with the reference kernels."""
    n, H, D = K.shape
    nb = n // grp
    kp = np.zeros((nb * grp // 16, H, D), np.int32)
    ks = np.zeros((nb, H, D), _meta(meta))
    kz = np.zeros((nb, H, D), _meta(meta))
    vq = np.zeros((nb * grp, H, D // 16), np.int32)
    vs = np.zeros((nb * grp, H), _meta(meta))
    vz = np.zeros((nb * grp, H), _meta(meta))
    wpb = grp // 16
    for b in range(nb):
        R.quantize_k_block(np.ascontiguousarray(K[b * grp:(b + 1) * grp]), kp[b * wpb:(b + 1) * wpb],
                           ks[b], kz[b], H, D, grp, meta)
        R.quantize_v_block(np.ascontiguousarray(V[b * grp:(b + 1) * grp]), vq[b * grp:(b + 1) * grp],
                           vs[b * grp:(b + 1) * grp], vz[b * grp:(b + 1) * grp], H, D, grp, meta)
    return kp, ks, kz, vq, vs, vz


def ref_attn(R, rng):
    out = {}
    # (nq, nkv, hd, dense, blocks, meta, group, ids_minus_one_every)
    cases = [(32, 8, 128, 36, 4, "fp32", 16, 0),        # microbench head shape, fewer tokens
             (32, 8, 128, 21, 3, "fp16", 16, 5),
             (8, 8, 64, 10, 2, "fp16", 32, 0),
             (28, 4, 128, 13, 3, "fp16", 16, 0),        # G = 7
             (4, 2, 64, 0, 5, "fp32", 16, 3),           # no dense tokens
             (16, 4, 128, 30, 0, "fp16", 16, 0),        # no PBS blocks
             (8, 2, 32, 17, 4, "fp32", 32, 0)]
    for ci, (nq, nkv, hd, dc, nb, meta, grp, m1) in enumerate(cases):
        Q = rng.standard_normal((nq, hd)).astype(np.float32)
        dK = rng.standard_normal((max(dc, 1), nkv, hd)).astype(np.float32)
        dV = rng.standard_normal((max(dc, 1), nkv, hd)).astype(np.float32)
        Kt = rng.standard_normal((max(nb, 1) * grp, nkv, hd)).astype(np.float32)
        Kt[:, :, 7] *= 8.0
        Vt = rng.standard_normal((max(nb, 1) * grp, nkv, hd)).astype(np.float32)
        kp, ks, kz, vq, vs, vz = _pbs_from_tokens(R, Kt, Vt, meta, grp)
        ids = np.arange(max(nb, 1) * grp, dtype=np.int64) + 1000
        if m1:
            ids[::m1] = -1
        o = np.zeros((nq, hd), np.float32)
        mw = np.zeros(dc + nb * grp, np.float32)
        R.fused_attention_decode(Q, dK, dV, dc, kp, ks, kz, vq, vs, vz, ids, nb, nq, nkv, hd, o, mw,
                                 grp, meta)
        for k, v in dict(Q=Q, dK=dK, dV=dV, kp=kp, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, ids=ids,
                         out=o, mw=mw,
                         cfg=np.array([nq, nkv, hd, dc, nb, 1 if meta == "fp16" else 0, grp])).items():
            out[f"c{ci}_{k}"] = v
    out["ncases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "ref_attn.npz"), **out)


ENGINE_STATE = ["S_K", "S_V", "RW_K", "RW_V", "HH_K", "HH_V", "HH_token_ids", "HH_scores",
                "PBS_K_Packed", "PBS_K_Scales", "PBS_K_Zeroes", "PBS_V_Packed", "PBS_V_Scales",
                "PBS_V_Zeroes", "PBS_token_ids", "global_attn_scores"]
COUNTERS = ["s_count", "rw_count", "rw_head_index", "hh_count", "pbs_count", "pbs_blocks_used",
            "total_processed_tokens", "total_evictions", "pbs_allocated_blocks"]


def ref_engine(R, rng):
    out = {}
    # (nq, nkv, hd, max_seq_len, sink, rw, h_ratio, decay, interval, group, meta, prefill, steps)
    cases = [(4, 2, 32, 1024, 4, 32, 0.1, 0.999, 32, 16, "fp16", 200, 260),
             (4, 4, 16, 512, 4, 16, 0.2, 0.99, 16, 32, "fp32", 96, 220),
             (4, 2, 16, 256, 4, 24, 0.1, 0.999, 8, 16, "fp32", 0, 330)]  # ids pass max_seq_len
    for ci, (nq, nkv, hd, msl, S, Rw, hr, dec, ui, grp, meta, P, N) in enumerate(cases):
        e = R.TriTierCacheEngine(nq, nkv, hd, msl, S, Rw, hr, dec, ui, grp, meta)
        Kp = rng.standard_normal((max(P, 1), nkv, hd)).astype(np.float32)
        Vp = rng.standard_normal((max(P, 1), nkv, hd)).astype(np.float32)
        if P:
            e.prefill(Kp, Vp, P)
        Qs = rng.standard_normal((N, nq * hd)).astype(np.float32)
        Ks = rng.standard_normal((N, nkv * hd)).astype(np.float32)
        Vs = rng.standard_normal((N, nkv * hd)).astype(np.float32)
        outs = np.zeros((N, nq * hd), np.float32)
        ctr = np.zeros((N, len(COUNTERS)), np.int64)
        for s in range(N):
            e.step(Qs[s], Ks[s], Vs[s], outs[s])
            ctr[s] = [getattr(e, c) for c in COUNTERS]
        st = {
            "S_K": e.get_S_K(), "S_V": e.get_S_V(), "RW_K": e.get_RW_K(), "RW_V": e.get_RW_V(),
            "HH_K": e.get_HH_K(), "HH_V": e.get_HH_V(), "HH_token_ids": e.get_HH_token_ids(),
            "HH_scores": e.get_HH_scores(), "PBS_K_Packed": e.get_PBS_K_Packed(),
            "PBS_K_Scales": e.get_PBS_K_Scales(), "PBS_K_Zeroes": e.get_PBS_K_Zeroes(),
            "PBS_V_Packed": e.get_PBS_V_Packed(), "PBS_V_Scales": e.get_PBS_V_Scales(),
            "PBS_V_Zeroes": e.get_PBS_V_Zeroes(), "PBS_token_ids": e.get_PBS_token_ids(),
            "global_attn_scores": e.get_global_attn_scores(),
        }
        for k, v in st.items():
            out[f"c{ci}_state_{k}"] = np.array(v)
        for k, v in dict(Kp=Kp, Vp=Vp, Qs=Qs, Ks=Ks, Vs=Vs, outs=outs, counters=ctr,
                         buffer_bytes=np.array(e.get_buffer_bytes()),
                         cfg=np.array([nq, nkv, hd, msl, S, Rw, ui, grp, 1 if meta == "fp16" else 0, P, N]),
                         fcfg=np.array([hr, dec], np.float32)).items():
            out[f"c{ci}_{k}"] = v
    out["ncases"] = np.array(len(cases))
    out["counter_names"] = np.array(COUNTERS)
    np.savez_compressed(os.path.join(HERE, "ref_engine.npz"), **out)


def main():
    from oracle import oracle as O
    kat_fixtures()
    R = O.load_reference()
    if R is None:
        raise SystemExit("reference build missing: run `make -C oracle ref` first")
    rng = np.random.default_rng(20261201)
    ref_quant(R, rng)
    ref_attn(R, rng)
    ref_engine(R, rng)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
