"""Pins the CPU oracle (oracle/tt_oracle.c) before it is trusted as the checker.

(a) the known-answer vectors of the reference's own C++ tests
    (tests/test_quantize_v.cpp, tests/tie_test_v.cpp of the reference), and
(b) outputs of the reference's own C++ kernels and engine (fixtures written by
    tests/golden/make_golden.py from the reference compiled by oracle/Makefile).
All comparisons are bit-exact: the oracle follows the reference's operation order.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint8)


def test_kat_quantize_v_reference_cpp_test(golden_dir):
    # reference tests/test_quantize_v.cpp:8-39 (fp32 metadata, default chunk 16)
    d = np.load(os.path.join(golden_dir, "kat_quantize_v.npz"))
    V = d["V"]
    T, H, D = V.shape
    packed = np.zeros((T, H, (D + 15) // 16), np.int32)
    scale = np.zeros((T, H), np.float32)
    zero = np.zeros((T, H), np.float32)
    O.quantize_v_block(V, packed, scale, zero, H, D, T)
    tol = float(d["tolerance"])
    assert np.all(np.abs(zero.ravel() - d["expected_min"]) <= tol)
    assert np.all(np.abs(scale.ravel() - d["expected_scale"]) <= tol)
    assert np.array_equal(packed.ravel().view(np.uint32), d["expected_packed"].view(np.uint32))
    # the constant row of the KAT clamps the scale to 1e-9 (test_quantize_v.cpp:12)
    assert np.any(scale == np.float32(1e-9))


def test_kat_round_half_to_even(golden_dir):
    # reference tests/tie_test_v.cpp:12-27: 0.5 -> 0, 1.5 -> 2, 2.5 -> 2
    d = np.load(os.path.join(golden_dir, "kat_tie_v.npz"))
    V = d["V"]
    packed = np.zeros((16, 1, 1), np.int32)
    scale = np.zeros((16, 1), np.float32)
    zero = np.zeros((16, 1), np.float32)
    O.quantize_v_block(V, packed, scale, zero, 1, 16, 16)
    w = int(packed[0, 0, 0]) & 0xFFFFFFFF
    for ch, want in zip(d["check_channels"], d["expected_codes"]):
        assert (w >> (2 * int(ch))) & 3 == int(want)
    assert scale[0, 0] == np.float32(2.0)


def test_quant_dequant_fixtures_bit_exact(golden_dir):
    d = np.load(os.path.join(golden_dir, "ref_quant.npz"))
    for ci in range(int(d["ncases"])):
        grp, f16, H, D = (int(x) for x in d[f"c{ci}_cfg"])
        mdt = np.uint16 if f16 else np.float32
        kp = np.zeros((grp // 16, H, D), np.int32)
        ks = np.zeros((H, D), mdt)
        kz = np.zeros((H, D), mdt)
        O.quantize_k_block(d[f"c{ci}_K"], kp, ks, kz, H, D, grp)
        assert np.array_equal(kp, d[f"c{ci}_kp"]), ci
        assert np.array_equal(_bits(ks), _bits(d[f"c{ci}_ks"])), ci
        assert np.array_equal(_bits(kz), _bits(d[f"c{ci}_kz"])), ci
        vq = np.zeros((grp, H, D // 16), np.int32)
        vs = np.zeros((grp, H), mdt)
        vz = np.zeros((grp, H), mdt)
        O.quantize_v_block(d[f"c{ci}_V"], vq, vs, vz, H, D, grp)
        assert np.array_equal(vq, d[f"c{ci}_vq"]), ci
        assert np.array_equal(_bits(vs), _bits(d[f"c{ci}_vs"])), ci
        assert np.array_equal(_bits(vz), _bits(d[f"c{ci}_vz"])), ci
        kd = np.zeros((grp, H, D), np.float32)
        O.dequantize_k(d[f"c{ci}_kp"], d[f"c{ci}_ks"], d[f"c{ci}_kz"], kd, 1, H, D, grp)
        assert np.array_equal(_bits(kd), _bits(d[f"c{ci}_kd"])), ci
        vd = np.zeros((grp, H, D), np.float32)
        O.dequantize_v(d[f"c{ci}_vq"], d[f"c{ci}_vs"], d[f"c{ci}_vz"], vd, grp, H, D)
        assert np.array_equal(_bits(vd), _bits(d[f"c{ci}_vd"])), ci


def test_fused_attention_fixtures_bit_exact(golden_dir):
    d = np.load(os.path.join(golden_dir, "ref_attn.npz"))
    for ci in range(int(d["ncases"])):
        nq, nkv, hd, dc, nb, f16, grp = (int(x) for x in d[f"c{ci}_cfg"])
        out = np.zeros((nq, hd), np.float32)
        mw = np.zeros(dc + nb * grp, np.float32)
        g = lambda k: d[f"c{ci}_{k}"]
        O.fused_attention_decode(g("Q"), g("dK"), g("dV"), dc, g("kp"), g("ks"), g("kz"), g("vq"),
                                 g("vs"), g("vz"), g("ids"), nb, nq, nkv, hd, out, mw, grp)
        assert np.array_equal(_bits(out), _bits(g("out"))), ci
        assert np.array_equal(_bits(mw), _bits(g("mw"))), ci


STATE_NAMES = ["S_K", "S_V", "RW_K", "RW_V", "HH_K", "HH_V", "HH_token_ids", "HH_scores",
               "PBS_K_Packed", "PBS_K_Scales", "PBS_K_Zeroes", "PBS_V_Packed", "PBS_V_Scales",
               "PBS_V_Zeroes", "PBS_token_ids", "global_attn_scores"]


def test_engine_trajectory_fixtures_bit_exact(golden_dir):
    d = np.load(os.path.join(golden_dir, "ref_engine.npz"))
    names = [str(n) for n in d["counter_names"]]
    for ci in range(int(d["ncases"])):
        nq, nkv, hd, msl, S, Rw, ui, grp, f16, P, N = (int(x) for x in d[f"c{ci}_cfg"])
        hr, dec = (float(x) for x in d[f"c{ci}_fcfg"])
        e = O.Engine(nq, nkv, hd, msl, S, Rw, hr, dec, ui, grp, "fp16" if f16 else "fp32")
        if P:
            e.prefill(d[f"c{ci}_Kp"], d[f"c{ci}_Vp"], P)
        for s in range(N):
            out = np.zeros(nq * hd, np.float32)
            e.step(d[f"c{ci}_Qs"][s], d[f"c{ci}_Ks"][s], d[f"c{ci}_Vs"][s], out)
            assert np.array_equal(_bits(out), _bits(d[f"c{ci}_outs"][s])), (ci, s)
            c = e.counters()
            assert [c[n] for n in names] == list(d[f"c{ci}_counters"][s]), (ci, s)
        for n in STATE_NAMES:
            mine = e.buffer(n)
            ref = d[f"c{ci}_state_{n}"].ravel()
            assert np.array_equal(_bits(mine), _bits(ref)), (ci, n)
        assert e.get_buffer_bytes() == int(d[f"c{ci}_buffer_bytes"])


@pytest.mark.skipif(O.load_reference() is None, reason="reference build (oracle/_ref) absent")
def test_oracle_vs_reference_build_fuzz():
    """Seeded fuzz against the reference compiled from its sources (when present)."""
    R = O.load_reference()
    rng = np.random.default_rng(7)
    for trial in range(20):
        grp = int(rng.choice([16, 32]))
        meta = str(rng.choice(["fp16", "fp32"]))
        mdt = np.uint16 if meta == "fp16" else np.float32
        H = int(rng.integers(1, 6))
        D = int(rng.choice([16, 32, 64, 128]))
        K = (rng.standard_normal((grp, H, D)) * rng.uniform(0.01, 50)).astype(np.float32)
        p1 = np.zeros((grp // 16, H, D), np.int32)
        s1, z1 = np.zeros((H, D), mdt), np.zeros((H, D), mdt)
        p2, s2, z2 = p1.copy(), s1.copy(), z1.copy()
        R.quantize_k_block(K, p1, s1, z1, H, D, grp, meta)
        O.quantize_k_block(K, p2, s2, z2, H, D, grp)
        assert np.array_equal(p1, p2) and np.array_equal(_bits(s1), _bits(s2)) and np.array_equal(_bits(z1), _bits(z2))
        V = (rng.standard_normal((grp, H, D)) * rng.uniform(0.01, 50)).astype(np.float32)
        q1 = np.zeros((grp, H, D // 16), np.int32)
        vs1, vz1 = np.zeros((grp, H), mdt), np.zeros((grp, H), mdt)
        q2, vs2, vz2 = q1.copy(), vs1.copy(), vz1.copy()
        R.quantize_v_block(V, q1, vs1, vz1, H, D, grp, meta)
        O.quantize_v_block(V, q2, vs2, vz2, H, D, grp)
        assert np.array_equal(q1, q2) and np.array_equal(_bits(vs1), _bits(vs2)) and np.array_equal(_bits(vz1), _bits(vz2))


def test_f16_conversion_round_trip_and_rne():
    # The oracle's binary16 conversion agrees with numpy's IEEE float16 cast (RNE).
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10,
                        (rng.standard_normal(5000) * 1e-5).astype(np.float32),
                        np.array([65504, 65520, 65519.99, 1e-8, 2.0 ** -24, 2.0 ** -25, -0.0, 0.0],
                                 np.float32)])
    lib = O.lib()
    mine = np.array([lib.orc_f32_to_f16(float(v)) for v in x], dtype=np.uint16)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, want)
