"""GPU parity of the stand-alone kernels against the reference fixtures and the oracle.

Bit-exact: packed words, scale/zero metadata bits, dequantized values.
Floating point: attention output |got - want| <= 1e-4 + 1e-5 * |want|
elementwise (max-abs 1e-4 / rel 1e-5, FP32); mean
attention weights relative, |got - want| <= 1e-9 + 1e-4 * |want| (they average
1/T, so an absolute 1e-4 bound would be vacuous), and each call's weights sum
to 1 within 1e-6.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-4, 1e-5
W_ATOL, W_RTOL, SUM_TOL = 1e-9, 1e-4, 1e-6


@pytest.fixture(scope="module")
def C_():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tritiercache_b200 import _C
    return _C


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint8)


def close(got, want, atol=ATOL, rtol=RTOL):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    lim = atol + rtol * np.abs(want.astype(np.float64))
    return bool(np.all(err <= lim)), float(err.max()) if err.size else 0.0


def weights_ok(got, want):
    ok, err = close(got, want, W_ATOL, W_RTOL)
    if not ok:
        return False, ("elementwise", err)
    if np.any(want != 0):
        tot = float(np.sum(got.astype(np.float64)))
        if abs(tot - 1.0) > SUM_TOL:
            return False, ("sum", tot)
    return True, err


def test_kat_quantize_v_on_gpu(C_, golden_dir):
    d = np.load(os.path.join(golden_dir, "kat_quantize_v.npz"))
    V = d["V"]
    T, H, D = V.shape
    p = torch.zeros((T, H, D // 16), dtype=torch.int32, device="cuda")
    s = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    z = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    C_.quantize_v_block(dev(V), p, s, z, H, D, T)
    assert np.array_equal(host(p).ravel().view(np.uint32), d["expected_packed"].view(np.uint32))
    assert np.all(np.abs(host(z).ravel() - d["expected_min"]) <= float(d["tolerance"]))
    assert np.all(np.abs(host(s).ravel() - d["expected_scale"]) <= float(d["tolerance"]))


def test_kat_round_half_to_even_on_gpu(C_, golden_dir):
    d = np.load(os.path.join(golden_dir, "kat_tie_v.npz"))
    p = torch.zeros((16, 1, 1), dtype=torch.int32, device="cuda")
    s = torch.zeros((16, 1), dtype=torch.float32, device="cuda")
    z = torch.zeros((16, 1), dtype=torch.float32, device="cuda")
    C_.quantize_v_block(dev(d["V"]), p, s, z, 1, 16, 16)
    w = int(host(p)[0, 0, 0]) & 0xFFFFFFFF
    for ch, want in zip(d["check_channels"], d["expected_codes"]):
        assert (w >> (2 * int(ch))) & 3 == int(want)


def test_quant_dequant_bit_exact_vs_reference_fixtures(C_, golden_dir):
    d = np.load(os.path.join(golden_dir, "ref_quant.npz"))
    for ci in range(int(d["ncases"])):
        grp, f16, H, D = (int(x) for x in d[f"c{ci}_cfg"])
        meta = "fp16" if f16 else "fp32"
        mdt = torch.int16 if f16 else torch.float32
        kp = torch.zeros((grp // 16, H, D), dtype=torch.int32, device="cuda")
        ks = torch.zeros((H, D), dtype=mdt, device="cuda")
        kz = torch.zeros((H, D), dtype=mdt, device="cuda")
        C_.quantize_k_block(dev(d[f"c{ci}_K"]), kp, ks, kz, H, D, grp, meta)
        assert np.array_equal(host(kp), d[f"c{ci}_kp"]), ci
        assert np.array_equal(bits(host(ks)), bits(d[f"c{ci}_ks"])), ci
        assert np.array_equal(bits(host(kz)), bits(d[f"c{ci}_kz"])), ci
        vq = torch.zeros((grp, H, D // 16), dtype=torch.int32, device="cuda")
        vs = torch.zeros((grp, H), dtype=mdt, device="cuda")
        vz = torch.zeros((grp, H), dtype=mdt, device="cuda")
        C_.quantize_v_block(dev(d[f"c{ci}_V"]), vq, vs, vz, H, D, grp, meta)
        assert np.array_equal(host(vq), d[f"c{ci}_vq"]), ci
        assert np.array_equal(bits(host(vs)), bits(d[f"c{ci}_vs"])), ci
        assert np.array_equal(bits(host(vz)), bits(d[f"c{ci}_vz"])), ci
        kd = torch.zeros((grp, H, D), dtype=torch.float32, device="cuda")
        C_.dequantize_k(dev(d[f"c{ci}_kp"]), dev(d[f"c{ci}_ks"]), dev(d[f"c{ci}_kz"]), kd, 1, H, D, grp, meta)
        assert np.array_equal(bits(host(kd)), bits(d[f"c{ci}_kd"])), ci
        vd = torch.zeros((grp, H, D), dtype=torch.float32, device="cuda")
        C_.dequantize_v(dev(d[f"c{ci}_vq"]), dev(d[f"c{ci}_vs"]), dev(d[f"c{ci}_vz"]), vd, grp, H, D, meta)
        assert np.array_equal(bits(host(vd)), bits(d[f"c{ci}_vd"])), ci


def test_host_buffers_are_staged_like_the_reference_binding(C_, golden_dir):
    # numpy arguments (the reference's own tests pass numpy arrays) run on the GPU
    d = np.load(os.path.join(golden_dir, "ref_quant.npz"))
    grp, f16, H, D = (int(x) for x in d["c1_cfg"])
    kp = np.zeros((grp // 16, H, D), np.int32)
    ks = np.zeros((H, D), np.uint16)
    kz = np.zeros((H, D), np.uint16)
    C_.quantize_k_block(d["c1_K"], kp, ks, kz, H, D, grp, "fp16")
    assert np.array_equal(kp, d["c1_kp"]) and np.array_equal(ks, d["c1_ks"]) and np.array_equal(kz, d["c1_kz"])


def test_quantize_fuzz_bit_exact_vs_oracle(C_):
    from oracle import oracle as O
    rng = np.random.default_rng(11)
    for trial in range(24):
        grp = int(rng.choice([16, 32]))
        f16 = bool(rng.integers(0, 2))
        H = int(rng.integers(1, 9))
        D = int(rng.choice([16, 32, 64, 128, 256]))
        scale = float(rng.choice([1e-6, 0.01, 1.0, 100.0, 1e4]))
        K = (rng.standard_normal((grp, H, D)) * scale).astype(np.float32)
        V = (rng.standard_normal((grp, H, D)) * scale).astype(np.float32)
        if trial % 5 == 0:
            K[:, 0, :3] = 1.5
            V[0, 0, :] = -3.0
        mnp = np.uint16 if f16 else np.float32
        mdt = torch.int16 if f16 else torch.float32
        meta = "fp16" if f16 else "fp32"
        ok = [np.zeros((grp // 16, H, D), np.int32), np.zeros((H, D), mnp), np.zeros((H, D), mnp)]
        O.quantize_k_block(K, *ok, H, D, grp)
        gk = [torch.zeros((grp // 16, H, D), dtype=torch.int32, device="cuda"),
              torch.zeros((H, D), dtype=mdt, device="cuda"), torch.zeros((H, D), dtype=mdt, device="cuda")]
        C_.quantize_k_block(dev(K), *gk, H, D, grp, meta)
        for a, b in zip(ok, gk):
            assert np.array_equal(bits(a), bits(host(b))), (trial, "K")
        ov = [np.zeros((grp, H, D // 16), np.int32), np.zeros((grp, H), mnp), np.zeros((grp, H), mnp)]
        O.quantize_v_block(V, *ov, H, D, grp)
        gv = [torch.zeros((grp, H, D // 16), dtype=torch.int32, device="cuda"),
              torch.zeros((grp, H), dtype=mdt, device="cuda"), torch.zeros((grp, H), dtype=mdt, device="cuda")]
        C_.quantize_v_block(dev(V), *gv, H, D, grp, meta)
        for a, b in zip(ov, gv):
            assert np.array_equal(bits(a), bits(host(b))), (trial, "V")


def _attn_gpu(C_, g, nq, nkv, hd, dc, nb, f16, grp):
    out = torch.zeros((nq, hd), dtype=torch.float32, device="cuda")
    mw = torch.zeros(dc + nb * grp, dtype=torch.float32, device="cuda")
    meta = "fp16" if f16 else "fp32"
    md = (lambda a: dev(a.view(np.int16))) if f16 else dev
    C_.fused_attention_decode(dev(g("Q")), dev(g("dK")), dev(g("dV")), dc, dev(g("kp")), md(g("ks")), md(g("kz")),
                              dev(g("vq")), md(g("vs")), md(g("vz")), dev(g("ids")), nb, nq, nkv, hd, out, mw, grp,
                              meta)
    return host(out), host(mw)


def test_fused_attention_vs_reference_fixtures(C_, golden_dir):
    d = np.load(os.path.join(golden_dir, "ref_attn.npz"))
    for ci in range(int(d["ncases"])):
        nq, nkv, hd, dc, nb, f16, grp = (int(x) for x in d[f"c{ci}_cfg"])
        g = lambda k: d[f"c{ci}_{k}"]
        out, mw = _attn_gpu(C_, g, nq, nkv, hd, dc, nb, f16, grp)
        ok, err = close(out, g("out"))
        assert ok, (ci, "out", err)
        ok, err = weights_ok(mw, g("mw"))
        assert ok, (ci, "mean weights", err)


@pytest.mark.parametrize("nq,nkv,hd,dc,nb,f16,grp,hole", [
    (32, 8, 128, 657, 100, 1, 16, 0),     # config-1 tiers at reduced length, GQA 4:1
    (32, 32, 128, 300, 61, 0, 16, 0),     # MHA (config 1 heads)
    (28, 4, 128, 200, 40, 1, 16, 9),      # G = 7 (config 5 heads), empty slots
    (32, 8, 128, 1886, 300, 1, 16, 0),    # config-2 dense tier size
    (8, 2, 64, 17, 33, 1, 32, 0),         # group 32
    (12, 3, 64, 5, 3, 0, 16, 2),          # odd kv-head count
    (16, 16, 256, 40, 8, 1, 16, 0),       # head_dim 256
    (4, 4, 16, 9, 2, 0, 16, 0),           # head_dim 16
])
def test_fused_attention_vs_oracle(C_, nq, nkv, hd, dc, nb, f16, grp, hole):
    from oracle import oracle as O
    rng = np.random.default_rng(nq * 1000 + nkv * 10 + hd + dc)
    Q = rng.standard_normal((nq, hd)).astype(np.float32)
    dK = rng.standard_normal((max(dc, 1), nkv, hd)).astype(np.float32)
    dV = rng.standard_normal((max(dc, 1), nkv, hd)).astype(np.float32)
    Kt = rng.standard_normal((nb * grp, nkv, hd)).astype(np.float32)
    Kt[:, :, rng.choice(hd, 4, replace=False)] *= 8.0
    Vt = rng.standard_normal((nb * grp, nkv, hd)).astype(np.float32)
    mnp = np.uint16 if f16 else np.float32
    kp = np.zeros((nb * grp // 16, nkv, hd), np.int32)
    ks = np.zeros((nb, nkv, hd), mnp)
    kz = np.zeros((nb, nkv, hd), mnp)
    vq = np.zeros((nb * grp, nkv, hd // 16), np.int32)
    vs = np.zeros((nb * grp, nkv), mnp)
    vz = np.zeros((nb * grp, nkv), mnp)
    w = grp // 16
    for b in range(nb):
        O.quantize_k_block(np.ascontiguousarray(Kt[b * grp:(b + 1) * grp]), kp[b * w:(b + 1) * w], ks[b], kz[b],
                           nkv, hd, grp)
        O.quantize_v_block(np.ascontiguousarray(Vt[b * grp:(b + 1) * grp]), vq[b * grp:(b + 1) * grp],
                           vs[b * grp:(b + 1) * grp], vz[b * grp:(b + 1) * grp], nkv, hd, grp)
    ids = np.arange(nb * grp, dtype=np.int64) + 7
    if hole:
        ids[::hole] = -1
    o_ref = np.zeros((nq, hd), np.float32)
    mw_ref = np.zeros(dc + nb * grp, np.float32)
    O.fused_attention_decode(Q, dK, dV, dc, kp, ks, kz, vq, vs, vz, ids, nb, nq, nkv, hd, o_ref, mw_ref, grp)
    arrs = dict(Q=Q, dK=dK, dV=dV, kp=kp, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, ids=ids)
    out, mw = _attn_gpu(C_, arrs.__getitem__, nq, nkv, hd, dc, nb, f16, grp)
    ok, err = close(out, o_ref)
    assert ok, ("out", err)
    ok, err = weights_ok(mw, mw_ref)
    assert ok, ("mean weights", err)


def test_fused_attention_edge_cases(C_):
    # zero tokens: output is zero (memset in fused_attn_avx2.cpp:265); argument validation
    out = torch.full((4, 64), 7.0, device="cuda")
    q = torch.randn(4, 64, device="cuda")
    C_.fused_attention_decode(q, None, None, 0, None, None, None, None, None, None, None, 0, 4, 2, 64, out)
    assert torch.count_nonzero(out).item() == 0
    with pytest.raises(ValueError):
        C_.fused_attention_decode(q, None, None, -1, None, None, None, None, None, None, None, 0, 4, 2, 64, out)
    with pytest.raises(ValueError):
        C_.fused_attention_decode(q, None, None, 0, None, None, None, None, None, None, None, -2, 4, 2, 64, out)
    with pytest.raises(ValueError):
        C_.fused_attention_decode(q, None, None, 0, None, None, None, None, None, None, None, 0, 0, 2, 64, out)
    with pytest.raises(ValueError):
        C_.fused_attention_decode(q.t(), None, None, 0, None, None, None, None, None, None, None, 0, 4, 2, 64, out)
