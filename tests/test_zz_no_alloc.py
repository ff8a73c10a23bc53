"""The allocation-free attention entry point against the allocating one.

tt_fused_attention_decode_noalloc exists for callers that must not allocate
device memory once they are running (memory reserved up front, an embedding
framework that owns the device allocator, loops where cudaMalloc's possible
device synchronisation is not allowed).  It uses a fixed scratch array in
device memory instead of the library's growable workspace.  This file checks,
through the C ABI, that two calls in a row agree with
tt_fused_attention_decode within the tolerance of the other attention tests,
and that a call needing more scratch than the array holds is refused with an
error instead of running.  It is collected last on purpose and also passes
when run alone.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-4, 1e-5


def _inputs(seed, nq, nkv, hd, dc, nb, grp):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    d = {}
    d["Q"] = torch.randn(nq, hd, device="cuda", generator=g)
    d["dK"] = torch.randn(max(dc, 1), nkv, hd, device="cuda", generator=g)
    d["dV"] = torch.randn(max(dc, 1), nkv, hd, device="cuda", generator=g)
    d["kp"] = torch.randint(-2 ** 31, 2 ** 31 - 1, (max(nb, 1) * grp // 16, nkv, hd), dtype=torch.int32,
                            device="cuda", generator=g)
    d["ks"] = (torch.rand(max(nb, 1), nkv, hd, device="cuda", generator=g) * 0.5).half()
    d["kz"] = torch.randn(max(nb, 1), nkv, hd, device="cuda", generator=g).half()
    d["vp"] = torch.randint(-2 ** 31, 2 ** 31 - 1, (max(nb, 1) * grp, nkv, hd // 16), dtype=torch.int32,
                            device="cuda", generator=g)
    d["vs"] = (torch.rand(max(nb, 1) * grp, nkv, device="cuda", generator=g) * 0.5).half()
    d["vz"] = torch.randn(max(nb, 1) * grp, nkv, device="cuda", generator=g).half()
    ids = torch.arange(max(nb, 1) * grp, dtype=torch.int64, device="cuda")
    ids[::5] = -1
    d["ids"] = ids
    return d


def _call(fn, d, nq, nkv, hd, dc, nb, grp):
    out = torch.full((nq, hd), float("nan"), device="cuda")
    mw = torch.full((dc + nb * grp,), float("nan"), device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    st = fn(p(d["Q"]), p(d["dK"]), p(d["dV"]), dc, p(d["kp"]), p(d["ks"]), p(d["kz"]), p(d["vp"]), p(d["vs"]),
            p(d["vz"]), p(d["ids"]), nb, nq, nkv, hd, p(out), p(mw), grp, 1,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return st, out, mw


def _close(a, b, atol=ATOL, rtol=RTOL):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    return bool(np.all(np.abs(a - b) <= atol + rtol * np.abs(b))), float(np.abs(a - b).max())


def test_no_alloc_entry_point_matches_allocating_one_on_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tritiercache_b200 import _lib
    L = _lib.lib()
    # two consecutive calls with different shapes: the second must not see the
    # first call's leftovers in the shared scratch array
    cases = [(32, 8, 128, 300, 100, 16, 11), (28, 4, 128, 45, 61, 32, 12)]
    for nq, nkv, hd, dc, nb, grp, seed in cases:
        d = _inputs(seed, nq, nkv, hd, dc, nb, grp)
        st, ref_out, ref_mw = _call(L.tt_fused_attention_decode, d, nq, nkv, hd, dc, nb, grp)
        assert st == 0, L.tt_last_error()
        st, out, mw = _call(L.tt_fused_attention_decode_noalloc, d, nq, nkv, hd, dc, nb, grp)
        assert st == 0, L.tt_last_error()
        torch.cuda.synchronize()
        ok, err = _close(out, ref_out)
        assert ok, ("attention output", err)
        ok, err = _close(mw, ref_mw, 1e-9, 1e-4)  # relative: the weights average 1/T
        assert ok, ("mean weights", err)
    err = ctypes.c_int(-1)
    assert L.tt_device_error(1, ctypes.byref(err)) == 0 and err.value == 0


def test_no_alloc_entry_point_allocates_nothing():
    """After one warm-up call (which loads the module holding the scratch array
    and every kernel the calls use), a larger call -- more scratch than the
    warm-up needed -- leaves the device's free memory unchanged."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tritiercache_b200 import _lib
    L = _lib.lib()
    small = (32, 8, 128, 300, 100, 16)
    large = (32, 8, 128, 1886, 3000, 16)
    ds = _inputs(21, *small)
    dl = _inputs(22, *large)
    st, _, _ = _call(L.tt_fused_attention_decode_noalloc, ds, *small)
    assert st == 0, L.tt_last_error()
    nq, nkv, hd, dc, nb, grp = large
    out = torch.empty((nq, hd), device="cuda")
    mw = torch.empty((dc + nb * grp,), device="cuda")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    st = L.tt_fused_attention_decode_noalloc(p(dl["Q"]), p(dl["dK"]), p(dl["dV"]), dc, p(dl["kp"]), p(dl["ks"]),
                                             p(dl["kz"]), p(dl["vp"]), p(dl["vs"]), p(dl["vz"]), p(dl["ids"]), nb,
                                             nq, nkv, hd, p(out), p(mw), grp, 1,
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, L.tt_last_error()
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, ("device memory changed across a no-alloc call", free0, free1)
    assert torch.isfinite(out).all()


def test_no_alloc_entry_point_refuses_calls_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tritiercache_b200 import _lib
    L = _lib.lib()
    # 64 query heads x 160k tokens of logits alone exceed the 32 MiB array; the
    # size check runs on the host before any kernel is launched (the buffers
    # are sized for the request all the same)
    nb = 10000
    d = _inputs(3, 64, 8, 128, 1, nb, 16)
    st, _, _ = _call(L.tt_fused_attention_decode_noalloc, d, 64, 8, 128, 0, nb, 16)
    assert st == _lib.TT_ERR_INVALID_ARGUMENT
    assert b"scratch" in L.tt_last_error()
