"""CPU checks of the drop-in boundary (no GPU needed, no compute calls).

* libtritier_b200.so builds for sm_100a and exports every entry point that
  include/tritier_b200.h declares;
* the Python `_C` mirror exposes the reference module's surface
  (src/tri_tier/cli.py:153-160 lists it);
* without a CUDA device the product path raises instead of falling back.
"""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tritier_b200.h")


@pytest.fixture(scope="module")
def libpath():
    from tritiercache_b200.csrc import build
    return build.build()


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tt_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_reference_surface():
    names = declared_symbols()
    for n in ["tt_fused_attention_decode", "tt_quantize_k_block", "tt_quantize_v_block", "tt_dequantize_k",
              "tt_dequantize_v", "tt_engine_create", "tt_engine_destroy", "tt_engine_step", "tt_engine_prefill",
              "tt_engine_get_counters", "tt_engine_get_buffer", "tt_engine_get_buffer_bytes", "tt_last_error"]:
        assert n in names


def test_library_exports_every_declared_symbol(libpath):
    lib = ctypes.CDLL(libpath)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (tt_[a-z0-9_]+)", out))
    assert exported == set(declared_symbols()), exported ^ set(declared_symbols())


def test_build_targets_sm100a_without_fast_math():
    from tritiercache_b200.csrc import build
    flags = " ".join(build.FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags
    assert "fast-math" not in flags and "fast_math" not in flags  # IEEE division is part of the contract


def test_python_mirror_exposes_reference_module_surface():
    from tritiercache_b200 import _C
    for n in ["TriTierCacheEngine", "fused_attention_decode", "quantize_k_block", "quantize_v_block",
              "dequantize_k", "dequantize_v"]:
        assert hasattr(_C, n)
    import inspect
    sig = inspect.signature(_C.fused_attention_decode)
    assert list(sig.parameters)[:4] == ["Q_ptr", "dense_K_ptr", "dense_V_ptr", "dense_count"]
    assert sig.parameters["k_group_size"].default == 16
    assert sig.parameters["pbs_metadata_dtype"].default == "fp32"
    esig = inspect.signature(_C.TriTierCacheEngine.__init__)
    assert esig.parameters["rw_size"].default == 64 and esig.parameters["update_interval"].default == 16
    assert esig.parameters["pbs_metadata_dtype"].default == "fp16"


def test_version_and_error_string_without_gpu(libpath):
    from tritiercache_b200 import _lib
    L = _lib.lib()
    assert b"sm_100a" in L.tt_version()
    # argument validation happens on the host before any device work
    st = L.tt_quantize_k_block(None, None, None, None, 0, 64, 16, 0, None)
    assert st == _lib.TT_ERR_INVALID_ARGUMENT
    assert b"positive" in L.tt_last_error()
    st = L.tt_fused_attention_decode(None, None, None, -1, None, None, None, None, None, None, None, 0, 4, 2, 64,
                                     None, None, 16, 0, None)
    assert st == _lib.TT_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.check(st, "fused_attention_decode")


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback_without_cuda():
    import numpy as np
    from tritiercache_b200 import _C
    K = np.zeros((16, 2, 32), np.float32)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.quantize_k_block(K, np.zeros((1, 2, 32), np.int32), np.zeros((2, 32), np.float32),
                            np.zeros((2, 32), np.float32), 2, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.TriTierCacheEngine(4, 2, 32, 128)
    from tritiercache_b200 import TriTierCache
    with pytest.raises(RuntimeError):
        TriTierCache(128, 32, 2, 16, 0.1)


def test_sharded_entry_points_validate_on_the_host(libpath):
    """The sequence-sharded calls refuse bad arguments before any device work."""
    import ctypes as C
    from tritiercache_b200 import _lib
    L = _lib.lib()
    x = C.c_void_p()
    h = (C.c_char * 64)()
    for world, rank in ((1, 0), (9, 0), (2, 2), (2, -1)):  # the peer exchange takes 2..8 ranks
        assert L.tt_sharded_xch_create(world, rank, 4, 32, 128, 0, C.byref(x), h) == _lib.TT_ERR_INVALID_ARGUMENT
    assert b"ranks" in L.tt_last_error()
    assert L.tt_sharded_xch_create(2, 0, 0, 32, 128, 0, C.byref(x), h) == _lib.TT_ERR_INVALID_ARGUMENT
    assert L.tt_sharded_xch_create(2, 0, 4, 32, 128, 0, None, h) == _lib.TT_ERR_INVALID_ARGUMENT
    assert L.tt_sharded_xch_open(None, None) == _lib.TT_ERR_INVALID_ARGUMENT
    assert L.tt_sharded_xch_destroy(None) == 0
    need = C.c_int(-1)
    assert L.tt_engine_sharded_sync_needed(None, 1, C.byref(need)) == _lib.TT_ERR_INVALID_ARGUMENT
    f = C.c_longlong(-1)
    assert L.tt_engine_sharded_scores_floats(None, 1, C.byref(f)) == _lib.TT_ERR_INVALID_ARGUMENT
    assert L.tt_engine_step_sharded_begin(None, 1, None, None, None, 0, 2, None, None, None) == \
        _lib.TT_ERR_INVALID_ARGUMENT
    assert L.tt_engine_step_sharded_merge(None, 1, 0, 2, None, None, None, None) == _lib.TT_ERR_INVALID_ARGUMENT
    assert L.tt_engine_step_sharded_begin_xch(None, 1, None, None, None, None, 0, None) == \
        _lib.TT_ERR_INVALID_ARGUMENT
    assert L.tt_engine_step_sharded_merge_xch(None, 1, None, None, None) == _lib.TT_ERR_INVALID_ARGUMENT
    # nothing to do for an empty batch
    assert L.tt_engine_step_sharded_begin(None, 0, None, None, None, 0, 2, None, None, None) == 0
