"""ctypes binding of libtritier_b200.so (the C ABI in include/tritier_b200.h).

The library is the only compute path: if it cannot be loaded, or no CUDA
device is present when a kernel is called, the call raises -- there is no
CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtritier_b200.so")

TT_OK = 0
TT_ERR_INVALID_ARGUMENT = 1
TT_ERR_OUT_OF_RANGE = 2
TT_ERR_OUT_OF_MEMORY = 3
TT_ERR_CUDA = 4
TT_ERR_TIMEOUT = 5
TT_ERR_UNSUPPORTED = 6

# Exception mapping of the reference binding (csrc/bindings.cpp:321-337).
_EXC = {
    TT_ERR_INVALID_ARGUMENT: ValueError,
    TT_ERR_UNSUPPORTED: ValueError,
    TT_ERR_OUT_OF_RANGE: IndexError,
    TT_ERR_OUT_OF_MEMORY: MemoryError,
    TT_ERR_CUDA: RuntimeError,
    TT_ERR_TIMEOUT: RuntimeError,
}


class EngineConfig(C.Structure):
    _fields_ = [("num_q_heads", C.c_int), ("num_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("max_seq_len", C.c_int), ("sink_size", C.c_int), ("rw_size", C.c_int),
                ("h_ratio", C.c_float), ("score_decay", C.c_float), ("update_interval", C.c_int),
                ("k_group_size", C.c_int), ("meta_fp16", C.c_int), ("device", C.c_int)]


class EngineCounters(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "s_count", "rw_count", "rw_head_index", "hh_count", "wr_count", "pbs_allocated_blocks",
        "pbs_blocks_used", "pbs_count", "total_processed_tokens", "total_evictions", "last_calc_pos",
        "max_hh", "chunk_size")] + [("cached_threshold", C.c_float)]


class KernelTimes(C.Structure):
    _fields_ = [("maintain_ms", C.c_double), ("partial_ms", C.c_double), ("finalize_ms", C.c_double),
                ("maintain_launches", C.c_int), ("partial_launches", C.c_int), ("finalize_launches", C.c_int)]


class BufferDesc(C.Structure):
    _fields_ = [("data", C.c_void_p), ("count", C.c_size_t), ("elem_size", C.c_int), ("dtype", C.c_int)]


EXPORTS = [
    "tt_last_error", "tt_version", "tt_pointer_is_device", "tt_fused_attention_decode", "tt_quantize_k_block",
    "tt_quantize_v_block", "tt_dequantize_k", "tt_dequantize_v", "tt_engine_create",
    "tt_engine_destroy", "tt_engine_step", "tt_engine_step_batched", "tt_engine_prefill",
    "tt_engine_get_counters", "tt_engine_get_buffer", "tt_engine_get_buffer_bytes",
    "tt_engine_device_bytes", "tt_engine_set_counters", "tt_profile_enable", "tt_profile_collect",
    "tt_device_error", "tt_fused_attention_decode_noalloc", "tt_engine_step_sharded_begin",
    "tt_engine_step_sharded_merge", "tt_engine_sharded_sync_needed", "tt_engine_sharded_scores_floats",
    "tt_engine_sharded_scores_pack", "tt_engine_sharded_scores_unpack", "tt_sharded_xch_create",
    "tt_sharded_xch_open", "tt_sharded_xch_destroy", "tt_engine_step_sharded_begin_xch",
    "tt_engine_step_sharded_merge_xch",
    "tt_engine_ingest", "tt_engine_full_count", "tt_engine_reconstruct", "tt_engine_accumulate_scores",
]

_lib = None
_lock = threading.Lock()


def _declare(L):
    vp, i, f = C.c_void_p, C.c_int, C.c_float
    L.tt_last_error.restype = C.c_char_p
    L.tt_last_error.argtypes = []
    L.tt_version.restype = C.c_char_p
    L.tt_version.argtypes = []
    L.tt_pointer_is_device.restype = C.c_int
    L.tt_pointer_is_device.argtypes = [vp]
    L.tt_fused_attention_decode.argtypes = [vp, vp, vp, i, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, vp, vp, i, i, vp]
    L.tt_quantize_k_block.argtypes = [vp, vp, vp, vp, i, i, i, i, vp]
    L.tt_quantize_v_block.argtypes = [vp, vp, vp, vp, i, i, i, i, vp]
    L.tt_dequantize_k.argtypes = [vp, vp, vp, vp, i, i, i, i, i, vp]
    L.tt_dequantize_v.argtypes = [vp, vp, vp, vp, i, i, i, i, vp]
    L.tt_engine_create.argtypes = [C.POINTER(EngineConfig), C.POINTER(vp)]
    L.tt_engine_destroy.argtypes = [vp]
    L.tt_engine_step.argtypes = [vp, vp, vp, vp, vp, vp]
    L.tt_engine_step_batched.argtypes = [C.POINTER(vp), i, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp),
                                         C.POINTER(vp), vp]
    L.tt_engine_prefill.argtypes = [vp, vp, vp, i, vp]
    L.tt_engine_get_counters.argtypes = [vp, C.POINTER(EngineCounters)]
    L.tt_engine_get_buffer.argtypes = [vp, i, C.POINTER(BufferDesc)]
    L.tt_engine_get_buffer_bytes.argtypes = [vp, C.POINTER(C.c_size_t)]
    L.tt_engine_device_bytes.argtypes = [vp, C.POINTER(C.c_size_t)]
    L.tt_engine_set_counters.argtypes = [vp, C.POINTER(EngineCounters), vp]
    L.tt_profile_enable.argtypes = [i]
    L.tt_profile_collect.argtypes = [C.POINTER(KernelTimes)]
    L.tt_device_error.argtypes = [i, C.POINTER(i)]
    L.tt_fused_attention_decode_noalloc.argtypes = [vp, vp, vp, i, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, vp, vp, i,
                                                    i, vp]
    pv = C.POINTER(vp)
    L.tt_engine_step_sharded_begin.argtypes = [pv, i, pv, pv, pv, i, i, vp, vp, vp]
    L.tt_engine_step_sharded_merge.argtypes = [pv, i, i, i, vp, pv, vp, vp]
    L.tt_engine_sharded_sync_needed.argtypes = [pv, i, C.POINTER(i)]
    L.tt_engine_sharded_scores_floats.argtypes = [pv, i, C.POINTER(C.c_longlong)]
    L.tt_engine_sharded_scores_pack.argtypes = [pv, i, i, i, vp, vp]
    L.tt_engine_sharded_scores_unpack.argtypes = [pv, i, vp, vp]
    L.tt_sharded_xch_create.argtypes = [i, i, i, i, i, i, C.POINTER(vp), vp]
    L.tt_sharded_xch_open.argtypes = [vp, vp]
    L.tt_sharded_xch_destroy.argtypes = [vp]
    L.tt_engine_step_sharded_begin_xch.argtypes = [pv, i, pv, pv, pv, vp, i, vp]
    L.tt_engine_step_sharded_merge_xch.argtypes = [pv, i, vp, pv, vp]
    L.tt_engine_ingest.argtypes = [vp, vp, vp, vp]
    L.tt_engine_full_count.argtypes = [vp, C.POINTER(i)]
    L.tt_engine_reconstruct.argtypes = [vp, vp, vp, vp, i, C.POINTER(i), vp]
    L.tt_engine_accumulate_scores.argtypes = [vp, vp, vp, i, i, vp]
    for name in EXPORTS:
        if name not in ("tt_last_error", "tt_version"):
            getattr(L, name).restype = C.c_int


def lib():
    """Loads libtritier_b200.so (raises ImportError when it is missing)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is not built; run `python -m tritiercache_b200.csrc.build` "
                        "(nvcc, sm_100a).")
                L = C.CDLL(LIB_PATH)
                _declare(L)
                _lib = L
    return _lib


def check(status: int, what: str = "") -> None:
    if status == TT_OK:
        return
    msg = lib().tt_last_error().decode(errors="replace")
    exc = _EXC.get(status, RuntimeError)
    raise exc(f"{what}: {msg}" if what and not msg.startswith(what) else msg)
