"""Drop-in for the reference extension module ``tri_tier._C`` (csrc/bindings.cpp).

Same callables, argument names, defaults and exception types as
``bindings.cpp:317-627``, implemented over the C ABI of libtritier_b200.so
(include/tritier_b200.h).  Every computation runs in the sm_100a kernels; when
the library or a CUDA device is missing the calls raise.

Argument rules follow ``get_contiguous_ptr`` (bindings.cpp:25-97): an argument
may be a raw integer address, a tensor exposing ``data_ptr()`` /
``is_contiguous()``, an object with ``__cuda_array_interface__`` or a
C-contiguous buffer (numpy).  Device memory is used in place.  Host memory
(numpy arrays, CPU tensors, host addresses) is staged through device memory:
inputs are copied in, outputs are copied back before the call returns, so the
reference's own numpy-based call sites keep working.  Kernels run on the
current torch CUDA stream of the device.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, lib

__all__ = ["fused_attention_decode", "quantize_k_block", "quantize_v_block", "dequantize_k",
           "dequantize_v", "TriTierCacheEngine", "engine_step_batched"]

_DT_BYTES = {"f32": 4, "i32": 4, "i64": 8, "u16": 2}
_TORCH_DT = {"f32": torch.float32, "i32": torch.int32, "i64": torch.int64, "u16": torch.int16}


def _require_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("tritiercache_b200 needs a CUDA device (B200, sm_100a); no CPU fallback exists.")
    lib()


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


class _Arg:
    """Resolved pointer argument: device address plus optional staging."""

    __slots__ = ("ptr", "host_ptr", "stage", "nbytes", "writable")

    def __init__(self):
        self.ptr = 0
        self.host_ptr = 0
        self.stage = None
        self.nbytes = 0
        self.writable = False

    def finish(self):
        if self.stage is not None and self.writable and self.nbytes:
            host = self.stage.cpu()  # synchronises the stream
            C.memmove(self.host_ptr, host.data_ptr(), self.nbytes)


def _stage_host(addr: int, nbytes: int, writable: bool) -> _Arg:
    a = _Arg()
    a.host_ptr, a.nbytes, a.writable = addr, nbytes, writable
    n = max(nbytes, 1)
    host = torch.empty(n, dtype=torch.uint8)
    if nbytes:
        C.memmove(host.data_ptr(), addr, nbytes)
    a.stage = host.to("cuda", non_blocking=False)
    a.ptr = a.stage.data_ptr()
    return a


def _arg(obj, name: str, nbytes: int, writable: bool = False, nullable: bool = False) -> _Arg:
    a = _Arg()
    if obj is None:
        if nullable:
            return a
        raise ValueError(f"Argument '{name}' cannot be None.")
    if isinstance(obj, (int, np.integer)) and not isinstance(obj, bool):
        addr = int(obj)
        if addr == 0:
            if nullable:
                return a
            raise ValueError(f"Argument '{name}' pointer address is NULL.")
        if lib().tt_pointer_is_device(C.c_void_p(addr)):
            a.ptr = addr
            return a
        return _stage_host(addr, nbytes, writable)
    if hasattr(obj, "data_ptr") and hasattr(obj, "is_contiguous"):
        if not obj.is_contiguous():
            raise ValueError(f"Argument '{name}' PyTorch tensor is not contiguous in memory. "
                             "Call .contiguous() before passing.")
        addr = int(obj.data_ptr())
        if addr == 0 and not nullable:
            raise ValueError(f"Argument '{name}' tensor data pointer is NULL.")
        if getattr(obj, "is_cuda", False):
            a.ptr = addr
            return a
        return _stage_host(addr, nbytes, writable) if addr else a
    cai = getattr(obj, "__cuda_array_interface__", None)
    if cai is not None:
        if cai.get("strides") not in (None,):
            shape, strides = cai["shape"], cai["strides"]
            item = np.dtype(cai["typestr"]).itemsize
            exp = item
            for d in range(len(shape) - 1, -1, -1):
                if shape[d] > 1 and strides[d] != exp:
                    raise ValueError(f"Argument '{name}' buffer is not C-contiguous in memory.")
                exp *= shape[d]
        a.ptr = int(cai["data"][0])
        if a.ptr == 0 and not nullable:
            raise ValueError(f"Argument '{name}' buffer data pointer is NULL.")
        return a
    try:
        mv = memoryview(obj)
    except TypeError:
        raise ValueError(f"Argument '{name}' has unsupported type '{type(obj)}'. Expected PyTorch tensor, "
                         "NumPy array, buffer object, or integer memory address.") from None
    if not mv.c_contiguous:
        raise ValueError(f"Argument '{name}' buffer is not C-contiguous in memory.")
    arr = np.asarray(obj)
    if writable and not arr.flags.writeable:
        raise ValueError(f"Argument '{name}' buffer is read-only.")
    addr = arr.__array_interface__["data"][0]
    if addr == 0:
        if nullable:
            return a
        raise ValueError(f"Argument '{name}' buffer data pointer is NULL.")
    return _stage_host(addr, min(nbytes, arr.nbytes) if nbytes else arr.nbytes, writable)


def _is_fp16(obj, pbs_metadata_dtype: str) -> bool:
    # bindings.cpp:130-136: the string says "fp16", or the scales' dtype
    # string contains "float16" / "half".
    fp16 = pbs_metadata_dtype == "fp16"
    dt = getattr(obj, "dtype", None)
    if dt is not None:
        s = str(dt)
        if "float16" in s or "half" in s:
            fp16 = True
    return fp16


def _finish(*args):
    for a in args:
        a.finish()


def fused_attention_decode(Q_ptr, dense_K_ptr, dense_V_ptr, dense_count, PBS_K_Packed_ptr, PBS_K_Scales_ptr,
                           PBS_K_Zeroes_ptr, PBS_V_Packed_ptr, PBS_V_Scales_ptr, PBS_V_Zeroes_ptr,
                           PBS_token_ids_ptr, num_blocks, num_q_heads, num_kv_heads, head_dim, attn_output_ptr,
                           mean_attn_weights_ptr=None, k_group_size=16, pbs_metadata_dtype="fp32"):
    """Fused decode attention (bindings.cpp:99-178, :340-363)."""
    if dense_count < 0:
        raise ValueError("dense_count must be non-negative.")
    if num_blocks < 0:
        raise ValueError("num_blocks must be non-negative.")
    if num_q_heads <= 0 or num_kv_heads <= 0 or head_dim <= 0:
        raise ValueError("num_q_heads, num_kv_heads, and head_dim must be positive integers.")
    _require_cuda()
    fp16 = _is_fp16(PBS_K_Scales_ptr, pbs_metadata_dtype)
    mb = 2 if fp16 else 4
    grp = int(k_group_size)
    kvs = num_kv_heads * head_dim
    qhd = (head_dim + 15) // 16
    ntok = num_blocks * grp
    z = num_blocks == 0
    q = _arg(Q_ptr, "Q", num_q_heads * head_dim * 4)
    dk = _arg(dense_K_ptr, "dense_K", dense_count * kvs * 4, nullable=dense_count == 0)
    dv = _arg(dense_V_ptr, "dense_V", dense_count * kvs * 4, nullable=dense_count == 0)
    kp = _arg(PBS_K_Packed_ptr, "PBS_K_Packed", num_blocks * max(grp // 16, 1) * kvs * 4, nullable=z)
    vp = _arg(PBS_V_Packed_ptr, "PBS_V_Packed", ntok * num_kv_heads * qhd * 4, nullable=z)
    ids = _arg(PBS_token_ids_ptr, "PBS_token_ids", ntok * 8, nullable=z)
    out = _arg(attn_output_ptr, "attn_output", num_q_heads * head_dim * 4, writable=True)
    mw = _arg(mean_attn_weights_ptr, "mean_attn_weights", (dense_count + ntok) * 4, writable=True, nullable=True)
    ks = _arg(PBS_K_Scales_ptr, "PBS_K_Scales", num_blocks * kvs * mb, nullable=z)
    kz = _arg(PBS_K_Zeroes_ptr, "PBS_K_Zeroes", num_blocks * kvs * mb, nullable=z)
    vs = _arg(PBS_V_Scales_ptr, "PBS_V_Scales", ntok * num_kv_heads * mb, nullable=z)
    vz = _arg(PBS_V_Zeroes_ptr, "PBS_V_Zeroes", ntok * num_kv_heads * mb, nullable=z)
    st = lib().tt_fused_attention_decode(q.ptr, dk.ptr, dv.ptr, dense_count, kp.ptr, ks.ptr, kz.ptr, vp.ptr,
                                         vs.ptr, vz.ptr, ids.ptr, num_blocks, num_q_heads, num_kv_heads, head_dim,
                                         out.ptr, mw.ptr, grp, 1 if fp16 else 0, _stream())
    check(st, "fused_attention_decode")
    _finish(out, mw)


def quantize_k_block(K, packed, scale, zero, num_heads, head_dim, k_group_size=16, pbs_metadata_dtype="fp32"):
    """2-bit channel-wise K block quantization (bindings.cpp:180-212)."""
    _require_cuda()
    fp16 = _is_fp16(scale, pbs_metadata_dtype)
    mb = 2 if fp16 else 4
    n = num_heads * head_dim
    a_k = _arg(K, "K", k_group_size * n * 4)
    a_p = _arg(packed, "packed", max(k_group_size // 16, 1) * n * 4, writable=True)
    a_s = _arg(scale, "scale", n * mb, writable=True)
    a_z = _arg(zero, "zero", n * mb, writable=True)
    check(lib().tt_quantize_k_block(a_k.ptr, a_p.ptr, a_s.ptr, a_z.ptr, num_heads, head_dim, k_group_size,
                                    1 if fp16 else 0, _stream()), "quantize_k_block")
    _finish(a_p, a_s, a_z)


def quantize_v_block(V, packed, scale, zero, num_heads, head_dim, chunk_size=16, pbs_metadata_dtype="fp32"):
    """2-bit token-wise V quantization (bindings.cpp:214-246)."""
    _require_cuda()
    fp16 = _is_fp16(scale, pbs_metadata_dtype)
    mb = 2 if fp16 else 4
    qhd = (head_dim + 15) // 16
    a_v = _arg(V, "V", chunk_size * num_heads * head_dim * 4)
    a_p = _arg(packed, "packed", chunk_size * num_heads * qhd * 4, writable=True)
    a_s = _arg(scale, "scale", chunk_size * num_heads * mb, writable=True)
    a_z = _arg(zero, "zero", chunk_size * num_heads * mb, writable=True)
    check(lib().tt_quantize_v_block(a_v.ptr, a_p.ptr, a_s.ptr, a_z.ptr, num_heads, head_dim, chunk_size,
                                    1 if fp16 else 0, _stream()), "quantize_v_block")
    _finish(a_p, a_s, a_z)


def dequantize_k(packed, scale, zero, out, num_blocks, num_heads, head_dim, k_group_size=16,
                 pbs_metadata_dtype="fp32"):
    """K dequantization (bindings.cpp:248-281)."""
    _require_cuda()
    fp16 = _is_fp16(scale, pbs_metadata_dtype)
    mb = 2 if fp16 else 4
    n = num_heads * head_dim
    a_p = _arg(packed, "packed", num_blocks * max(k_group_size // 16, 1) * n * 4)
    a_o = _arg(out, "out", num_blocks * k_group_size * n * 4, writable=True)
    a_s = _arg(scale, "scale", num_blocks * n * mb)
    a_z = _arg(zero, "zero", num_blocks * n * mb)
    check(lib().tt_dequantize_k(a_p.ptr, a_s.ptr, a_z.ptr, a_o.ptr, num_blocks, num_heads, head_dim, k_group_size,
                                1 if fp16 else 0, _stream()), "dequantize_k")
    _finish(a_o)


def dequantize_v(packed, scale, zero, out, total_tokens, num_heads, head_dim, pbs_metadata_dtype="fp32"):
    """V dequantization (bindings.cpp:283-315)."""
    _require_cuda()
    fp16 = _is_fp16(scale, pbs_metadata_dtype)
    mb = 2 if fp16 else 4
    qhd = (head_dim + 15) // 16
    a_p = _arg(packed, "packed", total_tokens * num_heads * qhd * 4)
    a_o = _arg(out, "out", total_tokens * num_heads * head_dim * 4, writable=True)
    a_s = _arg(scale, "scale", total_tokens * num_heads * mb)
    a_z = _arg(zero, "zero", total_tokens * num_heads * mb)
    check(lib().tt_dequantize_v(a_p.ptr, a_s.ptr, a_z.ptr, a_o.ptr, total_tokens, num_heads, head_dim,
                                1 if fp16 else 0, _stream()), "dequantize_v")
    _finish(a_o)


class _DeviceView:
    """__cuda_array_interface__ over engine memory; keeps the engine alive."""

    def __init__(self, ptr: int, shape, typestr: str, owner):
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None,
                                         "stream": None}


_BUF = {"S_K": 0, "S_V": 1, "RW_K": 2, "RW_V": 3, "HH_K": 4, "HH_V": 5, "HH_token_ids": 6, "HH_scores": 7,
        "WR_K": 8, "WR_V": 9, "WR_token_ids": 10, "PBS_K_Packed": 11, "PBS_K_Scales": 12, "PBS_K_Zeroes": 13,
        "PBS_V_Packed": 14, "PBS_V_Scales": 15, "PBS_V_Zeroes": 16, "PBS_token_ids": 17,
        "global_attn_scores": 18}
_TYPESTR = {0: "<f4", 1: "<i4", 2: "<i8", 3: "<u2"}


class TriTierCacheEngine:
    """Device-resident TriTierCache engine (bindings.cpp:383-627, cache_engine.h:10-123).

    Tier buffers live in GPU memory; ``get_*`` return zero-copy CUDA tensors
    (the reference returns writable numpy views, bindings.cpp:461-626).  The
    counter attributes read the device state and therefore wait for the
    engine's last stream.
    """

    def __init__(self, num_q_heads, num_kv_heads, head_dim, max_seq_len, sink_size=4, rw_size=64, h_ratio=0.1,
                 score_decay=0.999, update_interval=16, k_group_size=16, pbs_metadata_dtype="fp16", device=None):
        _require_cuda()
        dev = torch.cuda.current_device() if device is None else torch.device(device).index or 0
        self._h = None
        cfg = _lib.EngineConfig(int(num_q_heads), int(num_kv_heads), int(head_dim), int(max_seq_len),
                                int(sink_size), int(rw_size), float(h_ratio), float(score_decay),
                                int(update_interval), int(k_group_size),
                                1 if pbs_metadata_dtype == "fp16" else 0, int(dev))
        h = C.c_void_p()
        with torch.cuda.device(dev):
            check(lib().tt_engine_create(C.byref(cfg), C.byref(h)), "TriTierCacheEngine")
        self._h = h
        self._dev = dev
        self.num_q_heads = int(num_q_heads)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.max_seq_len = int(max_seq_len)
        self.sink_size = int(sink_size)
        self.rw_size = int(rw_size)
        self.h_ratio = float(np.float32(h_ratio))
        self.score_decay = float(np.float32(score_decay))
        self.update_interval = int(update_interval)
        self.k_group_size = 32 if int(k_group_size) == 32 else 16
        self.chunk_size = self.k_group_size
        self.pbs_metadata_dtype = pbs_metadata_dtype
        self.use_fp16_meta = pbs_metadata_dtype == "fp16"
        self.quant_head_dim = (self.head_dim + 15) // 16
        self.device = torch.device("cuda", dev)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().tt_engine_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self) -> int:
        return self._h.value

    # -- compute --------------------------------------------------------------
    def step(self, q_ptr, k_ptr, v_ptr, out_ptr):
        """Ingest one token, attend, update scores (bindings.cpp:399-417)."""
        kvs = self.num_kv_heads * self.head_dim
        q = _arg(q_ptr, "Q", self.num_q_heads * self.head_dim * 4)
        k = _arg(k_ptr, "K_new", kvs * 4)
        v = _arg(v_ptr, "V_new", kvs * 4)
        o = _arg(out_ptr, "attn_output", self.num_q_heads * self.head_dim * 4, writable=True)
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_step(self._h, q.ptr, k.ptr, v.ptr, o.ptr, _stream()), "step")
        _finish(o)
        self._keep = (q, k, v)

    def prefill(self, k_ptr, v_ptr, q_len):
        """Batch prompt ingestion (bindings.cpp:418-436)."""
        if q_len < 0:
            raise ValueError("q_len must be non-negative.")
        kvs = self.num_kv_heads * self.head_dim
        k = _arg(k_ptr, "K_all", q_len * kvs * 4)
        v = _arg(v_ptr, "V_all", q_len * kvs * 4)
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_prefill(self._h, k.ptr, v.ptr, int(q_len), _stream()), "prefill")
        self._keep = (k, v)

    # -- state ------------------------------------------------------------------
    def counters(self) -> dict:
        c = _lib.EngineCounters()
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_get_counters(self._h, C.byref(c)), "counters")
        return {n: getattr(c, n) for n, _ in _lib.EngineCounters._fields_}

    def set_counters(self, **kw) -> None:
        """Overwrite integer state (tt_engine_set_counters), stream-ordered on
        the current stream: with the writable buffer views this imports a tier
        layout built elsewhere.  Fields not given keep their current values.
        No reference counterpart (its counters are read-only, bindings.cpp:437-458)."""
        c = _lib.EngineCounters()
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_get_counters(self._h, C.byref(c)), "counters")
            for k, v in kw.items():
                if not hasattr(c, k):
                    raise ValueError(f"unknown counter '{k}'")
                setattr(c, k, v)
            check(lib().tt_engine_set_counters(self._h, C.byref(c), _stream()), "set_counters")

    def _ctr(self, name):
        return self.counters()[name]

    s_count = property(lambda self: self._ctr("s_count"))
    rw_count = property(lambda self: self._ctr("rw_count"))
    rw_head_index = property(lambda self: self._ctr("rw_head_index"))
    hh_count = property(lambda self: self._ctr("hh_count"))
    wr_count = property(lambda self: self._ctr("wr_count"))
    pbs_count = property(lambda self: self._ctr("pbs_count"))
    pbs_blocks_used = property(lambda self: self._ctr("pbs_blocks_used"))
    pbs_allocated_blocks = property(lambda self: self._ctr("pbs_allocated_blocks"))
    total_processed_tokens = property(lambda self: self._ctr("total_processed_tokens"))
    total_evictions = property(lambda self: self._ctr("total_evictions"))

    @property
    def max_hh(self) -> int:
        return self._ctr("max_hh")

    def get_buffer_bytes(self) -> int:
        n = C.c_size_t()
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_get_buffer_bytes(self._h, C.byref(n)), "get_buffer_bytes")
        return int(n.value)

    def get_device_bytes(self) -> int:
        n = C.c_size_t()
        check(lib().tt_engine_device_bytes(self._h, C.byref(n)), "get_device_bytes")
        return int(n.value)

    def _view(self, name: str, shape) -> torch.Tensor:
        d = _lib.BufferDesc()
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_get_buffer(self._h, _BUF[name], C.byref(d)), name)
        n = int(np.prod(shape)) if len(shape) else 1
        if n == 0 or not d.data:
            dt = {0: torch.float32, 1: torch.int32, 2: torch.int64, 3: torch.uint16}[d.dtype]
            return torch.empty(tuple(shape), dtype=dt, device=self.device)
        return torch.as_tensor(_DeviceView(d.data, shape, _TYPESTR[d.dtype], self), device=self.device)

    def get_global_attn_scores(self):
        return self._view("global_attn_scores", (self.max_seq_len,))

    def get_S_K(self):
        return self._view("S_K", (self.sink_size, self.num_kv_heads, self.head_dim))

    def get_S_V(self):
        return self._view("S_V", (self.sink_size, self.num_kv_heads, self.head_dim))

    def get_RW_K(self):
        return self._view("RW_K", (self.rw_size, self.num_kv_heads, self.head_dim))

    def get_RW_V(self):
        return self._view("RW_V", (self.rw_size, self.num_kv_heads, self.head_dim))

    def get_HH_K(self):
        return self._view("HH_K", (self.max_hh, self.num_kv_heads, self.head_dim))

    def get_HH_V(self):
        return self._view("HH_V", (self.max_hh, self.num_kv_heads, self.head_dim))

    def get_HH_token_ids(self):
        return self._view("HH_token_ids", (self.max_hh,))

    def get_HH_scores(self):
        return self._view("HH_scores", (self.max_hh,))

    def get_WR_K(self):
        return self._view("WR_K", (self.chunk_size, self.num_kv_heads, self.head_dim))

    def get_WR_V(self):
        return self._view("WR_V", (self.chunk_size, self.num_kv_heads, self.head_dim))

    def get_WR_token_ids(self):
        return self._view("WR_token_ids", (self.chunk_size,))

    def get_PBS_K_Packed(self):
        nb = self.pbs_allocated_blocks
        return self._view("PBS_K_Packed", (nb, self.k_group_size // 16, self.num_kv_heads, self.head_dim))

    def get_PBS_K_Scales(self):
        return self._view("PBS_K_Scales", (self.pbs_allocated_blocks, self.num_kv_heads, self.head_dim))

    def get_PBS_K_Zeroes(self):
        return self._view("PBS_K_Zeroes", (self.pbs_allocated_blocks, self.num_kv_heads, self.head_dim))

    def get_PBS_V_Packed(self):
        return self._view("PBS_V_Packed",
                          (self.pbs_allocated_blocks * self.chunk_size, self.num_kv_heads, self.quant_head_dim))

    def get_PBS_V_Scales(self):
        return self._view("PBS_V_Scales", (self.pbs_allocated_blocks * self.chunk_size, self.num_kv_heads, 1))

    def get_PBS_V_Zeroes(self):
        return self._view("PBS_V_Zeroes", (self.pbs_allocated_blocks * self.chunk_size, self.num_kv_heads, 1))

    def get_PBS_token_ids(self):
        return self._view("PBS_token_ids", (self.pbs_allocated_blocks * self.chunk_size,))

    # -- full-weights path (output_attentions) ----------------------------------
    def ingest(self, k_ptr, v_ptr) -> None:
        """Maintenance only: ingest one token and route the evicted one, no
        attention, no score feedback (tt_engine_ingest)."""
        kvs = self.num_kv_heads * self.head_dim
        k = _arg(k_ptr, "K_new", kvs * 4)
        v = _arg(v_ptr, "V_new", kvs * 4)
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_ingest(self._h, k.ptr, v.ptr, _stream()), "ingest")
        self._keep = (k, v)

    def reconstruct(self):
        """(K_full, V_full, ids) CUDA tensors of the whole cache in token-id
        order with the packed tier dequantized (tt_engine_reconstruct)."""
        n = C.c_int()
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_full_count(self._h, C.byref(n)), "reconstruct")
            cap = max(n.value, 1)
            K = torch.empty((cap, self.num_kv_heads, self.head_dim), device=self.device)
            V = torch.empty((cap, self.num_kv_heads, self.head_dim), device=self.device)
            ids = torch.empty(cap, dtype=torch.int64, device=self.device)
            got = C.c_int()
            check(lib().tt_engine_reconstruct(self._h, K.data_ptr(), V.data_ptr(), ids.data_ptr(), cap,
                                              C.byref(got), _stream()), "reconstruct")
        m = got.value
        return K[:m], V[:m], ids[:m]

    def accumulate_scores(self, weights: torch.Tensor, ids: Optional[torch.Tensor] = None) -> None:
        """global_attn_scores[ids] += weights.mean(0) (undecayed,
        tt_engine_accumulate_scores); weights [heads, n], ids [n] int64 or None."""
        w = weights.to(device=self.device, dtype=torch.float32).contiguous()
        if w.dim() != 2:
            raise ValueError("weights must be [heads, n].")
        n = w.shape[1]
        idp = None
        idt = None
        if ids is not None:
            idt = ids.to(device=self.device, dtype=torch.int64).contiguous()
            if idt.numel() != n:
                raise ValueError("ids must have one entry per position.")
            idp = idt.data_ptr()
        with torch.cuda.device(self._dev):
            check(lib().tt_engine_accumulate_scores(self._h, w.data_ptr(), idp, w.shape[0], n, _stream()),
                  "accumulate_scores")
        self._keep = (w, idt)


_row_arrays: dict = {}  # pointer arrays of 2-D row tensors, by (address, row bytes, rows)


def _ptr_array(ts, n: int, name: str):
    """ctypes array of n device pointers: `ts` is a sequence of contiguous
    CUDA tensors, or one 2-D CUDA tensor whose n rows (each contiguous, any
    row stride) are the entries (its pointers are computed without a Python
    loop)."""
    arr = C.c_void_p * n
    if isinstance(ts, torch.Tensor):
        if not (ts.is_cuda and ts.dim() == 2 and ts.shape[0] == n and (ts.stride(1) == 1 or ts.shape[1] == 1)):
            raise ValueError(f"{name}: expected a 2-D CUDA tensor with {n} contiguous rows.")
        row = ts.stride(0) * ts.element_size()
        key = (ts.data_ptr(), row, n)  # the array is a function of these alone
        a = _row_arrays.get(key)
        if a is None:
            p = np.arange(n, dtype=np.uint64) * np.uint64(row) + np.uint64(ts.data_ptr())
            a = arr.from_buffer_copy(p.tobytes())
            if len(_row_arrays) > 256:
                _row_arrays.clear()
            _row_arrays[key] = a
        return a
    if len(ts) != n:
        raise ValueError(f"{name}: expected {n} entries, got {len(ts)}.")
    out = []
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous()):
            raise ValueError(f"{name} entries must be contiguous CUDA tensors.")
        out.append(t.data_ptr())
    return arr(*out)


def _handles(engines):
    return (C.c_void_p * len(engines))(*[e._h.value for e in engines])


def engine_step_batched(engines, Qs, Ks, Vs, outs) -> None:
    """One decode step for several engines (layers / sequences) in one set of
    launches.  Each of Qs / Ks / Vs / outs is a sequence of contiguous FP32
    CUDA tensors, one per engine, or one contiguous tensor with a row per
    engine.  No reference counterpart (the reference is batch-1, one engine
    per call)."""
    n = len(engines)
    with torch.cuda.device(engines[0]._dev):
        check(lib().tt_engine_step_batched(_handles(engines), n, _ptr_array(Qs, n, "Q"), _ptr_array(Ks, n, "K_new"),
                                           _ptr_array(Vs, n, "V_new"), _ptr_array(outs, n, "attn_output"),
                                           _stream()), "engine_step_batched")


class ShardedStep:
    """The calls of one sequence-sharded decode step for this rank
    (tt_engine_step_sharded_begin / _merge and the score synchronisation).
    Every rank holds the same engines and feeds them the same inputs; each
    attends and scores the tokens it owns (ring, heavy-hitter and sink slot j
    on rank j % world, packed tokens in 256-token granules round-robin).
    Between begin and merge the caller all-gathers, in rank order, the exchange
    rows; after merge the routing rows, which the next begin takes.  No
    reference counterpart: the reference has no multi-GPU path."""

    ROUTE_FLOATS = 4  # one routing row: 16 bytes

    def __init__(self, engines, rank: int, world: int):
        self.engines = list(engines)
        self.rank, self.world = int(rank), int(world)
        self.n = len(self.engines)
        self._hs = _handles(self.engines)
        self.nq, self.hd = self.engines[0].num_q_heads, self.engines[0].head_dim
        self.xch_floats = self.n * self.nq * (self.hd + 2)   # per rank
        self.route_floats = self.n * self.ROUTE_FLOATS      # per rank

    def _ptrs(self, ts, name):
        return _ptr_array(ts, self.n, name)

    def sync_needed(self) -> bool:
        """Whether the next step recomputes the heavy-hitter threshold, so the
        scores must be synchronised first (and begin gets route_all=None)."""
        v = C.c_int()
        check(lib().tt_engine_sharded_sync_needed(self._hs, self.n, C.byref(v)), "sync_needed")
        return bool(v.value)

    def scores_floats(self) -> int:
        v = C.c_longlong()
        check(lib().tt_engine_sharded_scores_floats(self._hs, self.n, C.byref(v)), "scores_floats")
        return v.value

    def scores_pack(self, buf: torch.Tensor) -> None:
        with torch.cuda.device(self.engines[0]._dev):
            check(lib().tt_engine_sharded_scores_pack(self._hs, self.n, self.rank, self.world, buf.data_ptr(),
                                                      _stream()), "scores_pack")

    def scores_unpack(self, buf: torch.Tensor) -> None:
        with torch.cuda.device(self.engines[0]._dev):
            check(lib().tt_engine_sharded_scores_unpack(self._hs, self.n, buf.data_ptr(), _stream()),
                  "scores_unpack")

    def begin(self, Qs, Ks, Vs, xch_send: torch.Tensor, route_all: Optional[torch.Tensor]) -> None:
        with torch.cuda.device(self.engines[0]._dev):
            check(lib().tt_engine_step_sharded_begin(self._hs, self.n, self._ptrs(Qs, "Q"),
                                                     self._ptrs(Ks, "K_new"), self._ptrs(Vs, "V_new"), self.rank,
                                                     self.world, None if route_all is None else route_all.data_ptr(),
                                                     xch_send.data_ptr(), _stream()), "begin")

    def merge(self, xch_all: torch.Tensor, outs, route_send: torch.Tensor) -> None:
        with torch.cuda.device(self.engines[0]._dev):
            check(lib().tt_engine_step_sharded_merge(self._hs, self.n, self.rank, self.world, xch_all.data_ptr(),
                                                     self._ptrs(outs, "attn_output"), route_send.data_ptr(),
                                                     _stream()), "merge")

    # -- peer-memory exchange (tt_sharded_xch_*): the library exchanges the rows
    def xch_create(self) -> bytes:
        """Allocates this rank's exchange region; returns its 64-byte IPC handle."""
        x = C.c_void_p()
        h = (C.c_char * 64)()
        dev = self.engines[0]._dev
        with torch.cuda.device(dev):
            check(lib().tt_sharded_xch_create(self.world, self.rank, self.n, self.nq, self.hd, dev, C.byref(x), h),
                  "xch_create")
        self._x = x
        return bytes(h)

    def xch_open(self, handles: bytes) -> None:
        """Opens the other ranks' regions (handles: world x 64 bytes, rank order)."""
        with torch.cuda.device(self.engines[0]._dev):
            check(lib().tt_sharded_xch_open(self._x, handles), "xch_open")

    def xch_destroy(self) -> None:
        x = getattr(self, "_x", None)
        if x:
            lib().tt_sharded_xch_destroy(x)
            self._x = None

    def begin_xch(self, Qs, Ks, Vs, route_valid: bool) -> None:
        with torch.cuda.device(self.engines[0]._dev):
            check(lib().tt_engine_step_sharded_begin_xch(self._hs, self.n, self._ptrs(Qs, "Q"),
                                                         self._ptrs(Ks, "K_new"), self._ptrs(Vs, "V_new"), self._x,
                                                         1 if route_valid else 0, _stream()), "begin_xch")

    def merge_xch(self, outs) -> None:
        with torch.cuda.device(self.engines[0]._dev):
            check(lib().tt_engine_step_sharded_merge_xch(self._hs, self.n, self._x, self._ptrs(outs, "attn_output"),
                                                         _stream()), "merge_xch")


class ShardedEngineStep:
    """engine_step_batched over the ranks of a torch.distributed process group
    (NCCL, one process per GPU), for one fixed list of engines: every rank
    passes the same inputs and receives the same outputs; each attends and
    scores the tokens it owns.  Per step: begin, all-gather of the (m, l, acc)
    rows, merge, all-gather of the routing rows; before a step that recomputes
    the heavy-hitter threshold (every update_interval tokens) an all-reduce
    synchronises the scores.  The first call routes from each rank's own
    scores, which must then be current on every rank (after prefill or steps
    that were not sharded).  The exchange buffers are kept between calls.
    With phase_timing(True) every call also records CUDA events between its
    phases (device time per phase, phase_times())."""

    PHASES = ("sync", "begin", "allgather_rows", "merge", "allgather_route")
    PHASES_PEER = ("sync", "begin", "merge")

    def __init__(self, engines, rank=None, world=None, group=None, exchange="nccl"):
        """exchange: "nccl" (two all-gathers of the process group per step) or
        "peer" (the library writes the rows into every rank's memory over
        NVLink and waits on flags; ranks of one node, 2..8; call close() on
        every rank when done)."""
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group) if world is None else int(world)
        self.rank = dist.get_rank(group) if rank is None else int(rank)
        self.engines = list(engines)
        self.step = ShardedStep(self.engines, self.rank, self.world)
        self.dev = self.engines[0].device
        if exchange not in ("nccl", "peer"):
            raise ValueError("exchange must be 'nccl' or 'peer'.")
        self.exchange = exchange if self.world > 1 else "nccl"
        if self.exchange == "peer":
            self.PHASES = self.PHASES_PEER
            h = torch.tensor(list(self.step.xch_create()), dtype=torch.uint8, device=self.dev)
            allh = torch.empty(self.world * 64, dtype=torch.uint8, device=self.dev)
            dist.all_gather_into_tensor(allh, h, group=self.group)
            self.step.xch_open(bytes(allh.cpu().numpy().tobytes()))
            # a rank that leaves without close() (an exception) still waits for
            # the others at exit before its region goes away
            import atexit
            atexit.register(self.close)
        st = self.step
        self.xs = torch.empty(st.xch_floats, device=self.dev)
        self.xa = torch.empty(self.world * st.xch_floats, device=self.dev)
        self.rs = torch.zeros(st.route_floats, device=self.dev)
        self.ra = torch.zeros(self.world * st.route_floats, device=self.dev)
        self.scores = None
        self.route_valid = False
        self.syncs = 0
        self._timing = False
        self._acc = {p: 0.0 for p in self.PHASES}
        self._pending = []

    def phase_timing(self, on: bool) -> None:
        self._timing = bool(on)
        self._acc = {p: 0.0 for p in self.PHASES}
        self._pending = []

    def phase_times(self, steps: int) -> dict:
        """Device milliseconds per step of each phase over the timed calls."""
        torch.cuda.synchronize(self.dev)
        for ev in self._pending:
            for p, a, b in zip(self.PHASES, ev[:-1], ev[1:]):
                self._acc[p] += a.elapsed_time(b)
        self._pending = []
        return {p: round(v / max(steps, 1), 5) for p, v in self._acc.items()}

    def close(self) -> None:
        """Peer exchange: wait for every rank to finish its steps, then free the
        exchange regions (no rank may free its region while another can still
        write into it)."""
        import torch.distributed as dist
        if self.exchange == "peer" and getattr(self.step, "_x", None):
            if self.dev.type == "cuda":
                torch.cuda.synchronize(self.dev)
            if dist.is_initialized():
                dist.barrier(group=self.group)
            self.step.xch_destroy()

    def __call__(self, engines, Qs, Ks, Vs, outs) -> None:
        import torch.distributed as dist
        if len(engines) != self.step.n or any(a is not b for a, b in zip(engines, self.engines)):
            raise ValueError("ShardedEngineStep: called with a different list of engines.")
        st = self.step
        ev = None
        if self._timing:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.PHASES) + 1)]
            ev[0].record()
        if self.exchange == "peer":
            route_valid = self.route_valid
            if st.sync_needed():
                if self.scores is None:
                    self.scores = torch.empty(st.scores_floats(), device=self.dev)
                st.scores_pack(self.scores)
                dist.all_reduce(self.scores, group=self.group)
                st.scores_unpack(self.scores)
                route_valid = False
                self.syncs += 1
            if ev:
                ev[1].record()
            st.begin_xch(Qs, Ks, Vs, route_valid)
            if ev:
                ev[2].record()
            st.merge_xch(outs)
            self.route_valid = True
            if ev:
                ev[3].record()
                self._pending.append(ev)
            return
        route = self.ra if self.route_valid else None
        if self.world > 1 and st.sync_needed():
            if self.scores is None:
                self.scores = torch.empty(st.scores_floats(), device=self.dev)
            st.scores_pack(self.scores)
            dist.all_reduce(self.scores, group=self.group)
            st.scores_unpack(self.scores)
            route = None
            self.syncs += 1
        if ev:
            ev[1].record()
        st.begin(Qs, Ks, Vs, self.xs, route)
        if ev:
            ev[2].record()
        dist.all_gather_into_tensor(self.xa, self.xs, group=self.group)
        if ev:
            ev[3].record()
        st.merge(self.xa, outs, self.rs)
        if ev:
            ev[4].record()
        dist.all_gather_into_tensor(self.ra, self.rs, group=self.group)
        self.route_valid = True
        if ev:
            ev[5].record()
            self._pending.append(ev)


_shard_steps: dict = {}


def engine_step_batched_sharded(engines, Qs, Ks, Vs, outs, group=None, exchange="nccl") -> None:
    """engine_step_batched over the ranks of a torch.distributed process group
    (NCCL, one process per GPU): every rank passes the same engines' handles
    and the same inputs and receives the same outputs; each attends and scores
    the tokens it owns.  Keeps one ShardedEngineStep per (group, engine list,
    exchange); see ShardedEngineStep for the exchanges."""
    key = (id(group), tuple(e._h.value for e in engines), exchange)
    s = _shard_steps.get(key)
    if s is None:
        s = ShardedEngineStep(engines, group=group, exchange=exchange)
        _shard_steps[key] = s
    s(engines, Qs, Ks, Vs, outs)
