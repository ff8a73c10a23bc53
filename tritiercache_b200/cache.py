"""TriTierCache on the GPU engine (drop-in for src/tri_tier/cache.py).

The reference class wraps its C++ engine when ``tri_tier._C`` imports
(cache.py:31-59) and otherwise runs pure-torch tiers.  This class always
wraps the device engine of libtritier_b200: there is no CPU fallback, and
construction raises when CUDA or the library is missing.

Buffers are CUDA tensors aliasing the engine's tier memory (the reference
wraps writable numpy views with torch.from_numpy, cache.py:50-59).  The
counters (``Total_Processed_Tokens`` ...) are read from the device when
accessed instead of after every step (cache.py:110-116), so a decode step
does not synchronise the host with the GPU.
"""
from __future__ import annotations

import math

import torch

from . import _C
from .constants import CHUNK_SIZE, SINK_SIZE, UPDATE_THRESHOLD


class TriTierCache:
    def __init__(self, max_seq_len, head_dim, num_heads, R_size, H_ratio, num_q_heads=None, score_decay=0.999,
                 k_group_size=16, pbs_metadata_dtype="fp16", device=None):
        """Same arguments as cache.py:12 (plus ``device``, default the current CUDA device)."""
        self.R_size = R_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.num_q_heads = num_q_heads if num_q_heads is not None else num_heads
        self.score_decay = score_decay
        self.k_group_size = 32 if k_group_size == 32 else 16
        self.pbs_metadata_dtype = "fp32" if str(pbs_metadata_dtype).lower() == "fp32" else "fp16"
        self.current_threshold = 0.0
        self.max_heavy_hitters = math.ceil(max_seq_len * H_ratio)
        self.max_background_tokens = max_seq_len - R_size - self.max_heavy_hitters
        self.max_seq_len = max_seq_len
        decay_val = 1.0 if score_decay is None else float(score_decay)
        self._engine = _C.TriTierCacheEngine(self.num_q_heads, self.num_heads, self.head_dim, max_seq_len,
                                             SINK_SIZE, R_size, H_ratio, decay_val, UPDATE_THRESHOLD,
                                             self.k_group_size, self.pbs_metadata_dtype, device=device)
        self.device = self._engine.device
        self.S_K_Buffer = self._engine.get_S_K()
        self.S_V_Buffer = self._engine.get_S_V()
        self.RW_K_Buffer = self._engine.get_RW_K()
        self.RW_V_Buffer = self._engine.get_RW_V()
        self.HH_K_Buffer = self._engine.get_HH_K()
        self.HH_V_Buffer = self._engine.get_HH_V()
        self.HH_token_ids = self._engine.get_HH_token_ids()
        self.HH_scores = self._engine.get_HH_scores()
        self.Global_Attn_Scr = self._engine.get_global_attn_scores()
        self.WR_K_Buffer = self._engine.get_WR_K()
        self.WR_V_Buffer = self._engine.get_WR_V()
        self.WR_token_ids = self._engine.get_WR_token_ids()
        self.quant_head_dim = math.ceil(head_dim / 16)

    # -- counters (read from the device on access) ---------------------------
    def _c(self, name):
        return self._engine.counters()[name]

    Total_Processed_Tokens = property(lambda self: self._c("total_processed_tokens"))
    total_evictions = property(lambda self: self._c("total_evictions"))
    PBS_count = property(lambda self: self._c("pbs_count"))
    RW_count = property(lambda self: self._c("rw_count"))
    RW_head_index = property(lambda self: self._c("rw_head_index"))
    S_count = property(lambda self: self._c("s_count"))
    HH_count = property(lambda self: self._c("hh_count"))
    WR_count = property(lambda self: self._c("wr_count"))

    # -- hot path -------------------------------------------------------------
    def step(self, Q: torch.Tensor, K_new: torch.Tensor, V_new: torch.Tensor, attn_output: torch.Tensor):
        """Token ingestion, fused attention and score feedback in one engine call (cache.py:101-118)."""
        self._engine.step(Q, K_new, V_new, attn_output)

    def prefill(self, K_tokens: torch.Tensor, V_tokens: torch.Tensor) -> None:
        """Prompt ingestion; K_tokens, V_tokens: [q_len, num_heads, head_dim] (cache.py:120-139)."""
        q_len = K_tokens.shape[0]
        K = K_tokens.to(device=self.device, dtype=torch.float32).contiguous()
        V = V_tokens.to(device=self.device, dtype=torch.float32).contiguous()
        self._engine.prefill(K, V, q_len)

    def get_buffer_bytes(self) -> int:
        """The reference engine's byte formula (cache_engine.cpp:543-568)."""
        return self._engine.get_buffer_bytes()

    # -- full-weights path (output_attentions=True, patch_model.py:163-169) ----
    def ingest_token(self, K: torch.Tensor, V: torch.Tensor) -> None:
        """Ingests one token [num_heads, head_dim] and routes the evicted one
        (cache.py:206-233).  Routing and quantization are the engine's
        (cache_engine.cpp:209-269: cached percentile threshold, strict-min
        demotion, 16-token waiting room); the reference's pure-torch fallback
        routes with torch.quantile instead, a different rule."""
        Kd = K.to(device=self.device, dtype=torch.float32).contiguous()
        Vd = V.to(device=self.device, dtype=torch.float32).contiguous()
        self._engine.ingest(Kd, Vd)

    def reconstruct_full_cache(self):
        """(K_full, V_full, full_ids): sinks, heavy hitters and packed tokens in
        token-id order (packed ones dequantized), then the ring in logical
        order (cache.py:326-372); CUDA tensors."""
        return self._engine.reconstruct()

    def accumulate_attn_scrs(self, attn_weights: torch.Tensor, full_ids=None) -> None:
        """Adds the head-mean of one decode step's attention weights to the
        accumulated scores, undecayed (cache.py:164-187)."""
        if attn_weights.dim() == 4:
            if attn_weights.shape[2] > 1:
                raise RuntimeError("Multi-token prefill not supported in single-step accumulate")
            step = attn_weights.squeeze(0).squeeze(1)
        elif attn_weights.dim() == 3:
            step = attn_weights.squeeze(1)
        else:
            step = attn_weights
        if step.dim() == 1:
            step = step.unsqueeze(0)
        self._engine.accumulate_scores(step, full_ids)

    def fetch_or_calc_thresh(self, total_processed_tokens: int = 0):
        """The engine's cached heavy-hitter threshold (cache_engine.cpp:118-146),
        as a tensor (cache.py:189-204 returns its own quantile)."""
        return torch.tensor(float(self._engine.counters()["cached_threshold"]))

    def assert_evictions_occurred(self) -> None:
        """cache.py:156-162."""
        assert self.total_evictions > 0 or self.PBS_count > 0 or self.HH_count > 0, (
            f"TriTierCache ran with 0 evictions (total_tokens={self.Total_Processed_Tokens}, "
            f"R_size={self.R_size}, HH_count={self.HH_count}, PBS_count={self.PBS_count}). "
            "Quality benchmarks must run at context length >= 4x R_size to exercise compression tiers!")

    # -- packed tier views (sized by the engine's allocated blocks) ------------
    @property
    def PBS_K_Packed(self):
        return self._engine.get_PBS_K_Packed()

    @property
    def PBS_K_Scales(self):
        return self._engine.get_PBS_K_Scales()

    @property
    def PBS_K_Zeroes(self):
        return self._engine.get_PBS_K_Zeroes()

    @property
    def PBS_V_Packed(self):
        return self._engine.get_PBS_V_Packed()

    @property
    def PBS_V_Scales(self):
        return self._engine.get_PBS_V_Scales()

    @property
    def PBS_V_Zeroes(self):
        return self._engine.get_PBS_V_Zeroes()

    @property
    def PBS_token_ids(self):
        return self._engine.get_PBS_token_ids()
