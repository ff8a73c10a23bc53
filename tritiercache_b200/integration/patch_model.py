"""Hugging Face attention patch on the GPU engine (drop-in for
src/tri_tier/integration/patch_model.py).

Supports LlamaAttention, MistralAttention, Qwen2Attention and Qwen3Attention
(patch_model.py:176-206).  The patched forward keeps the reference's
structure (patch_model.py:54-169): lazy per-layer TriTierCache sized by the KV
heads, q/k/v projections, optional Qwen3 q/k RMSNorm, rotate-half RoPE,
causal SDPA plus ``cache.prefill`` for prompts, and one fused engine step per
decode token.  Unlike the reference, Q/K/V stay on the GPU (no ``.float()``
copies to host memory) and the step is stream-ordered.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple, Type

import torch

from ..cache import TriTierCache

HAS_CPP_EXT = True

MAX_SEQ_LEN = 32768
R_SIZE = 256
H_RATIO = 0.05
SCORE_DECAY = 0.999
K_GROUP_SIZE = 16
PBS_METADATA_DTYPE = "fp16"


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _reference_attention_path(self, cache: TriTierCache, Q: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                              head_dim: int):
    """Full-weights path of patch_model.py:33-51 (``output_attentions=True``):
    the whole cache reconstructed on the engine's device, softmax weights
    returned and added to the accumulated scores.  Runs on the engine's device;
    results come back on Q's device."""
    K_full, V_full, full_ids = cache.reconstruct_full_cache()
    dev = K_full.device
    Qd = Q.to(dev)
    if num_q_heads != num_kv_heads:
        rep = num_q_heads // num_kv_heads
        K_full = K_full.repeat_interleave(rep, dim=1)
        V_full = V_full.repeat_interleave(rep, dim=1)
    K_full = K_full.transpose(0, 1).unsqueeze(0).to(dtype=Qd.dtype)
    V_full = V_full.transpose(0, 1).unsqueeze(0).to(dtype=Qd.dtype)
    scaling = getattr(self, "scaling", None) or (head_dim ** -0.5)
    w = torch.softmax(torch.matmul(Qd, K_full.transpose(-2, -1)) * scaling, dim=-1)
    cache.accumulate_attn_scrs(w, full_ids)
    return torch.matmul(w, V_full).to(Q.device), w.to(Q.device)


def patched_forward(self, hidden_states: torch.Tensor,
                    position_embeddings: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                    attention_mask: Optional[torch.Tensor] = None, past_key_values: Optional[Any] = None,
                    **kwargs):
    """Forward for Llama/Mistral/Qwen2/Qwen3 attention modules (patch_model.py:54-169)."""
    bsz, q_len, _ = hidden_states.shape
    assert bsz == 1, "TriTierCache only supports batch_size=1"

    nq = self.config.num_attention_heads
    nkv = getattr(self.config, "num_key_value_heads", nq)
    hd = getattr(self, "head_dim", None) or (self.config.hidden_size // nq)
    cap = max(MAX_SEQ_LEN, getattr(self.config, "max_position_embeddings", MAX_SEQ_LEN))

    if getattr(self, "tri_tier_cache", None) is None:
        dev = hidden_states.device if hidden_states.is_cuda else None
        self.tri_tier_cache = TriTierCache(max_seq_len=cap, head_dim=hd, num_heads=nkv, R_size=R_SIZE,
                                           H_ratio=H_RATIO, num_q_heads=nq, score_decay=SCORE_DECAY,
                                           k_group_size=K_GROUP_SIZE, pbs_metadata_dtype=PBS_METADATA_DTYPE,
                                           device=dev)
    cache = self.tri_tier_cache

    q = self.q_proj(hidden_states).view(bsz, q_len, nq, hd)
    k = self.k_proj(hidden_states).view(bsz, q_len, nkv, hd)
    v = self.v_proj(hidden_states).view(bsz, q_len, nkv, hd)
    if getattr(self, "q_norm", None) is not None:
        q = self.q_norm(q)
    if getattr(self, "k_norm", None) is not None:
        k = self.k_norm(k)
    Q, K_new, V_new = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    cos, sin = position_embeddings
    if cos.ndim == 3:
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    Q = Q * cos + _rotate_half(Q) * sin
    K_new = K_new * cos + _rotate_half(K_new) * sin

    if q_len > 1:
        rep = nq // nkv
        K_exp = K_new.repeat_interleave(rep, dim=1) if rep > 1 else K_new
        V_exp = V_new.repeat_interleave(rep, dim=1) if rep > 1 else V_new
        ctx = torch.nn.functional.scaled_dot_product_attention(Q, K_exp, V_exp, is_causal=True)
        K_tok = K_new.squeeze(0).transpose(0, 1).contiguous()
        V_tok = V_new.squeeze(0).transpose(0, 1).contiguous()
        if getattr(self, "capture_needle_pos", None) is not None:
            self.captured_needle_k = K_tok[self.capture_needle_pos].clone()
            self.captured_needle_v = V_tok[self.capture_needle_pos].clone()
        cache.prefill(K_tok.float(), V_tok.float())
        return self.o_proj(ctx.transpose(1, 2).reshape(bsz, q_len, -1)), None

    if kwargs.get("output_attentions", False):
        cache.ingest_token(K_new.squeeze(0).squeeze(1).float(), V_new.squeeze(0).squeeze(1).float())
        ctx, w = _reference_attention_path(self, cache, Q, nq, nkv, hd)
        ctx = ctx.transpose(1, 2).reshape(bsz, q_len, -1).to(dtype=hidden_states.dtype)
        return self.o_proj(ctx), w

    dev = cache.device
    Qf = Q.reshape(nq * hd).to(device=dev, dtype=torch.float32).contiguous()
    Kf = K_new.reshape(nkv * hd).to(device=dev, dtype=torch.float32).contiguous()
    Vf = V_new.reshape(nkv * hd).to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty(nq * hd, dtype=torch.float32, device=dev)
    cache.step(Qf, Kf, Vf, out)
    ctx = out.view(bsz, q_len, -1).to(device=hidden_states.device, dtype=hidden_states.dtype)
    return self.o_proj(ctx), None


_SUPPORTED_ATTENTION_CLASSES: List[Type] = []
_ORIGINAL_FORWARDS: Dict[Type, Any] = {}
_IS_PATCHED: bool = False

for _mod, _cls in (("llama.modeling_llama", "LlamaAttention"), ("mistral.modeling_mistral", "MistralAttention"),
                   ("qwen2.modeling_qwen2", "Qwen2Attention"), ("qwen3.modeling_qwen3", "Qwen3Attention")):
    try:
        _m = __import__(f"transformers.models.{_mod}", fromlist=[_cls])
        _SUPPORTED_ATTENTION_CLASSES.append(getattr(_m, _cls))
    except Exception:  # transformers missing or model family absent
        pass


def apply_patch():
    """Patches every supported attention class (patch_model.py:209-216)."""
    global _IS_PATCHED
    for cls in _SUPPORTED_ATTENTION_CLASSES:
        if cls not in _ORIGINAL_FORWARDS:
            _ORIGINAL_FORWARDS[cls] = cls.forward
        cls.forward = patched_forward
    _IS_PATCHED = True


def remove_patch():
    """Restores the original forwards (patch_model.py:219-224)."""
    global _IS_PATCHED
    for cls, fwd in _ORIGINAL_FORWARDS.items():
        cls.forward = fwd
    _IS_PATCHED = False


def reset_caches(model):
    """Drops the lazily created caches of every layer (patch_model.py:227-231)."""
    for module in model.modules():
        if hasattr(module, "tri_tier_cache"):
            delattr(module, "tri_tier_cache")


def is_patched(model_or_module=None) -> bool:
    """patch_model.py:234-241."""
    if _IS_PATCHED:
        return True
    return any(getattr(cls, "forward", None) == patched_forward for cls in _SUPPORTED_ATTENTION_CLASSES)
