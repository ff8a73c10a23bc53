"""The drop-in Python layer on the GPU: TriTierCache and the Hugging Face
attention patch (integration/patch_model.py) driving the engine.

The first group mirrors the reference's own integration tests
(tests/test_patch_llama.py in the reference project: MHA and GQA single steps
through both paths, the 286-step decode across every tier with
output_attentions=True, a full LlamaForCausalLM.generate), with randomly
initialised models -- no checkpoint.  The second group checks parity:

* fused decode path: a GQA Llama attention layer on the GPU prefills a prompt
  and decodes 300 tokens through TriTierCache.step; every prefill / step call
  the patch makes is replayed into the CPU oracle engine with the same
  tensors, and every step's attention output (1e-4 + 1e-5|x|) and counters
  (exact) must match, with the oracle's scores copied into the GPU engine after
  each step (score sync, as in test_gpu_engine.py);
* full-weights path: reconstruct_full_cache is compared bit-exactly with a
  numpy restatement of the reference's cache.py:326-372 over the same engine
  state, and accumulate_attn_scrs with cache.py:164-187 (relative 1e-6).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")
from transformers.models.llama.configuration_llama import LlamaConfig  # noqa: E402
from transformers.models.llama.modeling_llama import LlamaAttention, LlamaForCausalLM, LlamaRotaryEmbedding  # noqa: E402

SINK_SIZE, R_SIZE, CHUNK_SIZE = 4, 256, 16


@pytest.fixture(scope="module", autouse=True)
def patched():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tritiercache_b200.integration import patch_model
    patch_model.apply_patch()
    yield patch_model
    patch_model.remove_patch()


def attention_layer(nq=4, nkv=4, hidden=64, hd=16, device="cuda", seed=0):
    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=hidden, num_attention_heads=nq, num_key_value_heads=nkv, head_dim=hd,
                      max_position_embeddings=4096, attention_bias=False)
    layer = LlamaAttention(cfg, layer_idx=0).to(device)
    rot = LlamaRotaryEmbedding(config=cfg).to(device)
    return layer, rot, cfg


def run(layer, rot, x, pos, **kw):
    cos, sin = rot(x, pos)
    return layer(x, position_embeddings=(cos, sin), **kw)


@pytest.mark.parametrize("nq,nkv,hidden", [(4, 4, 64), (8, 2, 128)])
def test_single_step_both_paths(nq, nkv, hidden):
    layer, rot, cfg = attention_layer(nq, nkv, hidden, 16)
    x = torch.randn(1, 1, hidden, device="cuda")
    pos = torch.tensor([[0]], device="cuda")
    with torch.no_grad():
        out, w = run(layer, rot, x, pos)
        assert out.shape == (1, 1, hidden) and w is None and not torch.isnan(out).any()
        out2, w2 = run(layer, rot, x, pos, output_attentions=True)
    assert out2.shape == (1, 1, hidden) and w2.shape == (1, nq, 1, 2)
    assert not torch.isnan(out2).any()
    assert torch.allclose(w2.sum(dim=-1), torch.ones(1, nq, 1, device="cuda"), atol=1e-5)
    cache = layer.tri_tier_cache
    assert cache.num_heads == nkv and cache.Total_Processed_Tokens == 2


def test_batched_prefill_and_batch_size_assertion():
    layer, rot, cfg = attention_layer()
    x = torch.randn(1, 4, cfg.hidden_size, device="cuda")
    with torch.no_grad():
        out, _ = run(layer, rot, x, torch.arange(4, device="cuda")[None])
    assert out.shape == (1, 4, cfg.hidden_size) and layer.tri_tier_cache.Total_Processed_Tokens == 4
    with pytest.raises(AssertionError, match="batch_size=1"):
        run(layer, rot, torch.randn(2, 1, cfg.hidden_size, device="cuda"), torch.tensor([[0], [0]], device="cuda"))


def test_multi_step_decode_full_weights_path_across_tiers():
    """286 decode steps with output_attentions=True: every tier fills and the
    weights cover exactly the attended tokens (all but the waiting room)."""
    layer, rot, cfg = attention_layer(4, 4, 64, 16)
    steps = SINK_SIZE + R_SIZE + CHUNK_SIZE + 10
    for s in range(steps):
        x = torch.randn(1, 1, cfg.hidden_size, device="cuda")
        with torch.no_grad():
            out, w = run(layer, rot, x, torch.tensor([[s]], device="cuda"), output_attentions=True)
        assert out.shape == (1, 1, cfg.hidden_size)
        assert torch.isfinite(out).all()
        cache = layer.tri_tier_cache
        assert w.shape == (1, 4, 1, (s + 1) - cache.WR_count)
    cache = layer.tri_tier_cache
    assert cache.Total_Processed_Tokens == steps
    assert cache.S_count == SINK_SIZE and cache.RW_count == R_SIZE
    assert cache.PBS_count >= CHUNK_SIZE or cache.HH_count > 0


def test_end_to_end_generate():
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=100, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=256,
                      pad_token_id=0, bos_token_id=1, eos_token_id=2)
    model = LlamaForCausalLM(cfg).cuda().eval()
    with torch.no_grad():
        out = model.generate(torch.tensor([[1]], device="cuda"), max_new_tokens=15, use_cache=True,
                             eos_token_id=None)
    assert out.shape == (1, 16)
    c0 = model.model.layers[0].self_attn.tri_tier_cache
    c1 = model.model.layers[1].self_attn.tri_tier_cache
    assert c0 is not c1
    assert c0.Total_Processed_Tokens == 15 and c1.Total_Processed_Tokens == 15
    assert float(c0.Global_Attn_Scr[:15].sum()) > 0


# ---------------------------------------------------------------------------
# parity
# ---------------------------------------------------------------------------
def test_fused_decode_path_matches_oracle_engine(patched, monkeypatch):
    """GQA layer (8 q / 2 kv heads, head_dim 64): prompt of 300 tokens, then 300
    decode steps through TriTierCache.step; every prefill / step call the patch
    makes is replayed into the oracle engine with the same tensors."""
    from oracle import oracle as O
    from tritiercache_b200.cache import TriTierCache
    log = []
    orig_prefill, orig_step = TriTierCache.prefill, TriTierCache.step

    def prefill(self, K, V):
        log.append(("prefill", K.detach().float().cpu().numpy().copy(), V.detach().float().cpu().numpy().copy()))
        orig_prefill(self, K, V)

    def step(self, Q, K, V, out):
        orig_step(self, Q, K, V, out)
        log.append(("step", Q.detach().cpu().numpy().copy(), K.detach().cpu().numpy().copy(),
                    V.detach().cpu().numpy().copy(), out.detach().cpu().numpy().copy()))

    monkeypatch.setattr(TriTierCache, "prefill", prefill)
    monkeypatch.setattr(TriTierCache, "step", step)
    nq, nkv, hd, hidden = 8, 2, 64, 256
    layer, rot, cfg = attention_layer(nq, nkv, hidden, hd, seed=3)
    P = 300
    with torch.no_grad():
        run(layer, rot, torch.randn(1, P, hidden, device="cuda"), torch.arange(P, device="cuda")[None])
    cache = layer.tri_tier_cache
    eng = cache._engine
    eo = O.Engine(nq, nkv, hd, cache.max_seq_len, SINK_SIZE, R_SIZE, patched.H_RATIO, patched.SCORE_DECAY, 32,
                  patched.K_GROUP_SIZE, patched.PBS_METADATA_DTYPE)
    kind, Kp, Vp = log[0]
    assert kind == "prefill" and Kp.shape == (P, nkv, hd)
    eo.prefill(np.ascontiguousarray(Kp), np.ascontiguousarray(Vp), P)
    g_view, hh_view = eng.get_global_attn_scores(), eng.get_HH_scores()
    counters = ["s_count", "rw_count", "rw_head_index", "hh_count", "wr_count", "pbs_count", "total_processed_tokens",
                "total_evictions"]
    for s in range(300):
        with torch.no_grad():
            run(layer, rot, torch.randn(1, 1, hidden, device="cuda"), torch.tensor([[P + s]], device="cuda"))
        kind, Qn, Kn, Vn, og = log[-1]
        assert kind == "step"
        oo = np.zeros(nq * hd, np.float32)
        eo.step(Qn, Kn, Vn, oo)
        err = np.abs(og.astype(np.float64) - oo)
        assert np.all(err <= 1e-4 + 1e-5 * np.abs(oo)), (s, float(err.max()))
        c, cg = eo.counters(), eng.counters()
        for key in counters:
            assert c[key] == cg[key], (s, key, c[key], cg[key])
        g_view.copy_(torch.from_numpy(eo.buffer("global_attn_scores").copy()))
        hh_view.copy_(torch.from_numpy(eo.buffer("HH_scores").copy()))
    assert eng.counters()["pbs_count"] > 0 and eng.counters()["hh_count"] > 0


def _state(eng):
    c = eng.counters()
    st = {k: getattr(eng, "get_" + k)().cpu().numpy() for k in
          ("S_K", "S_V", "RW_K", "RW_V", "HH_K", "HH_V", "PBS_K_Packed", "PBS_K_Scales", "PBS_K_Zeroes",
           "PBS_V_Packed", "PBS_V_Scales", "PBS_V_Zeroes", "PBS_token_ids")}
    st["HH_token_ids"] = eng.get_HH_token_ids().cpu().numpy()
    st.update(s_count=c["s_count"], hh_count=c["hh_count"], rw_count=c["rw_count"],
              rw_head_index=c["rw_head_index"], total=c["total_processed_tokens"],
              pbs_blocks_used=c["pbs_blocks_used"], rw_size=eng.rw_size, grp=eng.k_group_size,
              nkv=eng.num_kv_heads, hd=eng.head_dim, meta16=1 if eng.use_fp16_meta else 0)
    return st


@pytest.mark.parametrize("meta,grp", [("fp16", 16), ("fp32", 32)])
def test_full_weights_path_reconstruct_and_accumulate_match_reference_restatement(meta, grp):
    from oracle import oracle as O
    from tritiercache_b200.cache import TriTierCache
    nq, nkv, hd = 8, 2, 64
    cache = TriTierCache(max_seq_len=2048, head_dim=hd, num_heads=nkv, R_size=R_SIZE, H_ratio=0.05, num_q_heads=nq,
                         k_group_size=grp, pbs_metadata_dtype=meta)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    cache.prefill(torch.randn(700, nkv, hd, device="cuda", generator=g),
                  torch.randn(700, nkv, hd, device="cuda", generator=g))
    eng = cache._engine
    for s in range(120):
        cache.ingest_token(torch.randn(nkv, hd, device="cuda", generator=g),
                           torch.randn(nkv, hd, device="cuda", generator=g))
        if s % 40 == 0 or s == 119:
            K, V, ids = cache.reconstruct_full_cache()
            rK, rV, rid = O.reconstruct_full_cache(_state(eng))
            assert np.array_equal(ids.cpu().numpy(), rid), s
            assert np.array_equal(K.cpu().numpy().view(np.uint32), rK.view(np.uint32)), s
            assert np.array_equal(V.cpu().numpy().view(np.uint32), rV.view(np.uint32)), s
            # a full-weights step's attention and its score accumulation
            w = torch.softmax(torch.randn(1, nq, 1, ids.numel(), device="cuda", generator=g), dim=-1)
            g_ref = eng.get_global_attn_scores().cpu().numpy().copy()
            cache.accumulate_attn_scrs(w, ids)
            O.accumulate_attn_scrs(g_ref, w[0, :, 0].cpu().numpy(), ids.cpu().numpy())
            got = eng.get_global_attn_scores().cpu().numpy()
            assert np.all(np.abs(got - g_ref) <= 1e-9 + 1e-6 * np.abs(g_ref)), s
    c = eng.counters()
    assert c["hh_count"] > 0 and c["pbs_blocks_used"] > 0 and c["total_processed_tokens"] == 820
