"""The config-4 decoder stack's composition, checked on CPU.

``DecoderStack`` runs with the MXFP4 calls replaced by the reference's safe
path restated in PyTorch (CPU tensors) and is compared with transformers'
``Qwen3MoeDecoderLayer`` holding the same dequantized weights: RMSNorms, q/k
head norms, rotary embedding, grouped-query causal attention, the softmax
top-k router, the SiLU-gated experts and both residuals must agree.  A
prefill followed by decode steps through the KV cache must equal the prefill
of the whole sequence.  No GPU is needed.
"""

from types import SimpleNamespace

import torch

import _gpu_ref as gref
from _paths import PKG, load_by_path

ds = load_by_path("mxfp4_decoder_stack", PKG / "decoder_stack.py")
CFG = ds.StackConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, top_k=2, inter=128)


def _router(logits, top_k):
    p = torch.softmax(logits.float(), dim=-1)
    w, i = torch.topk(p, top_k, dim=-1)
    return w / w.sum(-1, keepdim=True), i.to(torch.int32)


REF_OPS = SimpleNamespace(linear_mxfp4_soft=gref.linear, moe_router=_router, moe_layer_mxfp4=gref.moe_layer)


def _small_scales(L):
    # scales near 2^-4 keep the random weights' outputs O(1) through the layers
    for name in ("qkv_s", "o_s", "router_s", "s13", "s2"):
        t = getattr(L, name)
        t.copy_(torch.randint(120, 124, t.shape, dtype=torch.uint8))
    return L


def _hf_layer(L, cfg):
    from transformers.models.qwen3_moe import modeling_qwen3_moe as hf

    hc = hf.Qwen3MoeConfig(hidden_size=cfg.hidden, num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads,
                           head_dim=cfg.head_dim, num_experts=cfg.experts, num_experts_per_tok=cfg.top_k,
                           moe_intermediate_size=cfg.inter, norm_topk_prob=True, rms_norm_eps=cfg.eps,
                           rope_theta=cfg.rope_theta, hidden_act="silu", attention_bias=False, decoder_sparse_step=1,
                           mlp_only_layers=[], max_position_embeddings=4096)
    hc._attn_implementation = "sdpa"
    layer = hf.Qwen3MoeDecoderLayer(hc, 0).to(torch.float32).eval()
    deq = lambda w, s: gref.dequant(w, s, torch.float32)  # noqa: E731
    qkv = deq(L.qkv_w, L.qkv_s)
    with torch.no_grad():
        a = layer.self_attn
        a.q_proj.weight.copy_(qkv[:cfg.q_size])
        a.k_proj.weight.copy_(qkv[cfg.q_size:cfg.q_size + cfg.kv_size])
        a.v_proj.weight.copy_(qkv[cfg.q_size + cfg.kv_size:])
        a.o_proj.weight.copy_(deq(L.o_w, L.o_s))
        a.q_norm.weight.copy_(L.q_norm.float())
        a.k_norm.weight.copy_(L.k_norm.float())
        layer.input_layernorm.weight.copy_(L.ln1.float())
        layer.post_attention_layernorm.weight.copy_(L.ln2.float())
        layer.mlp.gate.weight.copy_(deq(L.router_w, L.router_s))
        layer.mlp.experts.gate_up_proj.copy_(deq(L.w13, L.s13))
        layer.mlp.experts.down_proj.copy_(deq(L.w2, L.s2))
    return layer, hf.Qwen3MoeRotaryEmbedding(hc)


def test_layer_matches_transformers_qwen3_moe():
    torch.manual_seed(0)
    L = _small_scales(ds.random_layer(CFG, torch.device("cpu"), seed=1))
    seq = 24
    h = torch.randn(seq, CFG.hidden).to(torch.bfloat16)
    stack = ds.DecoderStack(ds.StackConfig(**{**CFG.__dict__, "layers": 1}), [L], max_ctx=64, ops=REF_OPS)
    stack.allocate_cache(1, seq)
    got = stack.prefill(h, 1).float()
    layer, rope = _hf_layer(L, CFG)
    pos = torch.arange(seq)[None]
    x = h.float()[None]
    cos, sin = rope(x, pos)
    mask = torch.full((seq, seq), float("-inf")).triu(1)[None, None]
    with torch.no_grad():
        want = layer(x, attention_mask=mask, position_ids=pos, position_embeddings=(cos, sin))
    want = (want[0] if isinstance(want, tuple) else want)[0]
    rel = ((got - want).norm(dim=-1) / want.norm(dim=-1))
    # BF16 activations between the ops here, FP32 in the transformers layer
    assert float(rel.median()) < 2e-2, rel
    assert float((rel < 5e-2).float().mean()) >= 0.9, rel


def test_decode_through_the_cache_equals_prefill():
    torch.manual_seed(1)
    layers = [_small_scales(ds.random_layer(CFG, torch.device("cpu"), seed=10 + i)) for i in range(CFG.layers)]
    seqs, prompt, steps = 2, 12, 3
    full = torch.randn(seqs, prompt + steps, CFG.hidden).to(torch.bfloat16)
    a = ds.DecoderStack(CFG, layers, max_ctx=64, ops=REF_OPS)
    a.allocate_cache(seqs, prompt + steps)
    want = a.prefill(full.reshape(-1, CFG.hidden), seqs).reshape(seqs, prompt + steps, -1)
    b = ds.DecoderStack(CFG, layers, max_ctx=64, ops=REF_OPS)
    b.allocate_cache(seqs, prompt + steps)
    first = b.prefill(full[:, :prompt].reshape(-1, CFG.hidden), seqs).reshape(seqs, prompt, -1)
    assert torch.allclose(first.float(), want[:, :prompt].float(), rtol=2e-2, atol=2e-2)
    for i in range(steps):
        got = b.decode(full[:, prompt + i], prompt + i)
        assert torch.allclose(got.float(), want[:, prompt + i].float(), rtol=2e-2, atol=2e-2), i
