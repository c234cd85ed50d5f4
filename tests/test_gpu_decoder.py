"""The full-model prefill runner (ugbsa.decoder) against transformers' Qwen2.

The runner computes transformers' Qwen2 decoder math with fused, tensor-
parallel weights.  Here a small random-init Qwen2 model
is built from the runner's own weights and run through transformers with
``attn_implementation="block_sparse"`` (this package's hook, registered at
import) and with ``"sdpa"``; the runner's logits must agree with it within
bf16 GEMM rounding (the runner's fused QKV / gate-up GEMMs sum in another
order than transformers' separate projections): max-abs difference at most
3% of the largest logit, mean-abs at most 0.3% of it.
"""
import numpy as np
import pytest
import torch

from ugbsa import decoder, ops
from ugbsa import sparse_attention as sa

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

SHAPE = decoder.DecoderShape(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, intermediate=1024,
                             vocab=1000, rope_theta=1.0e6, rms_eps=1e-6)
SEL = dict(mode="router", router_score="quest", router_mode="quantile", router_grain="row", router_quantile=0.25,
           budget_blocks=2, k_min=1, k_max=112)


def _hf_model(run: decoder.TPDecoder, attn_impl: str):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    s = run.shape
    cfg = Qwen2Config(hidden_size=s.hidden, intermediate_size=s.intermediate, num_attention_heads=s.heads,
                      num_key_value_heads=s.kv_heads, num_hidden_layers=s.layers, vocab_size=s.vocab,
                      rope_parameters={"rope_type": "default", "rope_theta": s.rope_theta}, rms_norm_eps=s.rms_eps,
                      max_position_embeddings=8192, tie_word_embeddings=False)
    cfg._attn_implementation = attn_impl
    m = Qwen2ForCausalLM(cfg)
    inv_freq = m.model.rotary_emb.inv_freq.clone()          # fp32
    m = m.to(DEV).to(torch.bfloat16).eval()
    # .to(bfloat16) also rounds the rotary frequencies (a buffer) to bf16, which a
    # model loaded with torch_dtype=bfloat16 keeps in fp32: restore them
    m.model.rotary_emb.inv_freq = inv_freq.to(DEV)
    H, Hk, D, I = s.heads, s.kv_heads, s.head_dim, s.intermediate
    with torch.no_grad():
        m.model.embed_tokens.weight.copy_(run.embed)
        m.lm_head.weight.copy_(run.lm_head.t())
        m.model.norm.weight.copy_(run.final_norm)
        for lw, layer in zip(run.layers, m.model.layers):
            at, mlp = layer.self_attn, layer.mlp
            w, b = lw["w_qkv"], lw["b_qkv"]
            at.q_proj.weight.copy_(w[:, :H * D].t())
            at.k_proj.weight.copy_(w[:, H * D:(H + Hk) * D].t())
            at.v_proj.weight.copy_(w[:, (H + Hk) * D:].t())
            at.q_proj.bias.copy_(b[:H * D])
            at.k_proj.bias.copy_(b[H * D:(H + Hk) * D])
            at.v_proj.bias.copy_(b[(H + Hk) * D:])
            at.o_proj.weight.copy_(lw["w_o"].t())
            mlp.gate_proj.weight.copy_(lw["w_gu"][:, :I].t())
            mlp.up_proj.weight.copy_(lw["w_gu"][:, I:].t())
            mlp.down_proj.weight.copy_(lw["w_down"].t())
            layer.input_layernorm.weight.copy_(lw["ln1"])
            layer.post_attention_layernorm.weight.copy_(lw["ln2"])
    return m


def _close(a, b):
    a, b = a.float().cpu().numpy(), b.float().cpu().numpy()
    top = np.abs(b).max()
    d = np.abs(a - b)
    assert d.max() <= 0.03 * top and d.mean() <= 0.003 * top, (d.max(), d.mean(), top)
    return d.max() / top


@pytest.mark.parametrize("attention", ["block_sparse", "dense"])
def test_decoder_matches_transformers_qwen2(attention):
    S = 2048
    cfg = ops.SelectorConfig(**SEL)
    run = decoder.TPDecoder(SHAPE, cfg, attention=attention, seed=3, device=torch.device(DEV))
    ids = torch.randint(0, SHAPE.vocab, (S,), generator=torch.Generator().manual_seed(5)).to(DEV)
    got = run.forward(ids)
    saved = {x: getattr(sa.SEL, x) for x in list(SEL) + ["kernel_v2"]}
    try:
        for x, val in SEL.items():
            setattr(sa.SEL, x, val)
        sa.SEL.kernel_v2 = True
        m = _hf_model(run, "block_sparse" if attention == "block_sparse" else "sdpa")
        with torch.no_grad():
            want = m(input_ids=ids[None], use_cache=False).logits[0]
    finally:
        for x, val in saved.items():
            setattr(sa.SEL, x, val)
    rel = _close(got, want)
    print(f"{attention}: logits max-abs {rel:.2e} of the largest logit")
