"""Pin the norm + rotary restatement (oracle.qk_norm_rope) to transformers'
own modules, which the reference's model path calls (it imports
apply_rotary_pos_emb from transformers, src/sparse_attention.py:47-48):
Qwen3RMSNorm + the Qwen3 rotary ("scale" mode) and Qwen3.5-MoE's RMSNorm
(1 + w) + its partial rotary ("offset" mode), on seeded bf16 inputs, CPU.

The restatement fixes the fp32 order of the sum of squares and uses a
correctly rounded 1/sqrt; torch's reduction order and rsqrt can move the
inverse norm by an ulp, so a rounded element may differ by one unit in its
last place.  The bar: at least 99.9% of elements bit-identical, none further
than two bf16 units in the last place of the row's largest magnitude.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

transformers = pytest.importorskip("transformers")


def _ulp_ok(a, b):
    """(every element within two bf16 units in the last place of its row's
    largest magnitude, fraction bit-identical)."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    m = np.maximum(np.abs(a), np.abs(b)).max(-1, keepdims=True)
    ulp = np.exp2(np.floor(np.log2(np.maximum(m, 1e-30))) - 7)
    return bool(np.all(np.abs(a - b) <= 2 * ulp)), float(np.mean(a == b))


def _rope_tables(B, S, R, seed):
    g = torch.Generator().manual_seed(seed)
    pos = torch.arange(S, dtype=torch.float32)[None].expand(B, S) + torch.randint(0, 100, (B, 1), generator=g)
    inv = 1.0 / (10000 ** (torch.arange(0, R, 2, dtype=torch.float32) / R))
    f = pos[..., None] * inv
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


@pytest.mark.parametrize("mode,D,R", [("scale", 128, 128), ("offset", 256, 64), ("offset", 128, 128),
                                      ("scale", 64, 64), ("offset", 64, 32)])
def test_norm_rope_matches_transformers(mode, D, R):
    B, S, H = 2, 96, 3
    g = torch.Generator().manual_seed(D + R)
    x = (torch.randn(B, S, H, D, generator=g) * 3).to(torch.bfloat16)
    cos, sin = _rope_tables(B, S, R, 7)
    if mode == "scale":
        from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb
        norm = Qwen3RMSNorm(D, eps=1e-6)
        w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
        assert R == D
    else:
        from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeRMSNorm as Norm
        from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import apply_rotary_pos_emb
        norm = Norm(D, eps=1e-6)
        w = (0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    norm = norm.to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(w)
        y = norm(x).transpose(1, 2)                  # [B, H, S, D]
        ref, _ = apply_rotary_pos_emb(y, y, cos, sin)
    got = oracle.qk_norm_rope(x.transpose(1, 2).float().numpy(), w.float().numpy(), 1e-6, cos.float().numpy(),
                              sin.float().numpy(), norm_mode=mode)
    ok, same = _ulp_ok(got, ref.float().numpy())
    assert ok and same >= 0.999, same


@pytest.mark.parametrize("D", [128, 64])
def test_rotary_only_matches_qwen2(D):
    """norm_mode "none": Qwen2's attention rotates Q and K without a per-head
    norm (transformers' modeling_qwen2.apply_rotary_pos_emb); bit for bit."""
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb
    B, S, H = 2, 96, 3
    g = torch.Generator().manual_seed(D)
    x = (torch.randn(B, H, S, D, generator=g) * 3).to(torch.bfloat16)
    cos, sin = _rope_tables(B, S, D, 11)
    with torch.no_grad():
        ref, _ = apply_rotary_pos_emb(x, x, cos, sin)
    got = oracle.qk_norm_rope(x.float().numpy(), None, 0.0, cos.float().numpy(), sin.float().numpy(),
                              norm_mode="none")
    assert np.array_equal(got, ref.float().numpy())
