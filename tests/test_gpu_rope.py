"""GPU parity of the fused per-head RMSNorm + rotary + K summary producer
(ugbsa_qk_norm_rope) against the oracle restatement, which
tests/test_rope_oracle.py pins to transformers' own modules.

Bars: at least 99.9% of output elements bit-identical to the oracle and none
further than two units in the last place of the row's largest magnitude (the
fp32 sum of squares runs in a different order); the K block summaries bit-exact against ugbsa_block_summary
of the kernel's own output; in place (Y = X) equals out of place; the
selection fed with the producer's summaries equals the selection that
computes them itself.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from ugbsa import ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _ulp_ok(a, b, dtype):
    """(every element within two units in the last place of its row's largest
    magnitude, fraction bit-identical): an input one ulp apart moves each
    rotated output by at most about one ulp of the terms it sums, which can
    be larger than the output itself when the two terms cancel."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    mant = 7 if dtype == torch.bfloat16 else 10
    m = np.maximum(np.abs(a), np.abs(b)).max(-1, keepdims=True)
    ulp = np.exp2(np.floor(np.log2(np.maximum(m, 1e-30))) - mant)
    return bool(np.all(np.abs(a - b) <= 2 * ulp)), float(np.mean(a == b))


def _tables(B, S, R, dtype):
    pos = torch.arange(S, dtype=torch.float32)[None].expand(B, S) + 3 * torch.arange(B)[:, None]
    inv = 1.0 / (10000 ** (torch.arange(0, R, 2, dtype=torch.float32) / R))
    f = pos[..., None] * inv
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


# B, H, S, D, R, mode, dtype, summary
CASES = [
    (1, 4, 2048, 128, 128, "scale", torch.bfloat16, "quest"),
    (2, 2, 1000, 256, 64, "offset", torch.bfloat16, "mean"),
    (1, 3, 777, 64, 32, "offset", torch.float16, "quest"),
    (2, 2, 512, 128, 16, "scale", torch.float16, None),
    (1, 4, 1000, 128, 128, "none", torch.bfloat16, "quest"),   # Qwen2: rotary without a per-head norm
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[5]}-d{c[3]}-r{c[4]}-S{c[2]}-{str(c[6])[6:]}" for c in CASES])
def test_norm_rope_matches_oracle(case):
    B, H, S, D, R, mode, dtype, summary = case
    g = torch.Generator().manual_seed(S + D)
    proj = (torch.randn(B, S, H, D, generator=g) * 2).to(dtype)         # a projection output [B, S, H, D]
    w = ((1.0 if mode == "scale" else 0.0) + 0.1 * torch.randn(D, generator=g)).to(dtype)
    cos, sin = _tables(B, S, R, dtype)
    want = oracle.qk_norm_rope(proj.transpose(1, 2).float().numpy(), w.float().numpy(), 1e-6,
                               cos.float().numpy(), sin.float().numpy(), norm_mode=mode,
                               dtype="bf16" if dtype == torch.bfloat16 else "fp16")
    xd = proj.to(DEV).transpose(1, 2)                                   # [B, H, S, D] view
    res = ops.qk_norm_rope(xd, w.to(DEV), 1e-6, cos.to(DEV), sin.to(DEV), norm_mode=mode, summary=summary)
    out, summ = (res if summary else (res, None))
    ok, same = _ulp_ok(out.float().cpu().numpy(), want, dtype)
    assert ok and same >= 0.999, same
    if mode == "none":   # no sum of squares: every element bit-identical
        assert same == 1.0
    if summary:
        ref = ops.block_summary(out, summary == "quest")
        if summary == "quest":
            assert torch.equal(summ[0], ref[0]) and torch.equal(summ[1], ref[1])
        else:
            assert torch.equal(summ, ref)
    # in place, into the projection buffer itself
    xi = proj.to(DEV)
    ops.qk_norm_rope(xi.transpose(1, 2), w.to(DEV), 1e-6, cos.to(DEV), sin.to(DEV), norm_mode=mode,
                     out=xi.transpose(1, 2))
    assert torch.equal(xi.transpose(1, 2), out)


def test_selection_with_producer_summaries():
    B, Hq, Hkv, S, D = 1, 8, 2, 4096, 128
    g = torch.Generator().manual_seed(5)
    qp = torch.randn(B, S, Hq, D, generator=g).to(torch.bfloat16).to(DEV)
    kp = torch.randn(B, S, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    wq = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).to(DEV)
    wk = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).to(DEV)
    cos, sin = (t.to(DEV) for t in _tables(B, S, D, torch.bfloat16))
    q = ops.qk_norm_rope(qp.transpose(1, 2), wq, 1e-6, cos, sin, norm_mode="scale")
    k, summ = ops.qk_norm_rope(kp.transpose(1, 2), wk, 1e-6, cos, sin, norm_mode="scale", summary="quest")
    cfg = ops.SelectorConfig(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                             router_quantile=0.25, budget_blocks=8, k_min=1, k_max=112)
    a = ops.select_kv_idx(q, k, D ** -0.5, cfg)
    b = ops.select_kv_idx(q, k, D ** -0.5, cfg, summ=summ)
    assert torch.equal(a, b)
