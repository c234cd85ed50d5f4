"""GPU parity of the block-sparse decode (ugbsa_decode_select / _attn,
ugbsa_block_summary_update) against the CPU restatement
(tests/test_decode_oracle.py pins it to the prefill oracle and to dense
attention).

Bars: kv_idx, sigma and trigger bit-exact; attention max-abs <= 2e-2 and
mean-abs <= 2e-3 against the float64 restatement; with every block kept, the
same bar against torch's SDPA over the cache (the reference's decode); the
incrementally refreshed cache summaries bit-exact against a full summary.
"""
import math
import zlib

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle
from ugbsa import ops, sparse_attention as sa
from ugbsa.synth import planted_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAX_ABS, MEAN_ABS = 2e-2, 2e-3

# name, B, Hq, Hkv, S, D, dtype, selector
CASES = [
    ("quest_row_gqa", 1, 8, 2, 4097, 128, torch.bfloat16, dict(mode="router", router_score="quest", budget_blocks=8)),
    ("mean_cell_b3", 3, 4, 4, 2000, 64, torch.float16,
     dict(mode="router", router_grain="cell", router_quantile=0.3, budget_blocks=4)),
    ("topk_d256", 2, 4, 1, 8192, 256, torch.bfloat16, dict(mode="topk", budget_blocks=16)),
    ("abs_row_b4", 4, 4, 2, 3000, 128, torch.bfloat16,
     dict(mode="router", router_mode="abs", router_tau=2e-41, budget_blocks=4)),
    # the bench's geometry at 100K: 1563 blocks over a cluster of 7 CTAs, 7 Q heads per KV head
    ("quest_gqa7_100k", 1, 28, 4, 100000, 128, torch.bfloat16,
     dict(mode="router", router_score="quest", budget_blocks=64, k_max=112)),
    # more than 1024 cells: the prefill finish kernels on one-tile rows
    ("cells_1280_cell_quantile", 40, 32, 8, 700, 64, torch.bfloat16,
     dict(mode="router", router_grain="cell", router_quantile=0.3, budget_blocks=2)),
    # 12 Q heads per KV head: the 16-accumulator selection, two heads ranked per cluster CTA
    ("gqa12_d64_quest", 1, 12, 1, 3000, 64, torch.bfloat16,
     dict(mode="router", router_score="quest", budget_blocks=8)),
    # head dim 256 in fp16: one staged round in flight
    ("gqa4_d256_quest_fp16", 1, 8, 2, 20000, 256, torch.float16,
     dict(mode="router", router_score="quest", budget_blocks=16)),
]


def _cfgs(kw):
    base = dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                router_quantile=0.25, router_tau=0.1, budget_blocks=4, k_min=1, k_max=112)
    base.update(kw)
    return oracle.OracleConfig(**base), ops.SelectorConfig(**base)


def _check_attn(got, want):
    d = np.abs(got.float().cpu().numpy() - want)
    assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (d.max(), d.mean())


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_decode_matches_oracle(case):
    name, B, Hq, Hkv, S, D, dtype, kw = case
    ocfg, gcfg = _cfgs(kw)
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=4, seed=zlib.crc32(name.encode()) % 1000,
                                bf16=(dtype == torch.bfloat16))
    if dtype == torch.float16:
        q, k, v = (x.astype(np.float16).astype(np.float32) for x in (q, k, v))
    q1 = np.ascontiguousarray(q[:, :, -1:])
    scale = D ** -0.5
    # cache with spare capacity: K/V allocated for more rows than S, summaries for more blocks
    cap_rows = S + 200
    kd = torch.zeros((B, Hkv, cap_rows, D), device=DEV, dtype=dtype)
    vd = torch.zeros_like(kd)
    kd[:, :, :S] = torch.from_numpy(k).to(dtype)
    vd[:, :, :S] = torch.from_numpy(v).to(dtype)
    nb = math.ceil(S / 64)
    cap = nb + 5
    a = torch.empty((B, Hkv, cap, D), device=DEV, dtype=torch.float32)
    summ = (a, torch.empty_like(a)) if gcfg.quest else a
    ops.block_summary_update(kd[:, :, :S], gcfg.quest, summ, 0)
    qd = torch.from_numpy(q1).to(DEV).to(dtype)
    kv, sig, trig = ops.decode_select(qd, summ, S, Hkv, scale, gcfg, return_router=True)
    want = oracle.decode_select(q1, oracle.block_summary(k, gcfg.quest), S, scale, ocfg)
    assert np.array_equal(kv.cpu().numpy(), want["kv_idx"])
    s_got, s_want = sig.cpu().numpy(), want["sigma_eff"]
    nan = np.isnan(s_want)
    assert np.array_equal(nan, np.isnan(s_got))
    assert np.array_equal(s_got[~nan].view(np.uint32), s_want[~nan].view(np.uint32))
    assert np.array_equal(trig.cpu().numpy(), want["trigger"])
    out = ops.decode_attn(qd, kd, vd, kv, S, scale)
    _check_attn(out, oracle.decode_attn(q1, k, v, want["kv_idx"], S, scale))


@pytest.mark.parametrize("G", [1, 7])
def test_decode_attn_repeated_and_invalid_ids(G):
    # hand-made lists: a block repeated within one head's list counts twice (the slot-by-slot
    # path), ids >= NB and negative ids are skipped
    B, Hkv, S, D, kmax = 2, 2, 3000, 128, 12
    Hq = G * Hkv
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=2, seed=21, bf16=True)
    nb = math.ceil(S / 64)
    rng = np.random.default_rng(5)
    kv = rng.integers(0, nb, size=(B, Hq, kmax)).astype(np.int32)
    kv[0, 0, 3] = kv[0, 0, 1]           # repeat
    kv[1, -1, 5] = nb                   # sentinel
    kv[1, -1, 6] = -1                   # negative id
    kv[0, -1, :] = nb                   # a head with nothing kept
    q1 = np.ascontiguousarray(q[:, :, -1:])
    qd, kd, vd = (torch.from_numpy(x).to(DEV).to(torch.bfloat16) for x in (q1, k, v))
    out = ops.decode_attn(qd, kd, vd, torch.from_numpy(kv).to(DEV), S, D ** -0.5)
    want = oracle.decode_attn(q1, k, v, kv, S, D ** -0.5)
    _check_attn(out, want)


def test_decode_attn_past_bitmap_limit():
    # more than 8192 blocks: the union bitmaps do not fit and the kernel goes slot by slot
    B, Hq, Hkv, D, kmax = 1, 2, 1, 64, 16
    S = 8192 * 64 + 100
    nb = math.ceil(S / 64)
    g = torch.Generator().manual_seed(23)
    k = torch.randn((B, Hkv, S, D), generator=g).to(torch.bfloat16)
    v = torch.randn((B, Hkv, S, D), generator=g).to(torch.bfloat16)
    q = torch.randn((B, Hq, 1, D), generator=g).to(torch.bfloat16)
    rng = np.random.default_rng(7)
    kv = np.stack([np.stack([rng.permutation(nb)[:kmax] for _ in range(Hq)])]).astype(np.int32)
    kv[0, 0, 0] = nb - 1                 # the ragged last block
    out = ops.decode_attn(q.to(DEV), k.to(DEV), v.to(DEV), torch.from_numpy(kv).to(DEV), S, D ** -0.5)
    want = oracle.decode_attn(q.float().numpy(), k.float().numpy(), v.float().numpy(), kv, S, D ** -0.5)
    _check_attn(out, want)


def test_decode_attn_union_without_repeats():
    # distinct ids per head, heavily shared across the group (the union path), ragged S
    B, Hq, Hkv, S, D, kmax = 1, 14, 2, 5000, 64, 20
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=2, seed=22, bf16=True)
    nb = math.ceil(S / 64)
    rng = np.random.default_rng(6)
    kv = np.stack([np.stack([rng.permutation(np.arange(nb // 2))[:kmax] for _ in range(Hq)])
                   for _ in range(B)]).astype(np.int32)
    kv[0, :, 0] = nb - 1                 # the ragged last block everywhere
    q1 = np.ascontiguousarray(q[:, :, -1:])
    qd, kd, vd = (torch.from_numpy(x).to(DEV).to(torch.bfloat16) for x in (q1, k, v))
    out = ops.decode_attn(qd, kd, vd, torch.from_numpy(kv).to(DEV), S, D ** -0.5)
    _check_attn(out, oracle.decode_attn(q1, k, v, kv, S, D ** -0.5))


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_decode_step_matches_separate_calls(case):
    # the fused step (refresh inside the selection, router inside the attention; the
    # separate calls past 256 cells) against refresh + decode_select + decode_attn:
    # identical outputs, lists, margins, triggers and refreshed summaries
    name, B, Hq, Hkv, S, D, dtype, kw = case
    if dtype == torch.float32:
        pytest.skip("the attention takes bf16 / fp16")
    _, gcfg = _cfgs(kw)
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=4, seed=zlib.crc32(name.encode()) % 1000,
                                bf16=(dtype == torch.bfloat16))
    qd = torch.from_numpy(np.ascontiguousarray(q[:, :, -1:])).to(DEV).to(dtype)
    kd = torch.from_numpy(k).to(DEV).to(dtype)
    vd = torch.from_numpy(v).to(DEV).to(dtype)
    nb = math.ceil(S / 64)
    cap = nb + 3
    scale = D ** -0.5

    def fresh_cache():
        a = torch.empty((B, Hkv, cap, D), device=DEV, dtype=torch.float32)
        summ = (a, torch.empty_like(a)) if gcfg.quest else a
        ops.block_summary_update(kd, gcfg.quest, summ, 0)
        for t in (summ if gcfg.quest else (summ,)):   # a stale last block
            t[:, :, nb - 1].fill_(123.0)
        return summ

    s1 = fresh_cache()
    ops.block_summary_update(kd, gcfg.quest, s1, nb - 1)
    kv1, sig1, trig1 = ops.decode_select(qd, s1, S, Hkv, scale, gcfg, return_router=True)
    out1 = ops.decode_attn(qd, kd, vd, kv1, S, scale)
    s2 = fresh_cache()
    out2, kv2, sig2, trig2 = ops.decode_step(qd, kd, vd, s2, S, scale, gcfg, return_router=True)
    assert torch.equal(kv1, kv2)
    assert torch.equal(trig1, trig2)
    a1, a2 = sig1.cpu().numpy(), sig2.cpu().numpy()
    assert np.array_equal(np.isnan(a1), np.isnan(a2))
    assert np.array_equal(a1[~np.isnan(a1)].view(np.uint32), a2[~np.isnan(a2)].view(np.uint32))
    assert torch.equal(out1, out2)
    for t1, t2 in (zip(s1, s2) if gcfg.quest else ((s1, s2),)):
        assert torch.equal(t1[:, :, :nb], t2[:, :, :nb])


def test_decode_with_every_block_kept_matches_sdpa():
    B, Hq, Hkv, S, D = 2, 8, 2, 5000, 128
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=4, seed=12, bf16=True)
    nb = math.ceil(S / 64)
    _, gcfg = _cfgs(dict(mode="topk", budget_blocks=nb, k_max=10 ** 6))
    qd, kd, vd = (torch.from_numpy(x).to(DEV).to(torch.bfloat16) for x in (q[:, :, -1:], k, v))
    summ = ops.block_summary(kd, False)
    kv = ops.decode_select(qd, summ, S, Hkv, D ** -0.5, gcfg)
    out = ops.decode_attn(qd, kd, vd, kv, S, D ** -0.5)
    ref = F.scaled_dot_product_attention(qd.float(), kd.float(), vd.float(), scale=D ** -0.5, enable_gqa=True)
    _check_attn(out, ref.cpu().numpy())


def test_summary_cache_refreshes_only_new_blocks():
    B, Hkv, D = 1, 2, 128
    S0, steps = 1000, 90
    _, k, _, _ = planted_inputs(B, Hkv, Hkv, S0 + steps, D, n_planted=2, seed=13, bf16=True)
    kd = torch.from_numpy(k).to(DEV).to(torch.bfloat16)
    cache = sa.SummaryCache()
    for quest in (True, False):
        cache.reset()
        for S in [S0] + list(range(S0 + 1, S0 + steps + 1)):
            got = cache.get(3, kd[:, :, :S], quest)
            if S in (S0, S0 + 24, S0 + steps):
                nb = math.ceil(S / 64)
                want = ops.block_summary(kd[:, :, :S], quest)
                if quest:
                    assert torch.equal(got[0][:, :, :nb], want[0]) and torch.equal(got[1][:, :, :nb], want[1])
                else:
                    assert torch.equal(got[:, :, :nb], want)


def test_hook_sparse_decode():
    B, Hq, Hkv, S, D = 1, 4, 2, 3000, 128
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=3, seed=14, bf16=True)
    qd, kd, vd = (torch.from_numpy(x).to(DEV).to(torch.bfloat16) for x in (q[:, :, -1:], k, v))
    saved = (sa.SEL.mode, sa.SEL.kernel_v2, sa.SEL.decode_sparse, sa.SEL.router_score, sa.SEL.budget_blocks,
             sa.SEL.k_min)
    sa.SEL.mode, sa.SEL.kernel_v2, sa.SEL.decode_sparse, sa.SEL.router_score = "router", True, True, "quest"
    sa.SEL.budget_blocks, sa.SEL.k_min = 4, 1

    class _M:
        layer_idx = 7
        num_key_value_groups = Hq // Hkv

    try:
        sa.SUMM_CACHE.reset()
        out, _ = sa.block_sparse_attention(_M(), qd, kd, vd, None, D ** -0.5)
        cfg = sa.SEL.config()
        kv = ops.decode_select(qd, ops.block_summary(kd, True), S, Hkv, D ** -0.5, cfg)
        ref = ops.decode_attn(qd, kd, vd, kv, S, D ** -0.5)
    finally:
        (sa.SEL.mode, sa.SEL.kernel_v2, sa.SEL.decode_sparse, sa.SEL.router_score, sa.SEL.budget_blocks,
         sa.SEL.k_min) = saved
        sa.SUMM_CACHE.reset()
    assert out.shape == (B, 1, Hq, D)
    assert torch.equal(out, ref.transpose(1, 2))
