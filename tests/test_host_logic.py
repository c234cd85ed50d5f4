"""Host-side logic that needs no GPU: head sharding, the Selector surface,
FLOP accounting, the synthetic generators."""
import numpy as np
import pytest
import torch

from ugbsa import parallel
from ugbsa import sparse_attention as sa
from ugbsa.synth import input_digest, planted_inputs, round_to_bf16


@pytest.mark.parametrize("Hq,Hkv,world", [(28, 4, 1), (28, 4, 2), (28, 4, 4), (28, 4, 8), (40, 8, 8),
                                          (16, 2, 2), (16, 2, 4), (16, 2, 8), (6, 2, 4)])
def test_head_shards_partition_heads_along_groups(Hq, Hkv, world):
    G = Hq // Hkv
    shards = parallel.all_shards(Hq, Hkv, world)
    covered = []
    for s in shards:
        covered += list(range(s.q0, s.q1))
        assert s.hq_local >= 1
        # every local Q head reads a KV head inside the rank's KV slice
        for h in range(s.q0, s.q1):
            assert s.kv0 <= h // G < s.kv1
        # the kernel's uniform GQA mapping h_local / (Hq_local / Hkv_local) is valid
        assert s.hq_local % s.hkv_local == 0
        for hl in range(s.hq_local):
            assert (s.q0 + hl) // G - s.kv0 == hl // (s.hq_local // s.hkv_local)
    assert covered == list(range(Hq))
    sizes = [s.hq_local for s in shards]
    assert max(sizes) - min(sizes) <= 1


def test_head_shard_rejects_unalignable_world():
    with pytest.raises(ValueError):
        parallel.HeadShard.make(28, 4, 3, 0)


def test_selector_defaults_match_reference():
    # src/sparse_attention.py:57-97
    s = sa.Selector()
    assert (s.mode, s.budget_blocks, s.k_min, s.k_max) == ("dense", 32, 8, 112)
    assert (s.router_mode, s.router_grain, s.router_tau, s.router_quantile, s.router_score) == \
        ("abs", "cell", 0.10, 0.20, "mean")
    assert s.kernel_v2 is False


def test_hook_rejects_out_of_scope_modes():
    class M:
        layer_idx = 0
        num_key_value_groups = 1
    old = sa.SEL.mode, sa.SEL.kernel_v2
    try:
        sa.SEL.mode, sa.SEL.kernel_v2 = "belief", True
        q = torch.zeros(1, 2, 128, 64)
        with pytest.raises(NotImplementedError):
            sa.block_sparse_attention(M(), q, q, q, None, 0.125)
    finally:
        sa.SEL.mode, sa.SEL.kernel_v2 = old


def test_sparse_decode_domain():
    bf = torch.bfloat16
    assert sa.sparse_decode_supported(torch.zeros(1, 8, 1, 128, dtype=bf), torch.zeros(1, 2, 4096, 128, dtype=bf))
    # fp32, head dim 96, 32 Q heads per KV head, more than 8192 blocks: outside it
    assert not sa.sparse_decode_supported(torch.zeros(1, 8, 1, 128), torch.zeros(1, 2, 4096, 128))
    assert not sa.sparse_decode_supported(torch.zeros(1, 8, 1, 96, dtype=bf), torch.zeros(1, 2, 4096, 96, dtype=bf))
    assert not sa.sparse_decode_supported(torch.zeros(1, 32, 1, 64, dtype=bf), torch.zeros(1, 1, 4096, 64, dtype=bf))
    assert not sa.sparse_decode_supported(torch.zeros(1, 2, 1, 64, dtype=bf),
                                          torch.zeros(1, 1, 8192 * 64 + 1, 64, dtype=bf))


def test_hook_decodes_densely_outside_the_sparse_decode_domain():
    # an fp32 decode row with SEL.decode_sparse set: the reference's dense SDPA decode
    class M:
        layer_idx = 0
        num_key_value_groups = 2
    old = sa.SEL.mode, sa.SEL.kernel_v2, sa.SEL.decode_sparse
    try:
        sa.SEL.mode, sa.SEL.kernel_v2, sa.SEL.decode_sparse = "router", True, True
        g = torch.Generator().manual_seed(3)
        q = torch.randn(1, 4, 1, 64, generator=g)
        k = torch.randn(1, 2, 300, 64, generator=g)
        v = torch.randn(1, 2, 300, 64, generator=g)
        out, _ = sa.block_sparse_attention(M(), q, k, v, None, 0.125)
        want = torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=0.125, enable_gqa=True)
        assert out.shape == (1, 1, 4, 64)
        assert torch.allclose(out, want.transpose(1, 2), atol=1e-6)
    finally:
        sa.SEL.mode, sa.SEL.kernel_v2, sa.SEL.decode_sparse = old


def test_selected_block_flops_counts_usable_slots():
    S, D = 256, 128
    nb = 4
    kv = torch.tensor([[[[0, 4, 4], [1, 0, 3], [2, 1, 0], [3, 0, 1]]]], dtype=torch.int32)
    # tile 0: {0}; tile 1: {1, 0} (3 is future); tile 2: {2,1,0}; tile 3: {3,0,1}
    assert parallel.selected_block_flops(kv, S, D) == 9 * 4 * 64 * 64 * D
    assert nb == 4


def test_planted_inputs_deterministic_and_bf16():
    a = planted_inputs(1, 4, 2, 512, 64, n_planted=3, seed=5, chained=True, bf16=True)
    b = planted_inputs(1, 4, 2, 512, 64, n_planted=3, seed=5, chained=True, bf16=True)
    assert input_digest(*a[:3]) == input_digest(*b[:3])
    q = a[0]
    assert np.array_equal(round_to_bf16(q), q)
    assert a[3].shape == (1, 2, 3)


def test_round_to_bf16_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32)
    t = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(round_to_bf16(x), t)


def test_decoder_tensor_parallel_layout_covers_everything_once():
    """ugbsa.decoder.TPLayout: every Q head, KV head (replicated only when the ranks
    outnumber the KV heads), intermediate column and vocab entry lands on a rank."""
    from ugbsa import decoder
    for shape in (decoder.QWEN25_7B, decoder.QWEN25_14B):
        for world in (1, 2, 4, 8):
            lays = [decoder.TPLayout.make(shape, world, r) for r in range(world)]
            q = sorted((L.shard.q0, L.shard.q1) for L in lays)
            assert q[0][0] == 0 and q[-1][1] == shape.heads
            assert all(a[1] == b[0] for a, b in zip(q, q[1:]))
            kv = {h for L in lays for h in range(L.shard.kv0, L.shard.kv1)}
            assert kv == set(range(shape.kv_heads))
            for L in lays:   # a rank's Q heads read only its KV heads
                G = shape.heads // shape.kv_heads
                assert L.shard.kv0 == L.shard.q0 // G and L.shard.kv1 == (L.shard.q1 - 1) // G + 1
            inter = sorted((L.inter0, L.inter1) for L in lays)
            assert inter[0][0] == 0 and inter[-1][1] == shape.intermediate
            assert all(a[1] == b[0] for a, b in zip(inter, inter[1:]))
            voc = sorted((L.vocab0, L.vocab1) for L in lays)
            assert voc[0][0] == 0 and voc[-1][1] == shape.vocab
            assert all(a[1] == b[0] for a, b in zip(voc, voc[1:]))


def test_decoder_flop_counts():
    from ugbsa import decoder
    s = decoder.QWEN25_7B
    # 7.07 B parameters in the linear layers and lm_head (embeddings excluded)
    assert abs(s.gemm_flops(1) / 2 - 7.07e9) / 7.07e9 < 0.01
    qt = 131072 // 64
    assert s.dense_attn_flops(131072) == 28 * 28 * qt * (qt + 1) / 2 * 4 * 64 * 64 * 128
