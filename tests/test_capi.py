"""C ABI checks that need no GPU: the library loads, exports what include/ugbsa.h
declares, and its host-side logic (budget arithmetic, argument validation)
matches the reference's rules."""
import ctypes
import os
import re

import pytest

from oracle import oracle
from ugbsa import _build, _lib, ops

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "ugbsa.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ugbsa_[a-z_0-9]+)\s*\(", src)))


def test_library_builds_and_loads():
    _build.build()
    assert os.path.exists(_lib.LIB_PATH)
    L = _lib.load()
    assert L.ugbsa_version() >= 100


def test_every_declared_symbol_is_exported():
    L = _lib.load()
    names = header_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/ugbsa.h but not exported"
    # and the ctypes table covers the header exactly
    assert set(names) == set(_lib.SIGNATURES)


def test_status_strings():
    for code in range(0, 10):
        assert _lib.status_string(code)
    assert "unknown" in _lib.status_string(999)


@pytest.mark.parametrize("mode", ["topk", "quest", "router"])
@pytest.mark.parametrize("S", [64, 200, 4096, 131072])
@pytest.mark.parametrize("budget,k_min,k_max", [(4, 1, 112), (2, 8, 112), (500, 1, 112), (64, 1, 112), (1, 1, 1)])
def test_budget_matches_reference_rule(mode, S, budget, k_min, k_max):
    g = ops.SelectorConfig(mode=mode, budget_blocks=budget, k_min=k_min, k_max=k_max)
    o = oracle.OracleConfig(mode=mode, budget_blocks=budget, k_min=k_min, k_max=k_max)
    assert ops.budget(g, S) == oracle.budget(o, S)


def test_bench_budget_is_nb_over_16():
    g = ops.SelectorConfig(mode="router", router_score="quest", budget_blocks=64, k_min=1, k_max=112)
    assert ops.budget(g, 131072) == (128, 256)


def _cfg():
    return ops.SelectorConfig(mode="router").to_c()


def test_argument_validation_without_device():
    L = _lib.load()
    st = _lib.Strides(1 << 20, 1 << 16, 128, 1)
    fake = ctypes.c_void_p(1 << 20)   # never dereferenced: validation fails first
    # unsupported head_dim
    assert L.ugbsa_block_summary(fake, _lib.BF16, st, 1, 1, 64, 100, 0, fake, None, None, None) == 5
    # null output
    assert L.ugbsa_block_summary(fake, _lib.BF16, st, 1, 1, 64, 128, 0, None, None, None, None) == 1
    # bad dtype
    assert L.ugbsa_block_summary(fake, 7, st, 1, 1, 64, 128, 0, fake, None, None, None) == 3
    # innermost stride must be 1
    bad = _lib.Strides(1 << 20, 1 << 16, 128, 2)
    assert L.ugbsa_block_summary(fake, _lib.BF16, bad, 1, 1, 64, 128, 0, fake, None, None, None) == 4
    # misaligned outer stride (bf16 rows of 100 elements)
    bad = _lib.Strides(1 << 20, 1 << 16, 100, 1)
    assert L.ugbsa_block_summary(fake, _lib.BF16, bad, 1, 1, 64, 128, 0, fake, None, None, None) == 4
    c = _cfg()
    # Hq not a multiple of Hkv
    assert L.ugbsa_select(fake, _lib.BF16, st, fake, None, 1, 6, 4, 4096, 128, ctypes.c_float(0.1),
                          ctypes.byref(c), fake, 16, None, None, fake, 1 << 20, None) == 2
    # kmax inconsistent with the budget
    assert L.ugbsa_select(fake, _lib.BF16, st, fake, None, 1, 8, 8, 4096, 128, ctypes.c_float(0.1),
                          ctypes.byref(c), fake, 17, None, None, fake, 1 << 20, None) == 2
    # workspace too small
    assert L.ugbsa_select(fake, _lib.BF16, st, fake, None, 1, 8, 8, 4096, 128, ctypes.c_float(0.1),
                          ctypes.byref(c), fake, 64, None, None, fake, 8, None) == 6
    # attention: an unknown dtype; fp32 (the CUDA-core kernel) has no output peers; head_dim 96 unsupported
    assert L.ugbsa_attn(fake, fake, fake, 7, st, st, st, fake, 16, 1, 8, 8, 4096, 4096, 128,
                        ctypes.c_float(0.1), fake, st, None) == 3
    peers = (ctypes.c_void_p * 1)(fake)
    assert L.ugbsa_attn_rows_peers(fake, fake, fake, _lib.F32, st, st, st, fake, 16, 1, 8, 8, 4096, 4096, 128, 0,
                                   1, ctypes.c_float(0.1), fake, st, peers, 1, None) == 3
    assert L.ugbsa_attn(fake, fake, fake, _lib.BF16, st, st, st, fake, 16, 1, 8, 8, 4096, 4096, 96,
                        ctypes.c_float(0.1), fake, st, None) == 5
    # arithmetic check: negative count, null operand
    assert L.ugbsa_check_bf16_fma(fake, fake, fake, fake, fake, -1, None) == 1
    assert L.ugbsa_check_bf16_fma(fake, None, fake, fake, fake, 4, None) == 1


def test_row_slice_validation_without_device():
    L = _lib.load()
    st = _lib.Strides(1 << 20, 1 << 16, 128, 1)
    fake = ctypes.c_void_p(1 << 20)
    c = _cfg()
    kb, km = ctypes.c_int(0), ctypes.c_int(0)
    assert L.ugbsa_select_budget(ctypes.byref(c), 4096, ctypes.byref(kb), ctypes.byref(km)) == 0

    def tiles(row_base, Sq, S=4096, stride=1):
        return L.ugbsa_select_tiles_rows(fake, _lib.BF16, st, fake, None, 1, 8, 8, S, 128, row_base, stride, Sq,
                                         ctypes.c_float(0.1), ctypes.byref(c), fake, km.value, fake, None, fake,
                                         1 << 30, None)
    assert tiles(64, 1024) == 2          # a slice starts on a tile pair (128 rows)
    assert tiles(-128, 1024) == 2
    assert tiles(128, 1000) == 2         # whole tiles unless the slice ends at S
    assert tiles(3072, 2048) == 2        # past the end of the sequence
    assert tiles(0, 0) == 2
    assert tiles(0, 1024, stride=0) == 2
    assert tiles(128, 2000, stride=2) == 2       # dealt pairs 1, 3, ..., 31: 32 whole tiles, 2048 rows
    assert tiles(128, 2048 + 64, stride=2) == 2  # a 33rd tile would be past the sequence

    def finish(row_base, Sq, S=4096, stride=1):
        return L.ugbsa_select_finish_rows(fake, fake, 1, 8, 8, S, row_base, stride, Sq, ctypes.byref(c), fake,
                                          km.value, None, None, fake, 1 << 30, None)
    assert finish(32, 1024) == 2
    assert finish(4032, 128) == 2
    assert finish(64, 1024, stride=2) == 2   # dealt slices start on a pair

    def attn(row_base, Sq, Sk=4096, stride=1):
        return L.ugbsa_attn_rows(fake, fake, fake, _lib.BF16, st, st, st, fake, 16, 1, 8, 8, Sq, Sk, 128, row_base,
                                 stride, ctypes.c_float(0.1), fake, st, None)
    assert attn(32, 1024) == 2           # tile-aligned rows only
    assert attn(3584, 1024) == 2         # rows past the keys
    assert attn(-64, 1024) == 2
    assert attn(0, 1000, Sk=1000, stride=3) == 2   # dealt: 3 pairs of 16 tiles dealt to rank 0: 6 tiles, 384 rows


def test_seq_shard_ranges_cover_pairs():
    from ugbsa import parallel
    cfg = ops.SelectorConfig(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                             router_quantile=0.25, budget_blocks=64, k_min=1, k_max=112)
    for S, world in ((131072, 2), (131072, 8), (65536, 3), (1000, 4), (4096, 8), (256, 2)):
        sh = parallel.all_seq_shards(S, world, cfg)
        qt = (S + 63) // 64
        assert sh[0].t0 == 0 and sh[-1].t1 == qt
        assert all(a.t1 == b.t0 for a, b in zip(sh, sh[1:]))
        assert all(s.t0 % 2 == 0 and s.t1 > s.t0 for s in sh)
        assert sum(s.rows for s in sh) == S and sh[-1].row1 == S
    costs = parallel.tile_costs(131072, *ops.budget(cfg, 131072), 0.25)
    for world in (2, 4, 8):
        sh = parallel.all_seq_shards(131072, world, cfg)
        share = [costs[s.t0:s.t1].sum() * world / costs.sum() for s in sh]
        assert max(share) < 1.01 and min(share) > 0.99, share
    with pytest.raises(ValueError):
        parallel.all_seq_shards(128, 2, cfg)     # two tiles: one pair for two ranks


def test_grid_shards_cover_heads_and_tiles_once():
    from ugbsa import parallel
    for Hq, Hkv, world in ((28, 4, 1), (28, 4, 2), (28, 4, 4), (28, 4, 8), (8, 2, 6), (8, 1, 3)):
        for S in (1000, 4096, 131072):
            nb = (S + 63) // 64
            seen = {}
            for r in range(world):
                sh = parallel.GridShard.make(Hq, Hkv, world, r)
                rows = sh.rows(S)
                assert len(rows) == ops.slice_rows(S, sh.row_base, sh.m, len(sh.tiles(S)))
                for h in range(sh.q0, sh.q1):
                    for t in sh.tiles(S):
                        seen[(h, t)] = seen.get((h, t), 0) + 1
            assert len(seen) == Hq * nb and set(seen.values()) == {1}
    with pytest.raises(ValueError):
        parallel.GridShard.make(28, 4, 6, 0)


def test_decode_validation_without_device():
    L = _lib.load()
    st = _lib.Strides(1 << 20, 1 << 16, 128, 1)
    fake = ctypes.c_void_p(1 << 20)
    c = _cfg()
    kb, km = ctypes.c_int(0), ctypes.c_int(0)
    L.ugbsa_select_budget(ctypes.byref(c), 4096, ctypes.byref(kb), ctypes.byref(km))

    def sel(nb_cap=64, kmax=km.value, ws=1 << 30, S=4096):
        return L.ugbsa_decode_select(fake, _lib.BF16, st, fake, fake, nb_cap, 1, 8, 2, S, 128, ctypes.c_float(0.1),
                                     ctypes.byref(c), fake, kmax, None, None, fake, ws, None)
    assert sel(nb_cap=63) == 2        # summaries hold fewer blocks than the cache
    assert sel(kmax=km.value + 1) == 2
    assert sel(ws=16) == 6

    def att(kmax=64, D=128, dtype=_lib.BF16):
        return L.ugbsa_decode_attn(fake, fake, fake, dtype, st, st, st, fake, kmax, 1, 8, 2, 4096, D,
                                   ctypes.c_float(0.1), fake, st, fake, 1 << 30, None)
    assert att(kmax=2048) == 2        # kept blocks staged in shared memory: at most 1024
    assert att(D=96) == 5
    assert att(dtype=_lib.F32) == 3
    assert L.ugbsa_block_summary_update(fake, _lib.BF16, st, 1, 2, 4096, 128, 1, 64, 64, fake, fake, None) == 2
    assert L.ugbsa_block_summary_update(fake, _lib.BF16, st, 1, 2, 4096, 128, 1, 0, 63, fake, fake, None) == 2
    assert L.ugbsa_decode_workspace_bytes(1, 28, 131072, 128, 256) >= 28 * 4

    def step(nb_cap=64, kmax=km.value, ws=1 << 30, D=128, dtype=_lib.BF16, kv=fake, S=4096):
        return L.ugbsa_decode_step(fake, fake, fake, dtype, st, st, st, fake, fake, nb_cap, 1, 8, 2, S, D,
                                   ctypes.c_float(0.1), ctypes.byref(c), kv, kmax, None, None, fake, st, fake, ws,
                                   None)
    assert step(nb_cap=63) == 2       # summaries hold fewer blocks than the cache
    assert step(kmax=km.value + 1) == 2
    assert step(ws=16) == 6
    assert step(D=96) == 5
    assert step(dtype=_lib.F32) == 3  # the attention takes bf16 / fp16
    assert step(kv=None) == 1         # kv_idx is written: required


def test_qk_norm_rope_validation_without_device():
    L = _lib.load()
    st = _lib.Strides(1 << 20, 1 << 16, 128, 1)
    fake = ctypes.c_void_p(1 << 20)

    def call(D=128, R=128, dtype=_lib.BF16, mode=0, summary=2, cs_s=128, eps=1e-6, sa=fake):
        return L.ugbsa_qk_norm_rope(fake, dtype, st, fake, mode, ctypes.c_float(eps), fake, fake, 0, cs_s, R, 1, 4,
                                    4096, D, fake, st, summary, sa, fake, None)
    assert call(D=96) == 5
    assert call(R=96) == 5            # rotated width: a power of two
    assert call(R=8) == 5
    assert call(dtype=_lib.F32) == 3
    assert call(mode=3) == 1          # modes: 0 scale, 1 offset, 2 none
    assert call(summary=3) == 1
    assert call(sa=None) == 1
    assert call(cs_s=100) == 4        # cos / sin rows not 16-byte aligned
    assert call(eps=float("nan")) == 1


def test_block_order_stats_validation_without_device():
    L = _lib.load()
    st = _lib.Strides(1 << 20, 1 << 16, 128, 1)
    fake = ctypes.c_void_p(1 << 20)

    def call(S, budget, D=128, tau=True):
        return L.ugbsa_block_order_stats(fake, _lib.BF16, st, fake, fake, 1, 4, 2, S, D, ctypes.c_float(0.1), 1,
                                         budget, fake, fake, fake, fake, fake if tau else None, fake,
                                         1 << 30, None)
    assert call(4096, 16) == 2     # NB 64: k_b 32, rho_k 64 = NB -> no rank rho_k
    assert call(4096, 40) == 2     # k_b = NB
    assert call(4096, 0) == 2
    assert call(1, 1) == 2
    assert call(4096, 4, D=100) == 5
    assert L.ugbsa_block_order_stats_workspace_bytes(1, 28, 131072) >= 28 * 1024 * 4
    assert L.ugbsa_block_order_stats_workspace_bytes(1, 28, 1) == 0


def test_workspace_sizes():
    L = _lib.load()
    c = _cfg()
    assert L.ugbsa_select_workspace_bytes(ctypes.byref(c), 1, 28, 131072) >= 28 * 2048 * 4
    assert L.ugbsa_select_finish_workspace_bytes(1, 131072) >= 2048 * 4
    assert L.ugbsa_select_workspace_bytes(ctypes.byref(c), 0, 28, 131072) == 0
    # the exact size depends on dtype, head dim and KV heads; the dtype-free query bounds all of them
    for dt in (_lib.F32, _lib.BF16, _lib.F16):
        for D in (64, 128, 256):
            for Hkv in (1, 4, 28):
                ex = L.ugbsa_select_workspace_bytes_ex(ctypes.byref(c), dt, 1, 28, Hkv, 8192, D)
                assert 0 < ex <= L.ugbsa_select_workspace_bytes(ctypes.byref(c), 1, 28, 8192)
    # bf16 head dim 256 with Hkv = Hq needs more than head dim 128 with Hkv = Hq
    e256 = L.ugbsa_select_workspace_bytes_ex(ctypes.byref(c), _lib.BF16, 1, 4, 4, 2048, 256)
    e128 = L.ugbsa_select_workspace_bytes_ex(ctypes.byref(c), _lib.BF16, 1, 4, 4, 2048, 128)
    assert e256 > e128
    assert L.ugbsa_select_workspace_bytes_ex(ctypes.byref(c), _lib.BF16, 1, 4, 0, 2048, 128) == 0


def test_ops_refuse_cpu_tensors():
    import torch
    q = torch.zeros(1, 2, 64, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.block_summary(q, False)
