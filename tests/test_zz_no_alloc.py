"""ugbsa_select_noalloc: the selector for callers that cannot allocate device memory.

Some callers of this library cannot hand it a scratch buffer -- for example a
serving runtime whose memory planner already owns all device memory, or a
binding that only holds the tensors it was given.  ugbsa_select_noalloc takes
its scratch from a fixed array inside libugbsa instead.  These tests call it
through the C ABI and require its results (kv_idx, sigma, trigger) to equal
those of ugbsa_select, which takes a caller workspace, bit for bit -- the same
exactness the selector's other tests use -- on two calls in a row with
different problems, so that contents left in the shared array by the first
call cannot leak into the second.  The file is collected last; it passes both
alone in a fresh process and after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

from ugbsa import _lib, ops
from ugbsa.synth import planted_inputs

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _st(t):
    s = t.stride()
    return _lib.Strides(s[0], s[1], s[2], s[3])


def _run(entry, q, k, cfg, with_workspace):
    L = _lib.load()
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    summ = ops.block_summary(k, cfg.quest)
    sa, sb = summ if cfg.quest else (summ, None)
    _, kmax = ops.budget(cfg, S)
    Qt = (S + 63) // 64
    kv = torch.full((B, Hq, Qt, kmax), -7, device=DEV, dtype=torch.int32)
    sigma = torch.full((B, Hq, Qt), -1.0, device=DEV)
    trig = torch.full((B, Hq, Qt), 9, device=DEV, dtype=torch.uint8)
    c = cfg.to_c()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [_p(q), _lib.BF16, _st(q), _p(sa), _p(sb), B, Hq, Hkv, S, D, ctypes.c_float(D ** -0.5), ctypes.byref(c),
            _p(kv), kmax, _p(sigma), _p(trig)]
    if with_workspace:
        nbytes = L.ugbsa_select_workspace_bytes_ex(ctypes.byref(c), _lib.BF16, B, Hq, Hkv, S, D)
        ws = torch.empty(nbytes, device=DEV, dtype=torch.uint8)
        rc = getattr(L, entry)(*args, _p(ws), ctypes.c_size_t(nbytes), stream)
    else:
        rc = getattr(L, entry)(*args, stream)
    assert rc == 0, _lib.status_string(rc)
    torch.cuda.synchronize()
    return kv.cpu().numpy(), sigma.cpu().numpy(), trig.cpu().numpy()


def _same(a, b):
    kv_a, s_a, t_a = a
    kv_b, s_b, t_b = b
    assert np.array_equal(kv_a, kv_b)
    assert np.array_equal(s_a.view(np.uint32), s_b.view(np.uint32))   # NaN bit patterns included
    assert np.array_equal(t_a, t_b)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    cases = [
        (dict(B=1, Hq=8, Hkv=2, S=4096, D=128, seed=31),
         ops.SelectorConfig(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                            router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112)),
        (dict(B=2, Hq=4, Hkv=4, S=1000, D=64, seed=32),
         ops.SelectorConfig(mode="router", router_score="mean", router_mode="quantile", router_grain="cell",
                            router_quantile=0.3, budget_blocks=3, k_min=1, k_max=112)),
        # head dim 256 with as many KV heads as query heads: the largest operand copies per head
        (dict(B=1, Hq=4, Hkv=4, S=2048, D=256, seed=33),
         ops.SelectorConfig(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                            router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112)),
    ]
    for inp, cfg in cases:   # two calls in a row on the shared fixed scratch
        q, k, _, _ = planted_inputs(inp["B"], inp["Hq"], inp["Hkv"], inp["S"], inp["D"], n_planted=4,
                                    seed=inp["seed"], bf16=True)
        qd = torch.from_numpy(q).to(DEV).to(torch.bfloat16)
        kd = torch.from_numpy(k).to(DEV).to(torch.bfloat16)
        got = _run("ugbsa_select_noalloc", qd, kd, cfg, with_workspace=False)
        want = _run("ugbsa_select", qd, kd, cfg, with_workspace=True)
        _same(got, want)
        assert (got[0] >= 0).all()


NOALLOC_LIMIT = 1 << 20   # bytes of the library's fixed scratch array


def _largest_accepted_seq(cfg, Hq, Hkv, D):
    """The longest sequence (a multiple of 64) whose selection scratch fits the array."""
    L = _lib.load()
    c = cfg.to_c()
    need = lambda S: L.ugbsa_select_workspace_bytes_ex(ctypes.byref(c), _lib.BF16, 1, Hq, Hkv, S, D)
    S = 64
    while need(S + 64) <= NOALLOC_LIMIT:
        S += 64
    return S


def test_noalloc_limit_boundary_28_heads():
    """At the bench's head layout (28 query / 4 KV heads, head dim 128, router on
    Quest envelopes) the last sequence length that fits runs and equals
    ugbsa_select; one block more is refused with UGBSA_ERR_TOO_LARGE."""
    cfg = ops.SelectorConfig(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                             router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112)
    S = _largest_accepted_seq(cfg, 28, 4, 128)
    assert 4096 <= S < 8192   # the limit the library documents: about 5K tokens at these heads
    q, k, _, _ = planted_inputs(1, 28, 4, S + 64, 128, n_planted=4, seed=34, bf16=True)
    qd = torch.from_numpy(q).to(DEV).to(torch.bfloat16)
    kd = torch.from_numpy(k).to(DEV).to(torch.bfloat16)
    got = _run("ugbsa_select_noalloc", qd[:, :, :S], kd[:, :, :S], cfg, with_workspace=False)
    want = _run("ugbsa_select", qd[:, :, :S], kd[:, :, :S], cfg, with_workspace=True)
    _same(got, want)
    L = _lib.load()
    summ = ops.block_summary(kd, True)
    _, kmax = ops.budget(cfg, S + 64)
    Qt = (S + 64) // 64
    kv = torch.empty((1, 28, Qt, kmax), device=DEV, dtype=torch.int32)
    c = cfg.to_c()
    rc = L.ugbsa_select_noalloc(_p(qd), _lib.BF16, _st(qd), _p(summ[0]), _p(summ[1]), 1, 28, 4, S + 64, 128,
                                ctypes.c_float(128 ** -0.5), ctypes.byref(c), _p(kv), kmax, None, None,
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 10   # UGBSA_ERR_TOO_LARGE


def test_noalloc_rejects_problems_beyond_its_scratch():
    L = _lib.load()
    c = ops.SelectorConfig(mode="router").to_c()
    fake = ctypes.c_void_p(1 << 20)
    st = _lib.Strides(1 << 30, 1 << 26, 128, 1)
    # 64 heads at 1M tokens: terabytes of tile scores > 1 MiB, refused before any device access
    rc = L.ugbsa_select_noalloc(fake, _lib.BF16, st, fake, None, 1, 64, 64, 1 << 20, 128, ctypes.c_float(0.1),
                                ctypes.byref(c), fake, 16, None, None, None)
    assert rc == 10   # UGBSA_ERR_TOO_LARGE
    assert "noalloc" in _lib.status_string(rc)
