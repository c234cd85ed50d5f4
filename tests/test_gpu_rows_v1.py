"""GPU parity of the v1 per-row selector and the per-row masked attention.

* ugbsa_select_rows against the oracle restatement (oracle.select_rows):
  the keep bits on the visible blocks, the margins after the grain step (+inf
  for ineligible rows) and the triggers bit for bit, for every case recorded
  from the reference (tests/golden/v1/), whose keep masks they must equal too;
* the tiles' union lists (ascending ids, sentinel NB) against the keep bits;
* ugbsa_attn_rowmask, the reference-API ``block_attn.block_sparse_attn(q, k, v,
  keep)`` and the Hugging Face hook with ``kernel_v2=False`` against the
  oracle's per-row masked attention: max-abs <= 2e-2, mean-abs <= 2e-3.
"""
import math
import types

import numpy as np
import pytest
import torch

from golden_util import load_v1, v1_names, visible_mask
from oracle import oracle
from ugbsa import block_attn, ops
from ugbsa import sparse_attention as sa

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
KNOBS = ("mode", "router_score", "router_mode", "router_grain", "router_quantile", "budget_blocks", "k_min", "k_max")


def _cfgs(sel):
    kw = {k: sel[k] for k in KNOBS}
    kw["router_tau"] = sel.get("router_tau", 0.10)
    return oracle.OracleConfig(**kw), ops.SelectorConfig(**kw)


def _msafe(eff, S, budget, nb):
    keff = max(1, min(budget, nb - 1))
    elig = (np.arange(S) // 64 + 1) > keff
    return np.where(elig[None, None] & ~np.isnan(eff), eff, np.inf).astype(np.float32)


@pytest.mark.parametrize("name", v1_names())
def test_select_rows_bit_exact_vs_oracle_and_reference(name):
    meta, (q, k, v), rec = load_v1(name)
    inp, sel = meta["inp"], meta["sel"]
    S = inp["S"]
    nb = math.ceil(S / 64)
    ocfg, gcfg = _cfgs(sel)
    dt = torch.bfloat16 if inp["bf16"] else torch.float32
    qd, kd = (torch.from_numpy(x).to(DEV).to(dt) for x in (q, k))
    bits, kv_idx, sigma, trig = ops.select_rows(qd, kd, float(rec["scale"]), gcfg, return_router=True)
    torch.cuda.synchronize()
    keep = ops.unpack_keep(bits, nb).cpu().numpy()
    vis = visible_mask(S)[None, None]
    want = oracle.select_rows(q, k, float(rec["scale"]), ocfg)
    assert np.array_equal(keep, keep & vis)                       # only visible blocks are ever set
    assert np.array_equal(keep, want["keep"] & vis)
    assert np.array_equal(keep, rec["keep"] & vis)                # the reference's own keep mask
    if sel["mode"] == "router":
        m_got = sigma.cpu().numpy()
        m_want = _msafe(want["sigma_eff"], S, sel["budget_blocks"], nb)
        assert np.array_equal(m_got.view(np.uint32), m_want.view(np.uint32))
        assert np.array_equal(trig.cpu().numpy(), want["trigger"])
    # each tile's list: the union of its rows' kept blocks, ascending, then the sentinel
    kv = kv_idx.cpu().numpy()
    for t in range(kv.shape[2]):
        u = keep[:, :, t * 64:(t + 1) * 64].any(2)               # [B, H, NB]
        for b in range(kv.shape[0]):
            for h in range(kv.shape[1]):
                ids = np.nonzero(u[b, h])[0]
                row = kv[b, h, t]
                assert np.array_equal(row[:len(ids)], ids)
                assert (row[len(ids):] == nb).all()


ATTN = [("v1_router_row_quantile", torch.bfloat16), ("v1_router_batch2_ragged", torch.bfloat16),
        ("v1_quest_gqa_bf16", torch.float16)]


@pytest.mark.parametrize("name,dtype", ATTN)
def test_rowmask_attention_vs_oracle(name, dtype):
    meta, (q, k, v), rec = load_v1(name)
    inp, sel = meta["inp"], meta["sel"]
    rnd = lambda x: torch.from_numpy(x).to(dtype).float().numpy()
    q, k, v = rnd(q), rnd(k), rnd(v)                             # the values the kernel reads
    _, gcfg = _cfgs(sel)
    qd, kd, vd = (torch.from_numpy(x).to(DEV).to(dtype) for x in (q, k, v))
    scale = float(rec["scale"])
    bits, kv_idx = ops.select_rows(qd, kd, scale, gcfg)
    out = ops.block_sparse_attn_rows(qd, kd, vd, kv_idx, bits, scale)
    keep = ops.unpack_keep(bits, math.ceil(inp["S"] / 64))
    ref = oracle.attn_keep(q, k, v, keep.cpu().numpy(), scale)
    d = np.abs(out.float().cpu().numpy() - ref)
    assert d.max() <= 2e-2 and d.mean() <= 2e-3, (d.max(), d.mean())
    # the reference's launcher API on a caller's keep mask
    out2 = block_attn.block_sparse_attn(qd, kd, vd, keep, scale)
    assert torch.equal(out2, out)


def test_hook_v1_path_matches_oracle():
    """kernel_v2 = False sends topk / quest / router through the per-row path
    (src/sparse_attention.py:790-803)."""
    meta, (q, k, v), rec = load_v1("v1_router_row_quantile")
    sel = meta["sel"]
    rnd = lambda x: torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    q, k, v = rnd(q), rnd(k), rnd(v)
    qd, kd, vd = (torch.from_numpy(x).to(DEV).to(torch.bfloat16) for x in (q, k, v))
    saved = {x: getattr(sa.SEL, x) for x in KNOBS + ("kernel_v2", "log")}
    try:
        for x in KNOBS:
            setattr(sa.SEL, x, sel[x])
        sa.SEL.kernel_v2, sa.SEL.log = False, True
        sa.SEL.reset_log()
        mod = types.SimpleNamespace(layer_idx=3, num_key_value_groups=1)
        out, w = sa.block_sparse_attention(mod, qd, kd, vd, None, float(rec["scale"]))
        keep = sa._block_select_mask(qd, kd, float(rec["scale"]), 3)
        assert list(sa.SEL.kept_blocks) == [3] and len(sa.SEL.router_trigger_rate) == 2
    finally:
        for x, val in saved.items():
            setattr(sa.SEL, x, val)
        sa.SEL.reset_log()
    assert w is None and tuple(out.shape) == (1, q.shape[2], q.shape[1], q.shape[3])
    ocfg, _ = _cfgs(sel)
    want_keep = oracle.select_rows(q, k, float(rec["scale"]), ocfg)["keep"]
    vis = visible_mask(q.shape[2])[None, None]
    assert np.array_equal(keep.cpu().numpy(), want_keep & vis)
    ref = oracle.attn_keep(q, k, v, want_keep & vis, float(rec["scale"]))
    d = np.abs(out.transpose(1, 2).float().cpu().numpy() - ref)
    assert d.max() <= 2e-2 and d.mean() <= 2e-3, (d.max(), d.mean())
