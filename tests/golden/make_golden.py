"""Generate the golden fixtures in tests/golden/*.npz from the reference itself.

Run in a container where the reference project is mounted (read-only), e.g.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --ref /path/to/reference

It imports the reference's own selector ``_block_select_kv_idx_v2``
(src/sparse_attention.py:588-748) and its masked-SDPA checker
``reference_attn`` (src/triton_block_attn.py:301-312), runs them on CPU on
seeded planted inputs (ugbsa.synth.planted_inputs), and records:

* ``kv_idx_ref``      the reference's kv_idx as returned;
* ``tile_score_ref``  the tensor the reference ranks with topk (after the
                      causal mask and the sink/self forcing, :697), captured by
                      wrapping ``torch.Tensor.topk`` for the duration of a call;
* ``margin_ref``, ``kquant_ref``, ``thresh_ref``  the flattened (expanded)
                      sigma margins handed to ``kthvalue`` and its result (:711-716);
* ``attn_ref``        reference_attn on the reference's own kv_idx (attention cases).

Inputs are not stored: tests regenerate them from the recorded seed and shape
and check ``input_digest`` first, so a generator change fails loudly.
The fixtures are small (a few hundred KB in total).

``--configs`` records the BASELINE configurations instead, into
tests/golden/configs/ (``CONFIG_CASES``):

* ``cfg1_layer``  config 1 in full (S=4096, 8/8 heads, d128, fp32, K-mean
  router, k_base 8): kv_idx, tile scores, the per-head margins before the
  row-grain mean (``cell_margin_ref``), the quantile, the ``SEL.log``
  diagnostics (``kept_blocks_ref``, ``trigger_rate_ref``) and reference_attn
  rows of a few (head, tile) samples;
* ``cfg2_select`` config 2's selection (S=32768, 28/4 heads, d128, bf16 inputs
  scored in fp32, Quest router, k_base 32, 16 chained planted blocks): the
  canonical block sets as a packed bit mask, the per-head margins, the quantile
  and the log diagnostics (its tile scores, 29 MB, are not stored).

``--v1`` records the reference's v1 per-row selector ``_block_select_mask``
(src/sparse_attention.py:208-382) into tests/golden/v1/ (``V1_CASES``): the
keep mask (packed bits), the per-row scores it ranks (captured at its first
topk), the router's masked margins, quantile and threshold, the SEL.log
records, and reference_attn on the keep mask for the attention cases.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "uncertainty-gated-block-sparse-attention_b200"))

from ugbsa.synth import input_digest, planted_inputs  # noqa: E402

# name -> (inputs, selector knobs, attention?)
CASES = {
    "router_mean_row_q25": dict(
        inp=dict(B=1, Hq=4, Hkv=4, S=1024, D=64, n_planted=4, seed=11, chained=False, bf16=False),
        sel=dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112), attn=False),
    "router_quest_gqa_bf16": dict(
        inp=dict(B=1, Hq=4, Hkv=2, S=1024, D=64, n_planted=6, seed=12, chained=True, bf16=True),
        sel=dict(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112), attn=False),
    "topk_mean": dict(
        inp=dict(B=1, Hq=2, Hkv=2, S=768, D=64, n_planted=3, seed=13, chained=False, bf16=False),
        sel=dict(mode="topk", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=3, k_min=1, k_max=112), attn=False),
    "quest_plain": dict(
        inp=dict(B=1, Hq=2, Hkv=1, S=1024, D=64, n_planted=4, seed=14, chained=True, bf16=True),
        sel=dict(mode="quest", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112), attn=False),
    "router_cell_abs": dict(
        inp=dict(B=1, Hq=2, Hkv=2, S=1024, D=64, n_planted=4, seed=15, chained=False, bf16=False),
        sel=dict(mode="router", router_score="mean", router_mode="abs", router_grain="cell",
                 router_quantile=0.25, router_tau=2e-41, budget_blocks=4, k_min=1, k_max=112),
        attn=False),
    "router_cell_quantile": dict(
        inp=dict(B=1, Hq=3, Hkv=3, S=1024, D=64, n_planted=4, seed=16, chained=False, bf16=False),
        sel=dict(mode="router", router_score="quest", router_mode="quantile", router_grain="cell",
                 router_quantile=0.3, budget_blocks=4, k_min=1, k_max=112), attn=False),
    "router_ragged_S1000": dict(
        inp=dict(B=1, Hq=2, Hkv=2, S=1000, D=64, n_planted=4, seed=17, chained=False, bf16=False),
        sel=dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=3, k_min=1, k_max=112), attn=True),
    "router_batch2_quest": dict(
        inp=dict(B=2, Hq=2, Hkv=1, S=512, D=64, n_planted=2, seed=18, chained=True, bf16=True),
        sel=dict(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=2, k_min=1, k_max=112), attn=False),
    "router_default_clamp": dict(
        # Selector defaults k_min=8, k_max=112: budget 2 is clamped up to 8 (k_base 16)
        inp=dict(B=1, Hq=2, Hkv=2, S=2048, D=64, n_planted=4, seed=19, chained=False, bf16=False),
        sel=dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.2, budget_blocks=2, k_min=8, k_max=112), attn=False),
    "attn_router_small": dict(
        inp=dict(B=1, Hq=2, Hkv=1, S=512, D=64, n_planted=2, seed=20, chained=False, bf16=True),
        sel=dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=1, k_min=1, k_max=112), attn=True),
}


CONFIG_CASES = {
    "cfg1_layer": dict(
        inp=dict(B=1, Hq=8, Hkv=8, S=4096, D=128, n_planted=4, seed=0, chained=False, bf16=False),
        sel=dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112),
        store="full", attn_samples=[(0, 1), (0, 40), (3, 63), (7, 40), (7, 63)]),
    "cfg2_select": dict(
        inp=dict(B=1, Hq=28, Hkv=4, S=32768, D=128, n_planted=16, seed=2, chained=True, bf16=True),
        sel=dict(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=16, k_min=1, k_max=112),
        store="sets", attn_samples=[]),
}


def pack_sets(kv_idx: np.ndarray, S: int) -> np.ndarray:
    """Canonical sets (sentinel and causally invisible ids dropped) as a bit mask
    [B, H, Qt, ceil(NB/8)] uint8 (np.packbits over the block axis)."""
    nb = math.ceil(S / 64)
    B, H, Qt, _ = kv_idx.shape
    mask = np.zeros((B, H, Qt, nb), bool)
    last_blk = np.minimum(np.arange(Qt) * 64 + 63, S - 1) // 64          # last visible block per tile
    ids = kv_idx.astype(np.int64)
    ok = (ids >= 0) & (ids < nb) & (ids <= last_blk[None, None, :, None])
    b, h, t, j = np.nonzero(ok)
    mask[b, h, t, ids[b, h, t, j]] = True
    return np.packbits(mask, axis=-1)


# v1 per-row selection (src/sparse_attention.py:208-382) + reference_attn with its keep mask
V1_CASES = {
    "v1_topk_mean": dict(
        inp=dict(B=1, Hq=4, Hkv=4, S=1024, D=64, n_planted=4, seed=61, chained=False, bf16=False),
        sel=dict(mode="topk", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112), attn=True),
    "v1_quest_gqa_bf16": dict(
        inp=dict(B=1, Hq=4, Hkv=2, S=1024, D=64, n_planted=4, seed=62, chained=True, bf16=True),
        sel=dict(mode="quest", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=3, k_min=1, k_max=112), attn=False),
    "v1_router_row_quantile": dict(
        inp=dict(B=1, Hq=4, Hkv=4, S=1024, D=64, n_planted=4, seed=63, chained=False, bf16=False),
        sel=dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112), attn=True),
    "v1_router_cell_quest": dict(
        inp=dict(B=1, Hq=3, Hkv=3, S=1024, D=64, n_planted=4, seed=64, chained=False, bf16=False),
        sel=dict(mode="router", router_score="quest", router_mode="quantile", router_grain="cell",
                 router_quantile=0.3, budget_blocks=4, k_min=1, k_max=112), attn=False),
    "v1_router_abs_row": dict(
        inp=dict(B=1, Hq=2, Hkv=2, S=1024, D=64, n_planted=4, seed=65, chained=False, bf16=False),
        sel=dict(mode="router", router_score="mean", router_mode="abs", router_grain="row",
                 router_quantile=0.25, router_tau=0.05, budget_blocks=4, k_min=1, k_max=112), attn=False),
    "v1_router_batch2_ragged": dict(
        inp=dict(B=2, Hq=2, Hkv=1, S=1000, D=64, n_planted=3, seed=66, chained=True, bf16=True),
        sel=dict(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                 router_quantile=0.25, budget_blocks=3, k_min=1, k_max=112), attn=True),
    "v1_default_clamp": dict(
        inp=dict(B=1, Hq=2, Hkv=2, S=1536, D=64, n_planted=4, seed=67, chained=False, bf16=False),
        sel=dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                 router_quantile=0.2, budget_blocks=2, k_min=8, k_max=112), attn=False),
}


def run_reference_v1(ref_src: str, name: str, spec: dict) -> dict:
    """The reference's v1 selector (and reference_attn on its keep mask), with the
    per-row scores it ranks, its margins and threshold, and its SEL.log records."""
    import torch

    if ref_src not in sys.path:
        sys.path.insert(0, ref_src)
    import sparse_attention as sa
    from transformers.models.qwen2.modeling_qwen2 import repeat_kv
    from triton_block_attn import reference_attn

    inp, sel = spec["inp"], spec["sel"]
    q, k, v, _ = planted_inputs(inp["B"], inp["Hq"], inp["Hkv"], inp["S"], inp["D"], n_planted=inp["n_planted"],
                                seed=inp["seed"], chained=inp["chained"], bf16=inp["bf16"])
    scale = inp["D"] ** -0.5
    X = sa.SEL
    X.kernel_v2 = False
    for key in ("mode", "router_score", "router_mode", "router_grain", "router_quantile", "budget_blocks",
                "k_min", "k_max"):
        setattr(X, key, sel[key])
    X.router_tau = sel.get("router_tau", 0.10)
    X.log = True
    X.reset_log()
    g = inp["Hq"] // inp["Hkv"]
    qt = torch.from_numpy(q)
    kt = repeat_kv(torch.from_numpy(k), g)
    captured = {}
    orig_topk, orig_kth = torch.Tensor.topk, torch.Tensor.kthvalue

    def topk_hook(self, *a, **kw):
        captured.setdefault("row_score", self.detach().clone())   # the first topk ranks the raw scores
        return orig_topk(self, *a, **kw)

    def kth_hook(self, *a, **kw):
        r = orig_kth(self, *a, **kw)
        captured["m_safe"] = self.detach().clone()
        captured["kquant"] = int(a[0] if a else kw["k"])
        captured["thresh"] = float(r.values)
        return r

    torch.Tensor.topk, torch.Tensor.kthvalue = topk_hook, kth_hook
    try:
        keep = sa._block_select_mask(qt, kt, scale, 0)
    finally:
        torch.Tensor.topk, torch.Tensor.kthvalue = orig_topk, orig_kth
    X.log = False
    keep_np = keep.numpy().astype(bool)
    # per-row scores and attention rows are stored for a few sampled tiles (size)
    qt_n = math.ceil(inp["S"] / 64)
    tiles = sorted({0, 3, qt_n // 2, qt_n - 1})
    rows = np.concatenate([np.arange(t * 64, min(inp["S"], (t + 1) * 64)) for t in tiles])
    out = {
        "input_digest": input_digest(q, k, v),
        "scale": np.float32(scale),
        "meta": json.dumps({"name": name, "inp": inp, "sel": sel, "sample_tiles": tiles}),
        "keep_ref": np.packbits(keep_np, axis=-1),
        "nb": np.int64(keep_np.shape[-1]),
        "sample_rows": rows.astype(np.int64),
        "row_score_ref": captured["row_score"].numpy().astype(np.float32)[:, :, rows],
        "kept_blocks_ref": np.stack([x.numpy() for x in X.kept_blocks.values()]),
        "budget_samples_ref": np.array(X.budget_samples, np.float64),
    }
    if sel["mode"] == "router":
        out["trigger_rate_ref"] = np.array(X.router_trigger_rate, np.float64)
        out["eff_budget_ref"] = np.array(X.router_eff_budget, np.float64)
        out["margin_mean_ref"] = np.array(X.router_margin_mean, np.float64)
    if "m_safe" in captured:
        out["m_safe_ref"] = captured["m_safe"].numpy().astype(np.float32)
        out["kquant_ref"] = np.int64(captured["kquant"])
        out["thresh_ref"] = np.float32(captured["thresh"])
    if spec["attn"]:
        vt = repeat_kv(torch.from_numpy(v), g)
        out["attn_ref"] = reference_attn(qt, kt, vt, keep, scale).numpy().astype(np.float32)[:, :, rows]
    return out


def run_reference_config(ref_src: str, name: str, spec: dict) -> dict:
    """One BASELINE configuration through the reference's selector with SEL.log on."""
    import torch

    if ref_src not in sys.path:
        sys.path.insert(0, ref_src)
    import sparse_attention as sa
    from transformers.models.qwen2.modeling_qwen2 import repeat_kv
    from triton_block_attn import reference_attn

    inp, sel = spec["inp"], spec["sel"]
    q, k, v, planted = planted_inputs(inp["B"], inp["Hq"], inp["Hkv"], inp["S"], inp["D"],
                                      n_planted=inp["n_planted"], seed=inp["seed"],
                                      chained=inp["chained"], bf16=inp["bf16"])
    S_, D = inp["S"], inp["D"]
    scale = D ** -0.5
    X = sa.SEL
    X.kernel_v2 = True
    for key in ("mode", "router_score", "router_mode", "router_grain", "router_quantile", "budget_blocks",
                "k_min", "k_max"):
        setattr(X, key, sel[key])
    X.router_tau = sel.get("router_tau", 0.10)
    X.log = True
    X.reset_log()
    g = inp["Hq"] // inp["Hkv"]
    qt = torch.from_numpy(q)
    kt = repeat_kv(torch.from_numpy(k), g)      # BASELINE's oracle: fp32 scores on repeat_kv'd keys
    captured = {}
    orig_topk, orig_kth, orig_mean = torch.Tensor.topk, torch.Tensor.kthvalue, torch.Tensor.mean

    def topk_hook(self, *a, **kw):
        if spec["store"] == "full":
            captured["tile_score"] = self.detach().clone()
        return orig_topk(self, *a, **kw)

    def kth_hook(self, *a, **kw):
        r = orig_kth(self, *a, **kw)
        captured["margin"] = self.detach().clone()
        captured["kquant"] = int(a[0] if a else kw["k"])
        captured["thresh"] = float(r.values)
        return r

    def mean_hook(self, *a, **kw):
        # the row-grain head mean of the per-tile margins (:708-710)
        if (a[:1] == (1,) or kw.get("dim") == 1) and kw.get("keepdim") and self.dim() == 3:
            captured["cell_margin"] = self.detach().clone()
        return orig_mean(self, *a, **kw)

    torch.Tensor.topk, torch.Tensor.kthvalue, torch.Tensor.mean = topk_hook, kth_hook, mean_hook
    try:
        kv = sa._block_select_kv_idx_v2(qt, kt, scale)
    finally:
        torch.Tensor.topk, torch.Tensor.kthvalue, torch.Tensor.mean = orig_topk, orig_kth, orig_mean
    X.log = False
    kv_np = kv.numpy().astype(np.int32)
    out = {
        "input_digest": input_digest(q, k, v),
        "scale": np.float32(scale),
        "meta": json.dumps({"name": name, "inp": inp, "sel": sel, "store": spec["store"],
                            "attn_samples": spec["attn_samples"]}),
        "kv_shape": np.array(kv_np.shape, np.int64),
        "sets_ref": pack_sets(kv_np, S_),
        "cell_margin_ref": captured["cell_margin"].numpy().astype(np.float32),
        "margin_ref": captured["margin"].numpy().astype(np.float32),
        "kquant_ref": np.int64(captured["kquant"]),
        "thresh_ref": np.float32(captured["thresh"]),
        "kept_blocks_ref": np.stack([x.numpy() for x in X.kept_blocks.values()]),
        "trigger_rate_ref": np.array(X.router_trigger_rate, np.float64),
        "budget_samples_ref": np.array(X.budget_samples, np.float64),
    }
    if spec["store"] == "full":
        out["kv_idx_ref"] = kv_np
        out["tile_score_ref"] = captured["tile_score"].numpy().astype(np.float32)
    if spec["attn_samples"]:
        vt = repeat_kv(torch.from_numpy(v), g)
        nb = math.ceil(S_ / 64)
        rows = []
        for (h, t) in spec["attn_samples"]:
            # reference_attn on one head with the tile-broadcast keep mask of that head
            keep = torch.zeros(1, 1, S_, nb, dtype=torch.bool)
            for tt in range(kv.shape[2]):
                ids = kv[0, h, tt].long()
                ids = ids[ids < nb]
                keep[0, 0, tt * 64:min(S_, (tt + 1) * 64), ids] = True
            o = reference_attn(qt[:, h:h + 1], kt[:, h:h + 1], vt[:, h:h + 1], keep, scale)
            rows.append(o[0, 0, t * 64:min(S_, (t + 1) * 64)].numpy().astype(np.float32))
        out["attn_rows_ref"] = np.stack(rows)
    return out


def run_reference(ref_src: str, name: str, spec: dict) -> dict:
    import torch

    if ref_src not in sys.path:
        sys.path.insert(0, ref_src)
    import sparse_attention as sa  # the reference module
    from transformers.models.qwen2.modeling_qwen2 import repeat_kv
    from triton_block_attn import reference_attn

    inp = spec["inp"]
    q, k, v, planted = planted_inputs(inp["B"], inp["Hq"], inp["Hkv"], inp["S"], inp["D"],
                                      n_planted=inp["n_planted"], seed=inp["seed"],
                                      chained=inp["chained"], bf16=inp["bf16"])
    D = inp["D"]
    scale = D ** -0.5
    sel = spec["sel"]
    S = sa.SEL
    S.kernel_v2 = True
    S.mode = sel["mode"]
    S.router_score = sel["router_score"]
    S.router_mode = sel["router_mode"]
    S.router_grain = sel["router_grain"]
    S.router_quantile = sel["router_quantile"]
    S.router_tau = sel.get("router_tau", 0.10)
    S.budget_blocks = sel["budget_blocks"]
    S.k_min = sel["k_min"]
    S.k_max = sel["k_max"]
    S.log = False

    qt = torch.from_numpy(q)
    g = inp["Hq"] // inp["Hkv"]
    kt = repeat_kv(torch.from_numpy(k), g)
    vt = repeat_kv(torch.from_numpy(v), g)

    captured = {}
    orig_topk = torch.Tensor.topk
    orig_kth = torch.Tensor.kthvalue

    def topk_hook(self, *a, **kw):
        captured["tile_score"] = self.detach().clone()
        return orig_topk(self, *a, **kw)

    def kth_hook(self, *a, **kw):
        r = orig_kth(self, *a, **kw)
        captured["margin"] = self.detach().clone()
        captured["kquant"] = int(a[0] if a else kw["k"])
        captured["thresh"] = float(r.values)
        return r

    torch.Tensor.topk = topk_hook
    torch.Tensor.kthvalue = kth_hook
    try:
        kv = sa._block_select_kv_idx_v2(qt, kt, scale)
    finally:
        torch.Tensor.topk = orig_topk
        torch.Tensor.kthvalue = orig_kth

    out = {
        "kv_idx_ref": kv.numpy().astype(np.int32),
        "tile_score_ref": captured["tile_score"].numpy().astype(np.float32),
        "input_digest": input_digest(q, k, v),
        "scale": np.float32(scale),
        "meta": json.dumps({"name": name, "inp": inp, "sel": sel}),
    }
    if "margin" in captured:
        out["margin_ref"] = captured["margin"].numpy().astype(np.float32)
        out["kquant_ref"] = np.int64(captured["kquant"])
        out["thresh_ref"] = np.float32(captured["thresh"])
    if spec["attn"]:
        nb = math.ceil(inp["S"] / 64)
        keep = torch.zeros(inp["B"], inp["Hq"], inp["S"], nb, dtype=torch.bool)
        for t in range(kv.shape[2]):
            ids = kv[:, :, t, :].long()
            ok = ids < nb
            rows = slice(t * 64, min(inp["S"], (t + 1) * 64))
            tile_keep = torch.zeros(inp["B"], inp["Hq"], nb + 1, dtype=torch.bool)
            tile_keep.scatter_(-1, torch.where(ok, ids, torch.full_like(ids, nb)), True)
            keep[:, :, rows, :] = tile_keep[:, :, None, :nb]
        o = reference_attn(qt, kt, vt, keep, scale)
        out["attn_ref"] = o.numpy().astype(np.float32)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("UGBSA_REFERENCE"), required="UGBSA_REFERENCE" not in os.environ,
                    help="root of the reference project (its src/ is imported); or set UGBSA_REFERENCE")
    ap.add_argument("--only", default=None)
    ap.add_argument("--configs", action="store_true", help="record the BASELINE configurations (CONFIG_CASES)")
    ap.add_argument("--v1", action="store_true", help="record the v1 per-row selector cases (V1_CASES)")
    args = ap.parse_args()
    ref_src = os.path.join(args.ref, "src")
    if args.v1:
        os.makedirs(os.path.join(HERE, "v1"), exist_ok=True)
        for name, spec in V1_CASES.items():
            if args.only and name != args.only:
                continue
            rec = run_reference_v1(ref_src, name, spec)
            path = os.path.join(HERE, "v1", f"{name}.npz")
            np.savez_compressed(path, **rec)
            print(f"wrote {path} ({os.path.getsize(path)} bytes)")
        return
    if args.configs:
        os.makedirs(os.path.join(HERE, "configs"), exist_ok=True)
        for name, spec in CONFIG_CASES.items():
            if args.only and name != args.only:
                continue
            rec = run_reference_config(ref_src, name, spec)
            path = os.path.join(HERE, "configs", f"{name}.npz")
            np.savez_compressed(path, **rec)
            print(f"wrote {path} ({os.path.getsize(path)} bytes)")
        return
    for name, spec in CASES.items():
        if args.only and name != args.only:
            continue
        rec = run_reference(ref_src, name, spec)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
