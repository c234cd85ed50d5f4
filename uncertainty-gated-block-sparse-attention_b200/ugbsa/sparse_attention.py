"""Drop-in for the reference's ``sparse_attention`` module (v2 prefill path).

Keeps the reference's user-facing surface:

* ``SEL`` (class ``Selector``) -- the global knob object harnesses set
  (src/sparse_attention.py:54-138).  The v2 path reads ``mode``,
  ``budget_blocks``, ``k_min``/``k_max``, ``router_mode``, ``router_grain``,
  ``router_quantile``, ``router_tau``, ``router_score`` and ``kernel_v2``.
* ``PROF`` -- CUDA-event profiler with the reference's buckets
  (``dense_sdpa``, ``v2_select``, ``v2_kernel``; :141-186).
* ``_block_select_kv_idx_v2(query, key_states, scaling, block_m=64)`` -- the
  selector (:588-748), now three sm_100a kernels.  ``key_states`` may have
  the KV head count (GQA resolved inside, no repeat_kv copy) or the Q head
  count, as in the reference.  Scores are fp32 whatever the input dtype.
* ``block_sparse_attention(module, query, key, value, attention_mask, scaling,
  dropout=0.0, **kwargs)`` -- the Hugging Face attention hook (:751-803),
  registered as ``"block_sparse"`` at import (:806).

The hook looks up ``_block_select_kv_idx_v2`` through this module's globals
at call time, so a diagnostics wrapper can monkey-patch it the way the
reference's dump hook does (src/dump_block_scores.py:64-69).

Scope: the modes topk / quest / router, per tile (``kernel_v2=True``, the v2
path) or per query row (``kernel_v2=False``, the v1 path with its per-row
inner mask: ``_block_select_mask``), plus the dense / decode path through SDPA.  ``SEL.decode_sparse = True`` (an addition,
off by default) sends decode calls (Q == 1) through the block-sparse decode
instead: the v2 policy on the decode row over the cache's block summaries
(``SUMM_CACHE``, refreshed incrementally per layer).  The research policies (belief, rollout,
rollout_peek) are outside this build and raise ``NotImplementedError``.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import ops

BLOCK = 64   # tokens per selection block (src/sparse_attention.py:51)


class Selector:
    """Global selector configuration (the v2 subset of the reference's knobs)."""

    def __init__(self):
        self.mode = "dense"          # "dense" | "topk" | "quest" | "router"
        self.budget_blocks = 32      # per-row budget; per-tile k_base = 2*clamp(budget, k_min, k_max)
        self.k_min, self.k_max = 8, 112
        self.router_mode = "abs"     # "abs" | "quantile"
        self.router_grain = "cell"   # "cell" | "row"
        self.router_tau = 0.10
        self.router_quantile = 0.20
        self.router_score = "mean"   # "mean" | "quest"
        self.kernel_v2 = False
        self.decode_sparse = False   # Q == 1: dense SDPA (the reference) unless set
        self.log = False
        self.reset_log()

    def reset_log(self):
        # filled by the v2 selector while ``log`` is set, as the reference does
        # (src/sparse_attention.py:726-744): per call, the blocks the last query
        # tile keeps unioned over heads (bool [n_blocks] on the host, keyed by
        # call order), the slot count, and the router's trigger fraction
        self.kept_blocks = {}
        self.budget_samples = []
        self.router_trigger_rate = []
        self.router_eff_budget = []
        self.router_margin_mean = []

    def config(self) -> ops.SelectorConfig:
        """Frozen snapshot of the knobs, as handed to the C ABI."""
        return ops.SelectorConfig(mode=self.mode, router_score=self.router_score, router_mode=self.router_mode,
                                  router_grain=self.router_grain, router_quantile=float(self.router_quantile),
                                  router_tau=float(self.router_tau), budget_blocks=int(self.budget_blocks),
                                  k_min=int(self.k_min), k_max=int(self.k_max))


SEL = Selector()


class _Profiler:
    """CUDA-event profiler; prefill calls only (src/sparse_attention.py:141-186)."""

    def __init__(self):
        self.enabled = False
        self.events = {}

    def reset(self):
        self.events = {}

    def start(self, name):
        if not self.enabled or not torch.cuda.is_available():
            return None
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        self.events.setdefault(name, []).append((s, e))
        return e

    @staticmethod
    def stop(ev):
        if ev is not None:
            ev.record()

    def summary(self):
        if not self.events:
            return {}
        torch.cuda.synchronize()
        out = {}
        for name, evs in self.events.items():
            ms = sorted(s.elapsed_time(e) for s, e in evs)
            out[name] = {"calls": len(ms), "total_ms": sum(ms), "mean_ms": sum(ms) / len(ms),
                         "p50_ms": ms[len(ms) // 2]}
        return out


PROF = _Profiler()


def _block_select_kv_idx_v2(query, key_states, scaling, block_m=64):
    """kv_idx [B, H, Q_tiles, kmax] int32 for the current ``SEL`` knobs.

    Same contract as src/sparse_attention.py:588-748: slots in descending tile
    score (ties -> lower block id), sink and self block always present, slots
    >= k_base of tiles the router did not trigger hold the sentinel NB.
    """
    if block_m != BLOCK:
        raise ValueError("block_m is fixed at 64")
    cfg = SEL.config()
    if not SEL.log:
        return ops.select_kv_idx(query, key_states, float(scaling), cfg)
    S = query.shape[-2]
    k_base, kmax = ops.budget(cfg, S)
    n_blocks = math.ceil(key_states.shape[-2] / BLOCK)
    if cfg.mode == "router" and k_base < kmax:
        kv_idx, sigma, trig = ops.select_kv_idx(query, key_states, float(scaling), cfg, return_router=True)
        # a host float per call, as the reference appends (:726-728; a sync only while logging)
        SEL.router_trigger_rate.append(float(trig.float().mean().item()))
    else:
        kv_idx = ops.select_kv_idx(query, key_states, float(scaling), cfg)
    # the last query tile's kept blocks of batch 0, unioned over heads, sentinels
    # dropped (:733-743); read by the reference's needle-hit metric
    last = kv_idx[0, :, -1, :].long().flatten()
    last = last[last < n_blocks]
    kept = torch.zeros(n_blocks, dtype=torch.bool, device=kv_idx.device)
    kept.scatter_(0, last, True)
    SEL.kept_blocks[len(SEL.kept_blocks)] = kept.cpu()
    SEL.budget_samples.append(float(kmax))
    return kv_idx


def _select_rows(query, key_states, scaling, layer_idx=0):
    """v1 per-row selection on the device: (keep bits, the tiles' union lists).
    Fills the SEL.log records as the reference's v1 selector does
    (src/sparse_attention.py:350-382)."""
    cfg = SEL.config()
    router = cfg.mode == "router"
    if SEL.log and router:
        bits, kv_idx, sigma, trig = ops.select_rows(query, key_states, float(scaling), cfg, return_router=True)
    else:
        bits, kv_idx = ops.select_rows(query, key_states, float(scaling), cfg)
    if SEL.log:
        nb = math.ceil(key_states.shape[-2] / BLOCK)
        last = ops.unpack_keep(bits[0, :, -1], nb)                       # [H, NB] of the last query row
        if router:
            keep_all = ops.unpack_keep(bits, nb)
            SEL.router_trigger_rate.append(float(trig.float().mean().item()))
            SEL.router_eff_budget.append(float(keep_all.float().sum(dim=-1).mean().item()))
            # the mean of the raw per-(head, row) margins: rows with at most k_eff visible
            # blocks (always the first ones) make it NaN, as in the reference
            SEL.router_margin_mean.append(float("nan"))
        SEL.kept_blocks[layer_idx] = last.any(dim=0).cpu()
        SEL.budget_samples.append(float(last.sum(dim=-1).float().mean().item()))
    return bits, kv_idx


def _block_select_mask(query, key_states, scaling, layer_idx):
    """The v1 per-row policy (src/sparse_attention.py:208-382, modes topk /
    quest / router): bool keep [B, H, Q, n_blocks] -- each query row's own top
    blocks (ties to the lower id), the sink and its own block, the router's
    triggered rows dense.  Scores are fp32 whatever the input dtype."""
    bits, _ = _select_rows(query, key_states, scaling, layer_idx)
    return ops.unpack_keep(bits, math.ceil(key_states.shape[-2] / BLOCK))


class SummaryCache:
    """Block summaries of each layer's growing KV cache, for the sparse decode:
    the first decode call of a layer summarises the whole cache, later calls
    only the blocks that received new keys (the last, growing one)."""

    def __init__(self):
        self.layers = {}

    def reset(self):
        self.layers = {}

    def get(self, layer_idx, key, quest: bool, last: bool = True):
        """The layer's summaries, refreshed from the first block with new keys
        (through the last block; with last=False up to the one before it, which
        the caller refreshes itself: ops.decode_step does)."""
        B, H, S, D = key.shape
        nb = math.ceil(S / BLOCK)
        ent = self.layers.get(layer_idx)
        fresh = (ent is None or ent["quest"] != quest or ent["shape"] != (B, H, D) or nb > ent["cap"]
                 or S < ent["S"] or ent["device"] != key.device)
        if fresh:
            cap = 64 * math.ceil((nb + 64) / 64)   # room for 64 more blocks before the next rebuild
            a = torch.empty((B, H, cap, D), device=key.device, dtype=torch.float32)
            summ = (a, torch.empty_like(a)) if quest else a
            ent = {"quest": quest, "shape": (B, H, D), "cap": cap, "S": 0, "summ": summ, "device": key.device}
            self.layers[layer_idx] = ent
        first = ent["S"] // BLOCK
        upto = nb if last else nb - 1
        if first < upto:
            ops.block_summary_update(key[:, :, :upto * BLOCK], quest, ent["summ"], first)
        ent["S"] = S
        return ent["summ"]


SUMM_CACHE = SummaryCache()


def sparse_decode_supported(query, key) -> bool:
    """The block-sparse decode's domain (ugbsa_decode_step): 16-bit Q / K / V,
    head dim 64 / 128 / 256, at most 16 Q heads per KV head, caches of at most
    8192 blocks (512K tokens).  Outside it the hook decodes densely, as the
    reference always does."""
    Hq, Hkv, S, D = query.shape[1], key.shape[1], key.shape[2], query.shape[-1]
    return (query.dtype in (torch.bfloat16, torch.float16) and key.dtype == query.dtype and D in (64, 128, 256)
            and Hq % Hkv == 0 and Hq // Hkv <= 16 and S <= 8192 * 64)


def block_sparse_decode(module, query, key, value, scaling):
    """One decode row per head over the cache (bf16 / fp16, see
    sparse_decode_supported): block selection on the cached summaries, then
    attention over the kept blocks.  Returns [B, 1, H, D]."""
    cfg = SEL.config()
    S = key.shape[2]
    # blocks before the last are refreshed here; the step refreshes the last one itself
    summ = SUMM_CACHE.get(getattr(module, "layer_idx", 0), key, cfg.quest, last=False)
    out = ops.decode_step(query, key, value, summ, S, float(scaling), cfg)
    return out.transpose(1, 2).contiguous()


def block_sparse_attention(module, query, key, value, attention_mask, scaling, dropout=0.0, **kwargs):
    """HF attention hook: dense SDPA for decode / ``mode == "dense"``, else the
    v2 sparse path.  Returns ``(attn_output [B, S, H, D] contiguous, None)``."""
    Q = query.shape[-2]
    is_prefill = Q > 1
    if Q == 1 and SEL.decode_sparse and SEL.kernel_v2 and SEL.mode in ("topk", "router", "quest") \
            and sparse_decode_supported(query, key):
        return block_sparse_decode(module, query, key, value, scaling), None
    if SEL.mode == "dense" or Q == 1:
        ev = PROF.start("dense_sdpa") if is_prefill else None
        out = F.scaled_dot_product_attention(query, key, value, is_causal=(Q > 1), scale=scaling,
                                             enable_gqa=query.shape[1] != key.shape[1])
        PROF.stop(ev)
        return out.transpose(1, 2).contiguous(), None
    if SEL.kernel_v2 and SEL.mode in ("topk", "router", "quest"):
        ev = PROF.start("v2_select") if is_prefill else None
        kv_idx = _block_select_kv_idx_v2(query, key, scaling)   # module global: patchable
        PROF.stop(ev)
        ev = PROF.start("v2_kernel") if is_prefill else None
        B, H, S, D = query.shape
        out = torch.empty((B, S, H, D), device=query.device, dtype=query.dtype)
        ops.block_sparse_attn(query, key, value, kv_idx, float(scaling), out=out.transpose(1, 2))
        PROF.stop(ev)
        return out, None
    if SEL.mode in ("topk", "router", "quest"):
        # v1 path (:790-803): per-row selection, the tile's union list, per-row inner mask
        B, H, S, D = query.shape
        bits, kv_idx = _select_rows(query, key, scaling, getattr(module, "layer_idx", 0))
        out = torch.empty((B, S, H, D), device=query.device, dtype=query.dtype)
        ops.block_sparse_attn_rows(query, key, value, kv_idx, bits, float(scaling), out=out.transpose(1, 2))
        return out, None
    raise NotImplementedError(
        f"SEL.mode={SEL.mode!r}: the research policies belief / rollout / rollout_peek are not built on B200; "
        "topk / quest / router (v1 per-row or v2 per-tile) and dense are")


def register():
    """Register the hook with transformers' AttentionInterface as "block_sparse"."""
    from transformers import AttentionInterface
    AttentionInterface.register("block_sparse", block_sparse_attention)


try:  # registration at import, as the reference does (:806)
    register()
except ImportError:  # transformers is optional for the kernel-level API
    pass
