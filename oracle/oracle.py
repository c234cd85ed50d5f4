"""Python face of the CPU restatement (oracle/ugbsa_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, always as the checker.  The product path (the
CUDA library and its Python host package) never imports this module.

Every function takes and returns numpy arrays.  Q/K/V are float32 (bf16 inputs
are passed as their exact float32 values, which is what the reference's
oracle definition does: ``_block_select_kv_idx_v2(q.float(), k.float(), ...)``).

Reference anchors (paths inside the reference project):
  block summary        src/sparse_attention.py:617-646
  tile scores          src/sparse_attention.py:638-666
  selection + router   src/sparse_attention.py:675-725
  attention semantics  src/triton_block_attn.py:184-264, :301-312
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass

import numpy as np

BLOCK = 64
_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

MODE = {"topk": 0, "quest": 1, "router": 2}
ROUTER_MODE = {"abs": 0, "quantile": 1}
GRAIN = {"cell": 0, "row": 1}


class _Cfg(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int), ("router_mode", ctypes.c_int),
                ("router_grain", ctypes.c_int), ("router_quantile", ctypes.c_double),
                ("router_tau", ctypes.c_double), ("budget_blocks", ctypes.c_int),
                ("k_min", ctypes.c_int), ("k_max", ctypes.c_int)]


@dataclass
class OracleConfig:
    """The Selector knobs read by the v2 path (src/sparse_attention.py:58-97)."""
    mode: str = "router"             # topk | quest | router
    router_score: str = "mean"       # mean | quest (router only)
    router_mode: str = "quantile"    # abs | quantile
    router_grain: str = "row"        # cell | row
    router_quantile: float = 0.25
    router_tau: float = 0.10
    budget_blocks: int = 4
    k_min: int = 1
    k_max: int = 112

    @property
    def quest(self) -> bool:
        """Quest envelope scoring (:630-632)."""
        return self.mode == "quest" or (self.mode == "router" and self.router_score == "quest")

    def c(self) -> _Cfg:
        return _Cfg(MODE[self.mode], ROUTER_MODE[self.router_mode], GRAIN[self.router_grain],
                    float(self.router_quantile), float(self.router_tau),
                    int(self.budget_blocks), int(self.k_min), int(self.k_max))


def build() -> str:
    """Compile the C restatement (gcc) if its shared object is missing or stale."""
    src = os.path.join(_HERE, "ugbsa_oracle.c")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I = ctypes.c_int
        F = ctypes.c_float
        L.oracle_block_summary.argtypes = [P, I64, I64, I64, I64, I, I, I, I, I, P, P]
        L.oracle_tile_scores.argtypes = [P, I64, I64, I64, I64, P, P, I, I, I, I, I, F, I, P]
        L.oracle_select_from_scores.argtypes = [P, I, I, I, ctypes.POINTER(_Cfg), P, P, P, P, P]
        L.oracle_budget.argtypes = [ctypes.POINTER(_Cfg), I, ctypes.POINTER(I), ctypes.POINTER(I)]
        L.oracle_budget.restype = None
        L.oracle_attn.argtypes = ([P, I64, I64, I64, I64] * 3) + [P, I, I, I, I, I, I, I, F, P]
        L.oracle_tile_scores_range.argtypes = [P, I64, I64, I64, I64, P, P, I, I, I, I, I, F, I, I, I, P]
        L.oracle_rank_tiles_range.argtypes = [P, I, I, I, ctypes.POINTER(_Cfg), I, I, P, P]
        L.oracle_attn_range.argtypes = ([P, I64, I64, I64, I64] * 3) + [P, I, I, I, I, I, I, I, F, I, I, P]
        L.oracle_decode_scores.argtypes = [P, I64, I64, I64, P, P, I, I, I, I, I, I, F, I, P]
        L.oracle_row_scores.argtypes = [P, I64, I64, I64, I64, P, P, I, I, I, I, I, F, I, P]
        L.oracle_select_rows_from_scores.argtypes = [P, I, I, I, ctypes.POINTER(_Cfg), P, P, P, P, P]
        L.oracle_attn_keep.argtypes = ([P, I64, I64, I64, I64] * 3) + [P, I, I, I, I, I, I, F, P]
        L.oracle_set_threads.argtypes = [I]
        L.oracle_set_threads.restype = None
        L.oracle_get_threads.argtypes = []
        L.oracle_get_threads.restype = I
        _lib = L
    return _lib


def set_threads(n: int) -> int:
    """Use n threads in the restatement's parallel regions; returns the count in effect."""
    lib().oracle_set_threads(int(n))
    return lib().oracle_get_threads()


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def budget(cfg: OracleConfig, S: int):
    """(k_base, kmax) for a sequence of S tokens (:688-695)."""
    nb = math.ceil(S / BLOCK)
    kb, km = ctypes.c_int(), ctypes.c_int()
    lib().oracle_budget(ctypes.byref(cfg.c()), nb, ctypes.byref(kb), ctypes.byref(km))
    return kb.value, km.value


def block_summary(k: np.ndarray, quest: bool):
    """K [B,Hkv,S,D] -> mean [B,Hkv,NB,D] or (Kmin, Kmax)."""
    k = _f32(k)
    B, H, S, D = k.shape
    nb = math.ceil(S / BLOCK)
    a = np.empty((B, H, nb, D), np.float32)
    b = np.empty((B, H, nb, D), np.float32) if quest else None
    rc = lib().oracle_block_summary(_ptr(k), H * S * D, S * D, D, 1, B, H, S, D, int(quest),
                                    _ptr(a), _ptr(b) if quest else None)
    assert rc == 0
    return (a, b) if quest else a


def tile_scores(q: np.ndarray, summ, scale: float, quest: bool) -> np.ndarray:
    """Raw tile scores [B,Hq,Qt,NB] (-inf for causally invisible blocks)."""
    q = _f32(q)
    B, Hq, S, D = q.shape
    if quest:
        sa, sb = _f32(summ[0]), _f32(summ[1])
    else:
        sa, sb = _f32(summ), None
    Hkv = sa.shape[1]
    nb = math.ceil(S / BLOCK)
    ts = np.empty((B, Hq, nb, nb), np.float32)
    rc = lib().oracle_tile_scores(_ptr(q), Hq * S * D, S * D, D, 1, _ptr(sa),
                                  _ptr(sb) if quest else None, B, Hq, Hkv, S, D,
                                  ctypes.c_float(scale), int(quest), _ptr(ts))
    assert rc == 0
    return ts


def select_from_scores(ts: np.ndarray, S: int, cfg: OracleConfig) -> dict:
    """Selection, sigma router and sentinel fill from raw tile scores."""
    ts = _f32(ts)
    B, H, Qt, nb = ts.shape
    kb, km = budget(cfg, S)
    kv = np.empty((B, H, Qt, km), np.int32)
    sig = np.empty((B, H, Qt), np.float32)
    eff = np.empty((B, H, Qt), np.float32)
    trig = np.empty((B, H, Qt), np.uint8)
    th = np.empty((1,), np.float32)
    rc = lib().oracle_select_from_scores(_ptr(ts), B, H, S, ctypes.byref(cfg.c()), _ptr(kv),
                                         _ptr(sig), _ptr(eff), _ptr(trig), _ptr(th))
    assert rc == 0
    return {"kv_idx": kv, "sigma": sig, "sigma_eff": eff, "trigger": trig.astype(bool),
            "thresh": float(th[0]), "k_base": kb, "kmax": km}


def select(q: np.ndarray, k: np.ndarray, scale: float, cfg: OracleConfig) -> dict:
    """Whole v2 selection: summaries -> tile scores -> kv_idx (+ router state)."""
    summ = block_summary(k, cfg.quest)
    ts = tile_scores(q, summ, scale, cfg.quest)
    out = select_from_scores(ts, q.shape[2], cfg)
    out["tile_scores"] = ts
    out["summary"] = summ
    return out


def attn(q, k, v, kv_idx, scale: float) -> np.ndarray:
    """Block-sparse attention in float64 accumulation; returns float32 [B,Hq,Sq,D]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    kv_idx = np.ascontiguousarray(kv_idx, dtype=np.int32)
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    out = np.empty((B, Hq, Sq, D), np.float32)
    rc = lib().oracle_attn(_ptr(q), Hq * Sq * D, Sq * D, D, 1,
                           _ptr(k), Hkv * Sk * D, Sk * D, D, 1,
                           _ptr(v), Hkv * Sk * D, Sk * D, D, 1,
                           _ptr(kv_idx), kv_idx.shape[-1], B, Hq, Hkv, Sq, Sk, D,
                           ctypes.c_float(scale), _ptr(out))
    assert rc == 0
    return out


def sample_step(q, k, v, scale: float, cfg: OracleConfig, t_begin: int, t_end: int, summ=None):
    """The per-tile work of the whole path for tiles [t_begin, t_end) of every head:
    tile scores, ranking + sigma, and attention over the selected blocks.

    Used by bench.py to time a bounded CPU sample of a large workload (the
    per-layer quantile over all tiles is skipped: it is O(Qt) and negligible).
    ``summ`` may carry precomputed block summaries.  Returns (kv_idx, out) for
    the sampled tiles (other tiles of the arrays are left unset).
    """
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    nb = math.ceil(S / BLOCK)
    if summ is None:
        summ = block_summary(k, cfg.quest)
    sa, sb = (summ if cfg.quest else (summ, None))
    sa = _f32(sa)
    sb = _f32(sb) if sb is not None else None
    ts = np.empty((B, Hq, nb, nb), np.float32)
    L = lib()
    rc = L.oracle_tile_scores_range(_ptr(q), Hq * S * D, S * D, D, 1, _ptr(sa), _ptr(sb) if sb is not None else None,
                                    B, Hq, Hkv, S, D, ctypes.c_float(scale), int(cfg.quest), t_begin, t_end, _ptr(ts))
    assert rc == 0
    kb, km = budget(cfg, S)
    kv = np.full((B, Hq, nb, km), nb, np.int32)
    sig = np.empty((B, Hq, nb), np.float32)
    rc = L.oracle_rank_tiles_range(_ptr(ts), B, Hq, S, ctypes.byref(cfg.c()), t_begin, t_end, _ptr(kv), _ptr(sig))
    assert rc == 0
    out = np.zeros((B, Hq, S, D), np.float32)
    rc = L.oracle_attn_range(_ptr(q), Hq * S * D, S * D, D, 1, _ptr(k), Hkv * S * D, S * D, D, 1,
                             _ptr(v), Hkv * S * D, S * D, D, 1, _ptr(kv), km, B, Hq, Hkv, S, S, D,
                             ctypes.c_float(scale), t_begin, t_end, _ptr(out))
    assert rc == 0
    return kv, out


def sampled_tiles(q, summ, scale: float, cfg: OracleConfig, tiles) -> dict:
    """Exact tile scores, the ranked kmax slots (before the router's sentinel
    fill) and the per-tile margin for the listed query tiles of every (b, h) of
    ``q`` -- the per-tile part of the selection (src/sparse_attention.py:638-707)
    at sizes where the whole [B,H,Qt,NB] array would not be worth computing.
    ``summ`` are the summaries of the KV heads ``q``'s heads read (GQA as usual)."""
    q = _f32(q)
    B, Hq, S, D = q.shape
    sa, sb = (summ if cfg.quest else (summ, None))
    sa = _f32(sa)
    sb = _f32(sb) if sb is not None else None
    Hkv = sa.shape[1]
    nb = math.ceil(S / BLOCK)
    tiles = [int(t) for t in tiles]
    ts = np.full((B, Hq, nb, nb), -np.inf, np.float32)
    L = lib()
    for t in tiles:
        rc = L.oracle_tile_scores_range(_ptr(q), Hq * S * D, S * D, D, 1, _ptr(sa), _ptr(sb) if sb is not None else None,
                                        B, Hq, Hkv, S, D, ctypes.c_float(scale), int(cfg.quest), t, t + 1, _ptr(ts))
        assert rc == 0
    _, km = budget(cfg, S)
    kv = np.full((B, Hq, nb, km), -1, np.int32)
    sig = np.full((B, Hq, nb), np.nan, np.float32)
    for t in tiles:
        rc = L.oracle_rank_tiles_range(_ptr(ts), B, Hq, S, ctypes.byref(cfg.c()), t, t + 1, _ptr(kv), _ptr(sig))
        assert rc == 0
    return {"kv_idx": kv[:, :, tiles], "sigma": sig[:, :, tiles], "tile_scores": ts[:, :, tiles]}


def attn_tiles(q, k, v, kv_idx, scale: float, tiles) -> np.ndarray:
    """Attention rows of the listed query tiles (float64 accumulation, slot
    semantics of triton_block_attn.py:184-264); returns [B, Hq, len(tiles), 64, D]
    (rows past S are zero).  kv_idx covers every tile [B, Hq, Qt, kmax]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    kv_idx = np.ascontiguousarray(kv_idx, dtype=np.int32)
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    out = np.zeros((B, Hq, Sq, D), np.float32)
    L = lib()
    for t in tiles:
        rc = L.oracle_attn_range(_ptr(q), Hq * Sq * D, Sq * D, D, 1, _ptr(k), Hkv * Sk * D, Sk * D, D, 1,
                                 _ptr(v), Hkv * Sk * D, Sk * D, D, 1, _ptr(kv_idx), kv_idx.shape[-1], B, Hq, Hkv,
                                 Sq, Sk, D, ctypes.c_float(scale), int(t), int(t) + 1, _ptr(out))
        assert rc == 0
    rows = np.zeros((B, Hq, len(tiles), BLOCK, D), np.float32)
    for i, t in enumerate(tiles):
        r1 = min(Sq, (t + 1) * BLOCK)
        rows[:, :, i, :r1 - t * BLOCK] = out[:, :, t * BLOCK:r1]
    return rows


def router_from_cells(cells: np.ndarray, cfg: OracleConfig) -> dict:
    """The router over per-(b, head, tile) margins (src/sparse_attention.py:708-718):
    row grain -> head sum in head order, then / H (torch's mean), broadcast back;
    quantile -> the k-th smallest of the expanded [B,H,Qt] values, NaN last
    (kthvalue), k = max(1, int(q * numel)), trigger where value <= threshold;
    abs -> value < fp32(tau)."""
    cells = np.ascontiguousarray(cells, dtype=np.float32)
    B, H, Qt = cells.shape
    if cfg.router_grain == "row":
        acc = cells[:, 0].copy()
        for h in range(1, H):
            acc = (acc + cells[:, h]).astype(np.float32)
        eff = np.broadcast_to((acc / np.float32(H)).astype(np.float32)[:, None, :], (B, H, Qt)).copy()
    else:
        eff = cells.copy()
    if cfg.router_mode == "quantile":
        kq = max(1, int(float(cfg.router_quantile) * eff.size))
        thresh = np.sort(eff.reshape(-1))[kq - 1]   # NaN sorts last
        trig = eff <= thresh
    else:
        thresh = np.float32(cfg.router_tau)
        trig = eff < thresh
    return {"sigma_eff": eff, "thresh": np.float32(thresh), "trigger": trig}


def row_scores(q: np.ndarray, summ, scale: float, quest: bool) -> np.ndarray:
    """Per-row block scores [B,Hq,S,NB] (-inf where the block starts after the row),
    the v1 selector's score matrix (src/sparse_attention.py:221-244) in the canonical order."""
    q = _f32(q)
    B, Hq, S, D = q.shape
    sa, sb = (summ if quest else (summ, None))
    sa = _f32(sa)
    sb = _f32(sb) if sb is not None else None
    nb = math.ceil(S / BLOCK)
    rs = np.empty((B, Hq, S, nb), np.float32)
    rc = lib().oracle_row_scores(_ptr(q), Hq * S * D, S * D, D, 1, _ptr(sa), _ptr(sb) if quest else None, B, Hq,
                                 sa.shape[1], S, D, ctypes.c_float(scale), int(quest), _ptr(rs))
    assert rc == 0
    return rs


def select_rows_from_scores(rs: np.ndarray, cfg: OracleConfig) -> dict:
    """v1 per-row selection from per-row scores (src/sparse_attention.py:245-352):
    keep [B,H,S,NB] bool, per-(head, row) margins, margins after the grain step,
    triggers and the quantile threshold."""
    rs = _f32(rs)
    B, H, S, nb = rs.shape
    keep = np.empty((B, H, S, nb), np.uint8)
    sig = np.empty((B, H, S), np.float32)
    eff = np.empty((B, H, S), np.float32)
    trig = np.empty((B, H, S), np.uint8)
    th = np.empty((1,), np.float32)
    rc = lib().oracle_select_rows_from_scores(_ptr(rs), B, H, S, ctypes.byref(cfg.c()), _ptr(keep), _ptr(sig),
                                              _ptr(eff), _ptr(trig), _ptr(th))
    assert rc == 0
    return {"keep": keep.astype(bool), "sigma": sig, "sigma_eff": eff, "trigger": trig.astype(bool),
            "thresh": float(th[0])}


def select_rows(q: np.ndarray, k: np.ndarray, scale: float, cfg: OracleConfig) -> dict:
    """The whole v1 selection: summaries -> per-row scores -> keep (+ router state)."""
    summ = block_summary(k, cfg.quest)
    rs = row_scores(q, summ, scale, cfg.quest)
    out = select_rows_from_scores(rs, cfg)
    out["row_scores"] = rs
    return out


def attn_keep(q, k, v, keep, scale: float) -> np.ndarray:
    """Attention with a per-row keep mask [B,Hq,S,NB] (the v1 kernel's semantics,
    src/triton_block_attn.py:39-122), float64 accumulation, float32 out."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    keep = np.ascontiguousarray(keep, dtype=np.uint8)
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    out = np.empty((B, Hq, Sq, D), np.float32)
    rc = lib().oracle_attn_keep(_ptr(q), Hq * Sq * D, Sq * D, D, 1, _ptr(k), Hkv * Sk * D, Sk * D, D, 1,
                                _ptr(v), Hkv * Sk * D, Sk * D, D, 1, _ptr(keep), B, Hq, Hkv, Sq, Sk, D,
                                ctypes.c_float(scale), _ptr(out))
    assert rc == 0
    return out


def canonical_sets(kv_idx: np.ndarray, S: int):
    """Per (b,h,t) the frozenset of kept block ids that the attention can use.

    Drops the sentinel (>= NB) and causally invisible ids: the reference's
    topk fills short tiles with arbitrary -inf entries (:697-698), which its
    kernel skips (triton_block_attn.py:231-233), so only this set is defined.
    """
    nb = math.ceil(S / BLOCK)
    B, H, Qt, _ = kv_idx.shape
    out = np.empty((B, H, Qt), dtype=object)
    for b in range(B):
        for h in range(H):
            for t in range(Qt):
                last = min(t * BLOCK + BLOCK - 1, S - 1)
                row = kv_idx[b, h, t]
                out[b, h, t] = frozenset(int(x) for x in row if 0 <= x < nb and x * BLOCK <= last)
    return out


def attn_from_sets_mask(q, k, v, kv_idx, scale):
    """Masked-softmax restatement of reference_attn (triton_block_attn.py:301-312)
    in float64 numpy, for small cases: keep[b,h,m,blk] from the tile's kv_idx."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    nb = math.ceil(S / BLOCK)
    out = np.zeros((B, Hq, S, D), np.float64)
    causal = np.arange(S)[None, :] <= np.arange(S)[:, None]
    for b in range(B):
        for h in range(Hq):
            keep = np.zeros((S, nb * BLOCK), bool)
            for t in range(kv_idx.shape[2]):
                for x in kv_idx[b, h, t]:
                    if 0 <= x < nb:
                        keep[t * BLOCK:(t + 1) * BLOCK, x * BLOCK:(x + 1) * BLOCK] = True
            mask = keep[:, :S] & causal
            lg = (q[b, h].astype(np.float64) @ k[b, h // g].astype(np.float64).T) * scale
            lg = np.where(mask, lg, -np.inf)
            mx = lg.max(-1, keepdims=True)
            p = np.exp(lg - mx)
            out[b, h] = (p @ v[b, h // g].astype(np.float64)) / p.sum(-1, keepdims=True)
    return out.astype(np.float32)


def dump_pairs(S: int):
    """Sampled adjacent query-row pairs of the noise-scale estimate
    (src/dump_block_scores.py:154-162): n_pairs = min(1024, S - 1) rows i spaced
    max(1, (S - 1) // n_pairs) apart, clamped to S - 2; each pairs row i with i + 1."""
    n_pairs = min(1024, S - 1)
    stride = max(1, (S - 1) // n_pairs)
    return np.minimum(np.arange(n_pairs) * stride, S - 2), n_pairs, stride


def block_order_stats(q: np.ndarray, k: np.ndarray, scale: float, quest: bool, budget_blocks: int):
    """The per-tile order statistics of the block-score diagnostic
    (src/dump_block_scores.py:100-181), from the canonical fp32 tile scores.

    Tile scores are unforced (no sink / self forcing) and causally masked with
    -inf; k_b = min(2 * budget_blocks, NB) with no k_min / k_max clamp,
    rho_k = min(2 * k_b, NB).  Over the descending sort s of each tile's NB
    scores: g = s[k_b-1] - s[k_b]; r = max(s[0] - s[k_b], 1e-9);
    sigma = clip(g / r, 0, 2); g_rho = s[rho_k-1] - s[rho_k] (float32, IEEE
    inf / NaN as they fall); valid[t] = (visible blocks of t) > rho_k.
    tau_hat [B, H] = sqrt(max(0, mean((bs[i+1] - bs[i])^2) / 2)) over the
    sampled row pairs (dump_pairs) and all NB blocks, bs the unmasked per-row
    block scores (float64 here).  Returns None where the reference records
    nothing (rho_k <= k_b, rho_k = NB, or no valid tile)."""
    q = _f32(q)
    B, H, S, D = q.shape
    nb = math.ceil(S / BLOCK)
    k_b = min(2 * int(budget_blocks), nb)
    rho_k = min(2 * k_b, nb)
    if rho_k <= k_b or rho_k >= nb:
        # the reference returns early, or its s[rho_k] index is out of range
        # (its wrapper catches the error and records nothing)
        return None
    last = np.minimum(np.arange(nb) * BLOCK + BLOCK - 1, S - 1)
    n_vis = last // BLOCK + 1
    valid = n_vis > rho_k
    if not valid.any():
        return None
    summ = block_summary(k, quest)
    ts = tile_scores(q, summ, scale, quest)
    s = -np.sort(-ts, axis=-1)
    f32 = np.float32
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        g = (s[..., k_b - 1] - s[..., k_b]).astype(f32)
        r = np.maximum(s[..., 0] - s[..., k_b], f32(1e-9)).astype(f32)
        sigma = np.clip(g / r, f32(0.0), f32(2.0)).astype(f32)
        g_rho = (s[..., rho_k - 1] - s[..., rho_k]).astype(f32)
    # noise scale from unmasked per-row scores of the sampled pairs
    i0, n_pairs, _ = dump_pairs(S)
    Hkv = k.shape[1]
    grp = H // Hkv
    if quest:
        kmin, kmax_ = (x.astype(np.float64) for x in summ)
    else:
        kmean = summ.astype(np.float64)
    tau = np.zeros((B, H), np.float64)
    for b in range(B):
        for h in range(H):
            qa = q[b, h, i0].astype(np.float64)
            qb = q[b, h, i0 + 1].astype(np.float64)
            kv = h // grp
            if quest:
                sa = (np.maximum(qa, 0) @ kmax_[b, kv].T + np.minimum(qa, 0) @ kmin[b, kv].T) * scale
                sb = (np.maximum(qb, 0) @ kmax_[b, kv].T + np.minimum(qb, 0) @ kmin[b, kv].T) * scale
            else:
                sa = qa @ kmean[b, kv].T * scale
                sb = qb @ kmean[b, kv].T * scale
            tau[b, h] = 0.5 * np.mean((sb - sa) ** 2)
    return {"g": g, "r": r, "sigma": sigma, "g_rho": g_rho, "valid": valid,
            "tau_hat": np.sqrt(np.maximum(tau, 0.0)).astype(f32), "tile_scores": ts,
            "k_b": k_b, "rho_k": rho_k}


def _round(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> bf16 / fp16 (round to nearest even) -> float32."""
    x = np.asarray(x, np.float32)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)


def qk_norm_rope(x: np.ndarray, weight: np.ndarray, eps: float, cos: np.ndarray, sin: np.ndarray,
                 norm_mode: str = "offset", dtype: str = "bf16") -> np.ndarray:
    """Per-head RMSNorm then rotary embedding, in the element order and rounding of
    transformers' modules (the reference imports apply_rotary_pos_emb from
    transformers, src/sparse_attention.py:47-48):
      r = 1 / sqrt(mean(fp32(x^2)) + eps)            (fp32)
      scale  (Qwen3RMSNorm):              y = T(w * T(x * r))
      offset (Qwen3.5-MoE / Qwen3-Next):  y = T((x * r) * (1 + w))
      none   (Qwen2 / Llama, no per-head norm): y = x
      first R = cos.shape[-1] columns: T(T(y * cos) + T(rotate_half(y) * sin)); the rest y.
    x [B, H, S, D] float32 holding T values; weight [D]; cos / sin [B or 1, S, R].
    T rounding is emulated (round to nearest even)."""
    x = _f32(x)
    D = x.shape[-1]
    if norm_mode == "none":   # rotary only (Qwen2 / Llama attention)
        y = x.copy()
        R = cos.shape[-1]
        c = np.asarray(cos, np.float32)[:, None]
        s = np.asarray(sin, np.float32)[:, None]
        yr = y[..., :R]
        rot = np.concatenate([-yr[..., R // 2:], yr[..., :R // 2]], axis=-1)
        y[..., :R] = _round(_round(yr * c, dtype) + _round(rot * s, dtype), dtype)
        return y
    w = np.asarray(weight, np.float32)
    sq = (x * x).astype(np.float32)
    var = (sq.sum(-1, keepdims=True, dtype=np.float32) / np.float32(D)).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt((var + np.float32(eps)).astype(np.float32))).astype(np.float32)
    n = (x * r).astype(np.float32)
    if norm_mode == "offset":
        y = _round(n * (np.float32(1.0) + w), dtype)
    else:
        y = _round(w * _round(n, dtype), dtype)
    R = cos.shape[-1]
    c = np.asarray(cos, np.float32)[:, None]
    s = np.asarray(sin, np.float32)[:, None]
    yr = y[..., :R]
    rot = np.concatenate([-yr[..., R // 2:], yr[..., :R // 2]], axis=-1)
    out = y.copy()
    out[..., :R] = _round(_round(yr * c, dtype) + _round(rot * s, dtype), dtype)
    return out


def decode_select(q: np.ndarray, summ, S: int, scale: float, cfg: OracleConfig) -> dict:
    """Block selection for one decode row per head (the row at position S-1)
    from cache summaries (block_summary of the cache's first S keys):
    canonical exact scores of every block (oracle_decode_scores), sink and own
    (last) block forced to FLT_MAX, top kmax in descending score with ties to
    the lower id, sigma margin, row / cell grain, quantile / abs router over
    the B x Hq cells, sentinel NB in the untriggered cells' slots >= k_base.
    The same rules as the prefill selection (src/sparse_attention.py:675-725)
    on a one-row tile.  q [B, Hq, 1, D] or [B, Hq, D]."""
    q = _f32(q)
    if q.ndim == 4:
        q = np.ascontiguousarray(q[:, :, 0])
    B, Hq, D = q.shape
    sa = _f32(summ[0] if cfg.quest else summ)
    sb = _f32(summ[1]) if cfg.quest else None
    Hkv, nbs = sa.shape[1], sa.shape[2]
    nb = math.ceil(S / BLOCK)
    sc = np.empty((B, Hq, nb), np.float32)
    rc = lib().oracle_decode_scores(_ptr(q), Hq * D, D, 1, _ptr(sa), _ptr(sb) if sb is not None else None, nbs,
                                    B, Hq, Hkv, S, D, ctypes.c_float(scale), int(cfg.quest), _ptr(sc))
    assert rc == 0
    kb, km = budget(cfg, S)
    v = (sc + np.float32(0.0)).astype(np.float32)        # -0 folded into +0, as the key order does
    v[..., 0] = np.finfo(np.float32).max
    v[..., nb - 1] = np.finfo(np.float32).max
    ids = np.broadcast_to(np.arange(nb), v.shape)
    order = np.lexsort((ids, -v.astype(np.float64)), axis=-1)   # descending value, then lower id
    kv = order[..., :km].astype(np.int32)
    vs = np.take_along_axis(v, order, axis=-1)
    router = cfg.mode == "router" and kb < km
    f32 = np.float32
    sig = np.full((B, Hq), np.nan, f32)
    if router:
        with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
            spread = (vs[..., 0] - vs[..., kb]).astype(f32)
            spread = np.where(spread < f32(1e-6), f32(1e-6), spread).astype(f32)
            sig = ((vs[..., kb - 1] - vs[..., kb]).astype(f32) / spread).astype(f32)
    eff = np.full((B, Hq), np.nan, f32)
    trig = np.zeros((B, Hq), bool)
    thresh = float("nan")
    if router:
        if cfg.router_grain == "row":
            rs = np.zeros(B, f32)
            for h in range(Hq):
                rs = (rs + sig[:, h]).astype(f32)
            row_eff = (rs / f32(Hq)).astype(f32)
            eff = np.broadcast_to(row_eff[:, None], (B, Hq)).copy()
            vals, n = row_eff, B
        else:
            eff = sig.copy()
            vals, n = sig.reshape(-1), B * Hq
        if cfg.router_mode == "quantile":
            numel = B * Hq
            kq = min(max(1, int(cfg.router_quantile * numel)), numel)
            k = (kq - 1) // Hq + 1 if cfg.router_grain == "row" else kq
            srt = np.sort(vals.astype(f32))                 # NaN last
            thresh = float(srt[k - 1])
            trig = eff <= f32(thresh)
        else:
            trig = eff < f32(cfg.router_tau)
        kv = kv.copy()
        kv[..., kb:][~trig] = nb
    return {"kv_idx": kv, "scores": sc, "sigma_eff": eff if router else np.full((B, Hq), np.nan, f32),
            "trigger": trig, "thresh": thresh, "k_base": kb, "kmax": km}


def decode_attn(q, k, v, kv_idx, S: int, scale: float) -> np.ndarray:
    """Softmax over the keys (< S) of the kept blocks, per (b, head), float64;
    q [B, Hq, 1, D], k / v [B, Hkv, >=S, D], kv_idx [B, Hq, kmax] (ids >= NB
    skipped, repeated ids counted again).  Returns float32 [B, Hq, 1, D]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Hq, _, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    nb = math.ceil(S / BLOCK)
    out = np.zeros((B, Hq, 1, D), np.float64)
    for b in range(B):
        for h in range(Hq):
            keys = [blk * BLOCK + r for blk in kv_idx[b, h] if 0 <= blk < nb for r in range(BLOCK)
                    if blk * BLOCK + r < S]
            if not keys:
                continue
            kk = np.asarray(keys)
            kr = k[b, h // g, kk].astype(np.float64)
            vr = v[b, h // g, kk].astype(np.float64)
            lg = kr @ q[b, h, 0].astype(np.float64) * scale
            p = np.exp(lg - lg.max())
            out[b, h, 0] = p @ vr / p.sum()
    return out.astype(np.float32)
