"""Torch-facing wrappers around the C ABI (device memory and stream plumbing only).

Each function validates its tensors, allocates outputs with torch's caching
allocator, and calls one ``ugbsa_*`` entry point on the current CUDA stream.
All computation happens in libugbsa's sm_100a kernels; nothing here falls back
to PyTorch or the CPU.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib

BLOCK = 64

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


@dataclass(frozen=True)
class SelectorConfig:
    """The Selector knobs read by the v2 path (src/sparse_attention.py:58-97)."""
    mode: str = "router"             # topk | quest | router
    router_score: str = "mean"       # mean | quest (router mode)
    router_mode: str = "quantile"    # abs | quantile
    router_grain: str = "row"        # cell | row
    router_quantile: float = 0.20
    router_tau: float = 0.10
    budget_blocks: int = 32
    k_min: int = 8
    k_max: int = 112

    @property
    def quest(self) -> bool:
        return self.mode == "quest" or (self.mode == "router" and self.router_score == "quest")

    def to_c(self) -> _lib.SelectorConfig:
        if self.mode not in _lib.MODE:
            raise ValueError(f"v2 selection supports modes {sorted(_lib.MODE)}, got {self.mode!r}")
        return _lib.SelectorConfig(_lib.MODE[self.mode], _lib.SCORE[self.router_score],
                                   _lib.ROUTER_MODE[self.router_mode], _lib.GRAIN[self.router_grain],
                                   float(self.router_quantile), float(self.router_tau),
                                   int(self.budget_blocks), int(self.k_min), int(self.k_max))


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _strides(t: torch.Tensor) -> _lib.Strides:
    s = t.stride()
    return _lib.Strides(s[0], s[1], s[2], s[3])


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _need_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("ugbsa ops run on CUDA tensors only (no CPU path)")


def _inner_contig(t: torch.Tensor) -> torch.Tensor:
    """Views must have a unit innermost stride and 16-byte-multiple outer strides."""
    esz = t.element_size()
    if t.stride(-1) != 1 or any((s * esz) % 16 for s in t.stride()[:-1]) or t.data_ptr() % 16:
        return t.contiguous()
    return t


def budget(cfg: SelectorConfig, S: int):
    """(k_base, kmax) for S tokens (src/sparse_attention.py:688-695)."""
    kb, km = ctypes.c_int(), ctypes.c_int()
    c = cfg.to_c()
    _lib.check(_lib.load().ugbsa_select_budget(ctypes.byref(c), S, ctypes.byref(kb), ctypes.byref(km)),
               "ugbsa_select_budget")
    return kb.value, km.value


def block_summary(key: torch.Tensor, quest: bool, with_norm: bool = False):
    """K [B,Hkv,S,D] -> mean [B,Hkv,NB,D] fp32, or (Kmin, Kmax); optional per-block norms."""
    _need_cuda(key)
    if key.dim() != 4 or key.dtype not in _DTYPES:
        raise ValueError("key must be a [B,H,S,D] float32/bfloat16/float16 tensor")
    key = _inner_contig(key)
    B, H, S, D = key.shape
    NB = math.ceil(S / BLOCK)
    a = torch.empty((B, H, NB, D), device=key.device, dtype=torch.float32)
    b = torch.empty_like(a) if quest else None
    n = torch.empty((B, H, NB), device=key.device, dtype=torch.float32) if with_norm else None
    rc = _lib.load().ugbsa_block_summary(_ptr(key), _DTYPES[key.dtype], _strides(key), B, H, S, D, int(quest),
                                         _ptr(a), _ptr(b), _ptr(n), _stream())
    _lib.check(rc, "ugbsa_block_summary")
    out = (a, b) if quest else a
    return (out, n) if with_norm else out


def select_kv_idx(query: torch.Tensor, key: torch.Tensor, scaling: float, cfg: SelectorConfig,
                  return_router: bool = False, summ=None):
    """v2 selection: kv_idx [B,Hq,Qt,kmax] int32 (+ sigma, trigger when asked).

    ``key`` may carry Hkv heads (GQA, Hq % Hkv == 0) or Hq heads (after repeat_kv).
    ``summ``: ``key``'s block summaries when already computed (qk_norm_rope with
    a summary, or block_summary); the summary pass is then skipped.
    """
    _need_cuda(query, key)
    if query.dim() != 4 or key.dim() != 4:
        raise ValueError("query/key must be [B,H,S,D]")
    B, Hq, S, D = query.shape
    if key.shape[0] != B or key.shape[2] != S or key.shape[3] != D or Hq % key.shape[1]:
        raise ValueError(f"incompatible query {tuple(query.shape)} / key {tuple(key.shape)} (prefill needs Sq == Sk)")
    if query.dtype not in _DTYPES or key.dtype not in _DTYPES:
        raise ValueError("unsupported dtype")
    query = _inner_contig(query)
    if summ is None:
        summ = block_summary(key, cfg.quest)
    sa, sb = (summ if cfg.quest else (summ, None))
    k_base, kmax = budget(cfg, S)
    Qt = math.ceil(S / BLOCK)
    kv_idx = torch.empty((B, Hq, Qt, kmax), device=query.device, dtype=torch.int32)
    c = cfg.to_c()
    ws_bytes = _lib.load().ugbsa_select_workspace_bytes_ex(ctypes.byref(c), _DTYPES[query.dtype], B, Hq,
                                                           key.shape[1], S, D)
    ws = torch.empty((ws_bytes,), device=query.device, dtype=torch.uint8)
    sigma = torch.empty((B, Hq, Qt), device=query.device, dtype=torch.float32) if return_router else None
    trig = torch.empty((B, Hq, Qt), device=query.device, dtype=torch.uint8) if return_router else None
    rc = _lib.load().ugbsa_select(_ptr(query), _DTYPES[query.dtype], _strides(query), _ptr(sa), _ptr(sb), B, Hq,
                                  key.shape[1], S, D, ctypes.c_float(scaling), ctypes.byref(c), _ptr(kv_idx), kmax,
                                  _ptr(sigma), _ptr(trig), _ptr(ws), ctypes.c_size_t(ws_bytes), _stream())
    _lib.check(rc, "ugbsa_select")
    if return_router:
        return kv_idx, sigma, trig.bool()
    return kv_idx


def block_sparse_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_idx: torch.Tensor, scale: float,
                      out: torch.Tensor | None = None, row_base: int = 0, peer_out=None,
                      pair_stride: int = 1) -> torch.Tensor:
    """Block-sparse causal attention: q [B,Hq,Sq,D], k/v [B,Hkv,Sk,D] (bf16/fp16).

    ``out`` (optional) is a [B,Hq,Sq,D] view to write into (any strides with a
    unit innermost stride), e.g. ``buf.transpose(1, 2)`` of a [B,S,H,D] buffer.
    ``row_base`` (a multiple of 64): q holds sequence rows row_base ..
    row_base + Sq - 1 and kv_idx their tiles (ugbsa_attn_rows); with
    ``pair_stride`` m > 1, q holds the tile pairs row_base/128 + k*m and
    ``out`` is the full [B,Hq,Sk,D] view (only those rows are written).
    ``peer_out``: device addresses of the same ``out`` view in other GPUs'
    buffers (PeerBuffer.peer_views); the kernel writes every tile there too
    (ugbsa_attn_rows_peers).
    """
    _need_cuda(q, k, v, kv_idx)
    if q.dtype not in (torch.bfloat16, torch.float16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("block_sparse_attn takes bf16, fp16 or fp32 q/k/v of one dtype")
    if peer_out and q.dtype == torch.float32:
        raise ValueError("output peers take bf16 / fp16 outputs")
    if kv_idx.dtype != torch.int32:
        raise ValueError("kv_idx must be int32")
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    if k.shape != v.shape or k.shape[0] != B or k.shape[3] != D or Hq % Hkv:
        raise ValueError(f"incompatible q {tuple(q.shape)} k {tuple(k.shape)} v {tuple(v.shape)}")
    Qt = math.ceil(Sq / BLOCK)
    if kv_idx.dim() != 4 or tuple(kv_idx.shape[:3]) != (B, Hq, Qt):
        raise ValueError(f"kv_idx must be [B,Hq,{Qt},kmax], got {tuple(kv_idx.shape)}")
    q, k, v = _inner_contig(q), _inner_contig(k), _inner_contig(v)
    kv_idx = kv_idx.contiguous()
    out_rows = Sq if pair_stride == 1 else Sk
    if out is None:
        out = torch.empty((B, Hq, out_rows, D), device=q.device, dtype=q.dtype)
    elif tuple(out.shape) != (B, Hq, out_rows, D) or out.dtype != q.dtype or out.stride(-1) != 1:
        raise ValueError(f"out must be a [B,Hq,{out_rows},D] view with unit innermost stride")
    L = _lib.load()
    if peer_out:
        arr = (ctypes.c_void_p * len(peer_out))(*peer_out)
        rc = L.ugbsa_attn_rows_peers(_ptr(q), _ptr(k), _ptr(v), _DTYPES[q.dtype], _strides(q), _strides(k),
                                     _strides(v), _ptr(kv_idx), kv_idx.shape[-1], B, Hq, Hkv, Sq, Sk, D,
                                     int(row_base), int(pair_stride), ctypes.c_float(scale), _ptr(out),
                                     _strides(out), arr, len(peer_out), _stream())
        _lib.check(rc, "ugbsa_attn_rows_peers")
        return out
    if row_base or pair_stride != 1:
        rc = L.ugbsa_attn_rows(_ptr(q), _ptr(k), _ptr(v), _DTYPES[q.dtype], _strides(q), _strides(k), _strides(v),
                               _ptr(kv_idx), kv_idx.shape[-1], B, Hq, Hkv, Sq, Sk, D, int(row_base),
                               int(pair_stride), ctypes.c_float(scale), _ptr(out), _strides(out), _stream())
        _lib.check(rc, "ugbsa_attn_rows")
        return out
    rc = L.ugbsa_attn(_ptr(q), _ptr(k), _ptr(v), _DTYPES[q.dtype], _strides(q), _strides(k), _strides(v),
                      _ptr(kv_idx), kv_idx.shape[-1], B, Hq, Hkv, Sq, Sk, D, ctypes.c_float(scale),
                      _ptr(out), _strides(out), _stream())
    _lib.check(rc, "ugbsa_attn")
    return out


# ------------------------------------------------------------------ v1 per-row selection
def select_rows(query: torch.Tensor, key: torch.Tensor, scaling: float, cfg: SelectorConfig,
                return_router: bool = False, summ=None, with_tiles: bool = True):
    """The v1 per-row selector (ugbsa_select_rows): keep bits [B,Hq,S,ceil(NB/32)]
    int32 (bit j of a row: block j kept) and, with ``with_tiles``, each tile's
    union list kv_idx [B,Hq,Qt,NB] (ascending, sentinel NB); with
    ``return_router`` also the margins after the grain step [B,Hq,S] (+inf for
    ineligible rows) and the triggers.  ``key`` may carry Hkv or Hq heads."""
    _need_cuda(query, key)
    B, Hq, S, D = query.shape
    if key.shape[0] != B or key.shape[2] != S or key.shape[3] != D or Hq % key.shape[1]:
        raise ValueError(f"incompatible query {tuple(query.shape)} / key {tuple(key.shape)}")
    query = _inner_contig(query)
    if summ is None:
        summ = block_summary(key, cfg.quest)
    sa, sb = (summ if cfg.quest else (summ, None))
    nb = math.ceil(S / BLOCK)
    nbw = (nb + 31) // 32
    bits = torch.empty((B, Hq, S, nbw), device=query.device, dtype=torch.int32)
    kv_idx = torch.empty((B, Hq, nb, nb), device=query.device, dtype=torch.int32) if with_tiles else None
    sigma = torch.empty((B, Hq, S), device=query.device, dtype=torch.float32) if return_router else None
    trig = torch.empty((B, Hq, S), device=query.device, dtype=torch.uint8) if return_router else None
    c = cfg.to_c()
    L = _lib.load()
    ws_bytes = L.ugbsa_select_rows_workspace_bytes(ctypes.byref(c), B, Hq, S)
    ws = torch.empty((ws_bytes,), device=query.device, dtype=torch.uint8)
    rc = L.ugbsa_select_rows(_ptr(query), _DTYPES[query.dtype], _strides(query), _ptr(sa), _ptr(sb), B, Hq,
                             key.shape[1], S, D, ctypes.c_float(scaling), ctypes.byref(c), _ptr(bits), _ptr(kv_idx),
                             _ptr(sigma), _ptr(trig), _ptr(ws), ctypes.c_size_t(ws_bytes), _stream())
    _lib.check(rc, "ugbsa_select_rows")
    if return_router:
        return bits, kv_idx, sigma, trig.bool()
    return bits, kv_idx


def keep_to_tiles(keep: torch.Tensor):
    """A keep mask [B,H,S,NB] (bool / uint8) -> (bits [B,H,S,ceil(NB/32)] int32,
    kv_idx [B,H,Qt,NB]: each tile's union of its rows' blocks, ascending)."""
    _need_cuda(keep)
    B, H, S, nb = keep.shape
    if nb != math.ceil(S / BLOCK):
        raise ValueError(f"keep must be [B,H,S,ceil(S/64)], got {tuple(keep.shape)}")
    k8 = keep.to(torch.uint8).contiguous()
    bits = torch.empty((B, H, S, (nb + 31) // 32), device=keep.device, dtype=torch.int32)
    kv_idx = torch.empty((B, H, nb, nb), device=keep.device, dtype=torch.int32)
    rc = _lib.load().ugbsa_keep_to_tiles(_ptr(k8), _ptr(bits), B, H, S, _ptr(kv_idx), _stream())
    _lib.check(rc, "ugbsa_keep_to_tiles")
    return bits, kv_idx


def unpack_keep(bits: torch.Tensor, nb: int) -> torch.Tensor:
    """keep bits [..., ceil(NB/32)] -> bool [..., NB] (device ops)."""
    shifts = torch.arange(32, device=bits.device, dtype=torch.int32)
    b = (bits.unsqueeze(-1) >> shifts) & 1
    return b.reshape(*bits.shape[:-1], -1)[..., :nb].bool()


def block_sparse_attn_rows(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_idx: torch.Tensor,
                           keep_bits: torch.Tensor, scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention over the tiles' union lists with the per-row keep mask
    (ugbsa_attn_rowmask): q [B,Hq,S,D], k/v [B,Hkv,S,D] bf16 / fp16."""
    _need_cuda(q, k, v, kv_idx, keep_bits)
    if q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("the per-row masked attention takes bf16 or fp16 q/k/v of one dtype")
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    q, k, v = _inner_contig(q), _inner_contig(k), _inner_contig(v)
    if out is None:
        out = torch.empty((B, Hq, S, D), device=q.device, dtype=q.dtype)
    kv_idx = kv_idx.contiguous()
    keep_bits = keep_bits.contiguous()
    rc = _lib.load().ugbsa_attn_rowmask(_ptr(q), _ptr(k), _ptr(v), _DTYPES[q.dtype], _strides(q), _strides(k),
                                        _strides(v), _ptr(kv_idx), kv_idx.shape[-1], _ptr(keep_bits), B, Hq, Hkv,
                                        S, D, ctypes.c_float(scale), _ptr(out), _strides(out), _stream())
    _lib.check(rc, "ugbsa_attn_rowmask")
    return out


def slice_rows(S: int, row_base: int, pair_stride: int, n_tiles: int) -> int:
    """Query rows of a slice of n_tiles local tiles (see ugbsa_select_tiles_rows):
    local tile t is sequence tile row_base/64 + t + 2*(t//2)*(pair_stride-1)."""
    tb = row_base // BLOCK
    rows = 0
    for t in range(n_tiles):
        g = tb + t + 2 * (t // 2) * (pair_stride - 1)
        rows += min(BLOCK, S - BLOCK * g)
    return rows


# ------------------------------------------------------------------ decode
def block_summary_update(key: torch.Tensor, quest: bool, summ, first_block: int):
    """Recompute the summaries of blocks first_block .. ceil(S/64)-1 of key
    [B,Hkv,S,D] into ``summ`` (mean [B,Hkv,cap,D], or (Kmin, Kmax)), in place."""
    _need_cuda(key)
    B, H, S, D = key.shape
    sa, sb = (summ if quest else (summ, None))
    cap = sa.shape[2]
    key = _inner_contig(key)
    rc = _lib.load().ugbsa_block_summary_update(_ptr(key), _DTYPES[key.dtype], _strides(key), B, H, S, D,
                                                int(quest), int(first_block), cap, _ptr(sa), _ptr(sb), _stream())
    _lib.check(rc, "ugbsa_block_summary_update")
    return summ


def _decode_ws(B, Hq, S, D, kmax, device):
    n = _lib.load().ugbsa_decode_workspace_bytes(B, Hq, S, D, kmax)
    return torch.empty((n,), device=device, dtype=torch.uint8), n


def decode_select(query: torch.Tensor, summ, S: int, n_kv_heads: int, scaling: float, cfg: SelectorConfig,
                  return_router: bool = False):
    """kv_idx [B,Hq,kmax] for one decode row per head (query [B,Hq,1,D]) over a
    cache of S keys whose block summaries ``summ`` (capacity >= ceil(S/64)
    blocks) are current (ugbsa_decode_select)."""
    _need_cuda(query)
    B, Hq, Q, D = query.shape
    if Q != 1:
        raise ValueError("decode_select takes one query row per head")
    sa, sb = (summ if cfg.quest else (summ, None))
    _, kmax = budget(cfg, S)
    kv_idx = torch.empty((B, Hq, kmax), device=query.device, dtype=torch.int32)
    sigma = torch.empty((B, Hq), device=query.device, dtype=torch.float32) if return_router else None
    trig = torch.empty((B, Hq), device=query.device, dtype=torch.uint8) if return_router else None
    ws, n = _decode_ws(B, Hq, S, D, kmax, query.device)
    c = cfg.to_c()
    rc = _lib.load().ugbsa_decode_select(_ptr(query), _DTYPES[query.dtype], _strides(query), _ptr(sa), _ptr(sb),
                                         sa.shape[2], B, Hq, n_kv_heads, S, D, ctypes.c_float(scaling),
                                         ctypes.byref(c), _ptr(kv_idx), kmax, _ptr(sigma), _ptr(trig), _ptr(ws),
                                         ctypes.c_size_t(n), _stream())
    _lib.check(rc, "ugbsa_decode_select")
    if return_router:
        return kv_idx, sigma, trig.bool()
    return kv_idx


def decode_attn(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, kv_idx: torch.Tensor, S: int,
                scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """out [B,Hq,1,D]: softmax over the keys (< S) of the kept blocks of kv_idx
    [B,Hq,kmax] (ugbsa_decode_attn); key / value [B,Hkv,>=S,D] (a cache)."""
    _need_cuda(query, key, value, kv_idx)
    B, Hq, Q, D = query.shape
    if Q != 1 or query.dtype not in (torch.bfloat16, torch.float16) or key.dtype != query.dtype \
            or value.dtype != query.dtype:
        raise ValueError("decode_attn takes one bf16/fp16 query row per head and K/V of its dtype")
    Hkv = key.shape[1]
    query, key, value = _inner_contig(query), _inner_contig(key), _inner_contig(value)
    kv_idx = kv_idx.contiguous()
    kmax = kv_idx.shape[-1]
    if out is None:
        out = torch.empty((B, Hq, 1, D), device=query.device, dtype=query.dtype)
    ws, n = _decode_ws(B, Hq, S, D, kmax, query.device)
    rc = _lib.load().ugbsa_decode_attn(_ptr(query), _ptr(key), _ptr(value), _DTYPES[query.dtype], _strides(query),
                                       _strides(key), _strides(value), _ptr(kv_idx), kmax, B, Hq, Hkv, S, D,
                                       ctypes.c_float(scale), _ptr(out), _strides(out), _ptr(ws),
                                       ctypes.c_size_t(n), _stream())
    _lib.check(rc, "ugbsa_decode_attn")
    return out


def decode_step(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, summ, S: int, scaling: float,
                cfg: SelectorConfig, return_router: bool = False, out: torch.Tensor | None = None):
    """One decode step (ugbsa_decode_step): the summary refresh of the cache's last
    block, the selection and the attention -- the results of block_summary_update
    (from the last block) + decode_select + decode_attn, in three launches.
    query [B,Hq,1,D]; key / value [B,Hkv,>=S,D] bf16 / fp16; summ the cache
    summaries (updated in place).  Returns out [B,Hq,1,D] (and kv_idx, sigma,
    trigger with return_router)."""
    _need_cuda(query, key, value)
    B, Hq, Q, D = query.shape
    if Q != 1 or query.dtype not in (torch.bfloat16, torch.float16) or key.dtype != query.dtype \
            or value.dtype != query.dtype:
        raise ValueError("decode_step takes one bf16/fp16 query row per head and K/V of its dtype")
    Hkv = key.shape[1]
    query, key, value = _inner_contig(query), _inner_contig(key), _inner_contig(value)
    sa, sb = (summ if cfg.quest else (summ, None))
    _, kmax = budget(cfg, S)
    kv_idx = torch.empty((B, Hq, kmax), device=query.device, dtype=torch.int32)
    sigma = torch.empty((B, Hq), device=query.device, dtype=torch.float32) if return_router else None
    trig = torch.empty((B, Hq), device=query.device, dtype=torch.uint8) if return_router else None
    if out is None:
        out = torch.empty((B, Hq, 1, D), device=query.device, dtype=query.dtype)
    ws, n = _decode_ws(B, Hq, S, D, kmax, query.device)
    c = cfg.to_c()
    rc = _lib.load().ugbsa_decode_step(_ptr(query), _ptr(key), _ptr(value), _DTYPES[query.dtype], _strides(query),
                                       _strides(key), _strides(value), _ptr(sa), _ptr(sb), sa.shape[2], B, Hq, Hkv,
                                       S, D, ctypes.c_float(scaling), ctypes.byref(c), _ptr(kv_idx), kmax,
                                       _ptr(sigma), _ptr(trig), _ptr(out), _strides(out), _ptr(ws),
                                       ctypes.c_size_t(n), _stream())
    _lib.check(rc, "ugbsa_decode_step")
    if return_router:
        return out, kv_idx, sigma, trig.bool()
    return out


def qk_norm_rope(x: torch.Tensor, weight: torch.Tensor, eps: float, cos: torch.Tensor, sin: torch.Tensor,
                 norm_mode: str = "offset", out: torch.Tensor | None = None, summary: str | None = None):
    """Per-head RMSNorm + rotary embedding in one pass (ugbsa_qk_norm_rope).

    x [B,H,S,D] bf16/fp16 view (e.g. proj.view(B,S,H,D).transpose(1,2));
    weight [D]; cos/sin [B or 1, S, R] (R rotated columns).  norm_mode
    "scale" (Qwen3RMSNorm), "offset" (Qwen3.5-MoE / Qwen3-Next, 1 + w) or
    "none" (rotary only, Qwen2 / Llama attention; ``weight`` may be None).
    ``out`` [B,H,S,D] view (default: new contiguous; ``x`` itself works).
    summary "mean" / "quest": also returns the block summaries of the output
    (as block_summary(out, ...) would): (out, summ).
    """
    if norm_mode == "none":
        _need_cuda(x, cos, sin)
    else:
        _need_cuda(x, weight, cos, sin)
    if x.dtype not in (torch.bfloat16, torch.float16) or (weight is not None and weight.dtype != x.dtype) \
            or cos.dtype != x.dtype or sin.dtype != x.dtype:
        raise ValueError("x, weight, cos and sin must share one dtype (bf16 or fp16)")
    B, H, S, D = x.shape
    if cos.dim() == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    if cos.shape != sin.shape or cos.shape[1] != S or cos.shape[0] not in (1, B) or cos.stride(-1) != 1 \
            or sin.stride() != cos.stride():
        raise ValueError("cos/sin must be [B or 1, S, R] with unit innermost stride and equal strides")
    R = cos.shape[-1]
    x = _inner_contig(x)
    weight = weight.contiguous() if norm_mode != "none" else None
    if out is None:
        out = torch.empty((B, H, S, D), device=x.device, dtype=x.dtype)
    elif tuple(out.shape) != (B, H, S, D) or out.dtype != x.dtype or out.stride(-1) != 1:
        raise ValueError("out must be a [B,H,S,D] view with unit innermost stride")
    mode = {"scale": _lib.NORM_SCALE, "offset": _lib.NORM_OFFSET, "none": _lib.NORM_NONE}[norm_mode]
    sm = {None: 0, "mean": 1, "quest": 2}[summary]
    nb = math.ceil(S / BLOCK)
    sa = torch.empty((B, H, nb, D), device=x.device, dtype=torch.float32) if sm else None
    sb = torch.empty((B, H, nb, D), device=x.device, dtype=torch.float32) if sm == 2 else None
    cb = cos.stride(0) if cos.shape[0] == B and B > 1 else 0
    rc = _lib.load().ugbsa_qk_norm_rope(_ptr(x), _DTYPES[x.dtype], _strides(x), _ptr(weight), mode,
                                        ctypes.c_float(eps), _ptr(cos), _ptr(sin), cb, cos.stride(1), R, B, H, S,
                                        D, _ptr(out), _strides(out), sm, _ptr(sa), _ptr(sb), _stream())
    _lib.check(rc, "ugbsa_qk_norm_rope")
    if not sm:
        return out
    return out, ((sa, sb) if sm == 2 else sa)


def block_order_stats(query: torch.Tensor, key: torch.Tensor, scaling: float, quest: bool, budget_blocks: int,
                      with_tau: bool = True):
    """Order statistics of the block-score diagnostic (ugbsa_block_order_stats):
    dict of g, r, sigma, g_rho [B,Hq,Qt] fp32, valid [Qt] bool and tau_hat [B,Hq]
    (None without with_tau), or None where the diagnostic records nothing
    (k_b = min(2*budget_blocks, NB) leaves no rank rho_k = min(2*k_b, NB) < NB
    above it, or no tile sees more than rho_k blocks).  ``key`` may carry Hkv
    heads (GQA) or Hq heads."""
    _need_cuda(query, key)
    B, Hq, S, D = query.shape
    nb = math.ceil(S / BLOCK)
    k_b = min(2 * int(budget_blocks), nb)
    rho_k = min(2 * k_b, nb)
    if S < 2 or rho_k <= k_b or rho_k >= nb:
        return None
    last = torch.clamp(torch.arange(nb) * BLOCK + BLOCK - 1, max=S - 1)
    valid = (last // BLOCK + 1) > rho_k
    if not bool(valid.any()):
        return None
    query = _inner_contig(query)
    summ = block_summary(key, quest)
    sa, sb = (summ if quest else (summ, None))
    dev = query.device
    out = {n: torch.empty((B, Hq, nb), device=dev, dtype=torch.float32) for n in ("g", "r", "sigma", "g_rho")}
    tau = torch.empty((B, Hq), device=dev, dtype=torch.float32) if with_tau else None
    L = _lib.load()
    ws_bytes = L.ugbsa_block_order_stats_workspace_bytes(B, Hq, S) if with_tau else 0
    ws = torch.empty((max(ws_bytes, 1),), device=dev, dtype=torch.uint8)
    rc = L.ugbsa_block_order_stats(_ptr(query), _DTYPES[query.dtype], _strides(query), _ptr(sa), _ptr(sb), B, Hq,
                                   key.shape[1], S, D, ctypes.c_float(scaling), int(quest), int(budget_blocks),
                                   _ptr(out["g"]), _ptr(out["r"]), _ptr(out["sigma"]), _ptr(out["g_rho"]),
                                   _ptr(tau), _ptr(ws), ctypes.c_size_t(ws_bytes), _stream())
    _lib.check(rc, "ugbsa_block_order_stats")
    out["valid"] = valid
    out["tau_hat"] = tau
    return out


def read_device_error() -> int:
    """Raw device error bits since the last call (host sync); 0 when healthy."""
    bits = ctypes.c_int(0)
    _lib.load().ugbsa_read_device_error(_stream(), ctypes.byref(bits))
    return bits.value


def select_tiles(query: torch.Tensor, summ, n_kv_heads: int, scaling: float, cfg: SelectorConfig,
                 want_rowsum: bool = True, row_base: int = 0, seq_len: int | None = None, pair_stride: int = 1):
    """First half of the selection for a shard of heads (ugbsa_select_tiles) or,
    with ``row_base`` / ``seq_len`` / ``pair_stride``, for a slice of the query
    rows of a ``seq_len``-token sequence (ugbsa_select_tiles_rows; ``summ`` then
    covers all seq_len keys).

    Returns (kv_idx [B,Hq,Qt,kmax] with all slots filled, sigma_cells [B,Hq,Qt],
    sigma_rowsum [B,Qt] or None), Qt the query tiles of this call."""
    _need_cuda(query)
    query = _inner_contig(query)
    B, Hq, Sq, D = query.shape
    S = Sq if seq_len is None else int(seq_len)
    sa, sb = (summ if cfg.quest else (summ, None))
    _, kmax = budget(cfg, S)
    Qt = math.ceil(Sq / BLOCK)
    kv_idx = torch.empty((B, Hq, Qt, kmax), device=query.device, dtype=torch.int32)
    cells = torch.empty((B, Hq, Qt), device=query.device, dtype=torch.float32)
    rowsum = torch.empty((B, Qt), device=query.device, dtype=torch.float32) if want_rowsum else None
    c = cfg.to_c()
    L = _lib.load()
    ws_bytes = L.ugbsa_select_workspace_bytes_ex(ctypes.byref(c), _DTYPES[query.dtype], B, Hq, n_kv_heads, S, D)
    ws = torch.empty((ws_bytes,), device=query.device, dtype=torch.uint8)
    if row_base or Sq != S or pair_stride != 1:
        rc = L.ugbsa_select_tiles_rows(_ptr(query), _DTYPES[query.dtype], _strides(query), _ptr(sa), _ptr(sb), B,
                                       Hq, n_kv_heads, S, D, int(row_base), int(pair_stride), Sq,
                                       ctypes.c_float(scaling), ctypes.byref(c), _ptr(kv_idx), kmax, _ptr(cells),
                                       _ptr(rowsum), _ptr(ws), ctypes.c_size_t(ws_bytes), _stream())
        _lib.check(rc, "ugbsa_select_tiles_rows")
        return kv_idx, cells, rowsum
    rc = L.ugbsa_select_tiles(_ptr(query), _DTYPES[query.dtype], _strides(query), _ptr(sa), _ptr(sb), B,
                              Hq, n_kv_heads, S, D, ctypes.c_float(scaling), ctypes.byref(c), _ptr(kv_idx),
                              kmax, _ptr(cells), _ptr(rowsum), _ptr(ws), ctypes.c_size_t(ws_bytes), _stream())
    _lib.check(rc, "ugbsa_select_tiles")
    return kv_idx, cells, rowsum


def select_finish(kv_idx: torch.Tensor, sigma_cells: torch.Tensor, sigma_all: torch.Tensor, n_heads_total: int,
                  S: int, cfg: SelectorConfig, return_router: bool = False, row_base: int = 0,
                  pair_stride: int = 1):
    """Second half: shared quantile over all heads and tiles, sentinel fill of
    this call's kv_idx (in place).  ``row_base``: kv_idx holds the tiles of the
    query rows starting there (ugbsa_select_finish_rows)."""
    B, Hq, Qt, kmax = kv_idx.shape
    L = _lib.load()
    ws_bytes = L.ugbsa_select_finish_workspace_bytes(B, S)
    ws = torch.empty((ws_bytes,), device=kv_idx.device, dtype=torch.uint8)
    sigma = torch.empty((B, Hq, Qt), device=kv_idx.device, dtype=torch.float32) if return_router else None
    trig = torch.empty((B, Hq, Qt), device=kv_idx.device, dtype=torch.uint8) if return_router else None
    c = cfg.to_c()
    Sq = slice_rows(S, int(row_base), int(pair_stride), Qt)
    if row_base or Sq != S or pair_stride != 1:
        rc = L.ugbsa_select_finish_rows(_ptr(sigma_cells), _ptr(sigma_all.contiguous()), B, Hq, n_heads_total, S,
                                        int(row_base), int(pair_stride), Sq, ctypes.byref(c), _ptr(kv_idx), kmax,
                                        _ptr(sigma), _ptr(trig), _ptr(ws), ctypes.c_size_t(ws_bytes), _stream())
        _lib.check(rc, "ugbsa_select_finish_rows")
    else:
        rc = L.ugbsa_select_finish(_ptr(sigma_cells), _ptr(sigma_all.contiguous()), B, Hq, n_heads_total, S,
                                   ctypes.byref(c), _ptr(kv_idx), kmax, _ptr(sigma), _ptr(trig), _ptr(ws),
                                   ctypes.c_size_t(ws_bytes), _stream())
        _lib.check(rc, "ugbsa_select_finish")
    if return_router:
        return kv_idx, sigma, trig.bool()
    return kv_idx
