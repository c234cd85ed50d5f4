"""Kernel-level API of the reference's ``triton_block_attn`` module, on B200.

``block_sparse_attn_v2`` keeps the reference's signature
(src/triton_block_attn.py:267-298) and runs libugbsa's sm_100a tcgen05 kernel
instead of Triton; ``block_sparse_attn`` is the v1 launcher (:150-181) with a
per-row keep mask, on the same kernel with its row mask.  K/V may carry fewer heads than Q (GQA, Hq % Hkv == 0); the
reference requires equal shapes after repeat_kv (:276), which still works.

``reference_attn`` is the reference's masked-SDPA checker (:301-312): a plain
PyTorch function kept for API compatibility and for users' own verification.
It is not on the product path.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops


def block_sparse_attn_v2(q, k, v, kv_idx, scale, block_n=64, block_m=64, num_warps=4, num_stages=1):
    """q [B,H,M,D], k/v [B,Hkv,N,D] bf16/fp16 CUDA; kv_idx [B,H,Q_tiles,MAX_KEPT] int32
    (sentinel = NB).  Returns [B,H,M,D].  ``num_warps``/``num_stages`` are accepted
    and ignored (the B200 kernel has a fixed warp-specialised schedule)."""
    if block_n != 64 or block_m != 64:
        raise ValueError("block_n and block_m are fixed at 64")
    return ops.block_sparse_attn(q, k, v, kv_idx, float(scale))


def block_sparse_attn(q, k, v, keep, scale, block_n=64, block_m=64, num_warps=4, num_stages=1):
    """The reference's v1 launcher (src/triton_block_attn.py:150-181): keep
    [B,H,M,NB] bool per query row; each tile attends to the union of its rows'
    blocks with every row masked to its own (triton_block_attn.py:87-104).
    q [B,H,M,D], k/v [B,Hkv,M,D] bf16 / fp16 CUDA.  Returns [B,H,M,D]."""
    if block_n != 64 or block_m != 64:
        raise ValueError("block_n and block_m are fixed at 64")
    bits, kv_idx = ops.keep_to_tiles(keep)
    return ops.block_sparse_attn_rows(q, k, v, kv_idx, bits, float(scale))


def reference_attn(q, k, v, keep, scale, block_n=64):
    """Masked SDPA with keep [B,H,M,NB] expanded to tokens and ANDed with causal."""
    B, H, M, D = q.shape
    N = k.shape[-2]
    NB = keep.shape[-1]
    kk = keep.unsqueeze(-1).expand(B, H, M, NB, block_n).reshape(B, H, M, NB * block_n)[..., :N]
    causal = torch.arange(N, device=q.device).view(1, N) <= torch.arange(M, device=q.device).view(M, 1)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=kk & causal, scale=scale)
