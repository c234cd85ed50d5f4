"""Qwen2-shaped decoder prefill, tensor-parallel over KV-head groups.

BASELINE configs 3 and 4 time a whole prefill of a random-init Qwen2.5-7B /
14B-shaped decoder with the block-sparse attention on every layer; the
reference does that through Hugging Face's Qwen2 modules with
``attn_implementation="block_sparse"`` (src/modal_app_profile.py:88-92,
129-132, the hook at src/sparse_attention.py:751-806).  This runner computes
the same per-layer math as transformers' Qwen2 decoder layer,

    x = RMSNorm(h);  q, k, v = x Wq + bq, x Wk + bk, x Wv + bv;  rotary(q, k)
    h = h + attention(q, k, v) Wo
    x = RMSNorm(h);  h = h + (silu(x Wg) * (x Wu)) Wd
    logits = RMSNorm(h) W_lm

with random-init weights of the same shapes, split Megatron-style over the
ranks of one node:

* column-parallel Q/K/V by KV-head groups (HeadShard: whole groups per rank;
  when the ranks outnumber the KV heads a group's Q heads are split and its
  K/V replicated), row-parallel o_proj, then one NCCL all-reduce of [S, hidden];
* column-parallel gate/up and row-parallel down_proj (intermediate split
  evenly), then one NCCL all-reduce;
* vocab-parallel lm_head (each rank returns its slice of the logits).

Per layer the attention is this package's path: the rotary kernel in place on
the fused QKV projection output (ugbsa_qk_norm_rope without a norm; it also
writes K's block summaries), the selection (the row-grain margin sums are
all-reduced over the ranks before the shared quantile, as the reference's
head mean couples all heads, :708-710) and the block-sparse attention kernel
writing straight into the o_proj input.  ``attention="dense"`` runs torch SDPA
instead (the dense denominator).  The projections and the MLP are cuBLAS GEMMs
through torch; RMSNorm and SwiGLU are torch element-wise ops.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from .parallel import HeadShard

BLOCK = 64


@dataclass(frozen=True)
class DecoderShape:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    rms_eps: float

    def gemm_flops(self, S: int) -> float:
        """2 * S * (weights of the linear layers, lm_head included)."""
        D, H, Hk = self.head_dim, self.heads, self.kv_heads
        per_layer = self.hidden * (H + 2 * Hk) * D + H * D * self.hidden + 3 * self.hidden * self.intermediate
        return 2.0 * S * (self.layers * per_layer + self.hidden * self.vocab)

    def dense_attn_flops(self, S: int) -> float:
        """Block-causal QK^T + PV over all layers (the dense-equivalent count)."""
        qt = math.ceil(S / BLOCK)
        return self.layers * self.heads * qt * (qt + 1) / 2 * 4 * BLOCK * BLOCK * self.head_dim


# BASELINE config 3 (Qwen2.5-7B geometry) and config 4 (Qwen2.5-14B geometry)
QWEN25_7B = DecoderShape(28, 3584, 28, 4, 128, 18944, 152064, 1.0e6, 1e-6)
QWEN25_14B = DecoderShape(48, 5120, 40, 8, 128, 13824, 152064, 1.0e6, 1e-5)


@dataclass(frozen=True)
class TPLayout:
    """What one rank of a tensor-parallel decoder holds."""
    shard: HeadShard
    inter0: int
    inter1: int
    vocab0: int
    vocab1: int

    @staticmethod
    def make(shape: DecoderShape, world: int, rank: int) -> "TPLayout":
        if shape.intermediate % world:
            raise ValueError(f"intermediate size {shape.intermediate} does not split over {world} ranks")
        shard = HeadShard.make(shape.heads, shape.kv_heads, world, rank)
        il = shape.intermediate // world
        vl = math.ceil(shape.vocab / world)
        return TPLayout(shard, rank * il, (rank + 1) * il, rank * vl, min(shape.vocab, (rank + 1) * vl))


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """transformers' Qwen2RMSNorm: w * T(x_fp32 * rsqrt(mean(x_fp32^2) + eps))."""
    xf = x.float()
    return w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


def rotary_tables(S: int, D: int, theta: float, device, dtype=torch.bfloat16):
    """cos / sin [1, S, D] as transformers' default rotary embedding computes them
    (fp32 angles, cast to the activation dtype)."""
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device=device, dtype=torch.int64).float() / D))
    pos = torch.arange(S, device=device, dtype=torch.float32)
    f = pos[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(dtype)[None], emb.sin().to(dtype)[None]


class TPDecoder:
    """A random-init Qwen2-shaped decoder on this rank (weights generated on the
    device from ``seed``; every rank draws the full weight matrices' values the
    same way and keeps its slice, so any world size computes the same model).

    forward(ids) -> this rank's logits slice [S, vocab1 - vocab0] (bf16)."""

    def __init__(self, shape: DecoderShape, sel: ops.SelectorConfig | None, world: int = 1, rank: int = 0,
                 group=None, attention: str = "block_sparse", seed: int = 0, device=None,
                 dtype=torch.bfloat16, mlp_chunk: int = 32768):
        if attention not in ("block_sparse", "dense"):
            raise ValueError("attention is 'block_sparse' or 'dense'")
        self.shape, self.sel, self.world, self.rank, self.group = shape, sel, world, rank, group
        self.attention = attention
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self.mlp_chunk = mlp_chunk
        self.layout = TPLayout.make(shape, world, rank)
        self.scale = shape.head_dim ** -0.5
        self.events = None   # optional per-layer CUDA events: list of (start, attn_start, attn_end, end)
        self.last_kv_idx = None
        L, sh = self.layout, self.layout.shard
        D, hid = shape.head_dim, shape.hidden
        gen = torch.Generator(device=self.device)

        def draw(rows, cols, key, std=0.02):
            # the full matrix's values for this key, so every world size gets the same model
            gen.manual_seed(seed * 1000003 + key)
            return (torch.randn((rows, cols), generator=gen, device=self.device, dtype=torch.float32) * std).to(dtype)

        self.embed = draw(shape.vocab, hid, 1)
        lm = draw(hid, shape.vocab, 2)
        self.lm_head = lm[:, L.vocab0:L.vocab1].contiguous()
        del lm
        self.final_norm = torch.ones(hid, device=self.device, dtype=dtype)
        self.layers = []
        qcols = slice(sh.q0 * D, sh.q1 * D)
        kcols = slice(sh.kv0 * D, sh.kv1 * D)
        for i in range(shape.layers):
            base = 100 + 10 * i
            wq, wk, wv = draw(hid, shape.heads * D, base), draw(hid, shape.kv_heads * D, base + 1), \
                draw(hid, shape.kv_heads * D, base + 2)
            bias = draw(1, (shape.heads + 2 * shape.kv_heads) * D, base + 3)[0]
            bq = bias[:shape.heads * D]
            bk = bias[shape.heads * D:(shape.heads + shape.kv_heads) * D]
            bv = bias[(shape.heads + shape.kv_heads) * D:]
            w_qkv = torch.cat([wq[:, qcols], wk[:, kcols], wv[:, kcols]], dim=1).contiguous()
            b_qkv = torch.cat([bq[qcols], bk[kcols], bv[kcols]]).contiguous()
            wo = draw(shape.heads * D, hid, base + 4)[qcols].contiguous()
            wg = draw(hid, shape.intermediate, base + 5)[:, L.inter0:L.inter1]
            wu = draw(hid, shape.intermediate, base + 6)[:, L.inter0:L.inter1]
            w_gu = torch.cat([wg, wu], dim=1).contiguous()
            wd = draw(shape.intermediate, hid, base + 7)[L.inter0:L.inter1].contiguous()
            del wq, wk, wv, wg, wu
            self.layers.append(dict(ln1=torch.ones(hid, device=self.device, dtype=dtype), w_qkv=w_qkv, b_qkv=b_qkv,
                                    w_o=wo, ln2=torch.ones(hid, device=self.device, dtype=dtype), w_gu=w_gu,
                                    w_down=wd))
        torch.cuda.empty_cache()

    # ------------------------------------------------------------------ pieces
    def _all_reduce(self, x):
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(x, group=self.group)

    def _select(self, q, k, summ):
        """kv_idx for this rank's heads; with several ranks the row-grain margin sums
        (or the cells) are combined over all ranks before the shared quantile."""
        cfg = self.sel
        if self.world == 1:
            return ops.select_kv_idx(q, k, self.scale, cfg, summ=summ)
        import torch.distributed as dist
        row = cfg.router_grain == "row"
        kv_idx, cells, rowsum = ops.select_tiles(q, summ, k.shape[1], self.scale, cfg, want_rowsum=row)
        if row:
            dist.all_reduce(rowsum, group=self.group)
            sigma_all = rowsum
        else:
            B, hl, Qt = cells.shape
            hmax = max(HeadShard.make(self.shape.heads, self.shape.kv_heads, self.world, r).hq_local
                       for r in range(self.world))
            pad = torch.full((B, hmax, Qt), float("nan"), device=cells.device, dtype=cells.dtype)
            pad[:, :hl] = cells
            g = torch.empty((self.world * B, hmax, Qt), device=cells.device, dtype=cells.dtype)
            dist.all_gather_into_tensor(g, pad, group=self.group)
            sigma_all = g.view(self.world, B, hmax, Qt).permute(1, 0, 2, 3).reshape(B, -1, Qt)
        return ops.select_finish(kv_idx, cells, sigma_all, self.shape.heads, q.shape[2], cfg)

    def _attention(self, x, lw, cos, sin):
        """x [S, hidden] (normed) -> attention output [S, hl * D] of this rank's heads."""
        S = x.shape[0]
        sh = self.layout.shard
        hl, hk, D = sh.hq_local, sh.hkv_local, self.shape.head_dim
        qkv = torch.addmm(lw["b_qkv"], x, lw["w_qkv"])                 # [S, (hl + 2 hk) D]
        v4 = qkv.view(1, S, hl + 2 * hk, D)
        q = v4[:, :, :hl].transpose(1, 2)                              # [1, hl, S, D] views, no copies
        k = v4[:, :, hl:hl + hk].transpose(1, 2)
        v = v4[:, :, hl + hk:].transpose(1, 2)
        out = torch.empty((S, hl * D), device=x.device, dtype=x.dtype)
        o4 = out.view(1, S, hl, D).transpose(1, 2)
        if self.attention == "dense":
            # the dense denominator: transformers' rotary (bit-identical to the kernel's)
            # and torch SDPA with GQA
            qr = ops.qk_norm_rope(q, None, 0.0, cos, sin, norm_mode="none", out=q)
            kr = ops.qk_norm_rope(k, None, 0.0, cos, sin, norm_mode="none", out=k)
            o4.copy_(F.scaled_dot_product_attention(qr, kr, v, is_causal=True, scale=self.scale,
                                                    enable_gqa=hl != hk))
            return out
        quest = self.sel.quest
        ops.qk_norm_rope(q, None, 0.0, cos, sin, norm_mode="none", out=q)
        _, summ = ops.qk_norm_rope(k, None, 0.0, cos, sin, norm_mode="none", out=k,
                                   summary="quest" if quest else "mean")
        kv_idx = self._select(q, k, summ)
        self.last_kv_idx = kv_idx
        ops.block_sparse_attn(q, k, v, kv_idx, self.scale, out=o4)
        return out

    def _mlp(self, x, lw):
        S = x.shape[0]
        il = self.layout.inter1 - self.layout.inter0
        out = torch.empty((S, self.shape.hidden), device=x.device, dtype=x.dtype)
        for r0 in range(0, S, self.mlp_chunk):
            r1 = min(S, r0 + self.mlp_chunk)
            gu = x[r0:r1] @ lw["w_gu"]
            a = F.silu(gu[:, :il]) * gu[:, il:]
            torch.mm(a, lw["w_down"], out=out[r0:r1])
        return out

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def layer(self, h: torch.Tensor, i: int, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """Decoder layer i on the residual stream h [S, hidden] (replicated on every rank)."""
        shape, lw = self.shape, self.layers[i]
        ev = self.events[i] if self.events is not None else None
        if ev is not None:
            ev[0].record()
        x = rms_norm(h, lw["ln1"], shape.rms_eps)
        if ev is not None:
            ev[1].record()
        a = self._attention(x, lw, cos, sin)
        if ev is not None:
            ev[2].record()
        o = a @ lw["w_o"]
        self._all_reduce(o)
        h = h + o
        x = rms_norm(h, lw["ln2"], shape.rms_eps)
        m = self._mlp(x, lw)
        self._all_reduce(m)
        h = h + m
        if ev is not None:
            ev[3].record()
        return h

    @torch.no_grad()
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        shape = self.shape
        S = ids.shape[0]
        cos, sin = rotary_tables(S, shape.head_dim, shape.rope_theta, ids.device, self.dtype)
        h = F.embedding(ids, self.embed)
        for i in range(shape.layers):
            h = self.layer(h, i, cos, sin)
        h = rms_norm(h, self.final_norm, shape.rms_eps)
        return h @ self.lm_head
