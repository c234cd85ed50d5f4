"""Head sharding of one attention layer across the GPUs of a node.

The reference is single-device (accelerate layer placement only,
src/modal_app_ruler.py:127-141).  Here a layer's heads are split over ranks,
one process per GPU, torch.distributed over NCCL:

* split: whole KV-head groups per rank when the rank count divides the KV head
  count (28/4 heads on 1, 2, 4 GPUs), otherwise each group's Q heads are split
  over world/Hkv ranks (28/4 on 8 GPUs: 4 + 3 Q heads, the group's K/V read by
  both ranks).  Every rank's Q heads lie in whole KV groups of its own slice.
* exchange 1 (the only cross-head coupling of the path): the row-grain sigma
  router averages the per-tile margin over ALL heads (src/sparse_attention.py:
  708-710) and takes one quantile over the layer (:711-718).  Each rank sums
  its heads' margins per tile ([B, Qt] fp32, 8 KB at 128K) and one SUM
  all-reduce gives every rank the same totals; the margins are subnormal, so
  the sums are exact in any order and the threshold is bit-identical on every
  rank (cell grain: the [B, Hq, Qt] margins are all-gathered instead).
* exchange 2: the per-rank outputs [B, Hq_local, S, D] are all-gathered into
  the [B, S, Hq, D] layer output.

Sequence sharding (SeqShard, SeqShardedPrefill) splits the query rows instead:
every rank holds all heads for a contiguous, tile-pair-aligned range of rows,
the ranges balanced by an estimate of each tile's cost (causal scoring grows
with the tile index, attention with min(tile + 1, budget)), so uneven head
counts (28 Q heads over 8 ranks) leave no rank idle.  Exchanges: the ranks'
K/V rows are all-gathered (every tile's attention reads all earlier keys);
the per-tile margins are gathered so that every rank takes the layer's one
quantile over all tiles; the output rows are all-gathered into [B, S, Hq, D].
Each rank's results equal the unsplit computation's rows bit for bit.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import ops

def pipelined_e2e(host_inputs, compute, out_shape, out_dtype, steps: int, warmup: int = 2, slots: int = 3):
    """Time `steps` end-to-end steps: each step copies `host_inputs` (pinned) to
    the device, runs compute(device_inputs) -> device output on the current
    stream, and copies the output back to pinned host memory.

    Two measurements: serial (copy in, compute, copy out, one step after the
    other on one stream) and pipelined (three streams, `slots` device input and
    host output buffers in rotation: the copy-in of step i+1 and the copy-out of
    step i-1 run while step i computes, as consecutive requests are served).  The
    pipelined figure is the throughput; every step still moves all its bytes
    inside the timed region.  Returns {"ms": pipelined, "serial_ms": serial}."""
    dev = torch.device("cuda", torch.cuda.current_device())
    cmp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    d_in = [[torch.empty_like(x, device=dev) for x in host_inputs] for _ in range(slots)]
    h_out = [torch.empty(out_shape, dtype=out_dtype).pin_memory() for _ in range(slots)]
    ev_in = [torch.cuda.Event() for _ in range(slots)]
    ev_done = [torch.cuda.Event() for _ in range(slots)]
    ev_out = [torch.cuda.Event() for _ in range(slots)]
    used = [False] * slots

    def serial_one():
        for d, h in zip(d_in[0], host_inputs):
            d.copy_(h, non_blocking=True)
        out = compute(d_in[0])
        h_out[0].copy_(out, non_blocking=True)

    def piped_one(i):
        k = i % slots
        with torch.cuda.stream(h2d):
            if used[k]:
                h2d.wait_event(ev_done[k])          # step i-2 has finished reading these inputs
            for d, h in zip(d_in[k], host_inputs):
                d.copy_(h, non_blocking=True)
            ev_in[k].record(h2d)
        cmp.wait_event(ev_in[k])
        if used[k]:
            cmp.wait_event(ev_out[k])               # step i-2's output has left for the host
        out = compute(d_in[k])
        ev_done[k].record(cmp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev_done[k])
            h_out[k].copy_(out, non_blocking=True)
            out.record_stream(d2h)
            ev_out[k].record(d2h)
        used[k] = True

    def timed(fn):
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(cmp)
        h2d.wait_stream(cmp)
        d2h.wait_stream(cmp)
        for i in range(steps):
            fn(i)
        cmp.wait_stream(h2d)
        cmp.wait_stream(d2h)
        e.record(cmp)
        torch.cuda.synchronize()
        return s.elapsed_time(e) / steps

    for _ in range(warmup):
        serial_one()
    serial = timed(lambda i: serial_one())
    for i in range(warmup):
        piped_one(i)
    torch.cuda.synchronize()
    piped = timed(lambda i: piped_one(i + warmup))
    return {"ms": piped, "serial_ms": serial}


class _DeviceArray:
    """__cuda_array_interface__ of a raw byte range (so torch can wrap it without a copy)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    """A [shape] device buffer on every rank of the group, each rank mapping the
    others' (CUDA IPC through libugbsa): a kernel given peer_views() writes its
    results into the other GPUs' copies over NVLink."""

    def __init__(self, shape, dtype: torch.dtype, device: torch.device, group=None):
        import ctypes

        import torch.distributed as dist

        from . import _lib
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        nbytes = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
        L = _lib.load()
        ptr = ctypes.c_void_p()
        h = _lib.IpcHandle()
        with torch.cuda.device(device):
            _lib.check(L.ugbsa_peer_buffer_alloc(nbytes, ctypes.byref(ptr), ctypes.byref(h)), "ugbsa_peer_buffer_alloc")
        self.ptr = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h.bytes), group=group)
        self.peer_base = {}
        with torch.cuda.device(device):
            for r, hb in enumerate(handles):
                if r == self.rank:
                    continue
                hr = _lib.IpcHandle()
                ctypes.memmove(ctypes.addressof(hr), hb, 64)
                pp = ctypes.c_void_p()
                _lib.check(L.ugbsa_peer_buffer_open(ctypes.byref(hr), ctypes.byref(pp)), "ugbsa_peer_buffer_open")
                self.peer_base[r] = pp.value
        raw = torch.as_tensor(_DeviceArray(self.ptr, nbytes), device=device)
        self.tensor = raw.view(dtype).view(*shape)
        self.nbytes = nbytes

    def peer_views(self, view: torch.Tensor):
        """Addresses of `view` (a view of self.tensor) in every other rank's buffer."""
        off = view.data_ptr() - self.ptr
        if not (0 <= off < self.nbytes):
            raise ValueError("view does not lie in this buffer")
        return [self.peer_base[r] + off for r in sorted(self.peer_base)]

    def close(self):
        """Collective: unmap the peers' buffers, then free this rank's once nobody maps it."""
        import torch.distributed as dist

        from . import _lib
        if self.ptr is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        L = _lib.load()
        for p in self.peer_base.values():
            L.ugbsa_peer_buffer_close(p)
        self.peer_base = {}
        self.tensor = None
        dist.barrier(group=self.group)
        L.ugbsa_peer_buffer_free(self.ptr)
        self.ptr = None


def launches_per_step(cfg: ops.SelectorConfig, k_base: int, kmax: int, tensor_core: bool = True) -> int:
    """libugbsa kernel launches per layer step: block summary; tile selection
    (tensor-core path: operand conversion, scoring, ranking; otherwise one
    kernel); [per-tile sigma row sum: router, row grain]; [quantile: router];
    [finalize: router]; attention."""
    router = cfg.mode == "router" and k_base < kmax
    n = 2 + (3 if tensor_core else 1)
    if router:
        n += 2 + (1 if cfg.router_grain == "row" else 0)
    return n


@dataclass(frozen=True)
class HeadShard:
    Hq: int
    Hkv: int
    world: int
    rank: int
    q0: int
    q1: int
    kv0: int
    kv1: int

    @staticmethod
    def make(Hq: int, Hkv: int, world: int, rank: int) -> "HeadShard":
        if Hq % Hkv:
            raise ValueError("Hq must be a multiple of Hkv")
        G = Hq // Hkv
        if world == 1:
            return HeadShard(Hq, Hkv, 1, 0, 0, Hq, 0, Hkv)
        if Hkv % world == 0:
            per = Hkv // world
            kv0, kv1 = rank * per, (rank + 1) * per
            return HeadShard(Hq, Hkv, world, rank, kv0 * G, kv1 * G, kv0, kv1)
        if world % Hkv == 0:
            parts = world // Hkv
            if parts > G:
                raise ValueError(f"{world} ranks exceed the {Hq} Q heads")
            kv = rank // parts
            j = rank % parts
            sizes = [G // parts + (1 if i < G % parts else 0) for i in range(parts)]
            start = kv * G + sum(sizes[:j])
            return HeadShard(Hq, Hkv, world, rank, start, start + sizes[j], kv, kv + 1)
        raise ValueError(f"cannot shard {Hq}/{Hkv} heads over {world} ranks along KV groups")

    @property
    def hq_local(self) -> int:
        return self.q1 - self.q0

    @property
    def hkv_local(self) -> int:
        return self.kv1 - self.kv0

    def slice(self, q, k, v):
        return q[:, self.q0:self.q1], k[:, self.kv0:self.kv1], v[:, self.kv0:self.kv1]


def all_shards(Hq: int, Hkv: int, world: int):
    return [HeadShard.make(Hq, Hkv, world, r) for r in range(world)]


class _PeerOutput:
    """Output all-gather done by the attention kernel: a [B, S, Hq, D] PeerBuffer
    on every rank; each rank's kernel writes its tiles into all ranks' copies,
    then one small all-reduce orders the step's end after every rank's writes.
    The attention launch itself follows the step's margin exchange, so no rank
    writes into a buffer whose previous contents a peer is still reading (as
    long as that reading is ordered before its next step on its stream).  The
    returned output is this persistent buffer: the next step overwrites it."""

    MAX_RANKS = 8   # this GPU and UGBSA_MAX_PEERS = 7 peers per attention launch (one node)

    def _setup_peer(self, peer_output, world):
        import torch.distributed as dist
        if peer_output is None:
            peer_output = (1 < world <= self.MAX_RANKS and dist.is_initialized()
                           and dist.get_backend(self.group) == "nccl")
        if peer_output and world > self.MAX_RANKS:
            raise ValueError(f"peer output reaches at most {self.MAX_RANKS} ranks (one node), got {world}")
        self.peer_output = bool(peer_output)
        self._peer = None
        self._flag = None

    def _peer_buffer(self, shape, dtype, device):
        if self._peer is None or tuple(self._peer.tensor.shape) != tuple(shape) or self._peer.tensor.dtype != dtype:
            if self._peer is not None:
                self._peer.close()
            self._peer = PeerBuffer(shape, dtype, device, self.group)
            self._flag = torch.zeros(1, device=device, dtype=torch.int32)
        return self._peer

    def _peer_done(self):
        import torch.distributed as dist
        dist.all_reduce(self._flag, group=self.group)

    def _close_peer(self):
        if self._peer is not None:
            self._peer.close()
            self._peer = None


class ShardedPrefill(_PeerOutput):
    """One layer's prefill (summary, selection, attention) on this rank's heads.

    peer_output (default: on with NCCL and several ranks): the attention kernel
    writes each output tile into every rank's [B, S, Hq, D] buffer over NVLink
    instead of an all-gather after it."""

    def __init__(self, shard: HeadShard, cfg: ops.SelectorConfig, scale: float, group=None, peer_output=None):
        self.shard = shard
        self.cfg = cfg
        self.scale = float(scale)
        self.group = group
        self.last_kv_idx = None
        self._setup_peer(peer_output, shard.world)
        shards = all_shards(shard.Hq, shard.Hkv, shard.world)
        self.hq_max = max(s.hq_local for s in shards)
        self.even = all(s.hq_local == self.hq_max for s in shards)
        # bytes of Q/K/V and of the output over all ranks (for the end-to-end accounting)
        self._qkv_heads = sum(s.hq_local + 2 * s.hkv_local for s in shards)

    def select(self, q, k):
        if self.shard.world == 1:
            return ops.select_kv_idx(q, k, self.scale, self.cfg)
        import torch.distributed as dist
        summ = ops.block_summary(k, self.cfg.quest)
        row = self.cfg.router_grain == "row"
        kv_idx, cells, rowsum = ops.select_tiles(q, summ, k.shape[1], self.scale, self.cfg, want_rowsum=row)
        if row:
            dist.all_reduce(rowsum, op=dist.ReduceOp.SUM, group=self.group)
            sigma_all = rowsum
        else:
            B, hl, Qt = cells.shape
            pad = torch.full((B, self.hq_max, Qt), float("nan"), device=cells.device, dtype=cells.dtype)
            pad[:, :hl] = cells
            gathered = torch.empty((self.shard.world * B, self.hq_max, Qt), device=cells.device, dtype=cells.dtype)
            dist.all_gather_into_tensor(gathered, pad, group=self.group)
            sigma_all = gathered.view(self.shard.world, B, self.hq_max, Qt).permute(1, 0, 2, 3).reshape(B, -1, Qt)
        return ops.select_finish(kv_idx, cells, sigma_all, self.shard.Hq, q.shape[2], self.cfg)

    def step(self, q, k, v, events=None, gather=True):
        """q/k/v: this rank's head slices.  Returns the layer output as a [B, S, Hq, D]
        tensor (gathered over ranks; with several ranks a view of head-major storage)
        or, with gather=False, this rank's heads [B, Hq_local, S, D]."""
        if events is not None:
            events[0].record()
        kv_idx = self.select(q, k)
        self.last_kv_idx = kv_idx
        if events is not None:
            events[1].record()
        B, hl, S, D = q.shape
        if self.shard.world == 1:
            out = torch.empty((B, S, hl, D), device=q.device, dtype=q.dtype)
            ops.block_sparse_attn(q, k, v, kv_idx, self.scale, out=out.transpose(1, 2))
            if events is not None:
                events[2].record()
            return out
        if gather and self.peer_output:
            sh = self.shard
            buf = self._peer_buffer((B, S, sh.Hq, D), q.dtype, q.device)
            local = buf.tensor[:, :, sh.q0:sh.q1].transpose(1, 2)     # [B, hl, S, D] view of [B, S, Hq, D]
            ops.block_sparse_attn(q, k, v, kv_idx, self.scale, out=local, peer_out=buf.peer_views(local))
            if events is not None:
                events[2].record()
            self._peer_done()
            return buf.tensor
        # head-major output: rank r's heads are contiguous, in rank order (HeadShard)
        local = torch.empty((B, self.hq_max, S, D), device=q.device, dtype=q.dtype)
        ops.block_sparse_attn(q, k, v, kv_idx, self.scale, out=local[:, :hl])
        if events is not None:
            events[2].record()
        if not gather:
            return local[:, :hl]
        import torch.distributed as dist
        world, Hq = self.shard.world, self.shard.Hq
        full = torch.empty((world * B, self.hq_max, S, D), device=q.device, dtype=q.dtype)
        dist.all_gather_into_tensor(full, local, group=self.group)
        if B == 1 and self.even:
            return full.view(1, Hq, S, D).transpose(1, 2)     # the gather already is [B, Hq, S, D]
        fullv = full.view(world, B, self.hq_max, S, D)
        out = torch.empty((B, Hq, S, D), device=q.device, dtype=q.dtype)
        for r, s in enumerate(all_shards(Hq, self.shard.Hkv, world)):
            out[:, s.q0:s.q1].copy_(fullv[r, :, :s.hq_local])   # padding heads dropped
        return out.transpose(1, 2)

    def time_e2e(self, q, k, v, steps: int, warmup: int = 2):
        """End to end through the public API: this rank's Q/K/V copied from pinned
        host memory every step, the output read back to pinned host memory.
        One GPU: the Hugging Face hook ugbsa.sparse_attention.block_sparse_attention.
        Several GPUs: ShardedPrefill.step; each rank reads back its own heads (the
        layer's output is head-sharded, as for a row-parallel output projection).
        Timed serially and pipelined over consecutive steps (pipelined_e2e).
        Byte counts are over all ranks."""
        from . import sparse_attention as sa

        hq, hk, hv = (x.contiguous().cpu().pin_memory() for x in (q, k, v))
        B, hl, S, D = q.shape
        out_shape = (B, S, hl, D) if self.shard.world == 1 else (B, hl, S, D)

        class _Module:
            layer_idx = 0
            num_key_value_groups = hl // k.shape[1]

        mod = _Module()

        def compute(d):
            if self.shard.world == 1:
                out, _ = sa.block_sparse_attention(mod, d[0], d[1], d[2], None, self.scale)
                return out
            return self.step(d[0], d[1], d[2], gather=False)

        t = pipelined_e2e([hq, hk, hv], compute, out_shape, q.dtype, steps, warmup)
        c = pipelined_e2e([hq, hk, hv], lambda d: torch.empty(out_shape, device=q.device, dtype=q.dtype),
                          out_shape, q.dtype, steps, warmup)
        per_head = B * S * D * q.element_size()
        if self.shard.world == 1:
            h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
            d2h = math.prod(out_shape) * q.element_size()
        else:
            h2d = self._qkv_heads * per_head
            d2h = self.shard.Hq * per_head
        return {"ms": t["ms"], "serial_ms": t["serial_ms"], "h2d": h2d, "d2h": d2h, "copy_only_ms": c["ms"]}

    def close(self):
        """Collective when peer output was used (releases the peer buffers)."""
        self._close_peer()


# ------------------------------------------------------------------ sequence sharding
# Relative cost of one (tile, block) unit of attention against one unit of
# causal scoring: attention ~76 ns per block of a 64-row tile over 28 heads,
# exact scoring ~3.1 ns per visible block (128K tokens, head_dim 128, one B200),
# and a fixed per-tile attention overhead of about three blocks.
ATTN_UNIT_COST = 24.0
ATTN_TILE_OVERHEAD = 3.0


def tile_costs(S: int, k_base: int, kmax: int, frac_boosted: float = 0.25):
    """Estimated cost of each query tile: scoring over its t + 1 visible blocks
    plus attention over min(t + 1, budget) blocks, the budget kmax for the
    router's boosted share of tiles and k_base for the rest."""
    import numpy as np
    qt = math.ceil(S / 64)
    vis = np.arange(1, qt + 1, dtype=np.float64)
    attn = (1.0 - frac_boosted) * np.minimum(vis, k_base) + frac_boosted * np.minimum(vis, kmax)
    return vis + ATTN_UNIT_COST * (attn + ATTN_TILE_OVERHEAD)


def balanced_tile_ranges(costs, world: int):
    """Split tiles 0 .. len(costs) - 1 into `world` contiguous ranges of nearly
    equal total cost, every boundary on an even tile (the scorer's tile pairs).
    Returns [(t0, t1), ...] in rank order."""
    import numpy as np
    qt = len(costs)
    npairs = (qt + 1) // 2
    if npairs < world:
        raise ValueError(f"{qt} query tiles cannot give each of {world} ranks a tile pair")
    pair_cost = np.add.reduceat(np.asarray(costs, dtype=np.float64), np.arange(0, qt, 2))
    cum = np.concatenate([[0.0], np.cumsum(pair_cost)])
    total = cum[-1]
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        j = int(np.searchsorted(cum, target))          # first pair boundary with cum >= target
        if j > 0 and target - cum[j - 1] < cum[j] - target:
            j -= 1
        j = max(j, bounds[-1] + 1)                      # at least one pair per rank
        j = min(j, npairs - (world - r))
        bounds.append(j)
    bounds.append(npairs)
    return [(2 * bounds[r], min(2 * bounds[r + 1], qt)) for r in range(world)]


@dataclass(frozen=True)
class SeqShard:
    """This rank's query rows: tiles t0 .. t1 - 1 (rows row0 .. row1 - 1) of S."""
    S: int
    world: int
    rank: int
    t0: int
    t1: int

    @staticmethod
    def make(S: int, world: int, rank: int, cfg: ops.SelectorConfig) -> "SeqShard":
        return all_seq_shards(S, world, cfg)[rank]

    @property
    def row0(self) -> int:
        return self.t0 * 64

    @property
    def row1(self) -> int:
        return min(self.t1 * 64, self.S)

    @property
    def rows(self) -> int:
        return self.row1 - self.row0


def all_seq_shards(S: int, world: int, cfg: ops.SelectorConfig):
    k_base, kmax = ops.budget(cfg, S)
    frac = cfg.router_quantile if (cfg.mode == "router" and cfg.router_mode == "quantile" and k_base < kmax) else 0.0
    ranges = balanced_tile_ranges(tile_costs(S, k_base, kmax, frac), world)
    return [SeqShard(S, world, r, a, b) for r, (a, b) in enumerate(ranges)]


def _gather_rows(local: torch.Tensor, full: torch.Tensor, dim: int, spans, group=None):
    """All-gather rank r's `local` (full.narrow(dim, *spans[r]) of every rank) into
    `full`.  NCCL with contiguous destinations: one uneven all-gather straight
    into place; otherwise a padded all-gather and per-rank copies."""
    import torch.distributed as dist
    world = len(spans)
    views = [full.narrow(dim, a, n) for a, n in spans]
    if dist.get_backend(group) == "nccl" and all(v.is_contiguous() for v in views):
        dist.all_gather(views, local.contiguous(), group=group)
        return full
    nmax = max(n for _, n in spans)
    shape = list(local.shape)
    shape[dim] = nmax
    pad = local.new_zeros(shape)
    pad.narrow(dim, 0, local.shape[dim]).copy_(local)
    out = local.new_empty([world] + shape)
    dist.all_gather_into_tensor(out, pad.unsqueeze(0), group=group)
    for r, (a, n) in enumerate(spans):
        views[r].copy_(out[r].narrow(dim, 0, n))
    return full


class SeqShardedPrefill(_PeerOutput):
    """One layer's prefill on this rank's query rows (all heads).

    step() takes this rank's rows of Q, K and V as [B, rows, H, D] tensors (the
    layout of a projection's output before the head transpose), all-gathers K
    and V, selects and attends for its rows and all-gathers the output rows
    into [B, S, Hq, D] (gather=False: this rank's rows only)."""

    def __init__(self, S: int, Hq: int, Hkv: int, D: int, cfg: ops.SelectorConfig, scale: float, world: int,
                 rank: int, group=None, peer_output=None):
        self.S, self.Hq, self.Hkv, self.D = S, Hq, Hkv, D
        self.cfg = cfg
        self.scale = float(scale)
        self.group = group
        self.shards = all_seq_shards(S, world, cfg)
        self.shard = self.shards[rank]
        self.world, self.rank = world, rank
        self.last_kv_idx = None
        self.row_spans = [(s.row0, s.rows) for s in self.shards]
        self.tile_spans = [(s.t0, s.t1 - s.t0) for s in self.shards]
        self._setup_peer(peer_output, world)

    def exchange_margins(self, cells: torch.Tensor, rowsum):
        """sigma_all for ugbsa_select_finish_rows: row grain, the [B, Qt] head sums in
        tile order; cell grain, every rank's [B, Hq, Qt_r] cells in rank order
        (the quantile ignores positions)."""
        B = cells.shape[0]
        nb = math.ceil(self.S / 64)
        if self.cfg.router_grain == "row":
            full = torch.empty((B, nb), device=cells.device, dtype=torch.float32)
            return _gather_rows(rowsum, full, 1, self.tile_spans, self.group)
        counts = [B * self.Hq * n for _, n in self.tile_spans]
        offs = [sum(counts[:r]) for r in range(self.world)]
        full = torch.empty((sum(counts),), device=cells.device, dtype=torch.float32)
        return _gather_rows(cells.reshape(-1), full, 0, list(zip(offs, counts)), self.group)

    def select(self, q, k):
        """q: [B, Hq, rows, D] view of this rank's rows; k: [B, Hkv, S, D] all keys."""
        summ = ops.block_summary(k, self.cfg.quest)
        row = self.cfg.router_grain == "row"
        sh = self.shard
        kv_idx, cells, rowsum = ops.select_tiles(q, summ, self.Hkv, self.scale, self.cfg, want_rowsum=row,
                                                 row_base=sh.row0, seq_len=self.S)
        sigma_all = self.exchange_margins(cells, rowsum)
        return ops.select_finish(kv_idx, cells, sigma_all, self.Hq, self.S, self.cfg, row_base=sh.row0)

    def gather_kv(self, k_rows, v_rows):
        B = k_rows.shape[0]
        kf = torch.empty((B, self.S, self.Hkv, self.D), device=k_rows.device, dtype=k_rows.dtype)
        vf = torch.empty_like(kf)
        _gather_rows(k_rows, kf, 1, self.row_spans, self.group)
        _gather_rows(v_rows, vf, 1, self.row_spans, self.group)
        return kf, vf

    def step(self, q_rows, k_rows, v_rows, events=None, gather=True):
        """q_rows [B, rows, Hq, D], k_rows / v_rows [B, rows, Hkv, D]: this rank's rows.
        Returns the layer output [B, S, Hq, D] (gather=False: [B, rows, Hq, D])."""
        if events is not None:
            events[0].record()
        kf, vf = self.gather_kv(k_rows, v_rows)
        q = q_rows.transpose(1, 2)
        k, v = kf.transpose(1, 2), vf.transpose(1, 2)
        kv_idx = self.select(q, k)
        self.last_kv_idx = kv_idx
        if events is not None:
            events[1].record()
        B = q_rows.shape[0]
        sh = self.shard
        if gather and self.peer_output:
            buf = self._peer_buffer((B, self.S, self.Hq, self.D), q_rows.dtype, q_rows.device)
            local = buf.tensor.narrow(1, sh.row0, sh.rows).transpose(1, 2)
            ops.block_sparse_attn(q, k, v, kv_idx, self.scale, out=local, row_base=sh.row0,
                                  peer_out=buf.peer_views(local))
            if events is not None:
                events[2].record()
            self._peer_done()
            return buf.tensor
        if gather:
            out = torch.empty((B, self.S, self.Hq, self.D), device=q_rows.device, dtype=q_rows.dtype)
            local = out.narrow(1, sh.row0, sh.rows)
        else:
            out = local = torch.empty((B, sh.rows, self.Hq, self.D), device=q_rows.device, dtype=q_rows.dtype)
        ops.block_sparse_attn(q, k, v, kv_idx, self.scale, out=local.transpose(1, 2), row_base=sh.row0)
        if events is not None:
            events[2].record()
        if gather:
            if local.is_contiguous():
                _gather_rows(local, out, 1, self.row_spans, self.group)
            else:
                _gather_rows(local.contiguous(), out, 1, self.row_spans, self.group)
        return out

    def time_e2e(self, q_rows, k_rows, v_rows, steps: int, warmup: int = 2):
        """End to end: this rank's rows of Q/K/V copied from pinned host memory
        every step, its output rows read back to pinned host memory (the layer
        output stays row-sharded, as for a sequence-parallel output
        projection); serial and pipelined (pipelined_e2e).  Byte counts are
        over all ranks."""
        hq, hk, hv = (x.contiguous().cpu().pin_memory() for x in (q_rows, k_rows, v_rows))
        t = pipelined_e2e([hq, hk, hv], lambda d: self.step(d[0], d[1], d[2], gather=False),
                          tuple(q_rows.shape), q_rows.dtype, steps, warmup)
        B, el = q_rows.shape[0], q_rows.element_size()
        per_row = B * self.D * el
        return {"ms": t["ms"], "serial_ms": t["serial_ms"], "h2d": self.S * (self.Hq + 2 * self.Hkv) * per_row,
                "d2h": self.S * self.Hq * per_row}

    def close(self):
        """Collective when peer output was used (releases the peer buffers)."""
        self._close_peer()


# ------------------------------------------------------------------ KV groups x dealt tile pairs
@dataclass(frozen=True)
class GridShard:
    """Rank `rank` of world = (KV head groups) x m: KV heads kv0 .. kv1 - 1 with
    their Q heads, and the query tile pairs j, j + m, j + 2m, ... (j = rank % m)
    of the whole sequence.  Dealing pairs round-robin gives the m ranks of a
    group the same mix of early (cheap) and late (expensive) causal tiles, for
    the scoring and the attention stage alike."""
    Hq: int
    Hkv: int
    world: int
    rank: int
    m: int
    j: int
    kv0: int
    kv1: int

    @staticmethod
    def make(Hq: int, Hkv: int, world: int, rank: int) -> "GridShard":
        if Hq % Hkv:
            raise ValueError("Hq must be a multiple of Hkv")
        if Hkv % world == 0:
            per, m = Hkv // world, 1
            kv0 = rank * per
            return GridShard(Hq, Hkv, world, rank, 1, 0, kv0, kv0 + per)
        if world % Hkv == 0:
            m = world // Hkv
            g = rank // m
            return GridShard(Hq, Hkv, world, rank, m, rank % m, g, g + 1)
        raise ValueError(f"{world} ranks neither divide nor are a multiple of {Hkv} KV heads")

    @property
    def q0(self) -> int:
        return self.kv0 * (self.Hq // self.Hkv)

    @property
    def q1(self) -> int:
        return self.kv1 * (self.Hq // self.Hkv)

    @property
    def row_base(self) -> int:
        return 128 * self.j

    def tiles(self, S: int):
        """Sequence tiles of this rank, in local order."""
        nb = math.ceil(S / 64)
        out = []
        p = self.j
        while 2 * p < nb:
            out.extend(t for t in (2 * p, 2 * p + 1) if t < nb)
            p += self.m
        return out

    def rows(self, S: int):
        """Sequence rows of this rank, in local order (a LongTensor index)."""
        idx = [torch.arange(64 * t, min(64 * t + 64, S)) for t in self.tiles(S)]
        return torch.cat(idx) if idx else torch.empty(0, dtype=torch.long)

    def slice(self, q, k, v):
        """This rank's inputs from full [B, H, S, D] tensors: its Q heads' dealt rows,
        its KV heads' full sequence."""
        S = q.shape[2]
        qh = q[:, self.q0:self.q1]
        if self.m > 1:
            qh = qh.index_select(2, self.rows(S).to(q.device))
        return qh, k[:, self.kv0:self.kv1], v[:, self.kv0:self.kv1]


class GridShardedPrefill(_PeerOutput):
    """One layer's prefill on a GridShard: scoring, ranking and attention for the
    shard's Q heads over its dealt query tiles.  Exchanges: the per-tile margin
    sums (row grain; a full-length vector per rank, zero outside its tiles, one
    SUM all-reduce) or the margins themselves (cell grain, an all-gather), then
    the output, which the attention kernel writes into every rank's
    [B, S, Hq, D] buffer (peer_output; required when tiles are dealt)."""

    def __init__(self, shard: GridShard, S: int, cfg: ops.SelectorConfig, scale: float, group=None,
                 peer_output=None):
        self.shard = shard
        self.S = S
        self.cfg = cfg
        self.scale = float(scale)
        self.group = group
        self.last_kv_idx = None
        self._setup_peer(peer_output, shard.world)
        self.tiles = torch.tensor(shard.tiles(S), dtype=torch.long)
        shards = [GridShard.make(shard.Hq, shard.Hkv, shard.world, r) for r in range(shard.world)]
        G = shard.Hq // shard.Hkv
        nb = math.ceil(S / 64)
        # cell-grain gather: rank r contributes B * (its Q heads) * (its tiles) cells
        self._cell_counts = [(s.kv1 - s.kv0) * G * len(s.tiles(S)) for s in shards]
        self._nb = nb
        self._tiles_dev = None
        # the m ranks that share a KV group (for the end-to-end path: each copies 1/m of
        # the group's K / V rows from the host and the group all-gathers them over NVLink);
        # every rank creates every group, in the same order
        self._kv_group = None
        if shard.world > 1 and shard.m > 1 and group is not None:
            import torch.distributed as dist
            for g in range(shard.world // shard.m):
                pg = dist.new_group(list(range(g * shard.m, (g + 1) * shard.m)))
                if g == shard.rank // shard.m:
                    self._kv_group = pg

    def exchange_margins(self, cells: torch.Tensor, rowsum):
        import torch.distributed as dist
        B = cells.shape[0]
        if self.shard.world == 1:
            return rowsum if self.cfg.router_grain == "row" else cells
        if self.cfg.router_grain == "row":
            if self._tiles_dev is None or self._tiles_dev.device != rowsum.device:
                self._tiles_dev = self.tiles.to(rowsum.device)
            full = torch.zeros((B, self._nb), device=rowsum.device, dtype=torch.float32)
            full.index_copy_(1, self._tiles_dev, rowsum)
            dist.all_reduce(full, op=dist.ReduceOp.SUM, group=self.group)   # margins subnormal: exact sums
            return full
        counts = [B * c for c in self._cell_counts]
        offs = [sum(counts[:r]) for r in range(len(counts))]
        full = torch.empty((sum(counts),), device=cells.device, dtype=torch.float32)
        return _gather_rows(cells.reshape(-1), full, 0, list(zip(offs, counts)), self.group)

    def select(self, q, k):
        sh = self.shard
        summ = ops.block_summary(k, self.cfg.quest)
        row = self.cfg.router_grain == "row"
        kv_idx, cells, rowsum = ops.select_tiles(q, summ, k.shape[1], self.scale, self.cfg, want_rowsum=row,
                                                 row_base=sh.row_base, seq_len=self.S, pair_stride=sh.m)
        sigma_all = self.exchange_margins(cells, rowsum)
        return ops.select_finish(kv_idx, cells, sigma_all, sh.Hq, self.S, self.cfg, row_base=sh.row_base,
                                 pair_stride=sh.m)

    def step(self, q, k, v, events=None, gather=True):
        """q [B, Hq_local, rows, D] (this rank's heads and dealt rows, GridShard.slice),
        k / v [B, Hkv_local, S, D].  Returns the layer output [B, S, Hq, D]; with
        gather=False this rank's heads [B, Hq_local, S, D] of which only its rows
        are written (pair_stride 1: all rows)."""
        if events is not None:
            events[0].record()
        kv_idx = self.select(q, k)
        self.last_kv_idx = kv_idx
        if events is not None:
            events[1].record()
        sh = self.shard
        B, hl, _, D = q.shape
        if gather and self.shard.world > 1:
            if not self.peer_output:
                raise RuntimeError("GridShardedPrefill gathers its output through peer buffers (NCCL ranks)")
            buf = self._peer_buffer((B, self.S, sh.Hq, D), q.dtype, q.device)
            local = buf.tensor[:, :, sh.q0:sh.q1].transpose(1, 2)
            ops.block_sparse_attn(q, k, v, kv_idx, self.scale, out=local, row_base=sh.row_base,
                                  pair_stride=sh.m, peer_out=buf.peer_views(local))
            if events is not None:
                events[2].record()
            self._peer_done()
            return buf.tensor
        out = torch.empty((B, hl, self.S, D), device=q.device, dtype=q.dtype)
        ops.block_sparse_attn(q, k, v, kv_idx, self.scale, out=out, row_base=sh.row_base, pair_stride=sh.m)
        if events is not None:
            events[2].record()
        return out.transpose(1, 2) if self.shard.world == 1 else out

    def _split_kv(self, S: int) -> bool:
        return self._kv_group is not None and S % self.shard.m == 0

    def gather_kv_rows(self, k_part, v_part):
        """K / V row blocks of this rank's KV heads (rows j*S/m .. (j+1)*S/m - 1 on rank j
        of the group) -> the whole sequence on every rank of the group (NCCL all-gather
        over NVLink)."""
        import torch.distributed as dist
        m = self.shard.m
        outs = []
        for x in (k_part, v_part):
            B, hk, r, D = x.shape
            full = torch.empty((m * B * hk, r, D), device=x.device, dtype=x.dtype)
            dist.all_gather_into_tensor(full, x.reshape(B * hk, r, D).contiguous(), group=self._kv_group)
            full = full.view(m, B, hk, r, D).permute(1, 2, 0, 3, 4).reshape(B, hk, m * r, D)
            outs.append(full)
        return outs

    def time_e2e(self, q, k, v, steps: int, warmup: int = 2):
        """End to end through the runner's public step(): every step this rank copies
        from pinned host memory its Q rows and its share of its KV heads' rows (with m
        ranks per KV group each copies 1/m of the group's K / V and the group
        all-gathers them over NVLink, so every K / V byte crosses PCIe once), runs the
        layer with the output gathered on every rank (gather=True), and reads back its
        1/world slice of the [B, S, Hq, D] output rows (the job reads the output once).
        Serial and pipelined (pipelined_e2e), plus the copy-only time of the same bytes
        (the host-link ceiling).  Byte counts are over all ranks."""
        sh = self.shard
        world = sh.world
        split = self._split_kv(self.S)
        hq = q.contiguous().cpu().pin_memory()
        if split:
            r = self.S // sh.m
            hk = k[:, :, sh.j * r:(sh.j + 1) * r].contiguous().cpu().pin_memory()
            hv = v[:, :, sh.j * r:(sh.j + 1) * r].contiguous().cpu().pin_memory()
        else:
            hk, hv = (x.contiguous().cpu().pin_memory() for x in (k, v))
        B, hl, rows, D = q.shape
        # this rank's slice of the gathered output: rows world-split
        r0 = (self.S * sh.rank) // world
        r1 = (self.S * (sh.rank + 1)) // world
        ridx = self.shard.rows(self.S).to(q.device) if self.shard.m > 1 else None

        def compute(d):
            kk, vv = self.gather_kv_rows(d[1], d[2]) if split else (d[1], d[2])
            if world > 1 and self.peer_output:
                out = self.step(d[0], kk, vv, gather=True)         # [B, S, Hq, D] on every rank
                # a copy: the gathered buffer is rewritten by the next step (ours and the peers')
                return out[:, r0:r1].clone()
            out = self.step(d[0], kk, vv, gather=False)
            return out.index_select(2, ridx) if ridx is not None else out

        if world > 1 and self.peer_output:
            out_shape, out_numel = (B, r1 - r0, sh.Hq, D), B * (r1 - r0) * sh.Hq * D
        else:
            out_shape, out_numel = (B, hl, rows, D), B * hl * rows * D
        t = pipelined_e2e([hq, hk, hv], compute, out_shape, q.dtype, steps, warmup)
        c = pipelined_e2e([hq, hk, hv], lambda d: torch.empty(out_shape, device=q.device, dtype=q.dtype),
                          out_shape, q.dtype, steps, warmup)
        el = q.element_size()
        per_head_rows = B * self.S * D * el
        kv_copies = 1 if split else sh.m
        h2d = sh.Hq * per_head_rows + 2 * sh.Hkv * kv_copies * per_head_rows
        d2h = sh.Hq * per_head_rows if (world > 1 and self.peer_output) else sh.Hq * per_head_rows
        return {"ms": t["ms"], "serial_ms": t["serial_ms"], "h2d": h2d, "d2h": d2h,
                "copy_only_ms": c["ms"], "rank_bytes": sum(x.numel() * el for x in (hq, hk, hv)) + out_numel * el}

    def close(self):
        """Collective when peer output was used (releases the peer buffers)."""
        self._close_peer()


def selected_block_flops(kv_idx: torch.Tensor, S: int, D: int, t0: int = 0, pair_stride: int = 1) -> float:
    """FLOPs of the attention kernel's work: 4*64*64*D per (tile, usable slot)
    (QK^T and PV over full 64x64 blocks), counted from the actual kv_idx
    (local tile t is sequence tile t0 + t + 2*(t//2)*(pair_stride-1))."""
    nb = math.ceil(S / 64)
    Qt = kv_idx.shape[2]
    t = torch.arange(Qt, device=kv_idx.device)
    last = ((t0 + t + 2 * (t // 2) * (pair_stride - 1)) * 64 + 63).view(1, 1, Qt, 1)
    ok = (kv_idx >= 0) & (kv_idx < nb) & (kv_idx.long() * 64 <= last)
    return float(ok.sum().item()) * 4 * 64 * 64 * D


def selection_flops(Hq: int, S: int, D: int, quest: bool = True) -> float:
    """fp32 FLOPs of exact tile scoring: one FMA per (row, visible block, d),
    two for Quest (positive and negative envelope chains)."""
    qt = math.ceil(S / 64)
    per = 4 if quest else 2
    return per * 64 * D * Hq * qt * (qt + 1) / 2


def stage_breakdown(q, k, v, cfg, scale, reps: int = 5):
    """Per-stage CUDA-event times (ms) of one layer on one GPU."""
    st = torch.cuda.current_stream()

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        for _ in range(reps):
            r = fn()
        e.record(st)
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps, r

    def timed_graph(fn):
        # device time of a short kernel: `reps` launches replayed from a CUDA graph
        # (timing them from the host would add the launch overhead)
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                r = fn()
        g.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        g.replay()
        e.record(st)
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps, r

    t_sum, summ = timed_graph(lambda: ops.block_summary(k, cfg.quest))
    t_sel, kv = timed(lambda: ops.select_kv_idx(q, k, scale, cfg))
    t_att, _ = timed(lambda: ops.block_sparse_attn(q, k, v, kv, scale))
    return {"summary": {"ms": t_sum}, "select": {"ms": t_sel - t_sum, "ms_incl_summary": t_sel},
            "attn": {"ms": t_att}}


def time_producer(q, k, quest: bool, reps: int = 5):
    """CUDA-event time (ms) and algorithmic bytes of the fused norm + rotary
    producer (ugbsa_qk_norm_rope) over the layer's Q and K heads (taken as the
    pre-norm projection outputs; full-width rotary, scale-mode norm), K with
    its block summaries."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    dev = q.device
    w = torch.ones(D, device=dev, dtype=q.dtype)
    pos = torch.arange(S, device=dev, dtype=torch.float32)[:, None]
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
    emb = torch.cat([pos * inv, pos * inv], dim=-1)[None]
    cos, sin = emb.cos().to(q.dtype), emb.sin().to(q.dtype)
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    summary = "quest" if quest else "mean"

    def run():
        ops.qk_norm_rope(q, w, 1e-6, cos, sin, norm_mode="scale", out=qo)
        ops.qk_norm_rope(k, w, 1e-6, cos, sin, norm_mode="scale", out=ko, summary=summary)

    run()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(st)
    for _ in range(reps):
        run()
    e.record(st)
    torch.cuda.synchronize()
    el = q.element_size()
    nb = math.ceil(S / 64)
    nbytes = 2 * (Hq + Hkv) * S * D * el + 2 * 2 * S * D * el + nb * Hkv * D * 4 * (2 if quest else 1)
    return {"ms": s.elapsed_time(e) / reps, "algorithmic_bytes": nbytes}


def time_decode_batch(B: int, Hq: int, Hkv: int, S: int, D: int, cfg: ops.SelectorConfig, scale: float,
                      reps: int = 20, seed: int = 0):
    """time_decode for B sequences of S cached keys each (seeded N(0,1) cache and
    query rows: decode batches several sequences, which the selection's many
    small launches amortise)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((B, Hkv, S, D), device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn((B, Hkv, S, D), device="cuda", dtype=torch.bfloat16, generator=g)
    q = torch.randn((B, Hq, 1, D), device="cuda", dtype=torch.bfloat16, generator=g)
    r = time_decode(q, k, v, cfg, scale, reps)
    del k, v
    r["batch"] = B
    return r


def time_decode(q, k, v, cfg: ops.SelectorConfig, scale: float, reps: int = 20):
    """One decode step per layer at this cache length (the last query row of
    each head against the whole K/V): the block-sparse decode (summary refresh
    of the last block, selection, attention) against torch SDPA over the whole
    cache (the reference's decode), CUDA events, ms per step.  Each stage is
    also captured alone in a CUDA graph and replayed, which gives its GPU time
    without the host's per-call cost; fused_step_graph_ms is the same step
    through ops.decode_step (three launches instead of five)."""
    import torch.nn.functional as F
    B, Hq, _, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    G = Hq // Hkv
    q1 = q[:, :, -1:].contiguous()
    summ = ops.block_summary(k, cfg.quest)
    nb = math.ceil(S / 64)
    st = torch.cuda.current_stream()

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        for _ in range(reps):
            r = fn()
        e.record(st)
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps, r

    def graphed(fn):
        try:
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(st)
            with torch.cuda.stream(side):
                fn()                      # warm the allocator pool on the capture stream
                with torch.cuda.graph(g, stream=side):
                    fn()
            st.wait_stream(side)
            return timed(lambda: g.replay())[0]
        except Exception:                 # capture unsupported here: eager only
            return None

    def refresh():
        ops.block_summary_update(k, cfg.quest, summ, nb - 1)

    def sparse():
        refresh()
        kv = ops.decode_select(q1, summ, S, Hkv, scale, cfg)
        return ops.decode_attn(q1, k, v, kv, S, scale), kv

    t_sparse, (_, kv) = timed(sparse)
    t_sel, _ = timed(lambda: ops.decode_select(q1, summ, S, Hkv, scale, cfg))
    t_att, _ = timed(lambda: ops.decode_attn(q1, k, v, kv, S, scale))
    t_graph = graphed(sparse)
    t_step = graphed(lambda: ops.decode_step(q1, k, v, summ, S, scale, cfg)) \
        if q1.dtype in (torch.bfloat16, torch.float16) else None
    g_refresh = graphed(refresh)
    g_sel = graphed(lambda: ops.decode_select(q1, summ, S, Hkv, scale, cfg))
    g_att = graphed(lambda: ops.decode_attn(q1, k, v, kv, S, scale))
    t_dense, _ = timed(lambda: F.scaled_dot_product_attention(q1, k, v, scale=scale, enable_gqa=Hq != Hkv))
    valid = (kv >= 0) & (kv < nb)
    kept = valid.sum().item()
    # the attention reads each KV group's union of its heads' lists once
    ids = torch.where(valid, kv, torch.full_like(kv, nb)).view(B, Hkv, G * kv.shape[-1])
    union = sum(int(torch.unique(ids[b_, h_]).numel()) - int((ids[b_, h_] == nb).any())
                for b_ in range(B) for h_ in range(Hkv))
    el = k.element_size()
    union_bytes = union * 64 * D * 2 * el
    summ_bytes = B * Hkv * nb * D * 4 * (2 if cfg.quest else 1)
    return {"sparse_ms": t_sparse, "sparse_graph_ms": t_graph, "fused_step_graph_ms": t_step,
            "select_ms": t_sel, "attn_ms": t_att,
            "graph_stage_ms": {"refresh": g_refresh, "select": g_sel, "attn": g_att},
            "dense_sdpa_ms": t_dense,
            "kept_blocks_per_head": kept / (B * Hq), "union_blocks_per_group": union / (B * Hkv),
            "attn_kv_bytes": union_bytes,
            "attn_GB_s": (union_bytes / (g_att / 1e3) / 1e9) if g_att else None, "summary_bytes": summ_bytes}


def time_dense(q, k, v, scale, reps: int = 3):
    """Dense causal attention on the same GPU: the faster of torch SDPA with
    enable_gqa (flash / cuDNN backends) and the reference's repeat_kv + SDPA
    (src/sparse_attention.py:761-770)."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    G = q.shape[1] // k.shape[1]
    st = torch.cuda.current_stream()
    cands = {}

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        for _ in range(reps):
            fn()
        e.record(st)
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps

    for name, be in (("sdpa_gqa_cudnn", SDPBackend.CUDNN_ATTENTION), ("sdpa_gqa_flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel([be]):
                cands[name] = timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale,
                                                                           enable_gqa=True))
        except RuntimeError:
            pass
    try:
        kr = k.repeat_interleave(G, dim=1)
        vr = v.repeat_interleave(G, dim=1)
        cands["repeat_kv_sdpa"] = timed(lambda: F.scaled_dot_product_attention(q, kr, vr, is_causal=True,
                                                                               scale=scale))
        del kr, vr
    except RuntimeError:
        pass
    if not cands:
        return None
    best = min(cands, key=cands.get)
    return {"ms": cands[best], "backend": best, "all": cands}
