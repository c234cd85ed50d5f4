"""Sharded prefill on several GPUs (NCCL) against the single-GPU result.

Runs only where at least two GPUs are visible.  Head sharding
(ugbsa.parallel.ShardedPrefill): each rank scores and ranks its heads, the
per-tile sigma sums are combined with one NCCL all-reduce, and the outputs are
all-gathered.  Sequence sharding (ugbsa.parallel.SeqShardedPrefill): each rank
takes a cost-balanced range of query rows for all heads, K/V rows and the
per-tile margins are all-gathered, then the output rows.  Every kernel is
deterministic and the margins are subnormal (sums exact in any order), so
kv_idx and the attention output must equal the unsharded computation bit for
bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, grain, peer, out_dir):
    import datetime
    import sys

    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "uncertainty-gated-block-sparse-attention_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)
    from ugbsa import ops, parallel
    from ugbsa.synth import planted_inputs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    B, Hq, Hkv, S, D = 1, 8, 4, 4096, 128
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=4, seed=41, chained=True, bf16=True)
    qd, kd, vd = (torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in (q, k, v))
    cfg = ops.SelectorConfig(mode="router", router_score="quest", router_mode="quantile", router_grain=grain,
                             router_quantile=0.25, budget_blocks=4, k_min=1, k_max=112)
    shard = parallel.HeadShard.make(Hq, Hkv, world, rank)
    runner = parallel.ShardedPrefill(shard, cfg, D ** -0.5, group=dist.group.WORLD, peer_output=peer)
    ql, kl, vl = shard.slice(qd, kd, vd)
    out = runner.step(ql, kl, vl)
    kv_local = runner.last_kv_idx
    torch.cuda.synchronize()
    # the unsharded reference, computed on this rank's GPU
    single = parallel.ShardedPrefill(parallel.HeadShard.make(Hq, Hkv, 1, 0), cfg, D ** -0.5)
    ref = single.step(qd, kd, vd)
    kv_ref = single.last_kv_idx[:, shard.q0:shard.q1]
    same_kv = bool(torch.equal(kv_local, kv_ref))
    same_out = bool(torch.equal(out, ref))
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{int(same_kv)} {int(same_out)}\n")
    runner.close()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("grain,peer", [("row", True), ("cell", True), ("row", False)])
def test_two_gpu_sharded_prefill_matches_single_gpu(tmp_path, grain, peer):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, grain, peer, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    res = [open(tmp_path / f"r{r}.txt").read().split() for r in range(2)]
    assert all(r == ["1", "1"] for r in res), res


def _seq_worker(rank, world, port, grain, peer, out_dir):
    import datetime
    import sys

    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "uncertainty-gated-block-sparse-attention_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)
    from ugbsa import ops, parallel
    from ugbsa.synth import planted_inputs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    B, Hq, Hkv, S, D = 1, 8, 2, 8000, 128
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=4, seed=43, chained=True, bf16=True)
    qd, kd, vd = (torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in (q, k, v))
    cfg = ops.SelectorConfig(mode="router", router_score="quest", router_mode="quantile", router_grain=grain,
                             router_quantile=0.25, budget_blocks=8, k_min=1, k_max=112)
    runner = parallel.SeqShardedPrefill(S, Hq, Hkv, D, cfg, D ** -0.5, world, rank, group=dist.group.WORLD,
                                        peer_output=peer)
    sh = runner.shard
    rows = lambda x: x[:, :, sh.row0:sh.row1].transpose(1, 2).contiguous()   # [B, rows, H, D]
    out = runner.step(rows(qd), rows(kd), rows(vd))
    kv_local = runner.last_kv_idx
    torch.cuda.synchronize()
    single = parallel.ShardedPrefill(parallel.HeadShard.make(Hq, Hkv, 1, 0), cfg, D ** -0.5)
    ref = single.step(qd, kd, vd)
    same_kv = bool(torch.equal(kv_local, single.last_kv_idx[:, :, sh.t0:sh.t1]))
    same_out = bool(torch.equal(out, ref))
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{int(same_kv)} {int(same_out)}\n")
    runner.close()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("grain,peer", [("row", True), ("cell", True), ("row", False)])
def test_two_gpu_sequence_sharded_prefill_matches_single_gpu(tmp_path, grain, peer):
    port = _free_port()
    mp.start_processes(_seq_worker, args=(2, port, grain, peer, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    res = [open(tmp_path / f"r{r}.txt").read().split() for r in range(2)]
    assert all(r == ["1", "1"] for r in res), res


def _grid_worker(rank, world, port, grain, Hkv, out_dir):
    import datetime
    import sys

    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "uncertainty-gated-block-sparse-attention_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)
    from ugbsa import ops, parallel
    from ugbsa.synth import planted_inputs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    B, Hq, S, D = 1, 8, 6000, 128
    q, k, v, _ = planted_inputs(B, Hq, Hkv, S, D, n_planted=4, seed=47, chained=True, bf16=True)
    qd, kd, vd = (torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in (q, k, v))
    cfg = ops.SelectorConfig(mode="router", router_score="quest", router_mode="quantile", router_grain=grain,
                             router_quantile=0.25, budget_blocks=8, k_min=1, k_max=112)
    sh = parallel.GridShard.make(Hq, Hkv, world, rank)
    runner = parallel.GridShardedPrefill(sh, S, cfg, D ** -0.5, group=dist.group.WORLD)
    out = runner.step(*sh.slice(qd, kd, vd))
    kv_local = runner.last_kv_idx
    torch.cuda.synchronize()
    single = parallel.ShardedPrefill(parallel.HeadShard.make(Hq, Hkv, 1, 0), cfg, D ** -0.5)
    ref = single.step(qd, kd, vd)
    tiles = torch.tensor(sh.tiles(S), device=dev)
    kv_ref = single.last_kv_idx[:, sh.q0:sh.q1].index_select(2, tiles)
    same_kv = bool(torch.equal(kv_local, kv_ref))
    same_out = bool(torch.equal(out, ref))
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{int(same_kv)} {int(same_out)}\n")
    runner.close()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("grain,Hkv", [("row", 1), ("cell", 1), ("row", 2)])
def test_two_gpu_grid_sharded_prefill_matches_single_gpu(tmp_path, grain, Hkv):
    """Hkv 1 over 2 ranks: both ranks hold the KV head, tile pairs dealt 0,2,4.. / 1,3,5..;
    Hkv 2: one KV group per rank."""
    port = _free_port()
    mp.start_processes(_grid_worker, args=(2, port, grain, Hkv, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    res = [open(tmp_path / f"r{r}.txt").read().split() for r in range(2)]
    assert all(r == ["1", "1"] for r in res), res


def _tp_worker(rank, world, port, out_dir):
    import datetime
    import sys

    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "uncertainty-gated-block-sparse-attention_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)
    from ugbsa import decoder, ops

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    shape = decoder.DecoderShape(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, intermediate=1024,
                                 vocab=1000, rope_theta=1.0e6, rms_eps=1e-6)
    cfg = ops.SelectorConfig(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                             router_quantile=0.25, budget_blocks=2, k_min=1, k_max=112)
    ids = torch.randint(0, shape.vocab, (2048,), generator=torch.Generator().manual_seed(5)).to(dev)
    tp = decoder.TPDecoder(shape, cfg, world, rank, group=dist.group.WORLD, seed=3, device=dev)
    one = decoder.TPDecoder(shape, cfg, 1, 0, seed=3, device=dev)
    sh = tp.layout.shard
    cos, sin = decoder.rotary_tables(2048, 128, shape.rope_theta, dev)
    # layer by layer from the same residual stream: the selection of this rank's heads is the
    # one-GPU selection bit for bit, and the layer output differs only by the bf16 rounding of
    # the row-parallel partial sums the all-reduce adds (a different kv_idx further down would
    # follow from that rounding, not from the split, so each layer starts from the same input)
    h = torch.nn.functional.embedding(ids, one.embed)
    ok, worst = True, 0.0
    for i in range(shape.layers):
        want = one.layer(h, i, cos, sin)
        got = tp.layer(h, i, cos, sin)
        ok &= bool(torch.equal(tp.last_kv_idx, one.last_kv_idx[:, sh.q0:sh.q1]))
        top = want.float().abs().max().item()
        d = (got.float() - want.float()).abs()
        rel = d.max().item() / top
        worst = max(worst, rel)
        ok &= rel <= 0.02 and d.mean().item() <= 0.002 * top
        h = want
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{int(ok)} {worst:.3e}\n")
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_tensor_parallel_decoder_matches_one_gpu(tmp_path):
    """ugbsa.decoder over 2 ranks (one KV group each, NCCL all-reduce after o_proj and
    down_proj): every layer selects the same blocks for its heads as one GPU and gives the
    one-GPU layer output within the bf16 rounding of the all-reduced partial sums."""
    port = _free_port()
    mp.start_processes(_tp_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    res = [open(tmp_path / f"r{r}.txt").read().split() for r in range(2)]
    assert all(r[0] == "1" for r in res), res
