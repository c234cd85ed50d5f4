#!/usr/bin/env python
"""bench.py -- block-sparse attention prefill on B200, the BASELINE.json metric.

Workload ("sparse-attn prefill ms + effective TFLOP/s at 128K;
ratio vs dense on same GPU"): one attention layer of the Qwen2.5-7B geometry at
128K tokens -- B=1, S=131072, 28 Q heads / 4 KV heads, head_dim 128, bf16,
block 64, router-on-Quest scoring, k_base = NB/16 = 128 slots per tile, q=0.25
quantile router (triggered tiles keep 256), causal.  Inputs are seeded
synthetic N(0,1) tensors with 16 chained planted key blocks per KV head.
``--workload cfg5`` measures BASELINE config 5 instead (head_dim 256, 16 Q / 2
KV heads, RMSNorm + RoPE on Q and K, 32 planted blocks, K-mean router, k_base
128).

A step is one pass of the hot path over that layer: block summaries, tile
scoring + top-k + sigma router + kv_idx, block-sparse attention.  ``value`` is
effective TFLOP/s = dense-equivalent block-causal FLOPs of the layer / step
time, with inputs resident in HBM; ``e2e`` is the same metric through the
public hook ``ugbsa.sparse_attention.block_sparse_attention`` with Q/K/V copied
from pinned host memory and the output copied back every step.

Multi-GPU (torchrun, one rank per GPU): KV-head groups are split over the
ranks, and when the ranks outnumber the KV heads, each group's query-tile pairs
are dealt round-robin over its ranks (ugbsa.parallel.GridShardedPrefill).  One
NCCL all-reduce of per-tile sigma sums feeds the shared quantile; the attention
kernel writes each output tile to every rank's buffer over NVLink (peer
stores), and one small all-reduce orders the step's end.  Total work is fixed:
"scaling": "strong".

``--impl reference`` times the CPU restatement of the reference path (the
reference itself is Python/PyTorch, absent from the GPU box) on every host
core, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "uncertainty-gated-block-sparse-attention_b200")
for _p in (PKG, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "sparse-attn prefill ms + effective TFLOP/s at 128K; ratio vs dense on same GPU"
UNIT = "TFLOP/s (dense-equivalent)"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# attention kernel DRAM traffic per launch at the 128K workload (dram__bytes_read.sum +
# dram__bytes_write.sum): the 64K capture summarised in profiles/ (680.0 + 450.5 MB =
# 1.131 GB, 1.05x its algorithmic bytes) scaled by 2, every term of which is linear in S at
# fixed heads
ATTN_TRAFFIC_BYTES = {("attn-layer", 131072): 2 * 1130506496, ("attn-layer", 65536): 1130506496}


# --workload: "attn-layer" (the metric's layer, Qwen2.5-7B geometry, router-on-Quest) or
# "cfg5" (head_dim 256, 16 Q / 2 KV heads, per-head RMSNorm + RoPE on
# Q and K, 32 planted blocks, K-mean router with k_base 128 at 128K)
WORKLOAD = "attn-layer"


def workload(seq):
    nb = seq // 64
    if WORKLOAD == "cfg5":
        return dict(name="cfg5", B=1, Hq=16, Hkv=2, S=seq, D=256, n_planted=32, seed=5, chained=False,
                    qk_norm_rope=True,
                    sel=dict(mode="router", router_score="mean", router_mode="quantile", router_grain="row",
                             router_quantile=0.25, budget_blocks=max(1, nb // 32), k_min=1,
                             k_max=max(112, nb // 32)))
    return dict(name="attn-layer", B=1, Hq=28, Hkv=4, S=seq, D=128, n_planted=16, seed=0, chained=True,
                qk_norm_rope=False,
                sel=dict(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                         router_quantile=0.25, budget_blocks=max(1, nb // 32), k_min=1, k_max=max(112, nb // 32)))


def parallel_kmax(cfg, S):
    """kmax of the selection (the budget's second value)."""
    from ugbsa import ops
    return ops.budget(cfg, S)[1]


def split_for(world, requested="auto"):
    """How a multi-GPU run divides the layer: "grid" (KV head groups x query tile
    pairs dealt round-robin), "heads" (Q heads, a KV group's split 4 + 3 when the
    ranks outnumber the KV heads) or "rows" (cost-balanced contiguous query-row
    ranges, all heads per rank).  auto: grid when the ranks divide, or are a
    multiple of, the KV heads; rows otherwise."""
    if requested != "auto":
        return requested
    w = workload(131072)
    return "grid" if w["Hkv"] % world == 0 or world % w["Hkv"] == 0 else "rows"


def parallelism_name(seq, world, split="auto"):
    w = workload(seq)
    sp = split_for(world, split)
    if sp == "grid":
        m = max(1, world // w["Hkv"])
        return f"kvheads{min(world, w['Hkv'])}" + (f"xdealt{m}" if m > 1 else "")
    return {"heads": "heads", "rows": "seq"}[sp] + str(world)


def config_for(seq, world, split="auto"):
    """The workload description both arms report (identical for a given S and rank count)."""
    w = workload(seq)
    s = w["sel"]
    nb = math.ceil(seq / 64)
    kb_row = max(min(s["budget_blocks"], s["k_max"]), s["k_min"])
    k_base = min(2 * kb_row, nb)
    kmax = min(2 * k_base, nb)
    gb = lambda n: f"{n / 1e6:.0f} MB"
    q_bytes = w["B"] * w["Hq"] * seq * w["D"] * 2
    kv_bytes = w["B"] * w["Hkv"] * seq * w["D"] * 2
    score = "router-on-Quest" if s["router_score"] == "quest" else "K-mean router"
    extra = " inputs: per-head RMSNorm + RoPE on Q and K" if w["qk_norm_rope"] else ""
    return {"workload": f"{w['name']}-{seq // 1024}K: B={w['B']} S={seq} Hq={w['Hq']} Hkv={w['Hkv']} D={w['D']} "
                        f"bf16 block=64 {score} quantile row-grain q={s['router_quantile']} k_base={k_base} "
                        f"kmax={kmax} causal{extra}",
            "global_batch": w["B"], "seq_len": seq,
            "parallelism": parallelism_name(seq, world, split) if world > 1 else "none",
            "l2": f"inputs larger than L2 (Q {gb(q_bytes)}, K {gb(kv_bytes)}, V {gb(kv_bytes)})"}


def dense_equiv_flops(Hq, S, D):
    qt = math.ceil(S / 64)
    return Hq * qt * (qt + 1) / 2 * 4 * 64 * 64 * D


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                     hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        load = [r for r in rows if r["power"] > 200.0] or rows
        reasons = set()
        for r in load:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("swp", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(load),
                "power_w_max": max(r["power"] for r in rows)}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------- reference arm
def run_reference(args, seq):
    """CPU restatement of the reference path, timed on a bounded sample."""
    import numpy as np
    import torch

    from oracle import oracle

    w = workload(seq)
    S, D = w["S"], w["D"]
    nb = math.ceil(S / 64)
    # every host core this process may run on, whatever OMP_NUM_THREADS torchrun exported
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(threads)
    threads = oracle.set_threads(threads)
    # sample: one Q head (and its KV head) of the layer, the heaviest `tiles` tiles
    tiles = args.ref_tiles
    t0, t1 = max(0, nb - tiles), nb
    gen = torch.Generator().manual_seed(w["seed"])
    q = torch.randn((1, 1, S, D), generator=gen).to(torch.bfloat16).float().numpy()
    k = torch.randn((1, 1, S, D), generator=gen).to(torch.bfloat16).float().numpy()
    v = torch.randn((1, 1, S, D), generator=gen).to(torch.bfloat16).float().numpy()
    s = w["sel"]
    cfg = oracle.OracleConfig(mode=s["mode"], router_score=s["router_score"], router_mode=s["router_mode"],
                              router_grain=s["router_grain"], router_quantile=s["router_quantile"],
                              budget_blocks=s["budget_blocks"], k_min=s["k_min"], k_max=s["k_max"])
    scale = D ** -0.5
    oracle.lib()
    sample_flops = sum((t + 1) * 4 * 64 * 64 * D for t in range(t0, t1))  # dense-equivalent, 1 head

    def step():
        summ = oracle.block_summary(k, cfg.quest)
        oracle.sample_step(q, k, v, scale, cfg, t0, t1, summ=summ)

    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        a = time.perf_counter()
        step()
        times.append(time.perf_counter() - a)
    sec = sum(times) / len(times)
    value = sample_flops / sec / 1e12
    sample = (f"1 of {w['Hq']} Q heads, tiles {t0}-{t1 - 1} of {nb} (the heaviest), S={S}: block summary of its KV head, "
              f"tile scores, ranking + sigma, attention over the selected blocks")
    line = {"metric": METRIC, "impl": "reference", "value": round(value, 6), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1), bf16-rounded)",
            "config": config_for(seq, args.gpus, getattr(args, "split", "auto")),
            "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": threads, "threads": threads,
                             "host_cpus": os.cpu_count(), "cpu_model": cpu_model(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 6), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "projected_full_layer_ms": round(sec * 1e3 * (dense_equiv_flops(w["Hq"], S, D) / sample_flops), 1)}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- GPU arm
def run_gpu(args, seq):
    import torch
    import torch.distributed as dist

    from ugbsa import ops, parallel
    from ugbsa import sparse_attention as sa
    from ugbsa.synth import planted_inputs_torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    w = workload(seq)
    B, Hq, Hkv, S, D = w["B"], w["Hq"], w["Hkv"], w["S"], w["D"]
    scale = D ** -0.5
    s = w["sel"]
    cfg = ops.SelectorConfig(**s)
    sa.SEL.mode, sa.SEL.kernel_v2 = s["mode"], True
    sa.SEL.router_score, sa.SEL.router_mode, sa.SEL.router_grain = s["router_score"], s["router_mode"], s["router_grain"]
    sa.SEL.router_quantile, sa.SEL.budget_blocks = s["router_quantile"], s["budget_blocks"]
    sa.SEL.k_min, sa.SEL.k_max = s["k_min"], s["k_max"]

    q, k, v = planted_inputs_torch(B, Hq, Hkv, S, D, n_planted=w["n_planted"], seed=w["seed"], chained=w["chained"],
                                   qk_norm_rope=w["qk_norm_rope"], dtype=torch.bfloat16, device=dev)
    split = split_for(world, args.split)
    t0, pstride = 0, 1
    if world > 1 and split == "grid":
        shard = parallel.GridShard.make(Hq, Hkv, world, rank)
        runner = parallel.GridShardedPrefill(shard, S, cfg, scale, group=dist.group.WORLD)
        ql, kl, vl = shard.slice(q, k, v)
        t0, pstride = 2 * shard.j, shard.m
    elif world > 1 and split == "rows":
        runner = parallel.SeqShardedPrefill(S, Hq, Hkv, D, cfg, scale, world, rank, group=dist.group.WORLD)
        sh = runner.shard
        t0 = sh.t0
        # this rank's rows in the [B, rows, H, D] layout of a projection's output
        ql, kl, vl = (x[:, :, sh.row0:sh.row1].transpose(1, 2).contiguous() for x in (q, k, v))
    else:
        shard = parallel.HeadShard.make(Hq, Hkv, world, rank)
        runner = parallel.ShardedPrefill(shard, cfg, scale, group=dist.group.WORLD if world > 1 else None)
        ql, kl, vl = shard.slice(q, k, v)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # warm-up (also builds the allocator cache)
    for _ in range(args.warmup):
        runner.step(ql, kl, vl)
    torch.cuda.synchronize()

    peaks, peak_kind = load_peaks()
    sampler = ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else
                           os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    # the clock sampler first, then the barrier: every rank records its start event
    # right after the same collective (a skewed start would be counted as step time)
    sampler.start()
    time.sleep(0.25)
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        runner.step(ql, kl, vl, events=ev[i])
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    total_ms = t_start.elapsed_time(t_end)
    sel_ms = [e[0].elapsed_time(e[1]) for e in ev]
    attn_ms = [e[1].elapsed_time(e[2]) for e in ev]
    t = torch.tensor([total_ms, sum(sel_ms), sum(attn_ms)], device=dev, dtype=torch.float64)
    per_rank = None
    if world > 1:
        g = torch.empty((world, 3), device=dev, dtype=torch.float64)
        dist.all_gather_into_tensor(g, t.view(1, 3))
        # per rank: [step, select stage, attention stage] ms (the imbalance across ranks)
        per_rank = [[round(x / args.steps, 3) for x in r] for r in g.tolist()]
        t = g.max(dim=0).values
    total_ms, sel_sum, attn_sum = t.tolist()
    ms_per_step = total_ms / args.steps

    # algorithmic work from the actual selection
    kv_idx = runner.last_kv_idx
    sel_flops = parallel.selected_block_flops(kv_idx, S, D, t0, pstride)
    ft = torch.tensor([sel_flops], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ft)
    sel_flops_total = ft.item()
    deq = dense_equiv_flops(Hq, S, D)
    value = deq / (ms_per_step / 1e3) / 1e12
    attn_ms_avg = attn_sum / args.steps
    achieved = sel_flops / (attn_ms_avg / 1e3) / 1e12 if attn_ms_avg > 0 else 0.0   # this rank's launch
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))

    # stage split (N=1 only): summary vs select, for the HBM roofline of the summary kernel
    stages = None
    if world == 1:
        stages = parallel.stage_breakdown(ql, kl, vl, cfg, scale, reps=5)
        summ_bytes = S * Hkv * D * 2 + math.ceil(S / 64) * Hkv * D * 4 * (2 if cfg.quest else 1)
        stages["summary"]["GB_s"] = summ_bytes / (stages["summary"]["ms"] / 1e3) / 1e9
        stages["summary"]["frac_hbm"] = stages["summary"]["GB_s"] / float(peaks.get("hbm_gbs", 6650.0))
        stages["summary"]["algorithmic_bytes"] = summ_bytes
        prod = parallel.time_producer(ql, kl, cfg.quest)
        prod["GB_s"] = prod["algorithmic_bytes"] / (prod["ms"] / 1e3) / 1e9
        prod["frac_hbm"] = prod["GB_s"] / float(peaks.get("hbm_gbs", 6650.0))
        prod["what"] = "fused per-head RMSNorm + rotary over Q and K, K block summaries (qk_norm_rope)"
        stages["producer"] = prod
        stages["decode"] = parallel.time_decode(ql, kl, vl, cfg, scale)
        small = ops.SelectorConfig(**{**s, "budget_blocks": 8, "k_max": 112})
        stages["decode_budget8"] = parallel.time_decode(ql, kl, vl, small, scale)
        stages["decode_b8_budget8"] = parallel.time_decode_batch(8, Hq, Hkv, S, D, small, scale)
        stages["decode"]["what"] = ("one decode step at this cache length: block-sparse decode (last-block summary "
                                    "refresh, selection, split-K attention) vs torch SDPA over the whole cache")
        sel_fl = parallel.selection_flops(Hq, S, D)
        stages["select"]["scoring_TFLOPs"] = sel_fl / 1e12
        stages["select"]["fp32_scoring_TFLOP_s"] = sel_fl / (stages["select"]["ms"] / 1e3) / 1e12
        # roofline on the algorithmic work: one multiply-add per (query row, visible block, d)
        # (Quest: the same count with a sign select) against the sustained bf16 peak, and the
        # bytes that must move (Q once, the summaries, kv_idx written), whichever bounds
        nb_ = math.ceil(S / 64)
        alg_fl = 2.0 * 64 * D * Hq * nb_ * (nb_ + 1) / 2
        alg_by = (B * Hq * S * D * 2 + B * Hkv * nb_ * D * 4 * (2 if cfg.quest else 1)
                  + B * Hq * nb_ * parallel_kmax(cfg, S) * 4)
        pk_tf = float(peaks.get("bf16_tflops_sustained", 1399.5))
        pk_gb = float(peaks.get("hbm_gbs", 6650.0))
        t_fl, t_by = alg_fl / (pk_tf * 1e12), alg_by / (pk_gb * 1e9)
        stages["select"]["roofline"] = {
            "bound": "tensor" if t_fl >= t_by else "hbm", "algorithmic_TFLOPs": alg_fl / 1e12,
            "algorithmic_bytes": alg_by, "roofline_ms": max(t_fl, t_by) * 1e3,
            "frac": max(t_fl, t_by) / (stages["select"]["ms"] / 1e3),
            "peaks": f"{pk_tf} TFLOP/s sustained bf16, {pk_gb} GB/s (measured)"}

    # dense denominator on the same GPU (N=1; rank 0 of a sharded run reports the 1-GPU figure)
    dense = None
    if world == 1 and not args.no_dense:
        dense = parallel.time_dense(q, k, v, scale, reps=3)

    # e2e: public hook, pinned host inputs, output read back every step
    e2e = None
    if not args.no_e2e:
        e2e = runner.time_e2e(ql, kl, vl, steps=args.steps, warmup=2)
        te = torch.tensor([e2e["ms"]], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = te.item()
        ts = torch.tensor([e2e["serial_ms"]], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(ts, op=dist.ReduceOp.MAX)
        tc = torch.tensor([e2e.get("copy_only_ms", float("nan"))], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tc, op=dist.ReduceOp.MAX)
        copy_ms = tc.item()
        e2e = {"value": round(deq / (e2e_ms / 1e3) / 1e12, 3), "unit": UNIT,
               "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],   # over all ranks
               "ms_per_step": round(e2e_ms, 3),
               "pipelined": "copy-in of step i+1 and copy-out of step i-1 overlap step i (three streams)",
               "serial_ms_per_step": round(ts.item(), 3),
               # the same host<->device copies with no compute: the host-link ceiling of this e2e
               "copy_only_ms_per_step": round(copy_ms, 3),
               "frac_of_copy_ceiling": round(copy_ms / e2e_ms, 4) if e2e_ms > 0 else None}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_sample(seq, args.ref_tiles)

    if world > 1:
        runner.close()
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": (f"synthetic (seeded N(0,1) + {w['n_planted']} {'chained ' if w['chained'] else ''}planted blocks "
                     f"per KV head{', RMSNorm + RoPE applied' if w['qk_norm_rope'] else ''})"),
            "config": config_for(seq, world, split),
            "sparse_ms_per_layer": round(ms_per_step, 3),
            "select_ms": round(sel_sum / args.steps, 3), "attn_ms": round(attn_ms_avg, 3),
            "selected_block_TFLOPs": round(sel_flops_total / 1e12, 3),
            "dense_equivalent_TFLOPs": round(deq / 1e12, 3),
            "roofline": {"bound": "tensor", "kernel": "attn_fwd_kernel", "achieved": round(achieved, 2),
                         "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_kind": f"bf16_tflops_sustained ({peak_kind})",
                         "traffic": ATTN_TRAFFIC_BYTES.get((w["name"], seq)) if world == 1 else None},
            "gpu_launches": parallel.launches_per_step(cfg, *ops.budget(cfg, S)) * args.steps,
            "clocks": clocks, "e2e": e2e, "cpu_baseline": cpu}
    if dense is not None:
        line["dense_ms"] = round(dense["ms"], 3)
        line["dense_backend"] = dense["backend"]
        line["ratio_vs_dense"] = round(ms_per_step / dense["ms"], 4)
    if stages is not None:
        line["stages"] = stages
    if per_rank is not None:
        line["per_rank_ms"] = per_rank
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- full-model prefill
def run_model(args):
    """BASELINE configs 3 / 4: a whole prefill of a random-init Qwen2.5-7B (cfg3) or
    14B (cfg4) shaped decoder, tensor-parallel over the ranks (ugbsa.decoder), with
    the block-sparse attention on every layer, beside the same model with dense
    SDPA attention.  A step is one forward over S uniform random token ids."""
    import torch
    import torch.distributed as dist

    from ugbsa import decoder, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    shape = decoder.QWEN25_7B if args.workload == "cfg3" else decoder.QWEN25_14B
    S = args.seq
    nb = math.ceil(S / 64)
    if args.workload == "cfg3":   # router-on-Quest, k_base = NB/16, q = 0.25
        sel = dict(mode="router", router_score="quest", router_mode="quantile", router_grain="row",
                   router_quantile=0.25, budget_blocks=max(1, nb // 32), k_min=1, k_max=max(112, nb // 32))
        policy = "router-on-Quest"
    else:                         # top-k 32 blocks: router-on-Quest, Quest or K-mean top-k
        m = args.policy
        sel = dict(mode={"router": "router", "quest": "quest", "topk": "topk"}[m], router_score="quest",
                   router_mode="quantile", router_grain="row", router_quantile=0.25, budget_blocks=16, k_min=1,
                   k_max=112)
        policy = {"router": "router-on-Quest", "quest": "Quest", "topk": "K-mean top-k"}[m]
    cfg = ops.SelectorConfig(**sel)
    k_base, kmax = ops.budget(cfg, S)
    model = decoder.TPDecoder(shape, cfg, world, rank, group=dist.group.WORLD if world > 1 else None,
                              seed=0, device=dev)
    gen = torch.Generator().manual_seed(1)
    ids_host = torch.randint(0, shape.vocab, (S,), generator=gen).pin_memory()
    ids = ids_host.to(dev)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def timed(n):
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            model.forward(ids)
        b.record(stream)
        torch.cuda.synchronize()
        barrier()
        t = torch.tensor([a.elapsed_time(b) / n], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for _ in range(args.warmup):
        model.forward(ids)
    sampler = ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else
                           os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
    sampler.start()
    time.sleep(0.25)
    ms = timed(args.steps)
    clocks = sampler.stop()
    # attention share of one forward (per-layer events; this rank)
    model.events = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(shape.layers)]
    model.forward(ids)
    torch.cuda.synchronize()
    attn_ms = sum(e[1].elapsed_time(e[2]) for e in model.events)
    model.events = None
    # end to end: token ids from pinned host memory, the last position's logits read back
    vl = model.layout.vocab1 - model.layout.vocab0
    host_out = torch.empty((vl,), dtype=torch.bfloat16).pin_memory()
    barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        d_ids = ids_host.to(dev, non_blocking=True)
        logits = model.forward(d_ids)
        host_out.copy_(logits[-1], non_blocking=True)
    b.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([a.elapsed_time(b) / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = te.item()
    dense_ms = None
    if not args.no_dense:
        model.attention = "dense"
        model.forward(ids)
        dense_ms = timed(max(1, min(args.steps, 2)))
        model.attention = "block_sparse"
    flops = shape.gemm_flops(S) + shape.dense_attn_flops(S)
    value = flops / (ms / 1e3) / 1e12
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    name = "Qwen2.5-7B" if args.workload == "cfg3" else "Qwen2.5-14B"
    # tensor work actually done: the GEMMs, and the sparse attention at about its
    # selected fraction (k_base..kmax of the visible blocks) -- the GEMMs dominate
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform random token ids, random-init weights)",
            "config": {"workload": f"{args.workload}-{S // 1024}K: full prefill of a random-init {name}-shaped decoder "
                                   f"({shape.layers} layers, hidden {shape.hidden}, {shape.heads}/{shape.kv_heads} "
                                   f"heads, d{shape.head_dim}, MLP {shape.intermediate}, vocab {shape.vocab}), "
                                   f"{policy} block 64 k_base={k_base} kmax={kmax} on every layer, "
                                   f"tensor parallel over KV-head groups, NCCL all-reduce after o_proj and down_proj",
                       "global_batch": 1, "seq_len": S, "parallelism": f"tp{world}" if world > 1 else "none",
                       "l2": "activations and weights larger than L2"},
            "prefill_ms": round(ms, 3), "tokens_per_s": round(S / (ms / 1e3), 1),
            "attention_ms_rank0": round(attn_ms, 3),
            "roofline": {"bound": "tensor", "kernel": "whole prefill (cuBLAS GEMMs + this package's attention)",
                         "achieved": round(shape.gemm_flops(S) / (ms / 1e3) / 1e12, 2), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(shape.gemm_flops(S) / (ms / 1e3) / 1e12 / peak, 4),
                         "peak_kind": f"bf16_tflops_sustained ({peak_kind})", "traffic": None,
                         "note": "achieved counts the GEMM FLOPs only"},
            "gpu_launches": None, "clocks": clocks,
            "e2e": {"value": round(flops / (e2e_ms / 1e3) / 1e12, 3), "unit": UNIT,
                    "h2d_bytes_per_step": S * 8, "d2h_bytes_per_step": vl * 2 * world, "ms_per_step": round(e2e_ms, 3)},
            "cpu_baseline": None}
    if dense_ms is not None:
        line["dense_ms"] = round(dense_ms, 3)
        line["dense_backend"] = "torch SDPA (enable_gqa), same model"
        line["ratio_vs_dense"] = round(ms / dense_ms, 4)
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(seq, tiles):
    """Rank-0 CPU leg: the oracle restatement on a bounded sample, all host cores."""
    import types
    a = types.SimpleNamespace(steps=1, warmup=0, gpus=1, ref_tiles=tiles)
    import io
    import contextlib
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        run_reference(a, seq)
    d = json.loads(buf.getvalue().strip().splitlines()[-1])
    return d["cpu_baseline"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ugbsa", choices=["ugbsa", "reference"])
    ap.add_argument("--seq", type=int, default=131072)
    ap.add_argument("--workload", default="attn-layer", choices=["attn-layer", "cfg5", "cfg3", "cfg4"],
                    help="attn-layer: the metric's 28/4-head d128 layer; cfg5: BASELINE config 5 (d256, 16/2 heads); "
                         "cfg3 / cfg4: full prefill of a Qwen2.5-7B / 14B-shaped decoder, tensor parallel")
    ap.add_argument("--policy", default="router", choices=["router", "quest", "topk"],
                    help="cfg4's selection policy (router-on-Quest, Quest, K-mean top-k)")
    ap.add_argument("--ref-tiles", type=int, default=32, help="tiles in the CPU sample")
    ap.add_argument("--no-dense", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--split", default="auto", choices=["auto", "grid", "heads", "rows"],
                    help="multi-GPU division of the layer (auto: grid when the ranks divide or are a multiple of "
                         "the KV heads, rows otherwise)")
    args = ap.parse_args()
    global WORKLOAD
    WORKLOAD = args.workload
    if args.warmup < 3 and args.impl == "ugbsa":
        args.warmup = 3
    if args.workload in ("cfg3", "cfg4"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the full-model workloads have no CPU reference "
                              "arm; the attention layer's is --workload attn-layer"}))
            return
        run_model(args)
        return
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        run_reference(args, args.seq)
        return
    run_gpu(args, args.seq)


if __name__ == "__main__":
    main()
