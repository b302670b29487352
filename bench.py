"""RCSA benchmark on B200: one Matrix-shaped DiT attention layer (config 2).

A step is one RCSA layer call: pooled-QK block selection + per-block int8
quantisation (one fused pass over Q/K) and the tcgen05 block-sparse
attention, on H=24 heads x d128, 3520 queries (4 frames of 880 tokens), 32
history + 4 current key frames, budget 8 blocks, block-causal.

Usage::

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--policy auto|int8|bf16] [--shard head|rollout]

Multi-GPU (torchrun, one process per GPU): ``--shard head`` (default) splits
the 24 heads of every call across the GPUs (24/12/6/3 per GPU at 1/2/4/8) and
all-gathers the bf16 head outputs over NCCL inside the timed step (strong
scaling: ``value`` is microseconds per layer call of the whole job, the
slowest rank's time); the same run also reports rollout sharding (every GPU
runs its own full call, no collective) under ``rollout``.  ``--shard
rollout`` makes that the headline instead.  ``--impl reference`` times the
reference's PyTorch path (a CPU port, ``oracle/cpu_reference.py``) on all
host cores, all 24 heads per step, on rank 0.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "RCSA int8 sparse-attn µs/call & % tensor-core peak; scaling at 1/2/4/8 B200"
BLOCK, BUDGET, HEADS, D = 880, 8, 24, 128
# kernels of one layer call: pooling + quantisation, selection, attention, and
# under the auto policy the code pass for the blocks int8 query blocks read
KERNELS_PER_CALL = {"auto": 4, "int8": 3, "bf16": 3}
HIST, CUR = 32, 4
# Algorithmic work of one config-2 attention call (every score pair of the
# budget-8 block-causal selection, 24 heads): int8 QK^T ops and bf16 P.V FLOP.
ALG_OPS_INT8 = ALG_OPS_BF16 = 199.83e9
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            return json.load(fh), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
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
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [int(r[1]) for r in rows]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": int(statistics.median(sm)), "sm_max_mhz": int(rows[0][2]),
                "samples": len(rows), "reasons": sorted(reasons)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def attention_ops(counts, qk_mode, block):
    """Algorithmic ops of one attention launch: (int8 QK^T ops, bf16 ops)."""
    pairs = counts.double() * block * block  # [B,H,nQb] score pairs
    qk = 2.0 * D * pairs
    pv = 2.0 * D * pairs
    if qk_mode is None:
        return 0.0, float(qk.sum() + pv.sum())
    m = qk_mode.double()
    return float((qk * m).sum()), float((qk * (1 - m)).sum() + pv.sum())


CONFIG2_WORKLOAD = ("config2: RCSA layer (select+int8 quant+block-sparse attention), H=24 d128, "
                    "Lq=3520 (4x880), 32+4 key frames, budget 8, block-causal")


def layer_config(world: int, shard: str) -> dict:
    """The ``config`` of both arms' lines (identical for the same N and shard)."""
    return {"workload": CONFIG2_WORKLOAD, "parallelism": f"{shard}-sharded x{world}",
            "l2": "inputs larger than L2 (Q+K 216 MB read per call by the selection pass)"}


def _cpu_layer_us(w, threads: int, repeats: int) -> float:
    """Median wall time of the reference's CPU path over all 24 heads."""
    import torch

    from oracle import cpu_reference

    torch.set_num_threads(threads)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        cpu_reference.rcsa_layer(w.q, w.k, w.v, BLOCK, BUDGET)
        times.append(time.perf_counter() - t0)
    return statistics.median(times) * 1e6


def run_reference(args, world, rank):
    """CPU reference arm: the reference's PyTorch path (selection + explicit
    softmax attention, all 24 heads per step) on all host cores, rank 0."""
    import torch

    from cast_b200 import workloads
    from oracle import cpu_reference

    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = workloads.config2()
    for _ in range(args.warmup):
        cpu_reference.rcsa_layer(w.q, w.k, w.v, BLOCK, BUDGET)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference.rcsa_layer(w.q, w.k, w.v, BLOCK, BUDGET)
    per_call_us = (time.perf_counter() - t0) / args.steps * 1e6
    line = {
        "impl": "reference", "metric": METRIC, "value": per_call_us, "unit": "us/call",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_call_us / 1000.0, "higher_is_better": False,
        "scaling": "strong" if args.shard == "head" else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded config 2: N(0,1)*U(0.5,2) per head)",
        "config": layer_config(world, args.shard),
        "cpu_baseline": {"value": per_call_us, "unit": "us/call", "cores": threads, "kind": "port",
                         "sample": f"the whole config-2 call (all 24 heads), {args.steps} timed steps"},
        "e2e": {"value": per_call_us, "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "timing": "host wall clock over the timed steps (the reference path runs on the CPU)",
    }
    print(json.dumps(line))
    return 0


def cpu_baseline_sample():
    """The reference's CPU path on this host: the whole config-2 call on all
    cores (median of 3) and on one core (one run), and the config-4 PAR
    correction restated in numpy (``oracle/par.py``) on all cores."""
    import torch

    from cast_b200 import workloads
    from oracle import par as opar

    threads = os.cpu_count() or 1
    w = workloads.config2()
    _cpu_layer_us(w, threads, 1)  # warm-up
    all_cores = _cpu_layer_us(w, threads, 3)
    one_core = _cpu_layer_us(w, 1, 1)
    torch.set_num_threads(threads)
    p4 = workloads.config4()
    full = p4.full_residual.float().numpy()
    act = p4.active_residual.float().numpy()
    opar.correct(full, act, p4.active_frames, p4.memory_length, 22, 40)
    t0 = time.perf_counter()
    opar.correct(full, act, p4.active_frames, p4.memory_length, 22, 40)
    par_us = (time.perf_counter() - t0) * 1e6
    return {"value": all_cores, "unit": "us/call", "cores": threads, "kind": "port",
            "sample": "the whole config-2 call (all 24 heads: selection + explicit-softmax attention), "
                      "median of 3",
            "one_core_us": one_core, "one_core_sample": "the same call on 1 thread, one run",
            "par_config4_us": par_us,
            "par_config4_sample": "config-4 FC-PASM correct() restated in numpy, one run, all cores"}


def attention_traffic(policy: str, heads: int, config: int):
    """DRAM bytes per attention launch from the committed ncu capture of the
    same workload, if that capture was taken of the current kernel source."""
    import hashlib

    path = os.path.join(ROOT, "profiles", "attention_traffic.json")
    key = f"config{config}_{policy}_{heads}heads"
    if not os.path.exists(path):
        return None, "no capture"
    with open(path) as fh:
        rec = json.load(fh).get(key)
    if rec is None:
        return None, f"no capture of {key}"
    with open(os.path.join(ROOT, "cast_b200", "csrc", "attention.cuh"), "rb") as fh:
        sha = hashlib.sha256(fh.read()).hexdigest()
    if sha != rec.get("attention_cuh_sha256"):
        return None, f"capture of {key} predates the current kernel source"
    return float(rec["dram_bytes_per_launch"]), f"ncu capture of {key}: {rec['command']}"


def _graph_us(fn, n, dev):
    """Mean device time of fn() replayed from a CUDA graph, n replays."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        fn()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    del graph
    return a.elapsed_time(b) / n * 1000.0


def compact_measure(dev, peaks, steps):
    """The compact path's packing with the RoPE phase at config-2 compact
    scale (31,680 tokens of 36 frames x 22x40, 24 heads, 880-token frame
    blocks; q/k/v 195 MB each, larger than L2), and the control-barycentric
    pair writer on config 4's frame (880 x 3072 fp32, targets 1 and 2 between
    anchors 0 and 3).  Graph replay; GB/s on the algorithmic bytes."""
    import numpy as np
    import torch

    from cast_b200 import barycentric, compact, workloads

    c = workloads.compact_case(heads=24, frames=36, hw=(22, 40), cell=(1, 22, 40), seed=9)
    order = torch.argsort(c.block_id, stable=True)  # frame blocks: full, no padding
    idx = order.to(torch.int32).to(dev)
    g = torch.Generator().manual_seed(9)
    phase = torch.polar(torch.ones(c.q.shape[1], 1, 64), torch.rand(c.q.shape[1], 1, 64, generator=g))
    qd, kd, vd, ph = c.q.to(dev), c.k.to(dev), c.v.to(dev), phase.to(dev)
    out = compact.pack(qd, kd, vd, idx, ph)
    n = max(10, steps)
    us_pack = _graph_us(lambda: compact.pack(qd, kd, vd, idx, ph, out=out), n, dev)
    pack_bytes = 6 * qd.numel() * 2
    act = torch.randn(1, 4, 880, 3072, generator=g).to(dev)
    wts = torch.softmax(torch.randn(1, 2, 2, generator=g), dim=-1).to(dev)
    prs = torch.tensor([[0, 1], [0, 1]], dtype=torch.int32, device=dev)
    tgs = torch.tensor([1, 2], dtype=torch.int32, device=dev)
    full = torch.zeros(1, 5, 880, 3072, device=dev)
    us_pair = _graph_us(lambda: barycentric.direct_control_barycentric_pair_write(
        act, wts, prs, tgs, full, arithmetic_mode="left_then_right_fma"), n, dev)
    pair_bytes = 4 * 880 * 3072 * 4  # two shared anchor frames read, two targets written
    lift = lift_measure(dev, n)
    del np
    return {
        "lift": lift,
        "compact_pack": {"us_per_call": us_pack, "algorithmic_bytes": pack_bytes,
                         "achieved_gbs": pack_bytes / us_pack / 1e3,
                         "frac": pack_bytes / us_pack / 1e3 / peaks["hbm_gbs"],
                         "workload": "31,680 tokens x 24 heads x 128, bf16, RoPE phase, 880-token blocks"},
        "pair_write": {"us_per_call": us_pair, "algorithmic_bytes": pair_bytes,
                       "achieved_gbs": pair_bytes / us_pair / 1e3,
                       "frac": pair_bytes / us_pair / 1e3 / peaks["hbm_gbs"],
                       "workload": "config-4 frame 880 x 3072 fp32, targets 1, 2 between anchors 0, 3; "
                                   "graph of one call (L2 holds the 43 MB, an upper bound)"},
        "note": "HBM peak measured; CUDA graph replay, device time",
    }


def lift_measure(dev, n):
    """The whole control-barycentric lift (``control_barycentric_residual_lift``:
    targets on the host, the weights kernel, the pair writer, the anchors
    copied in) on an 8-frame residual of 880 x 3072 fp32 rows, anchors 0, 3,
    5, 7, mouse and keyboard controls: wall clock per call including its host
    work and small index copies, synchronised every call."""
    import time

    import torch

    from cast_b200 import barycentric

    g = torch.Generator().manual_seed(12)
    frames, active = 8, (0, 3, 5, 7)
    act = torch.randn(1, len(active), 880, 3072, generator=g).to(dev)
    af = torch.tensor(active, device=dev)
    plucker = torch.randn(1, frames * 880, 6, generator=g).to(dev)
    mouse = torch.randn(1, 4 * frames - 3, 2, generator=g).to(dev)
    keyboard = (torch.rand(1, 4 * frames - 3, 4, generator=g) > 0.5).float().to(dev)

    def call():
        return barycentric.control_barycentric_residual_lift(
            act, af, frames, 0, None, plucker, mouse, keyboard, None, None, (1.0, 1.0, 1.0), True)

    for _ in range(3):
        call()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(n):
        call()
        torch.cuda.synchronize(dev)
    us = (time.perf_counter() - t0) / n * 1e6
    return {"us_per_call_wall": us, "targets": 4, "launches_per_call": 3,
            "workload": "8 frames x 880 x 3072 fp32, anchors 0, 3, 5, 7, mouse + keyboard controls",
            "note": "wall clock, synchronised per call: host targets, weights kernel, pair writer, "
                    "anchor copy"}


def swap_measure(dev, steps, cpu_leg=True):
    """The FC-PASM swap router's whole ``refine`` on a 24-head layer of pooled
    blocks: 32 memory blocks plus 4 current cells of 2x4 blocks, 64 keys,
    D=128, 16 selected per row, a published FC sketch, the factory's knobs
    (one round, one swap, same-bank, transport gate 0.5).  ``device_us``: the
    call's kernels (objective + gates: 2 launches; proxies, one round, the
    closing pass: 3) replayed from a CUDA graph; ``refine_us``: the Python
    call end to end (host gates, the launches, its one stats read, the
    record), wall clock.  Beside it the CPU oracle on the same call."""
    import time

    import torch

    from cast_b200 import swap_router, workloads

    w = workloads.swap_case(heads=24, memory_blocks=32, cells=4, spatial_shape=(2, 4), dim=128,
                            width=16, exact_frames=(0, 3), transport=True, seed=21)
    M = w.memory_blocks
    for e in w.transport["pairs"].values():
        e["theta"], e["affinity"] = e["theta"].to(dev), e["affinity"].to(dev)
        e["mean_affinity"] = e["mean_affinity"].to(dev)
    router = swap_router.FCPASMLocalCoordinateSwapRouter(swap_router.FCPASMSwapRoutingConfig(
        num_swap_rounds=1, swap_eps=0.10, max_swaps_per_call=1, same_bank_only=True,
        require_fc_transport=True, min_transport_affinity=0.5, active_layers=(22, 26)))
    sel = w.selected.to(dev)
    kw = dict(score=w.score.to(dev), pooled_value=w.pooled_value.to(dev), selected=sel,
              counts=w.counts.to(dev), local=w.local.to(dev), memory_blocks=M, spatial_shape=(2, 4),
              exact_current_frames=(0, 3), temporal_group_size=1, current_boundary=4,
              transport=w.transport, layer_index=22)
    _, rec = router.refine(**kw)
    us = _graph_us(lambda: router.enqueue(**kw), max(10, steps), dev)
    n = max(10, steps)
    router.refine(**kw)
    t0 = time.perf_counter()
    for _ in range(n):
        router.refine(**kw)
    refine_us = (time.perf_counter() - t0) / n * 1e6
    line = {"device_us": us, "refine_us": refine_us, "launches_per_call": 5,
            "status": rec["status"], "swaps": rec["swap_count"],
            "workload": "24 heads, 32 memory + 32 current pooled blocks, D=128, 16 selected, "
                        "FC transport, 1 round / 1 swap / same-bank",
            "note": "device_us: CUDA graph replay of the call's 5 kernels; refine_us: the whole Python "
                    "refine, wall clock, one host synchronisation per call"}
    if cpu_leg:
        from oracle import swap_router as osr
        tr_cpu = workloads.swap_case(heads=24, memory_blocks=32, cells=4, spatial_shape=(2, 4), dim=128,
                                     width=16, exact_frames=(0, 3), transport=True, seed=21)
        ops = {}

        def op(pair, x):
            key = (pair, round(float(x), 12))
            if key not in ops:
                ops[key] = swap_router.transport_operator(tr_cpu.transport, pair, spatial_shape=(2, 4),
                                                          exponent=x, device="cpu")[0].numpy()
            return ops[key]

        args = dict(score=tr_cpu.score.numpy(), pooled_value=tr_cpu.pooled_value.numpy(),
                    selected=tr_cpu.selected.numpy(), counts=tr_cpu.counts.numpy(),
                    local=tr_cpu.local.numpy(), memory_blocks=M, spatial=8, exact_frames=(0, 3), group=1,
                    boundary=4, config=osr.SwapConfig(num_swap_rounds=1, swap_eps=0.1, max_swaps_per_call=1,
                                                      same_bank_only=True), operator=op)
        osr.refine(**args)
        ops.clear()
        t0 = time.perf_counter()
        osr.refine(**args)
        line["cpu_oracle_us"] = (time.perf_counter() - t0) * 1e6
        line["cpu_oracle"] = ("numpy restatement (oracle/swap_router.py) with the torch transport operators, "
                              "same call, host cores")
    return line


def par_measure(dev, peaks, peak_src, steps):
    """PAR (FC-PASM) on BASELINE config 4: bf16 residual [1, 1+4, 880, 3072]
    (one memory frame), anchors = current frames 0 and 3, targets 1 and 2.
    One call replayed from a CUDA graph; GB/s on the algorithmic bytes (read
    the two anchor frames, write the two target frames)."""
    import torch

    from cast_b200 import par, workloads

    w = workloads.config4(device=dev)
    corr = par.FCPASMCorrector()
    corr.begin_model_call(chunk_index=1, step_index=0)
    full = w.full_residual.clone()
    act = w.active_residual.contiguous()
    frames = tuple(w.active_frames)
    kw = dict(layer_index=0, full_input=None, full_residual=full, active_residual=act,
              active_frames=torch.tensor(frames), memory_length=w.memory_length,
              spatial_height=w.height, spatial_width=w.width, active_frame_values=frames)
    for _ in range(3):
        corr.correct(**kw)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        corr.correct(**kw)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        corr.correct(**kw)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    n = max(20, steps)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) / n * 1000.0
    hw, c = full.shape[-2], full.shape[-1]
    alg = (2 + 2) * hw * c * full.element_size()
    gbs = alg / (us * 1e-6) / 1e9
    del graph
    return {"workload": "config4: FC-PASM, bf16 residual [1, 1+4, 880 (22x40), 3072], anchors 0 and 3, "
                        "targets 1 and 2", "us_per_call": us, "algorithmic_bytes": alg,
            "achieved_gbs": gbs, "peak_gbs": peaks["hbm_gbs"], "frac": gbs / peaks["hbm_gbs"],
            "note": f"HBM peak {peak_src}; CUDA graph replay of one correct() call, device time"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--policy", default="auto", choices=["auto", "int8", "bf16"])
    ap.add_argument("--shard", default="head", choices=["head", "rollout"])
    ap.add_argument("--gather", default="peer", choices=["peer", "fused", "ce", "nccl"],
                    help="head sharding: NCCL's all-gather after the attention (nccl), one streaming launch "
                         "of peer stores after it (peer) or peer stores in the attention's epilogue (fused)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the PAR / compact / swap-router lines (profiling runs)")
    ap.add_argument("--heads", type=int, default=HEADS,
                    help="heads of the config-2 layer (smaller values only for profiling captures)")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3],
                    help="2: the headline layer (default); 3: BASELINE config 3, 128 history frames, "
                         "anchor-only queries (Lq=1760), budget 16")
    ap.add_argument("--sweep", action="store_true",
                    help="BASELINE config 5 instead: 30 layers x 3 denoise steps x 8 rollouts of "
                         "config-2 layer calls per chunk (a step = one chunk)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch
    import torch.distributed as dist

    from cast_b200 import _lib
    from cast_b200 import distributed as cdist
    from cast_b200 import rcsa, workloads

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    peaks, peak_src = load_peaks()
    if args.sweep:
        return run_sweep(args, world, rank, local, dev, peaks, peak_src)

    if args.config == 3:
        w = workloads.config3(heads=args.heads)
    else:
        w = workloads.config2(heads=args.heads, seed=1)
    budget = w.budget
    stream = torch.cuda.current_stream(dev)

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return a.elapsed_time(b)

    def setup(lo, hi):
        q_h, k_h, v_h = (t[:, lo:hi].contiguous() for t in (w.q, w.k, w.v))
        q, k, v = q_h.to(dev), k_h.to(dev), v_h.to(dev)
        b_, h_, lq_, d_ = q.shape
        plan = rcsa.RCSAPlan(b_, h_, lq_, k.shape[2], d_, block_size=BLOCK, budget=budget,
                             policy=args.policy, device=dev)
        for _ in range(args.warmup):  # eager warm-up (the plan allocates nothing per call)
            plan(q, k, v)
        torch.cuda.synchronize()
        return (q_h, k_h, v_h), (q, k, v), plan

    # ---- the headline: this rank's share of one call (all heads, or H/N heads
    # plus the all-gather of the head outputs)
    head = args.shard == "head"
    lo, hi = cdist.head_range(args.heads, world, rank) if head else (0, args.heads)
    host_in, (q, k, v), plan = setup(lo, hi)
    h0 = time.perf_counter()
    for _ in range(5):
        plan(q, k, v)
    host_us = (time.perf_counter() - h0) / 5 * 1e6
    torch.cuda.synchronize()
    # one call = the plan's kernels captured once in a CUDA graph and replayed;
    # every replay recomputes everything from the input buffers
    g_all = plan.capture(q, k, v, "all")
    g_att = plan.capture(q, k, v, "attend")
    g_sel = plan.capture(q, k, v, "select")
    gathered = None
    if head and world > 1:
        gathered = torch.empty((world * q.shape[0], *q.shape[1:]), dtype=q.dtype, device=dev)

    def nccl_step():
        g_all.replay()
        if gathered is not None:
            dist.all_gather_into_tensor(gathered, plan.out)

    # Head sharding with the gather fused into the attention (default): every
    # rank's attention stores its rows into every rank's gathered buffer over
    # NVLink, then waits for the peers' rows; one CUDA graph per gathered
    # buffer, alternating.
    peer = None
    if gathered is not None and args.gather in ("peer", "fused", "ce"):
        peer = cdist.PeerGather(q.shape[0], q.shape[1], q.shape[2], q.shape[3], device=dev)
        peer_graphs, gather_graphs = [], []
        for par in (0, 1):
            for graphs, with_select in ((peer_graphs, True), (gather_graphs, False)):
                gph = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream(dev)
                side.wait_stream(stream)
                with torch.cuda.stream(side), torch.cuda.graph(gph, stream=side):
                    if with_select:
                        plan.select(q, k)
                    if args.gather == "fused":
                        plan.attend(q, k, v, out=peer.slot(par), peers=peer.peers(par))
                    elif args.gather == "ce":
                        plan.attend(q, k, v, out=peer.slot(par))
                        peer.send(par)
                    else:
                        plan.attend(q, k, v, out=peer.slot(par))
                        peer.push(par)
                    peer.wait()
                stream.wait_stream(side)
                graphs.append(gph)
        turn = [0]

        def step():
            peer_graphs[turn[0] & 1].replay()
            turn[0] += 1

        def gather_step():  # the attention with its gather and the wait, alone
            gather_graphs[turn[0] & 1].replay()
            turn[0] += 1
    else:
        step = nccl_step

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if gathered is not None and peer is None:  # the gathered heads are the single-call output
        g_all.replay()
        dist.all_gather_into_tensor(gathered, plan.out)
        torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    total_ms = timed(step, args.steps)
    clocks = sampler.stop()
    if peer is not None:
        _lib.check_device(stream.cuda_stream, "fused gather")
    att_ms = timed(g_att.replay, args.steps) / args.steps
    sel_ms = timed(g_sel.replay, args.steps) / args.steps
    gather_ms = nccl_ms = gather_call_ms = 0.0
    if gathered is not None:
        if peer is not None:
            gather_call_ms = timed(gather_step, args.steps) / args.steps
        gather_ms = timed(lambda: dist.all_gather_into_tensor(gathered, plan.out), args.steps) / args.steps
        if peer is not None:  # the same call with the NCCL all-gather after it, for comparison
            for _ in range(3):
                nccl_step()
            nccl_ms = timed(nccl_step, args.steps) / args.steps
            del peer_graphs, gather_graphs
            peer.close()
    sel = plan.selection()
    counts_cpu = sel.counts.cpu()
    mode_cpu = sel.qk_mode.cpu() if sel.qk_mode is not None else None

    # ---- rollout sharding at the same N: every GPU runs its own full call
    rollout_ms = None
    if world > 1 and head:
        _, (rq, rk, rv), rplan = setup(0, args.heads)
        g_roll = rplan.capture(rq, rk, rv, "all")
        for _ in range(3):
            g_roll.replay()
        rollout_ms = timed(g_roll.replay, args.steps) / args.steps
        del g_roll, rplan, rq, rk, rv

    # ---- end to end through the public API with host buffers: pinned host
    # inputs copied in, the plan call, the output copied back and checked,
    # every step
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (t.pin_memory() for t in host_in)
        hout = torch.empty(hq.shape, dtype=hq.dtype).pin_memory()
        b_, h_, lq_, d_ = q.shape
        host_plan = rcsa.RCSAHostPlan(b_, h_, lq_, k.shape[2], d_, block_size=BLOCK, budget=budget,
                                      policy=args.policy, groups=min(4, h_), device=dev)
        e_steps = max(3, min(10, args.steps))

        def e2e_step():
            host_plan(hq, hk, hv, hout)

        for _ in range(2):
            e2e_step()
        e2e_ms = timed(e2e_step, e_steps) / e_steps
        # bytes of the whole job: every rank copies its heads' Q, K and
        # selected value blocks in and its output out (the same selection
        # every step, so the last call's counts hold for each)
        moved = torch.tensor([host_plan.last_h2d_bytes, host_plan.last_d2h_bytes], dtype=torch.float64,
                             device=dev)
        if world > 1:
            dist.all_reduce(moved)
        e2e = {"ms": e2e_ms, "h2d": int(moved[0]), "d2h": int(moved[1]),
               "h2d_all_values": world * sum(t.numel() * t.element_size() for t in (hq, hk, hv))}
    extras = rank == 0 and world == 1 and not args.no_extras
    par_line = par_measure(dev, peaks, peak_src, args.steps) if extras else None
    compact_line = compact_measure(dev, peaks, args.steps) if extras else None
    swap_line = swap_measure(dev, args.steps, not args.no_cpu_baseline) if extras else None
    # the same layer call under the other QK^T precision policies (same inputs)
    policy_line = None
    if extras and args.config == 2:
        policy_line = {}
        for pol in ("int8", "bf16"):
            if pol == args.policy:
                continue
            pplan = rcsa.RCSAPlan(q.shape[0], q.shape[1], q.shape[2], k.shape[2], q.shape[3], block_size=BLOCK,
                                  budget=budget, policy=pol, device=dev)
            for _ in range(args.warmup):
                pplan(q, k, v)
            graphs = {part: pplan.capture(q, k, v, part) for part in ("all", "attend", "select")}
            for _ in range(3):
                graphs["all"].replay()
            policy_line[pol] = {part: timed(g.replay, args.steps) / args.steps * 1000.0
                                for part, g in graphs.items()}
            del graphs, pplan
        policy_line["unit"] = "us/call"
        policy_line["note"] = ("device time of the same layer call (all), its attention and its selection "
                               "under the other QK^T precision policies, CUDA graph replay")

    # ---- max over ranks
    vals = torch.tensor([total_ms, att_ms, e2e["ms"] if e2e else 0.0, sel_ms, gather_ms,
                         rollout_ms or 0.0, nccl_ms, gather_call_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, att_ms, e2e_ms, sel_ms, gather_ms, rollout_ms, nccl_ms, gather_call_ms = (
        float(x) for x in vals.tolist())
    ms_per_step = total_ms / args.steps
    value_us = ms_per_step * 1000.0

    # ---- roofline of the attention kernel on this rank's heads
    i8_ops, bf_ops = attention_ops(counts_cpu, mode_cpu, BLOCK)
    p_bf16 = peaks["bf16_tflops"] * 1e12
    p_i8 = 2.0 * p_bf16
    share = (hi - lo) / HEADS
    alg_i8, alg_bf = ALG_OPS_INT8 * share, ALG_OPS_BF16 * share
    t_alg = alg_i8 / p_i8 + alg_bf / p_bf16          # the fixed algorithmic roofline
    t_ww = i8_ops / p_i8 + bf_ops / p_bf16           # the work this launch chose
    att_s = att_ms * 1e-3
    traffic, traffic_src = attention_traffic(args.policy, hi - lo, args.config)
    int8_frac = float(mode_cpu.float().mean()) if mode_cpu is not None else 0.0
    sq_read = (q.numel() + k.numel()) * 2
    if args.policy == "auto" and sel.qk_mode is not None:
        # codes only for the blocks the int8 query blocks read, which the code
        # pass reads again (bf16) and writes (int8)
        idx = sel.indices.cpu()
        coded = 0
        for b in range(mode_cpu.shape[0]):
            for h in range(mode_cpu.shape[1]):
                kset = set()
                for i in range(mode_cpu.shape[2]):
                    if mode_cpu[b, h, i]:
                        coded += 1
                        kset.update(int(x) for x in idx[b, h, i, :counts_cpu[b, h, i]])
                coded += len(kset)
        sq_bytes = sq_read + coded * BLOCK * q.shape[-1] * 3
    else:
        sq_bytes = sq_read + (q.numel() + k.numel())  # bf16 read + int8 codes written

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value_us, "unit": "us/call", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": False, "scaling": "strong" if head else "weak",
        "vs_baseline": None, "dtype": "int8+bf16" if args.policy != "bf16" else "bf16",
        "data": ("synthetic (seeded config 2: N(0,1)*U(0.5,2) per head)" if args.config == 2 else
                 "synthetic (seeded config 3: N(0,1)*U(0.5,2) per head, linear drift over history frames)"),
        "config": (layer_config(world, args.shard) if args.config == 2 and args.heads == HEADS else
                   {"workload": f"config{args.config}, {args.heads} heads",
                    "parallelism": f"{args.shard}-sharded x{world}"}),
        "details": {"policy": args.policy, "int8_row_fraction": int8_frac, "heads_per_gpu": hi - lo},
        "attention_us": att_ms * 1000.0,
        "select_quant_us": sel_ms * 1000.0,
        "select_quant_roofline": {
            "bound": "hbm", "algorithmic_bytes": sq_bytes, "achieved_gbs": sq_bytes / (sel_ms * 1e-3) / 1e9,
            "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": sq_bytes / (sel_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
            "note": ("selection + quantisation kernels: Q+K bf16 read once; int8 codes written for every block "
                     "(int8/bf16 policy) or, under auto, only for the blocks int8 query blocks read (those read "
                     "again); pooled/RMS/scales ignored"),
        },
        "host_enqueue_us_eager": host_us,
        "timing": (f"CUDA graph replay of the {KERNELS_PER_CALL[args.policy]}-kernel layer call"
                   + ("" if gathered is None else
                      " with the head outputs' all-gather fused into the attention (peer stores over "
                      "NVLink) and the wait for the peers' rows" if args.gather == "fused" else
                      " + one launch streaming the head outputs into every peer over NVLink and the "
                      "wait for the peers' rows" if args.gather == "peer" else
                      " + NCCL all-gather of the head outputs")
                   + "; CUDA events on the launching stream, max over ranks"),
        "roofline": {
            "bound": "tensor", "achieved": (alg_i8 + alg_bf) / att_s / 1e12,
            "peak": (alg_i8 + alg_bf) / t_alg / 1e12, "unit": "TFLOP/s", "frac": t_alg / att_s,
            "traffic": traffic,
            "note": (f"attention kernel, this GPU's {hi - lo} heads; algorithmic work of the call "
                     f"({alg_i8:.4g} int8 QK^T ops + {alg_bf:.4g} bf16 P.V FLOP, all score pairs of the "
                     f"selection) at int8 = 2x bf16 and bf16 {peaks['bf16_tflops']} TFLOP/s ({peak_src} "
                     f"cuBLAS burst; no measured int8 peak); traffic: {traffic_src}"),
            "work_weighted": {"frac": t_ww / att_s, "ops_int8": i8_ops, "ops_bf16": bf_ops,
                              "note": "the same kernel against the work it chose (int8 QK^T only for "
                                      "the auto policy's int8 query blocks)"},
        },
        "par": par_line,
        "compact_and_lift": compact_line,
        "swap_router": swap_line,
        "other_policies": policy_line,
        "gpu_launches": (KERNELS_PER_CALL[args.policy]
                         + (0 if peer is None else 2 if args.gather == "peer" else
                            world if args.gather == "ce" else 1)) * args.steps,
        "clocks": clocks,
    }
    if gathered is not None:
        line["all_gather_us"] = gather_ms * 1000.0
        line["gather"] = args.gather
        if peer is not None:
            link_bytes = (world - 1) * q.numel() * 2  # this rank's heads to every other rank
            t_link = link_bytes / 770e9
            line["peer_gather_roofline"] = {
                "kernel_us": gather_call_ms * 1000.0, "nvlink_bytes_per_gpu": link_bytes,
                "link_us": t_link * 1e6, "compute_us": t_alg * 1e6,
                "frac": max(t_alg, t_link) / (gather_call_ms * 1e-3),
                "note": ("attention with its gather (fused into the epilogue, or the streaming launch "
                         "after it) and the peers' wait (CUDA graph, max over ranks) against the slower of "
                         "its tensor-core roofline and its NVLink bytes at the measured 770 GB/s per "
                         "direction")}
            line["nccl_gather_value"] = {
                "value": nccl_ms * 1000.0, "unit": "us/call",
                "note": "the same call with a separate NCCL all-gather after it, max over ranks"}
        line["rollout"] = {"value": rollout_ms * 1000.0 / world, "unit": "us/call",
                           "note": f"rollout sharding: each of {world} GPUs runs its own full call, no "
                                   "collective; value = slowest GPU's call time / N"}
    if e2e:
        line["e2e"] = {"value": e2e_ms * 1000.0, "unit": "us/call",
                       "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                       "h2d_bytes_all_values": e2e["h2d_all_values"],
                       "path": "RCSAHostPlan: pinned host q and k in, each head group's selection read back "
                               "and only its selected value blocks copied in, copies overlapped with the "
                               "compute, output copied back and the device error word checked"
                               + (" (each rank its own heads, in parallel)" if world > 1 else "")}
    if not args.no_cpu_baseline and world == 1 and args.config == 2 and args.heads == HEADS:
        line["cpu_baseline"] = cpu_baseline_sample()
    print(json.dumps(line))
    return 0


SWEEP_LAYERS, SWEEP_STEPS, SWEEP_ROLLOUTS = 30, 3, 8


def run_sweep(args, world, rank, local, dev, peaks, peak_src):
    """per chunk, 30 layers x 3 denoise steps x 8 rollouts
    = 720 config-2 layer calls (random-init layers: two seeded input sets of
    the layer shape, alternating, each far larger than L2).  ``--shard head``
    gives every GPU H/N heads of every call and all-gathers the bf16 head
    outputs after each call on NCCL's stream (async), overlapped with the next
    call's selection and attention; ``--shard rollout`` gives every GPU 8/N
    rollouts with all heads and no collective.  Each layer call is one CUDA
    graph replay; a ring of three output / gather buffers keeps in-flight
    gathers off the buffer the next call writes."""
    import torch
    import torch.distributed as dist

    from cast_b200 import distributed as cdist
    from cast_b200 import rcsa, workloads

    head = args.shard == "head"
    if not head and SWEEP_ROLLOUTS % world:
        raise SystemExit(f"{SWEEP_ROLLOUTS} rollouts do not split over {world} GPUs")
    lo, hi = cdist.head_range(args.heads, world, rank) if head else (0, args.heads)
    calls = SWEEP_LAYERS * SWEEP_STEPS * (SWEEP_ROLLOUTS if head else SWEEP_ROLLOUTS // world)
    sets = []
    for i in range(2):
        w = workloads.config2(heads=args.heads, seed=11 + i + (0 if head else 100 * rank))
        sets.append(tuple(t[:, lo:hi].contiguous().to(dev) for t in (w.q, w.k, w.v)))
    b_, h_, lq_, d_ = sets[0][0].shape
    plan = rcsa.RCSAPlan(b_, h_, lq_, sets[0][1].shape[2], d_, block_size=BLOCK, budget=BUDGET,
                         policy=args.policy, device=dev)
    ring = 3
    outs = [torch.empty_like(sets[0][0]) for _ in range(ring)]
    gath = [torch.empty((world * b_, h_, lq_, d_), dtype=torch.bfloat16, device=dev)
            for _ in range(ring)] if head and world > 1 else None
    graphs = {(si, r): plan.capture(*sets[si], "all", out=outs[r]) for si in range(2) for r in range(ring)}
    works = [None] * ring
    stream = torch.cuda.current_stream(dev)

    def chunk():
        for c in range(calls):
            r = c % ring
            if works[r] is not None:  # the gather that last read this slot
                works[r].wait()
                works[r] = None
            graphs[(c % 2, r)].replay()
            if gath is not None:
                works[r] = dist.all_gather_into_tensor(gath[r], outs[r], async_op=True)
        for r in range(ring):
            if works[r] is not None:
                works[r].wait()
                works[r] = None

    for _ in range(args.warmup):
        chunk()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        chunk()
    e.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = torch.tensor([a.elapsed_time(e) / args.steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms_chunk = float(ms.item())
    sel = plan.selection()
    i8_ops, bf_ops = attention_ops(sel.counts.cpu(), sel.qk_mode.cpu() if sel.qk_mode is not None else None, BLOCK)
    p_bf16 = peaks["bf16_tflops_sustained"] * 1e12
    ideal_ms = calls * (i8_ops / (2.0 * p_bf16) + bf_ops / p_bf16) * 1e3
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": "config 5 sweep: ms per chunk (30 layers x 3 denoise steps x 8 rollouts of the config-2 layer)",
        "value": ms_chunk, "unit": "ms/chunk", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": False, "scaling": "strong", "dtype": "int8+bf16", "vs_baseline": None,
        "data": "synthetic (two seeded config-2 input sets, alternating per call)",
        "config": {"workload": "config5", "parallelism": f"{args.shard}-sharded x{world}",
                   "heads_per_gpu": hi - lo, "calls_per_gpu_per_chunk": calls, "policy": args.policy},
        "ms_per_layer_call_per_gpu": ms_chunk / calls,
        "roofline": {"bound": "tensor", "ideal_ms_per_gpu": ideal_ms, "frac": ideal_ms / ms_chunk,
                     "note": f"selection + attention of every call vs the attention tensor work at the "
                             f"{peak_src} sustained bf16 peak ({peaks['bf16_tflops_sustained']} TFLOP/s, int8 = 2x)"},
        "collective": ("all-gather of bf16 head outputs after every call on NCCL's stream, overlapped with "
                       "the next call" if gath is not None else "none"),
        "gpu_launches": KERNELS_PER_CALL[args.policy] * calls * args.steps,
        "clocks": clocks,
    }
    print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
