#!/usr/bin/env python
"""Benchmark of the B200 quantised MoE block: MoE-layer prefill tok/s and
decode µs/layer, each with its roofline fraction.

Headline (every N, N=1 included): the expert-parallel prefill step — 36 MoE
layers of the Qwen3-Next-80B-A3B shape (H=2048, 512 routed experts + 1
shared, I=512, top-10, int4 g64 affine weights, 32.6 GB, so L2 never holds
them), 8192 tokens per step split over the N ranks, router logits drawn so
expert popularity follows Zipf(1.1).  Experts are sharded over the ranks by a
load-balanced placement; tokens travel to their experts' owners and back
over NVLink peer memory.  value = global tokens per second (strong scaling).
The same code path runs at N=1 (a one-rank exchange).  Each rank checks a
token subset of layer 0 bit for bit against the single-GPU block
(`ep_check`).

At N=1 the same JSON line also carries: the 48-layer decode sweep (T in
{1,2,4,8,32}) with its HBM roofline and e2e, the cold-prefill block (H=3072,
512 experts, I=768, shared 3072) at T in {4096, 16384, 65536}, the CPU
baseline (the oracle on the host cores) and the single-layer CPU timing.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl titan|reference]
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG2 = dict(H=2048, E=512, k=10, I=512, Is=512)
CFG3 = dict(H=3072, E=512, k=10, I=768, Is=3072)
DECODE_T = (1, 2, 4, 8, 32)
HEADLINE_T = 1
EXPERT_BYTES_CFG2 = 1_769_472      # one expert's int4 weights + bf16 scales/biases


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("titan", "reference"), default="titan")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--prefill-T", default="4096,16384,65536", help="comma list; empty to skip")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--traffic-file", default=os.path.join(ROOT, "profiles", "traffic.txt"))
    ap.add_argument("--profile", choices=("decode", "prefill", "ep"), default=None,
                    help="run a small untimed case for an ncu capture and exit")
    ap.add_argument("--gemm-kernel", type=int, default=0,
                    help="prefill grouped GEMMs: 0 tcgen05 (default), 1 mma.sync baseline")
    ap.add_argument("--spec-streams", type=int, default=64, help="config 5: streams per step")
    ap.add_argument("--spec-draft", type=int, default=3, help="config 5: draft tokens per stream")
    ap.add_argument("--spec-layers", type=int, default=48, help="config 5: layers per step")
    ap.add_argument("--headline-only", action="store_true",
                    help="only the expert-parallel headline (no decode / prefill / CPU extras)")
    ap.add_argument("--ref-tokens", type=int, default=64,
                    help="tokens per oracle call of the CPU baseline and the reference arm")
    ap.add_argument("--ep-tokens", type=int, default=8192, help="ep: global tokens per step")
    ap.add_argument("--ep-layers", type=int, default=36, help="ep: layers per step")
    ap.add_argument("--ep-placement", choices=("balanced", "contiguous"), default="balanced",
                    help="ep: balanced = experts placed by load measured on a separate "
                         "calibration batch (balanced_placement); contiguous = E/N in order")
    ap.add_argument("--ep-exchange", choices=("peer", "nccl"), default="peer",
                    help="ep: peer = NVLink stores into IPC-mapped buffers with the return "
                         "fused into the down GEMM; nccl = two all-to-alls per layer")
    return ap.parse_args()


# ----------------------------------------------------------------- plumbing

def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class Clocks:
    """nvidia-smi sampling during a timed region (every 200 ms)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs"), d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


def measured_peaks_all():
    """HBM GB/s and dense bf16 TF/s, burst and sustained (MEASURED_PEAKS.json,
    else the pool's earlier measurement)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    d = json.load(open(p)) if os.path.exists(p) else {}
    return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16_tflops": d.get("bf16_tflops", 1590.0),
            "bf16_tflops_sustained": d.get("bf16_tflops_sustained", 1400.0),
            "source": "measured" if d else "fallback"}


def read_traffic(path):
    """profiles/traffic.txt: lines 'kernel_stage: <dram bytes per launch>' from
    an ncu capture (see the summary next to it)."""
    out = {}
    if os.path.exists(path):
        for l in open(path):
            if ":" in l and not l.lstrip().startswith("#"):
                k, v = l.split(":", 1)
                try:
                    out[k.strip()] = float(v.split()[0])
                except (ValueError, IndexError):
                    pass
    return out


# --------------------------------------------------------------- workloads

def build_decode_layers(n_layers, device, seed):
    import torch
    from titan_b200 import SparseMoeBlock
    torch.manual_seed(seed)
    c = CFG2
    return [SparseMoeBlock(c["H"], c["E"], c["k"], c["I"], c["Is"], device=device,
                           weight_std=0.02, router_std=0.02) for _ in range(n_layers)]


def decode_opts():
    from titan_b200 import _lib
    o = _lib.Options()
    o.min_tokens, o.int8_prefill, o.down_int8, o.wsum_mode = 512, 1, 1, 0
    return o


def stage_profile(calls, reps=3):
    """Per-kernel device time via the library's stage hook: an event before
    every launch and one after each call, all enqueued behind a sleep kernel
    so the GPU never waits for the host between them."""
    import torch
    from titan_b200 import _lib
    marks = []

    def hook(name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((name, ev))

    torch.cuda.synchronize()
    torch.cuda._sleep(int(4e8))
    _lib.set_stage_hook(hook)
    try:
        for _ in range(reps):
            for fn in calls:
                fn()
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append(("<end>", ev))
    finally:
        _lib.set_stage_hook(None)
    torch.cuda.synchronize()
    agg = {}
    for (name, a), (_, b) in zip(marks, marks[1:]):
        if name == "<end>":
            continue
        t, n = agg.get(name, (0.0, 0))
        agg[name] = (t + a.elapsed_time(b), n + 1)
    launches = sum(1 for n, _ in marks if n != "<end>") // reps
    return {k: {"ms_total": t / reps, "launches": n // reps, "us_per_launch": 1000 * t / n}
            for k, (t, n) in agg.items()}, launches


def time_graph(fn, steps, warmup, world):
    """Capture fn in a CUDA graph; time `steps` replays with CUDA events."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(max(warmup, 3)):
        g.replay()
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = a.elapsed_time(b) / steps
    del g
    return max_over_ranks(ms, world)


def decode_bytes(blocks, x, opts):
    """Algorithmic bytes of one step: each layer streams its distinct selected
    experts, the shared expert, the router and the activations once."""
    import torch
    c = CFG2
    total, uniq = 0, []
    for b in blocks:
        _, idx, _ = b(x, options=opts, return_routing=True)
        u = int(torch.unique(idx).numel())
        uniq.append(u)
        T = x.shape[0]
        total += (u + 1) * EXPERT_BYTES_CFG2 + c["E"] * c["H"] * 2 + c["H"] * 2 + 2 * T * c["H"] * 2
    return total, uniq


def bench_decode(args, world, device, blocks):
    import torch
    opts = decode_opts()
    gen = torch.Generator(device=device).manual_seed(7)
    hbm, _, src = measured_peaks()
    sweep, head = {}, None
    for T in DECODE_T:
        x = torch.randn(T, CFG2["H"], generator=gen, device=device).to(torch.bfloat16)

        def step(x=x):
            for b in blocks:
                b(x, options=opts)

        ms = time_graph(step, args.steps, args.warmup, world)
        nbytes, uniq = decode_bytes(blocks, x, opts)
        us = 1000 * ms / len(blocks)
        gbs = nbytes / (ms * 1e-3) / 1e9
        sweep[str(T)] = {"us_per_layer": round(us, 3), "ms_per_step": round(ms, 4),
                         "GBps": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
                         "unique_experts_mean": round(float(np.mean(uniq)), 1),
                         "bytes_per_layer": int(nbytes / len(blocks))}
        if T <= 4:
            # the same step on the three-launch pipeline (options.decode_kernel = 1)
            o1 = decode_opts()
            o1.decode_kernel = 1

            def step1(x=x, o1=o1):
                for b in blocks:
                    b(x, options=o1)

            ms1 = time_graph(step1, args.steps, args.warmup, world)
            sweep[str(T)]["three_launch_us_per_layer"] = round(1000 * ms1 / len(blocks), 3)
        if T == HEADLINE_T:
            head = (x, ms, us, nbytes)
    return blocks, opts, sweep, head


def bench_e2e(blocks, opts, T, steps, warmup, world):
    """The same decode through the public API with a pinned host->device copy
    of every layer's input and a device->host read of its output."""
    import torch
    H = CFG2["H"]
    xh = torch.randn(T, H).to(torch.bfloat16).pin_memory()
    yh = torch.empty(len(blocks), T, H, dtype=torch.bfloat16).pin_memory()
    dev = blocks[0].gate_weight.device

    def step():
        for i, b in enumerate(blocks):
            xd = xh.to(dev, non_blocking=True)
            y = b(xd, options=opts)
            yh[i].copy_(y, non_blocking=True)

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1000 / steps
    barrier(world)
    ms = max_over_ranks(max(a.elapsed_time(b) / steps, wall), world)
    per = T * H * 2 * len(blocks)
    return {"value": round(1000 * ms / len(blocks), 3), "unit": "us/layer",
            "h2d_bytes_per_step": per, "d2h_bytes_per_step": per, "ms_per_step": round(ms, 4)}


def prefill_ops_per_token(c):
    return 2 * c["k"] * (c["H"] * 2 * c["I"] + c["I"] * c["H"]) + \
        2 * (c["H"] * 2 * c["Is"] + c["Is"] * c["H"]) + 2 * c["H"] * c["E"]


def bench_prefill(args, world, device):
    """The cold-prefill block (H=3072, 512 experts, I=768, top-10, shared
    expert 3072) at each --prefill-T on the default persistent tile kernel, and
    the swap-AB kernel at the first T: ms, tok/s, TOP/s and the fraction of
    the measured dense bf16 peak (the kernels issue f16 MMAs; the nominal
    int8 fraction is given for context)."""
    import torch
    from titan_b200 import SparseMoeBlock, _lib
    Ts = [int(t) for t in args.prefill_T.split(",") if t.strip()]
    if not Ts:
        return {}
    peaks = measured_peaks_all()
    c = CFG3
    torch.manual_seed(99)
    blk = SparseMoeBlock(c["H"], c["E"], c["k"], c["I"], c["Is"], device=device, weight_std=0.02)
    blk.prepare()
    out = {"ops_per_token": prefill_ops_per_token(c)}
    runs = [(T, 0) for T in Ts] + [(Ts[0], 2)]
    for T, kernel in runs:
        o = _lib.Options()
        o.min_tokens, o.int8_prefill, o.down_int8, o.wsum_mode = 512, 1, 1, 0
        o.gemm_kernel = kernel
        x = torch.randn(T, c["H"], device=device).to(torch.bfloat16)
        for _ in range(max(args.warmup, 3)):
            blk(x, options=o)
        torch.cuda.synchronize()
        steps = max(3, min(args.steps, 10 if T <= 16384 else 4))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            blk(x, options=o)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        ops = prefill_ops_per_token(c) * T
        tops = ops / (ms * 1e-3) / 1e12
        stages, launches = stage_profile([lambda: blk(x, options=o)], reps=1)
        key = str(T) if kernel == 0 else f"{T}_swap_ab_kernel"
        out[key] = {"gemm": "tcgen05 persistent tile (TMA)" if kernel == 0 else "tcgen05 swap-AB persistent",
                    "ms": round(ms, 4), "tok_per_s": round(T / (ms * 1e-3), 1),
                    "TOPs": round(tops, 2),
                    "frac_of_measured_bf16_peak": round(tops / peaks["bf16_tflops"], 4),
                    "frac_int8_nominal_4500": round(tops / 4500.0, 4),
                    "gpu_launches": launches,
                    "stages_us": {k: round(v["us_per_launch"], 2) for k, v in stages.items()}}
        gu = stages.get("gemm_gate_up")
        if gu:
            fl = 2.0 * T * c["k"] * 2 * c["I"] * c["H"]
            out[key]["gemm_gate_up_TFLOPs"] = round(fl / (gu["us_per_launch"] * 1e-6) / 1e12, 1)
        del x
        torch.cuda.empty_cache()
    del blk
    torch.cuda.empty_cache()
    return out


def zipf_router_(blk, gen, s=1.1):
    """Expert popularity ~ Zipf(s): column 0 of the router carries
    -s*log(rank) for a seeded random ranking of the experts (the tokens'
    x[:, 0] is 1), the other columns N(0, 1.28/sqrt(H)) so that every
    logit gets noise of the Gumbel's spread and top-k approximates sampling
    k experts without replacement from the Zipf law."""
    import torch
    E, H = blk.gate_weight.shape
    perm = torch.randperm(E, generator=gen).to(blk.gate_weight.device)
    bias = torch.empty(E, device=blk.gate_weight.device)
    bias[perm] = -s * torch.log(torch.arange(1, E + 1, device=bias.device, dtype=torch.float32))
    w = torch.randn(E, H, generator=gen).to(blk.gate_weight.device) * (1.28 / math.sqrt(H - 1))
    w[:, 0] = bias
    with torch.no_grad():
        blk.gate_weight.copy_(w.to(torch.bfloat16))


def run_ep(args, world, rank, local):
    """Config 4: expert parallelism over the N ranks, strong scaling.  Every
    rank builds the same layers (same seeds) and keeps experts
    [rank*E/N, (rank+1)*E/N); it serves ep_tokens/N tokens per layer: router,
    shared expert and weighted sum on its own tokens, the routed experts of
    the tokens of every rank that chose one of its experts (rows stored into
    the owners' peer-mapped buffers, expert outputs stored back by the down
    GEMM's epilogue; --ep-exchange nccl: two all-to-alls per layer).
    value = global tokens per second."""
    import torch
    from titan_b200 import SparseMoeBlock, _lib
    from titan_b200.expert_parallel import ExpertParallelMoE
    import torch.distributed as dist
    _lib.load()
    device = torch.device("cuda", torch.cuda.current_device())
    own_group = not dist.is_initialized()
    if own_group:                     # N=1: a one-rank group, so the same code path runs
        import socket
        so = socket.socket()
        so.bind(("127.0.0.1", 0))
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(so.getsockname()[1]))
        so.close()
        dist.init_process_group("nccl", rank=0, world_size=1,
                                timeout=datetime.timedelta(seconds=300))
    try:
        return _run_ep(args, world, rank, local, device)
    finally:
        if own_group:
            dist.destroy_process_group()


def run_spec_group(args, world, rank, local):
    """run_spec inside a process group (a one-rank group at N=1)."""
    import torch
    import torch.distributed as dist
    device = torch.device("cuda", torch.cuda.current_device())
    own_group = not dist.is_initialized()
    if own_group:
        import socket
        so = socket.socket()
        so.bind(("127.0.0.1", 0))
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(so.getsockname()[1])
        so.close()
        dist.init_process_group("nccl", rank=0, world_size=1,
                                timeout=datetime.timedelta(seconds=300))
    try:
        return run_spec(args, world, rank, local, device)
    finally:
        if own_group:
            dist.destroy_process_group()


def _run_ep(args, world, rank, local, device):
    """Returns the measurement dict of the config-4 expert-parallel step on
    this rank (the caller prints rank 0's)."""
    import torch
    from titan_b200 import SparseMoeBlock, _lib, ops
    from titan_b200.expert_parallel import ExpertParallelMoE, balanced_placement
    c = CFG2
    if args.ep_tokens % world:
        raise SystemExit(f"--ep-tokens {args.ep_tokens} does not split over {world} ranks")
    T = args.ep_tokens // world
    epr = c["E"] // world
    ex = None
    if args.ep_exchange == "peer":
        from titan_b200.expert_parallel import PeerExchange
        ex = PeerExchange(T, c["H"], c["k"], device=device)
    gen = torch.Generator(device=device).manual_seed(9000 + rank)
    x = torch.randn(T, c["H"], generator=gen, device=device)
    x[:, 0] = 1.0
    x = x.to(torch.bfloat16)
    layers, full0, pairs_r0 = [], None, []
    for l in range(args.ep_layers):
        torch.manual_seed(4321 + l)
        blk = SparseMoeBlock(c["H"], c["E"], c["k"], c["I"], c["Is"], device=device,
                             weight_std=0.02)
        zipf_router_(blk, torch.Generator().manual_seed(777 + l))
        placement = None
        if args.ep_placement == "balanced":
            # expert load from a calibration batch (other tokens than the
            # timed ones), summed over the ranks
            gc = torch.Generator(device=device).manual_seed(7000 + 97 * l + rank)
            xc = torch.randn(T, c["H"], generator=gc, device=device)
            xc[:, 0] = 1.0
            ic, _ = ops.router_topk(xc.to(torch.bfloat16), blk.gate_weight, c["k"])
            load = torch.bincount(ic.reshape(-1).long(), minlength=c["E"]).to(torch.int64)
            if world > 1:
                import torch.distributed as dist
                dist.all_reduce(load)
            placement = balanced_placement(load.cpu().tolist(), world)
        ep = ExpertParallelMoE(blk, exchange=ex, placement=placement)
        layers.append(ep)
        # pairs each rank's experts serve in this layer (for the GEMM roofline)
        il, _ = ops.router_topk(x, blk.gate_weight, c["k"])
        owner = (ep.place[il.long()].long() if ep.place is not None else il.long()) // epr
        cnt = torch.bincount(owner.reshape(-1), minlength=world).to(torch.int64)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(cnt)
        pairs_r0.append(int(cnt[0]))
        if l == 0:
            full0 = blk                       # the single-GPU block of layer 0, for ep_check
        del blk
    torch.cuda.empty_cache()
    opts = _lib.Options()
    opts.min_tokens, opts.int8_prefill, opts.down_int8, opts.wsum_mode = 1, 1, 1, 0
    idx, _ = ops.router_topk(x, layers[0].gate_weight, c["k"])
    dest = (idx.long() // epr) if layers[0].place is None else \
        (layers[0].place[idx.long()].long() // epr)
    member = torch.zeros(T, world, dtype=torch.bool, device=device)
    member.scatter_(1, dest, True)
    ranks_per_token = float(member.sum(1).float().mean())
    counts = torch.bincount(idx.reshape(-1).long(), minlength=c["E"]).float()
    top_share = float(counts.sort(descending=True).values[:10].sum() / counts.sum())

    def step():
        for ep in layers:
            ep(x, options=opts)

    torch.cuda.synchronize()
    barrier(world)                    # ranks start together (bounded device waits)
    clk = Clocks(local).__enter__()
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    clk.__exit__(None, None, None)
    ms = max_over_ranks(a.elapsed_time(b) / args.steps, world)
    # phase breakdown of one more step (events between phases, summed over layers)
    marks_all = []
    for ep in layers:
        marks = []
        ep(x, options=opts, marks=marks)
        marks_all.append(marks)
    torch.cuda.synchronize()
    phases = {}
    for marks in marks_all:
        for (_, a0), (name, b0) in zip(marks, marks[1:]):
            phases[name] = phases.get(name, 0.0) + a0.elapsed_time(b0)
    phases = {k: round(1000 * v / len(layers), 1) for k, v in phases.items()}
    # per-kernel device time of one step (events before every launch, the
    # queue kept full behind a sleep kernel): the dominant kernel's roofline
    barrier(world)
    stages, launches = stage_profile([step], reps=1)
    barrier(world)
    I, H, Is = c["I"], c["H"], c["Is"]
    pairs = sum(pairs_r0) / len(pairs_r0) if rank == 0 else None
    flops = {"gemm_gate_up": (2.0 * pairs * 2 * I * H) if pairs else None,
             "gemm_down": (2.0 * pairs * H * I) if pairs else None,
             "gemm_shared_gate_up": 2.0 * T * 2 * Is * H,
             "gemm_shared_down": 2.0 * T * H * Is}
    _, _, peak_src = measured_peaks()
    peaks = measured_peaks_all()
    dom = max(stages.items(), key=lambda kv: kv[1]["ms_total"])
    gemms = {k: v for k, v in stages.items() if flops.get(k)}
    top = max(gemms.items(), key=lambda kv: kv[1]["ms_total"]) if gemms else None
    roof = None
    if top is not None:
        name, st = top
        ach = flops[name] / (st["us_per_launch"] * 1e-6) / 1e12
        pk = peaks["bf16_tflops_sustained"]
        traffic = read_traffic(args.traffic_file)
        roof = {"kernel": name, "bound": "tensor", "achieved": round(ach, 1), "peak": pk,
                "unit": "TFLOP/s", "frac": round(ach / pk, 4),
                "peak_source": f"{peak_src} bf16 sustained (a kernel timed inside a long step)",
                "algorithmic_flops_per_launch": flops[name],
                "us_per_launch": round(st["us_per_launch"], 2),
                "launches_per_step": st["launches"],
                "dominant_of_step": dom[0],
                # captured at N = 1 (one rank serves every expert); at N > 1 a
                # rank's launch reads another weight set, so none is claimed
                "traffic": traffic.get(f"{name}_ep") if world == 1 else None,
                "note": "f16 MMA per 64-wide group (exact int8 x int4 sums) and the "
                        "reference's fp32 rescale; flops = 2 x routed pairs of rank 0 x N x K, "
                        "no padding counted"}
    # the public API end to end: the step's tokens copied in from pinned host
    # memory, the last layer's output copied back, every step
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()

    def step_e2e():
        xd = xh.to(device, non_blocking=True)
        y = None
        for ep in layers:
            y = ep(xd, options=opts)
        yh.copy_(y, non_blocking=True)

    for _ in range(2):
        step_e2e()
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    ke = max(3, args.steps // 2)
    for _ in range(ke):
        step_e2e()
    b.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1000 / ke
    barrier(world)
    ms_e2e = max_over_ranks(max(a.elapsed_time(b) / ke, wall), world)
    e2e = {"value": round(args.ep_tokens / (ms_e2e * 1e-3), 1), "unit": "tok/s",
           "h2d_bytes_per_step": args.ep_tokens * H * 2,
           "d2h_bytes_per_step": args.ep_tokens * H * 2, "ms_per_step": round(ms_e2e, 4),
           "api": "ExpertParallelMoE.forward over the layers, pinned host x in, last y out"}
    # in-run correctness: a token subset of layer 0's expert-parallel output
    # against the single-GPU block on the same tokens, bit for bit
    n_chk = min(64, T)
    y_ep = layers[0](x, options=opts)[:n_chk]
    y_one = full0(x[:n_chk].contiguous(), options=opts)
    diff = int((y_ep.view(torch.int16) != y_one.view(torch.int16)).sum())
    ep_check = {"layer": 0, "tokens": n_chk, "bit_identical": diff == 0, "mismatches": diff,
                "against": "SparseMoeBlock.forward on one GPU, same tokens and options"}
    ok = torch.tensor([1 if diff == 0 else 0], device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    ep_check["all_ranks_bit_identical"] = bool(int(ok) == 1)
    if ex is not None:
        ex.check()                    # no device wait gave up
        ex.close()
    del layers, full0
    torch.cuda.empty_cache()
    return {"ms": ms, "value": round(args.ep_tokens / (ms * 1e-3), 1), "T_rank": T,
            "phases": phases, "roofline": roof, "gpu_launches": launches * args.steps,
            "e2e": e2e, "ep_check": ep_check, "clocks": clk.summary(),
            "routing": {"ranks_per_token": round(ranks_per_token, 2),
                        "top10_expert_share": round(top_share, 4),
                        "pairs_rank0_per_layer": round(pairs, 1) if pairs else None},
            "stages_us": {k: round(v["us_per_launch"], 1) for k, v in stages.items()}}


def spec_tokens(streams, draft, H, E, k, shared=7, s=1.2, seed=0):
    """Tokens of a batched speculative-decode verify step with prescribed
    routing: `streams` streams of 1 + `draft` tokens; expert popularity
    follows Zipf(s) over a seeded ranking; the tokens of a stream share
    `shared` of their k experts (drawn per stream) and draw the rest per
    token.  With the one-hot router of spec_router (logit of expert e =
    x[:, e]) the chosen experts get distinct logits in [3, 3 + k/8) and every
    other logit stays below 2, so the top-k sets are known exactly (no bf16
    ties at the boundary).  Returns x [streams, 1 + draft, H] fp32 and the
    sets [streams * (1 + draft), k] (ascending)."""
    rng = np.random.default_rng(seed)
    Tq = 1 + draft
    rank = rng.permutation(E)
    p = 1.0 / np.arange(1, E + 1) ** s
    p /= p.sum()
    x = rng.standard_normal((streams * Tq, H)).astype(np.float32)
    x[:, :E] = np.clip(rng.normal(0.0, 0.4, size=(streams * Tq, E)), -1.5, 1.5)
    sets = np.zeros((streams * Tq, k), np.int64)
    for st in range(streams):
        base = rank[rng.choice(E, size=shared, replace=False, p=p)]
        for j in range(Tq):
            t = st * Tq + j
            q = p.copy()
            q[np.isin(rank, base)] = 0.0
            q /= q.sum()
            own = rank[rng.choice(E, size=k - shared, replace=False, p=q)]
            chosen = np.concatenate([base, own])
            lv = 3.0 + 0.125 * rng.permutation(k)          # distinct, exact in bf16
            x[t, chosen] = lv
            sets[t] = np.sort(chosen)
    return x.reshape(streams, Tq, H), sets


def spec_router_(blk):
    """One-hot router: the logit of expert e is x[:, e] exactly."""
    import torch
    E, H = blk.gate_weight.shape
    w = torch.zeros(E, H, device=blk.gate_weight.device)
    w[torch.arange(E), torch.arange(E)] = 1.0
    with torch.no_grad():
        blk.gate_weight.copy_(w.to(torch.bfloat16))


def run_spec(args, world, rank, local, device):
    """Batched speculative decode: 64 streams x (1 + 3 draft) = 256 tokens per
    verify step through `spec_layers` layers of the decode shape, the experts
    sharded over the N ranks (the streams split over the ranks), verify
    semantics (the reference's unsorted stock gathers).  Every step checks
    each rank's top-k sets against the prescribed ones bit for bit; after the
    timing, layer 0's expert-parallel output of the rank's tokens against the
    single-GPU block (the combine)."""
    import torch
    from titan_b200 import SparseMoeBlock, _lib, ops
    from titan_b200.expert_parallel import ExpertParallelMoE, PeerExchange
    c = CFG2
    S, D = args.spec_streams, args.spec_draft
    Tq = 1 + D
    if S % world:
        raise SystemExit(f"--spec-streams {S} does not split over {world} ranks")
    xs, sets = spec_tokens(S, D, c["H"], c["E"], c["k"], seed=77)
    sl = slice(rank * (S // world), (rank + 1) * (S // world))
    xr = torch.from_numpy(xs[sl]).to(device).to(torch.bfloat16).contiguous()
    want = torch.from_numpy(sets.reshape(S, Tq, -1)[sl].reshape(-1, c["k"])).to(device)
    T = xr.shape[0] * Tq
    ex = PeerExchange(T, c["H"], c["k"], device=device)
    layers, full0 = [], None
    for l in range(args.spec_layers):
        torch.manual_seed(5000 + l)
        blk = SparseMoeBlock(c["H"], c["E"], c["k"], c["I"], c["Is"], device=device,
                             weight_std=0.02)
        spec_router_(blk)
        layers.append(ExpertParallelMoE(blk, exchange=ex))
        if l == 0:
            full0 = blk
        del blk
    torch.cuda.empty_cache()
    opts = SparseMoeBlock.verify_options()
    xf = xr.reshape(T, c["H"])
    bad_routing = 0

    def step(check=False):
        nonlocal bad_routing
        for ep in layers:
            ep(xf, options=opts)
        if check:
            idx, _ = ops.router_topk(xf, layers[0].gate_weight, c["k"])
            got = torch.sort(idx.long(), dim=1).values
            bad_routing += int((got != want).any(dim=1).sum())

    torch.cuda.synchronize()
    barrier(world)
    for _ in range(max(args.warmup, 3)):
        step(check=True)
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b) / args.steps, world)
    for _ in range(args.steps):          # the per-step checks, outside the timed region
        step(check=True)
    y_ep = layers[0](xf, options=opts)
    y_one = full0(xf, options=opts)
    mism = int((y_ep.view(torch.int16) != y_one.view(torch.int16)).sum())
    flags = torch.tensor([bad_routing, mism], device=device, dtype=torch.int64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(flags)
    ex.check()
    ex.close()
    del layers, full0
    torch.cuda.empty_cache()
    return {"workload": f"batched speculative decode: {S} streams x (1 + {D} draft) = {S * Tq} "
                        f"tokens per verify step, {args.spec_layers} layers of the decode shape, "
                        "Zipf(1.2) expert popularity, the tokens of a stream share 7 of their 10 "
                        "experts, verify semantics (unsorted stock gathers, token-major combine)",
            "ms_per_step": round(ms, 4), "us_per_layer": round(1000 * ms / args.spec_layers, 2),
            "tok_per_s": round(S * Tq / (ms * 1e-3), 1),
            "topk_mismatched_tokens_all_steps": int(flags[0]),
            "combine_mismatches_vs_single_gpu": int(flags[1]),
            "checked_steps": args.steps + max(args.warmup, 3), "parallelism": f"ep{world}"}


# -------------------------------------------------------------- CPU baseline

def host_layer(rng, c):
    """Host-synthesised layer of shape c for the CPU oracle: random int4 words
    and scales/biases with the magnitudes N(0, 0.02) weights quantise to
    (the oracle's work does not depend on the values)."""
    from oracle import oracle as O

    def q(E, N, K):
        w = rng.integers(0, 2 ** 31, size=(E, N, K // 8), dtype=np.int32).view(np.uint32)
        s = O.f32_to_bf16(rng.uniform(0.0045, 0.0065, size=(E, N, K // 64)).astype(np.float32))
        b = O.f32_to_bf16((-7.5 * O.bf16_to_f32(s) + rng.normal(0, 1e-3, size=s.shape)).astype(np.float32))
        return w, s, b

    H, E, k, I, Is = c["H"], c["E"], c["k"], c["I"], c["Is"]
    wr = O.f32_to_bf16(rng.normal(0, 0.02, size=(E, H)).astype(np.float32))
    gu = q(E, 2 * I, H)
    dn = q(E, H, I)
    L = O.Layer(H, E, k, I, Is, wr, *gu, *dn)
    sg = q(1, 2 * Is, H)
    sd = q(1, H, Is)
    L.sgu_w, L.sgu_s, L.sgu_b = sg
    L.sdn_w, L.sdn_s, L.sdn_b = sd
    L.wg = O.f32_to_bf16(rng.normal(0, 0.02, size=(H,)).astype(np.float32))
    return L


def cpu_baseline(seconds, T=HEADLINE_T, n_layers=2):
    from oracle import oracle as O
    O.set_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    layers = [host_layer(rng, CFG2) for _ in range(n_layers)]
    x = O.f32_to_bf16(rng.standard_normal((T, CFG2["H"])).astype(np.float32))
    O.moe_decode(layers[0], x)
    n, t0 = 0, time.perf_counter()
    while True:
        O.moe_decode(layers[n % n_layers], x)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    us = 1e6 * el / n
    return {"value": round(us, 1), "unit": "us/layer", "cores": O.threads(), "kind": "port",
            "sample": f"config-2 decode layer (H=2048, E=512+1, I=512, k=10), T={T}, "
                      f"{n} layer calls cycling {n_layers} host-synthesised layers over "
                      f"{el:.1f} s (oracle/moe_oracle.c, fp64 sums, OpenMP)"}


def cpu_prefill_baseline(seconds, tokens=64, cfg=None, shared=True):
    """The oracle's prefill semantics (router, int8 routed experts in the
    reference's fp32 order, SwiGLU, weighted sum, shared expert) on a bounded
    sample of tokens of one host-synthesised layer: tokens per second on all
    host cores."""
    from oracle import oracle as O
    cfg = cfg or CFG2
    O.set_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    L = host_layer(rng, cfg)
    if not shared:
        L.Is = 0
        L.sgu_w = L.sgu_s = L.sgu_b = L.sdn_w = L.sdn_s = L.sdn_b = L.wg = None
    x = O.f32_to_bf16(rng.standard_normal((tokens, cfg["H"])).astype(np.float32))
    O.moe_prefill(L, x, int8_mode=3)
    n, t0 = 0, time.perf_counter()
    while True:
        O.moe_prefill(L, x, int8_mode=3)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"tok_per_s": round(n * tokens / el, 2), "ms_per_call": round(1000 * el / n, 2),
            "calls": n, "tokens_per_call": tokens, "seconds": round(el, 2),
            "cores": O.threads()}


# ------------------------------------------------------------------- arms

def ep_config(args, world):
    """The headline workload's config dict, printed identically by both arms."""
    c = CFG2
    return {"workload": f"expert-parallel prefill step: {args.ep_layers} MoE layers of the "
                        f"80B-A3B decode shape (H={c['H']}, {c['E']} routed + 1 shared expert, "
                        f"I={c['I']}, top-{c['k']}, int4 g64 affine), {args.ep_tokens} tokens per "
                        "step split over the ranks, Zipf(1.1) expert popularity",
            "layers": args.ep_layers, "tokens_per_step": args.ep_tokens,
            "tokens_per_rank": args.ep_tokens // world, "experts_per_rank": c["E"] // world,
            "parallelism": f"ep{world}",
            "placement": ("experts placed by the load of a separate calibration batch "
                          "(balanced_placement)" if args.ep_placement == "balanced"
                          else "contiguous E/N per rank"),
            "collective": ("2 NCCL all-to-alls per layer" if args.ep_exchange == "nccl" else
                           "NVLink stores into CUDA-IPC-mapped peer buffers, epoch flags, the "
                           "return stored by the down GEMM's epilogue, no host sync"),
            "l2": f"inputs larger than L2: {args.ep_layers} layers x 906 MB of expert weights "
                  "cycled every step",
            "timing": "CUDA events around the steps, max over ranks"}


def run_reference(args, world, rank):
    """The reference algorithm on the host cores (the CPU oracle: the
    overlay's int8 x int4 algebra in its fp32 order, MLX's rounding points):
    each step one bounded sample of the headline workload (tokens through one
    layer), reported per 36-layer step like the GPU arm."""
    if rank != 0:
        return 0
    from oracle import oracle as O
    O.set_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    L = host_layer(rng, CFG2)
    tok = args.ref_tokens
    x = O.f32_to_bf16(rng.standard_normal((tok, CFG2["H"])).astype(np.float32))
    for _ in range(max(1, min(args.warmup, 2))):
        O.moe_prefill(L, x, int8_mode=3)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.moe_prefill(L, x, int8_mode=3)
    el = time.perf_counter() - t0
    v = tok * args.steps / el / args.ep_layers
    sample = (f"{tok} tokens through one host-synthesised layer per step, {args.steps} steps "
              f"in {el:.1f} s on {O.threads()} threads (oracle/moe_oracle.c, OpenMP), scaled "
              f"to the {args.ep_layers}-layer step")
    line = {"metric": "moe_prefill_tokens_per_s", "value": round(v, 3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000 * el / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 x int4, fp32 epilogue (the reference's order)", "data": "synthetic",
            "impl": "reference", "config": ep_config(args, world),
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": O.threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "CPU restatement of the reference block (MLX is not installable here)"}
    print(json.dumps(line), flush=True)
    return 0


def run_titan(args, world, rank, local):
    import torch
    from titan_b200 import _lib
    _lib.load()
    device = torch.device("cuda", torch.cuda.current_device())
    peaks = measured_peaks_all()
    ep = run_ep(args, world, rank, local)
    extras, cb = {}, None
    if not args.headline_only:
        extras["spec_decode_config5"] = run_spec_group(args, world, rank, local)
    if world == 1 and not args.headline_only:
        hbm = peaks["hbm_gbs"]
        blocks = build_decode_layers(args.layers, device, seed=1234 + rank)
        torch.cuda.synchronize()
        clk = Clocks(local).__enter__()
        blocks, opts, sweep, head = bench_decode(args, world, device, blocks)
        x, ms, us, nbytes = head
        gbs = nbytes / (ms * 1e-3) / 1e9
        extras["decode_config2"] = {
            "us_per_layer_T1": round(us, 3), "sweep": sweep,
            "roofline": {"kernel": "decode_layer (the whole layer in one launch)",
                         "bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4),
                         "algorithmic_bytes_per_layer": int(nbytes / args.layers),
                         "source": "CUDA graph of one 48-layer step, CUDA events, per layer"},
            "e2e": bench_e2e(blocks, opts, HEADLINE_T, max(3, args.steps // 2), args.warmup,
                             world),
            "config": "H=2048, 512 routed + 1 shared expert, I=512, top-10, int4 g64, "
                      f"{args.layers} layers resident in HBM (43.5 GB, larger than L2)"}
        st1, _ = stage_profile([lambda b=b: b(x, options=opts) for b in blocks], reps=2)
        extras["decode_config2"]["stages_us_T1"] = {k: round(v["us_per_launch"], 3)
                                                    for k, v in st1.items()}
        del blocks
        torch.cuda.empty_cache()
        extras["prefill_config3"] = bench_prefill(args, world, device)
        clk.__exit__(None, None, None)
        extras["clocks_extras"] = clk.summary()
        if not args.no_cpu_baseline:
            r = cpu_prefill_baseline(args.cpu_seconds, tokens=args.ref_tokens)
            v = r["tok_per_s"] / args.ep_layers
            cb = {"value": round(v, 3), "unit": "tok/s", "cores": r["cores"], "kind": "port",
                  "sample": f"{r['calls']} calls of {r['tokens_per_call']} tokens through one "
                            f"host-synthesised layer in {r['seconds']} s (oracle, fp32 int8 "
                            f"algebra, OpenMP), scaled to the {args.ep_layers}-layer step"}
            c1 = dict(H=2048, E=64, k=10, I=512, Is=0)
            r1 = cpu_prefill_baseline(min(args.cpu_seconds, 8.0), tokens=128, cfg=c1,
                                      shared=False)
            extras["cpu_config1"] = {"workload": "single layer T=128, H=2048, 64 experts, "
                                                 "top-10, I=512, no shared expert",
                                     "ms_per_layer": r1["ms_per_call"], "cores": r1["cores"],
                                     "tok_per_s": r1["tok_per_s"]}
    if rank != 0:
        return 0
    line = {
        "metric": "moe_prefill_tokens_per_s", "value": ep["value"], "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ep["ms"], 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 x int4 (exact per-group f16 tcgen05 MMA), f32 epilogue",
        "data": "synthetic (seeded weights and tokens; no dataset)",
        "config": ep_config(args, world),
        "roofline": ep["roofline"], "cpu_baseline": cb, "e2e": ep["e2e"],
        "gpu_launches": ep["gpu_launches"], "clocks": ep["clocks"], "ep_check": ep["ep_check"],
        "phases_us_per_layer_rank0": ep["phases"], "routing": ep["routing"],
        "stages_us_rank0": ep["stages_us"],
    }
    line.update(extras)
    print(json.dumps(line), flush=True)
    return 0


def run_profile_case(args):
    """A small untimed case of one path, for ncu captures (bench numbers are
    never taken from it): decode = 2 decode-shape layers at T=1, 3 steps;
    prefill = one cold-prefill block at the first --prefill-T, 2 calls;
    ep = one decode-shape layer with the Zipf(1.1) router on --ep-tokens
    tokens on one GPU (the grouped GEMMs of the headline step at N=1), 2 calls."""
    import torch
    from titan_b200 import SparseMoeBlock, _lib
    device = torch.device("cuda", 0)
    if args.profile == "decode":
        blocks = build_decode_layers(2, device, seed=1234)
        x = torch.randn(HEADLINE_T, CFG2["H"], device=device).to(torch.bfloat16)
        opts = decode_opts()
        for _ in range(3):
            for b in blocks:
                b(x, options=opts)
    elif args.profile == "ep":
        c = CFG2
        torch.manual_seed(4321)
        blk = SparseMoeBlock(c["H"], c["E"], c["k"], c["I"], c["Is"], device=device,
                             weight_std=0.02)
        zipf_router_(blk, torch.Generator().manual_seed(777))
        blk.prepare()
        o = _lib.Options()
        o.min_tokens, o.int8_prefill, o.down_int8, o.wsum_mode = 1, 1, 1, 0
        o.gemm_kernel = args.gemm_kernel
        g = torch.Generator(device=device).manual_seed(9000)
        x = torch.randn(args.ep_tokens, c["H"], generator=g, device=device)
        x[:, 0] = 1.0
        x = x.to(torch.bfloat16)
        for _ in range(2):
            blk(x, options=o)
    else:
        c = CFG3
        T = int(args.prefill_T.split(",")[0])
        torch.manual_seed(99)
        blk = SparseMoeBlock(c["H"], c["E"], c["k"], c["I"], c["Is"], device=device,
                             weight_std=0.02)
        blk.prepare()
        o = _lib.Options()
        o.min_tokens, o.int8_prefill, o.down_int8, o.wsum_mode = 512, 1, 1, 0
        o.gemm_kernel = args.gemm_kernel
        x = torch.randn(T, c["H"], device=device).to(torch.bfloat16)
        for _ in range(2):
            blk(x, options=o)
    torch.cuda.synchronize()
    rc = _lib.load().tmoe_device_status()
    print(json.dumps({"profile": args.profile, "device_status": rc}))
    return 0 if rc == 0 else 1


def main():
    args = parse()
    if args.profile:
        return run_profile_case(args)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, world, rank)
    world, rank, local = dist_setup(args)
    try:
        return run_titan(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
