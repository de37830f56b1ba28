#!/usr/bin/env python
"""Batch-one SwiGLU FFN decode layer (4096 -> 14336) on B200: us per layer and % of HBM peak.

One step = one full layer (gate = Wg x + bg, up = Wu x + bu, h = SiLU(gate) * up,
y = Wd h + bd + x; fp16 weights, fp32 accumulation, fp16 h, fp32 y) on seeded
synthetic inputs, weights cycling through rotating copies whose total exceeds
twice the 126 MB L2, so every step streams its weights from HBM.

* N = 1: the layer on one B200, as whichever is faster on this GPU: the two
  product kernels (gate, then down launched programmatically), or the whole
  layer in one persistent kernel (gate, grid barrier, down).
* N > 1 (torchrun, one rank per GPU): tensor parallel. Wg/Wu split by
  intermediate row, Wd by its K dimension; the down kernel sums the ranks'
  partial y over NVLink peer memory and adds bias + residual once (fused
  all-reduce). The NCCL all-reduce path is timed beside it as the baseline.

Steps are captured in CUDA graphs: the timed steps run as graphs that each hold
up to 32 consecutive layer steps (the FFN layers of one decode step);
the reference's protocol, one step per graph replay, is timed and reported
beside it (``one_step_graph_us``), and so are the baselines.

Prints ONE JSON line on rank 0. ``--impl reference`` times the reference's own
CPU path (its include/contract.hpp matvec, compiled under oracle/_ref) on the
host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "cuda-kernel_b200"))

METRIC = "SwiGLU FFN µs/layer and % of HBM peak, batch 1 (4096→14336), 1/2/4/8 B200"
UNIT = "us/layer"
L2_BYTES = 126 * 1024 * 1024
# NVLink 5 peer copy per direction per GPU measured on this pool's B200s (nominal 900 GB/s):
# the denominator of the fused exchange's NVLink fraction.
NVLINK_PEER_GBS = 770.0


def parse():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--intermediate", type=int, default=14336)
    p.add_argument("--gate-config", type=int, default=0, help="registry id (0 = tune)")
    p.add_argument("--down-config", type=int, default=0, help="registry id (0 = tune)")
    p.add_argument("--graph-steps", type=int, default=0,
                   help="layer steps per CUDA graph (0 = a decode step of up to 32 layers, 1 = one step per graph)")
    p.add_argument("--no-prefetch-weights", action="store_true",
                   help="launch each step's gate in plain stream order (no SWB_PREFETCH_WEIGHTS)")
    p.add_argument("--layer-config", type=int, default=0,
                   help="fused whole-layer kernel id (0 = tune against the two-kernel path, -1 = never)")
    p.add_argument("--fixture", type=Path, default=None,
                   help="captured layer directory (swiglu_b200.fixtures) of --hidden x --intermediate")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-cublas", action="store_true")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# --------------------------------------------------------------- reference arm

def reference_arm(args) -> None:
    """The reference's CPU implementation of the layer on all host threads (rank 0 only)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT))
    import oracle  # the checker package: used here only as the timed reference arm
    H, I = args.hidden, args.intermediate
    threads = len(os.sched_getaffinity(0))
    w = oracle.normal_workload(0, H, I)
    if oracle.ref_available():
        kind = "reference"
        run = lambda: oracle.ref_ffn(w, threads=threads)  # noqa: E731
    else:
        kind = "port"
        threads = 1
        run = lambda: oracle.ffn(w)  # noqa: E731
    for _ in range(max(args.warmup, 0)):
        run()
    samples = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s = time.perf_counter()
        run()
        samples.append(time.perf_counter() - s)
    total = time.perf_counter() - t0
    us = total / args.steps * 1e6
    line = {
        "impl": "reference", "metric": METRIC, "value": us, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16 in, f64 accumulate (CPU)", "data": "synthetic",
        "config": {"workload": f"SwiGLU FFN {H}->{I} batch 1", "hidden": H, "intermediate": I, "batch": 1,
                   "parallelism": "host threads", "seed": 0},
        "cpu_baseline": {"value": us, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{args.steps} full {H}->{I} layers (decode::matvec x3 + SiLU + residual; "
                                   f"fp16->fp32 conversion of the weights included, block by block), "
                                   f"rows split over {threads} threads",
                         "median_step_us": statistics.median(samples) * 1e6},
        "e2e": {"value": us, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm

def make_weights(torch, H, I, copies, device, seed=0):
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def normal(shape, scale):
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * scale).half()

    sets = []
    for _ in range(copies):
        sets.append({"wg": normal((I, H), 1 / math.sqrt(H)), "wu": normal((I, H), 1 / math.sqrt(H)),
                     "wd": normal((H, I), 1 / math.sqrt(I))})
    common = {"x": normal((H,), 1.0), "bg": normal((I,), 0.02), "bu": normal((I,), 0.02), "bd": normal((H,), 0.02)}
    return sets, common


def time_kernel(torch, fn, reps, stream):
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(reps):
        fn(i)
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) * 1e3 / reps


def tune(torch, binding, launch_gate, launch_down, ids, stream, reps=8, down_ids=None):
    """Pick the fastest gate and down geometry by median over rotating copies."""
    best = {}
    for name, launch, cand in (("gate", launch_gate, ids), ("down", launch_down, down_ids or ids)):
        times = {}
        for cid in cand:
            launch(cid, 0)
            torch.cuda.synchronize()
            samples = [time_kernel(torch, lambda i, c=cid: launch(c, i), reps, stream) for _ in range(3)]
            times[cid] = statistics.median(samples)
        best[name] = min(times, key=times.get)
        best[name + "_times"] = times
    return best


def traffic_from_profile(tag: str, cfg: int, H: int, I: int, shard: int, world: int):
    """DRAM bytes (read + write) per launch of kernel `tag` at registry id `cfg`, from the committed
    ncu summary of that kernel: profiles/<tag>_<H>x<rows>.txt holds one line
    ``traffic_bytes_per_launch[<id>]: <bytes>`` per profiled geometry. A tensor-parallel shard
    uses its own shape's summary when one exists, else the full layer's figure over N (weight
    traffic scales with the shard). Returns (bytes or None, where it came from)."""
    import re
    cands = [(shard, 1)] if world > 1 else []
    cands.append((I, world))
    for rows, div in cands:
        path = ROOT / "profiles" / f"{tag}_{H}x{rows}.txt"
        try:
            text = path.read_text()
        except OSError:
            continue
        m = re.search(r"^traffic_bytes_per_launch\[%d\]:\s*([0-9.eE+]+)" % cfg, text, flags=re.M)
        if m:
            how = "ncu dram__bytes_read.sum + dram__bytes_write.sum"
            return int(float(m.group(1)) // div), (f"{path.relative_to(ROOT)} ({how}, config {cfg}"
                                                   + (f", full layer / {div}" if div > 1 else "") + ")")
    return None, f"no committed ncu summary of {tag} config {cfg} at this shape"


def cpu_baseline(sets, common, H, I, budget_s):
    """The reference's CPU path (oracle/_ref, one thread) on a bounded sample of whole layers."""
    sys.path.insert(0, str(ROOT))
    import oracle  # the checker package: used here only as the timed CPU baseline
    w = {k: sets[0][k].cpu().numpy() for k in ("wg", "wu", "wd")}
    w.update({k: common[k].cpu().numpy() for k in ("x", "bg", "bu", "bd")})
    if oracle.ref_available():
        kind, run = "reference", (lambda: oracle.ref_ffn(w, threads=1))
    else:
        kind, run = "port", (lambda: oracle.ffn(w))
    run()  # warm caches / page in
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 1000:
            break
    return {"value": el / n * 1e6, "unit": UNIT, "cores": 1, "kind": kind,
            "sample": f"{n} full {H}->{I} layers on 1 host thread (decode::matvec x3 + SiLU + residual, "
                      f"as src/benchmark.cu:131-141; fp16->fp32 conversion of the weights included, "
                      f"block by block), {el:.1f} s"}


def ours(args) -> None:
    import torch
    import torch.distributed as dist
    from swiglu_b200 import binding, _lib, intensity
    from swiglu_b200.clocks import ClockSampler

    world, rank, local = dist_env()
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    _lib.lib()  # fail loudly now if the native library is missing
    if world > 1:
        import datetime
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")  # a timed-out collective ends the process
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=device)

    H, I = args.hidden, args.intermediate
    if I % world:
        raise SystemExit("intermediate size must divide by the GPU count")
    shard = I // world
    layer = intensity.layer(H, I)
    if world == 1:
        rank_bytes = layer["bytes"]
        gate_bytes = layer["gate"]["bytes"]
    else:
        tpb = intensity.tp_rank(H, I, world)
        rank_bytes = tpb["bytes"]
        gate_bytes = tpb["gate"]["bytes"]
    weight_bytes_rank = 3 * H * shard * 2
    copies = max(2, math.ceil(2 * L2_BYTES / weight_bytes_rank) + 1)

    # All work runs on one dedicated stream (graph capture cannot use the legacy default stream).
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream

    # Full weights are drawn on every rank from the same seed, then each rank keeps its shard.
    full_sets, common = make_weights(torch, H, I, copies, device)
    if args.fixture is not None:
        # a captured layer (src/benchmark.cu:122-127): every rotating copy holds its weights
        from swiglu_b200.fixtures import as_layer, load
        cap = {k: torch.from_numpy(v.copy()).to(device) for k, v in as_layer(load(args.fixture, H, I)).items()}
        for s in full_sets:
            for k in ("wg", "wu", "wd"):
                s[k].copy_(cap[k])
        common = {"x": cap["x"], "bg": cap["bg"], "bu": cap["bu"], "bd": cap["bd"]}
    r0, r1 = rank * shard, (rank + 1) * shard
    sets = []
    for s in full_sets:
        sets.append({"wg": s["wg"][r0:r1].contiguous(), "wu": s["wu"][r0:r1].contiguous(),
                     "wd": s["wd"][:, r0:r1].contiguous()})
    bg, bu = common["bg"][r0:r1].contiguous(), common["bu"][r0:r1].contiguous()
    x, bd = common["x"], common["bd"]
    w0 = full_sets[0]
    del full_sets
    torch.cuda.synchronize()

    h = torch.empty(shard, dtype=torch.float16, device=device)
    y = torch.empty(H, dtype=torch.float32, device=device)
    L = _lib.lib()

    def launch_gate(cid, i):
        s = sets[i % copies]
        _lib.check(L.swb_gate(cid, s["wg"].data_ptr(), s["wu"].data_ptr(), x.data_ptr(), bg.data_ptr(),
                              bu.data_ptr(), h.data_ptr(), shard, H, 0, sp))

    if world == 1:
        def launch_down(cid, i):
            s = sets[i % copies]
            _lib.check(L.swb_project(cid, s["wd"].data_ptr(), h.data_ptr(), bd.data_ptr(), x.data_ptr(),
                                     y.data_ptr(), H, shard, _lib.SWB_RESIDUAL, sp))
    else:
        def launch_down(cid, i):
            s = sets[i % copies]
            _lib.check(L.swb_project(cid, s["wd"].data_ptr(), h.data_ptr(), None, None, y.data_ptr(), H, shard,
                                     0, sp))

    ids = binding.config_ids()
    down_ids = ids
    if world > 1:
        # the fused all-reduce epilogue lives in the RBULK kernel: tune the down geometry among those
        down_ids = [c for c in ids if binding.config_info(c)["family"] == _lib.SWB_FAMILY_RBULK]
    if args.gate_config and args.down_config:
        gcfg, dcfg, tuned = args.gate_config, args.down_config, None
    else:
        tuned = tune(torch, binding, launch_gate, launch_down, ids, stream, down_ids=down_ids)
        gcfg = args.gate_config or tuned["gate"]
        dcfg = args.down_config or tuned["down"]
        if world > 1:  # every rank runs the same geometry: take rank 0's choice
            t = torch.tensor([gcfg, dcfg], dtype=torch.int64, device=device)
            dist.broadcast(t, 0)
            gcfg, dcfg = int(t[0]), int(t[1])

    exchange = None
    if world > 1:
        from swiglu_b200.tp import Exchange
        exchange = Exchange(rank, world, H, device)  # one-time set-up: IPC handles shared by all_gather
    workspace = binding.layer_workspace(device)  # grid-barrier slots of the one-GPU fused layer kernel

    # The weights are written once, before any step: each step's gate may start streaming them
    # while the previous step's down kernel (and exchange) still runs (SWB_PREFETCH_WEIGHTS).
    flags = 0 if args.no_prefetch_weights else _lib.SWB_PREFETCH_WEIGHTS

    def layer_step(cfg, g, d, i):
        # cfg = 0: gate kernel, then the down kernel launched programmatically (for N > 1 the
        # down kernel also sums the ranks' partials over NVLink); cfg > 0: the whole layer
        # (and, for N > 1, the exchange) in one persistent kernel
        s = sets[i % copies]
        if world == 1 and cfg:
            _lib.check(L.swb_ffn_fused_ex(cfg, s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(),
                                          x.data_ptr(), bg.data_ptr(), bu.data_ptr(), bd.data_ptr(), h.data_ptr(),
                                          y.data_ptr(), H, shard, workspace.data_ptr(), flags, sp))
        elif world == 1:
            _lib.check(L.swb_ffn_ex(g, d, s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(),
                                    x.data_ptr(), bg.data_ptr(), bu.data_ptr(), bd.data_ptr(), h.data_ptr(),
                                    y.data_ptr(), H, shard, flags, sp))
        else:
            _lib.check(L.swb_ffn_tp_fused_ex(exchange.handle, cfg or g, 0 if cfg else d, s["wg"].data_ptr(),
                                             s["wu"].data_ptr(), s["wd"].data_ptr(), x.data_ptr(), bg.data_ptr(),
                                             bu.data_ptr(), bd.data_ptr(), h.data_ptr(), y.data_ptr(), H, shard,
                                             flags, sp))

    def median_step_us(fn):
        torch.cuda.synchronize()
        return statistics.median(time_kernel(torch, fn, 8, stream) for _ in range(3))

    def agree(values):
        # rank 0's choice, on every rank (all ranks then take the same steps in the same order)
        if world == 1:
            return values
        t = torch.tensor(values, dtype=torch.int64, device=device)
        dist.broadcast(t, 0)
        return [int(v) for v in t.tolist()]

    # Gate and down tuned one at a time cannot see how the pair shares the GPU (the
    # down kernel's CTAs become resident, and prefetch Wd, as the gate's leave room):
    # the best few of each are timed again as whole steps.
    pair_times = {}
    if tuned is not None:
        top = lambda times: sorted(times, key=times.get)[:4]  # noqa: E731
        cands = agree(top(tuned["gate_times"]) + top(tuned["down_times"]))
        for g in cands[:4]:
            for d in cands[4:]:
                try:
                    layer_step(0, g, d, 0)
                except RuntimeError:  # geometry does not hold this shape (same answer on every rank)
                    continue
                pair_times[(g, d)] = median_step_us(lambda i, g=g, d=d: layer_step(0, g, d, i))
        best = min(pair_times, key=pair_times.get)
        gcfg, dcfg = agree(list(best))

    # the fused whole-layer kernels against the tuned two-kernel step, timed the same way
    # (every rank times the same candidates in the same order; rank 0's choice is broadcast)
    lcfg = max(args.layer_config, 0)
    layer_times = {}
    if args.layer_config == 0:
        cands = [0] + binding.layer_config_ids()
        for c in cands:
            try:
                layer_step(c, gcfg, dcfg, 0)
            except RuntimeError:  # geometry does not hold this shape (same answer on every rank)
                continue
            layer_times[c] = median_step_us(lambda i, c=c: layer_step(c, gcfg, dcfg, i))
        lcfg = agree([min(layer_times, key=layer_times.get)])[0]

    def step(i):
        layer_step(lcfg, gcfg, dcfg, i)

    def step_nccl(i):
        # the baseline tensor-parallel step: partial y, NCCL all-reduce, then bias + residual
        s = sets[i % copies]
        _lib.check(L.swb_ffn_tp(gcfg, dcfg, s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(),
                                x.data_ptr(), bg.data_ptr(), bu.data_ptr(), h.data_ptr(), y.data_ptr(), H, shard,
                                sp))
        dist.all_reduce(y)
        _lib.check(L.swb_residual_epilogue(y.data_ptr(), bd.data_ptr(), x.data_ptr(), H, sp))

    # ---- sanity check of the (sharded) layer against a plain torch fp32 computation
    step(0)
    torch.cuda.synchronize()
    xf = x.float()
    gref = w0["wg"].float() @ xf + common["bg"].float()
    uref = w0["wu"].float() @ xf + common["bu"].float()
    href = (torch.nn.functional.silu(gref) * uref).half()
    yref = w0["wd"].float() @ href.float() + common["bd"].float() + xf
    # atol_j: the change one fp16 rounding of h can make in y_j (h is fp16 by contract)
    atol = 2.0 ** -11 * (w0["wd"].float().abs() @ href.float().abs())
    rel = ((y - yref).abs() / (yref.abs() + atol)).max().item()
    del w0, gref, uref, href, yref
    if world > 1:  # every rank takes the same exit decision
        t = torch.tensor([rel], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        rel = float(t.item())
    if not rel <= 2e-3:
        raise SystemExit(f"bench sanity check failed: max relative error {rel}")
    if world > 1:  # the NCCL baseline must agree with the fused path too
        # Both sum the same fp32 partials, in different orders: they differ by a few
        # ulps of sum_i |Wd[j,i] h_i| = 2^11 atol_j. A missing or doubled partial would
        # be off by about that sum / N, orders of magnitude above the bound.
        y_fused = y.clone()
        step_nccl(0)
        torch.cuda.synchronize()
        dn = ((y - y_fused).abs() / (y_fused.abs() + atol)).max()
        dist.all_reduce(dn, op=dist.ReduceOp.MAX)
        if not float(dn) <= 2e-3:  # the tolerance of the check against the fp32 reference above
            raise SystemExit(f"fused and NCCL tensor-parallel paths disagree: {float(dn)}")
    del atol
    launches_per_step = 1 if lcfg else 2

    # ---- CUDA graphs. One graph per rotating copy holds one whole step (the reference's
    # protocol: src/benchmark.cu:46-83, one captured call replayed); the timed steps are
    # issued as graphs that each hold `chain` consecutive layer steps, as the FFN layers of
    # one decode step run back to back in one graph: up to 32 (the layer count of the
    # 32-layer model this 4096 -> 14336 FFN belongs to) and at most K, a whole number of
    # passes over the rotating weight copies, so consecutive steps never share a copy. Every
    # step does all of its work; `one_step_graph_us` reports the one-step-per-graph protocol.
    chain = args.graph_steps if args.graph_steps > 0 else min(args.steps, 32)
    if chain > copies:
        chain = chain // copies * copies

    def capture(fn, first, n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for k in range(n):
                fn((first + k) % copies)
        return g

    for c in range(copies):
        step(c)  # warm every copy (and NCCL) before capture
    torch.cuda.synchronize()
    graphs = [capture(step, c, 1) for c in range(copies)]
    chained = [capture(step, 0, chain)] if chain > 1 else []
    torch.cuda.synchronize()

    def run_steps(n, one_per_graph=False):
        # n steps in order: whole chains first, then single-step graphs for the rest
        i = 0
        if chained and not one_per_graph:
            for _ in range(n // chain):
                chained[0].replay()
            i = (n // chain) * chain
        for k in range(i, n):
            graphs[k % copies].replay()

    def run_step(i):
        graphs[i % copies].replay()

    sampler = ClockSampler(local, interval_s=0.002).start()
    run_steps(max(args.warmup, chain))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_window = [time.time()]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    run_steps(args.steps)
    end.record(stream)
    end.synchronize()
    t_window.append(time.time())
    if world > 1:
        dist.barrier()
    elapsed_ms = start.elapsed_time(end)
    if world > 1:  # max over ranks; every rank then holds the same number
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    # A timed region shorter than a few NVML samples is followed by a soak of the same
    # graph replays (not timed) so the clock record reflects this load. The replay
    # count comes from the rank-agreed time, so every rank issues the same collectives.
    soak_window = None
    if elapsed_ms < 300.0:
        soak_steps = int(math.ceil(300.0 / max(elapsed_ms, 1e-3) * args.steps))
        t0 = time.time()
        run_steps(soak_steps)
        torch.cuda.synchronize()
        soak_window = (t0, time.time())
        if world > 1:
            dist.barrier()
    us_per_layer = elapsed_ms * 1e3 / args.steps
    # the reference's protocol: the same steps, one step per graph replay (max over ranks)
    if world > 1:
        dist.barrier()
    one_step_us = time_kernel(torch, lambda i: run_step(i), args.steps, stream)
    if world > 1:
        t = torch.tensor([one_step_us], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        one_step_us = float(t.item())

    # ---- each kernel alone: `kn` back-to-back launches over the rotating copies captured in
    # one CUDA graph, in plain stream order (no programmatic overlap with a neighbour), timed
    # with CUDA events on the launching stream around whole replays; per-launch time = replay
    # time / kn (median of 3 replays, max over ranks). With the fused layer kernel the
    # dominant kernel is that one launch per step; otherwise the gate kernel.
    kn = copies * max(1, args.steps // copies)

    def alone_us(launch):
        for c in range(copies):
            launch(c)
        torch.cuda.synchronize()
        g = capture(launch, 0, kn)
        g.replay()
        torch.cuda.synchronize()
        t = statistics.median(time_kernel(torch, lambda i: g.replay(), 1, stream) for _ in range(3)) / kn
        g.reset()
        if world > 1:
            tt = torch.tensor([t], dtype=torch.float64, device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    peaks = intensity.measured_peaks(ROOT / "MEASURED_PEAKS.json")
    down_bytes = rank_bytes - gate_bytes

    def kernel_record(tag, cfg, nbytes, us):
        traffic, source = traffic_from_profile(tag, cfg, H, I, shard, world)
        gbs = nbytes / (us * 1e-6) / 1e9
        return {"config": cfg, "launch_us": us, "bytes_per_launch": nbytes, "achieved": gbs,
                "frac": gbs / peaks["hbm_gbs"], "traffic": traffic, "traffic_source": source,
                "launches_timed": kn}

    kernels = {}
    if lcfg:
        kernels["layer"] = kernel_record("layer", lcfg, rank_bytes,
                                         alone_us(lambda i: layer_step(lcfg, gcfg, dcfg, i)))
    kernels["gate"] = kernel_record("gate", gcfg, gate_bytes, alone_us(lambda i: launch_gate(gcfg, i)))
    kernels["down"] = kernel_record("down", dcfg, down_bytes, alone_us(lambda i: launch_down(dcfg, i)))
    # The pair is chosen by whole chained steps, where a deep ring prefetches more of the
    # next kernel's weights behind this one's tail; launched alone, a shallow ring (SMs kept
    # even) can be faster. The fastest of the three best-tuned geometries of each kernel,
    # timed alone the same way, is recorded beside the pair's.
    if tuned is not None:
        for tag, launch, nbytes, pair_cfg in (("gate", launch_gate, gate_bytes, gcfg),
                                              ("down", launch_down, down_bytes, dcfg)):
            times = tuned[tag + "_times"]
            cands = agree(sorted(times, key=times.get)[:3])
            alone = {c: (kernels[tag]["launch_us"] if c == pair_cfg else
                         alone_us(lambda i, c=c, f=launch: f(c, i)))
                     for c in cands}
            best = min(alone, key=alone.get)
            rec = kernel_record(tag, best, nbytes, alone[best])
            rec["candidates_us"] = {str(c): round(v, 3) for c, v in alone.items()}
            kernels[tag + "_best_alone"] = rec
    dom = kernels["layer" if lcfg else "gate"]
    kname = (f"fused layer (config {lcfg})" + (" with the NVLink exchange" if world > 1 else "")) if lcfg \
        else f"gate (config {gcfg})"
    roofline = {"bound": "hbm", "kernel": kname, "achieved": dom["achieved"], "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": dom["frac"],
                "peak_source": f"{peaks['source']} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"
                               if peaks["source"] == "measured" else f"{peaks['source']} copy bandwidth",
                "traffic": dom["traffic"], "traffic_source": dom["traffic_source"],
                "bytes_per_launch": dom["bytes_per_launch"], "launch_us": dom["launch_us"],
                "timing": f"{kn} back-to-back launches of the kernel alone in one CUDA graph, "
                          "plain stream order, CUDA events around whole replays",
                "kernels": kernels}
    layer_gbs = rank_bytes / (us_per_layer * 1e-6) / 1e9
    layer_roofline = {"achieved": layer_gbs, "frac": layer_gbs / peaks["hbm_gbs"], "unit": "GB/s",
                      "bytes_per_step_per_rank": rank_bytes}

    # ---- all-reduce alone (tensor parallel): reported separately, it is latency-bound
    tp = None
    if world > 1:
        # the NCCL baseline step, captured and timed the same two ways (max over ranks)
        for c in range(copies):
            step_nccl(c)
        torch.cuda.synchronize()
        ngraphs = [capture(step_nccl, c, 1) for c in range(copies)]
        nchain = capture(step_nccl, 0, chain) if chain > 1 else None
        for i in range(args.warmup):
            ngraphs[i % copies].replay()
        dist.barrier()
        nccl_one = time_kernel(torch, lambda i: ngraphs[i % copies].replay(), args.steps, stream)
        nccl_us = nccl_one
        if nchain is not None and args.steps >= chain:
            dist.barrier()
            nccl_us = time_kernel(torch, lambda i: nchain.replay(), args.steps // chain, stream) / chain
            nchain.reset()
        for gr in ngraphs:
            gr.reset()
        ngraphs.clear()
        t = torch.tensor([nccl_us, nccl_one], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        nccl_us, nccl_one = float(t[0]), float(t[1])
        # 20 all-reduces captured in one graph, replayed: device-side latency, not host launch rate
        ag = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ag, stream=stream):
            for _ in range(20):
                dist.all_reduce(y)
        ag.replay()
        torch.cuda.synchronize()
        ar = time_kernel(torch, lambda i: ag.replay(), 10, stream) / 20
        ag.reset()
        del ag
        t = torch.tensor([ar], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        nccl_ar = float(t.item())

        # The exchange's own cost: the rank's step with the fused exchange against the same
        # kernels with none (the partial y stays local), both as `kn` steps in one graph in
        # plain stream order (no weight prefetch), max over ranks.
        def step_local(i):
            s = sets[i % copies]
            if lcfg:
                _lib.check(L.swb_ffn_fused(lcfg, s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(),
                                           x.data_ptr(), bg.data_ptr(), bu.data_ptr(), bd.data_ptr(), h.data_ptr(),
                                           y.data_ptr(), H, shard, workspace.data_ptr(), sp))
            else:
                _lib.check(L.swb_ffn_tp(gcfg, dcfg, s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(),
                                        x.data_ptr(), bg.data_ptr(), bu.data_ptr(), h.data_ptr(), y.data_ptr(), H,
                                        shard, sp))

        def step_fused_plain(i):
            s = sets[i % copies]
            _lib.check(L.swb_ffn_tp_fused_ex(exchange.handle, lcfg or gcfg, 0 if lcfg else dcfg, s["wg"].data_ptr(),
                                             s["wu"].data_ptr(), s["wd"].data_ptr(), x.data_ptr(), bg.data_ptr(),
                                             bu.data_ptr(), bd.data_ptr(), h.data_ptr(), y.data_ptr(), H, shard,
                                             0, sp))

        def graph_step_us(fn):
            for c in range(copies):
                fn(c)
            torch.cuda.synchronize()
            g = capture(fn, 0, kn)
            g.replay()
            torch.cuda.synchronize()
            dist.barrier()
            v = statistics.median(time_kernel(torch, lambda i: g.replay(), 1, stream) for _ in range(3)) / kn
            g.reset()
            return v

        local_us = graph_step_us(step_local)
        fused_plain_us = graph_step_us(step_fused_plain)
        t = torch.tensor([local_us, fused_plain_us], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        local_us, fused_plain_us = float(t[0]), float(t[1])
        exchange_us = max(fused_plain_us - local_us, 1e-3)
        # what must cross NVLink per rank and step: this rank's fp32 partial of every row to each
        # peer (the payload), sent as 8-byte {value, epoch} words (the wire bytes)
        payload = (world - 1) * H * 4
        wire = (world - 1) * H * 8
        nvlink = {"bytes_per_rank_step": payload, "wire_bytes_per_rank_step": wire, "exchange_us": exchange_us,
                  "achieved": wire / (exchange_us * 1e-6) / 1e9, "peak": NVLINK_PEER_GBS, "unit": "GB/s",
                  "frac": wire / (exchange_us * 1e-6) / 1e9 / NVLINK_PEER_GBS,
                  "peak_source": "measured NVLink peer copy per direction on this pool's B200s",
                  "how": "exchange_us = fused rank step - the same kernels without the exchange, each "
                         f"{kn} steps in one CUDA graph without weight prefetch (max over ranks)",
                  "local_step_us": local_us, "fused_step_no_prefetch_us": fused_plain_us,
                  "latency_bound": True}
        tp = {"ranks": world, "shard_rows": shard, "exchange": "fused one-shot all-reduce over NVLink peer memory "
              "in the down kernel", "nccl_step_us": nccl_us, "fused_speedup_vs_nccl": nccl_us / us_per_layer,
              "nccl_one_step_graph_us": nccl_one,
              "nccl_allreduce_us": nccl_ar, "allreduce_bytes": H * 4, "nvlink_roofline": nvlink}

    # ---- end to end through the public C-ABI call with host buffers (N=1). As the
    # reference's transfer-inclusive timing (src/benchmark.cu:177-206): each step copies
    # x from pinned host memory, runs the captured layer call, copies y back to pinned host.
    e2e = None
    if world > 1:
        # Every rank: the reference's transfer-inclusive step (src/benchmark.cu:177-206) through
        # swb_ffn_tp_host_ex -- x in from page-locked host memory (the same x on every rank), the
        # rank's gate and fused down + exchange, the reduced y out to page-locked host memory --
        # `chain` steps per CUDA graph as for `value`, each step with its own pinned x and y,
        # max over ranks. Beside it, one step per graph with copy operations.
        from swiglu_b200 import tp as T
        n_host = max(chain, 1)
        x_hosts = [(x.float() * (1.0 + 0.01 * k)).half().cpu().pin_memory() for k in range(n_host)]
        y_hosts = [torch.empty(H, dtype=torch.float32).pin_memory() for _ in range(n_host)]
        x_dev = torch.empty_like(x)
        g_id, d_id = (lcfg, 0) if lcfg else (gcfg, dcfg)

        def rank_shard(k):
            s = sets[k % copies]
            return {"wg": s["wg"], "wu": s["wu"], "wd": s["wd"], "bg": bg, "bu": bu}

        def host_step(k):
            T.ffn_tp_host(exchange, x_hosts[k], rank_shard(k), bd, x_dev, h, y, y_hosts[k], g_id, d_id, stream=sp,
                          prefetch_weights=True)

        for k in range(n_host):
            host_step(k)
        torch.cuda.synchronize()
        hg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(hg, stream=stream):
            for k in range(n_host):
                host_step(k)
        for _ in range(max(args.warmup, 3)):
            hg.replay()
        torch.cuda.synchronize()
        dist.barrier()
        reps = max(1, args.steps // n_host)
        e2e_us = time_kernel(torch, lambda i: hg.replay(), reps, stream) / n_host
        hg.reset()
        del hg
        # every step's host y against the device-buffer call on that step's x (all ranks agree)
        bad = 0
        for k in range(n_host):
            T.ffn_tp_fused(exchange, x_hosts[k].to(device), rank_shard(k), bd, h, y, g_id, d_id, stream=sp)
            torch.cuda.synchronize()
            bad += int(not torch.equal(y_hosts[k], y.cpu()))
        x_host, y_host = x_hosts[0], y_hosts[0]
        x_keep = x.clone()

        def e2e_step_tp(i):
            x.copy_(x_host, non_blocking=True)
            graphs[i % copies].replay()
            y_host.copy_(y, non_blocking=True)

        for i in range(max(args.warmup, 3)):
            e2e_step_tp(i)
        dist.barrier()
        copy_us = time_kernel(torch, e2e_step_tp, args.steps, stream)
        x.copy_(x_keep)
        t = torch.tensor([e2e_us, copy_us, bad], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if t[2].item() > 0:
            raise SystemExit("end-to-end output mismatch on some rank")
        e2e = {"value": float(t[0]), "unit": UNIT, "h2d_bytes_per_step": world * H * 2,
               "d2h_bytes_per_step": world * H * 4,
               "path": f"every rank: pinned host x -> swb_ffn_tp_host_ex (C ABI: x in, gate, fused down + "
                       f"exchange, y out as one programmatic chain, SWB_PREFETCH_WEIGHTS) -> pinned host y; "
                       f"{n_host} steps per CUDA graph, each with its own pinned x and y; every step's y checked "
                       f"against swb_ffn_tp_fused_ex",
               "one_step_copy_graph_us": float(t[1]),
               "one_step_copy_graph_path": "every rank: pinned x -> H2D copy -> one captured swb_ffn_tp_fused per "
                                           "graph replay -> D2H copy -> pinned y"}
    if world == 1:
        # The reference's transfer-inclusive protocol (src/benchmark.cu:177-206): every step
        # copies its x in from page-locked host memory, runs the layer and copies y back out,
        # steps back to back in one stream. Through swb_ffn_host_ex (binding.ffn_host): the
        # transfers are kernels in the layer's programmatic chain, so with SWB_PREFETCH_WEIGHTS
        # the next step's gate streams its weights while this step's y and the next x cross
        # PCIe. `chain` steps per CUDA graph as above, each step with its own pinned x and y.
        n_host = max(chain, 1)
        x_hosts = [(common["x"].float() * (1.0 + 0.01 * k)).half().cpu().pin_memory() for k in range(n_host)]
        y_hosts = [torch.empty(H, dtype=torch.float32).pin_memory() for _ in range(n_host)]
        x_dev = torch.empty_like(x)

        def host_step(k):
            s = sets[k % copies]
            binding.ffn_host(x_hosts[k], s["wg"], s["wu"], s["wd"], bg, bu, bd, x_dev, h, y, y_hosts[k], gcfg,
                             dcfg, stream=sp, prefetch_weights=True)

        for k in range(n_host):
            host_step(k)
        torch.cuda.synchronize()
        hg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(hg, stream=stream):
            for k in range(n_host):
                host_step(k)
        for _ in range(max(args.warmup, 3)):
            hg.replay()
        torch.cuda.synchronize()
        reps = max(1, args.steps // n_host)
        e2e_us = time_kernel(torch, lambda i: hg.replay(), reps, stream) / n_host
        hg.reset()
        del hg
        # every step's host y against the device-buffer layer on that step's x
        for k in range(n_host):
            s = sets[k % copies]
            binding.ffn(x_hosts[k].to(device), s["wg"], s["wu"], s["wd"], bg, bu, bd, h, y, gcfg, dcfg, stream=sp)
            torch.cuda.synchronize()
            if not torch.equal(y_hosts[k], y.cpu()):
                raise SystemExit(f"end-to-end output mismatch at step {k}")

        # beside it, the one-step-per-graph protocol with copy operations: pinned x -> H2D ->
        # captured swb_ffn (C ABI) -> D2H -> pinned y, one graph replay per step
        x_host, y_host = x_hosts[0], y_hosts[0]
        e2e_graphs = []

        def public_call(c):
            binding.ffn(x_dev, sets[c]["wg"], sets[c]["wu"], sets[c]["wd"], bg, bu, bd, h, y, gcfg, dcfg,
                        stream=sp)

        for c in range(copies):
            public_call(c)
        torch.cuda.synchronize()
        for c in range(copies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                public_call(c)
            e2e_graphs.append(g)

        def e2e_step(i):
            x_dev.copy_(x_host, non_blocking=True)
            e2e_graphs[i % copies].replay()
            y_host.copy_(y, non_blocking=True)

        for i in range(max(args.warmup, 3)):
            e2e_step(i)
        torch.cuda.synchronize()
        copy_us = time_kernel(torch, e2e_step, args.steps, stream)
        for g in e2e_graphs:
            g.reset()
        del e2e_graphs
        e2e = {"value": e2e_us, "unit": UNIT,
               "h2d_bytes_per_step": x_hosts[0].numel() * x_hosts[0].element_size(),
               "d2h_bytes_per_step": y_hosts[0].numel() * y_hosts[0].element_size(),
               "path": f"pinned host x -> swb_ffn_host_ex (C ABI: x in, gate, down, y out as one programmatic "
                       f"chain, SWB_PREFETCH_WEIGHTS) -> pinned host y; {n_host} steps per CUDA graph, "
                       f"each with its own pinned x and y; every step's y checked against swb_ffn",
               "one_step_copy_graph_us": copy_us,
               "one_step_copy_graph_path": "pinned x -> H2D copy -> one captured swb_ffn per graph replay -> D2H "
                                           "copy -> pinned y"}

    # ---- cuBLAS GemmEx + pointwise on the same GPU (baseline, N=1)
    cublas = None
    if world == 1 and not args.no_cublas:
        base = binding.CublasBaseline(device)
        gbuf = torch.empty(I, dtype=torch.float32, device=device)
        ubuf = torch.empty_like(gbuf)
        hb = torch.empty(I, dtype=torch.float16, device=device)
        yb = torch.empty(H, dtype=torch.float32, device=device)
        res, res_one = {}, {}
        for algo in (0, 1):
            # warm (cuBLAS workspaces), capture and time replays -- the same two protocols as
            # our layer: chained steps per graph, and one step per graph (src/benchmark.cu:46-83)
            def cstep(c, algo=algo):
                base.ffn(x, sets[c]["wg"], sets[c]["wu"], sets[c]["wd"], bg, bu, bd, gbuf, ubuf, hb, yb, algo=algo,
                         stream=sp)
            for c in range(copies):
                cstep(c)
            torch.cuda.synchronize()
            cg = [capture(cstep, c, 1) for c in range(copies)]
            fn = lambda i, cg=cg: cg[i % copies].replay()  # noqa: E731
            for i in range(args.warmup):
                fn(i)
            res_one[algo] = time_kernel(torch, fn, args.steps, stream)
            res[algo] = res_one[algo]
            if chain > 1 and args.steps >= chain:
                cc = capture(cstep, 0, chain)
                cc.replay()
                res[algo] = time_kernel(torch, lambda i: cc.replay(), args.steps // chain, stream) / chain
                cc.reset()
            for g in cg:
                g.reset()
        algo = min(res, key=res.get)
        cublas = {"value": res[algo], "unit": UNIT, "algo": ["default", "default_tensor_op"][algo],
                  "kernels_per_step": 5, "speedup_vs_cublas": res[algo] / us_per_layer,
                  "one_step_graph_us": res_one[algo], "speedup_vs_cublas_one_step_graph": res_one[algo] / one_step_us}
        base.close()

    clocks = sampler.stop(window=tuple(t_window), fallback_window=soak_window)
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(sets, common, H, I, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": us_per_layer, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "one_step_graph_us": one_step_us,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 (fp32 accumulate)",
            "data": "captured-model-fixture" if args.fixture is not None else "synthetic",
            "config": {"workload": f"SwiGLU FFN {H}->{I} batch 1", "hidden": H, "intermediate": I, "batch": 1,
                       "parallelism": f"tp{world}", "gate_config": gcfg, "down_config": dcfg,
                       "layer_config": lcfg or None,
                       "prefetch_weights": bool(flags),
                       "graph": f"{chain} consecutive layer steps per CUDA graph replay (a decode step's FFN "
                                f"layers; weights rotate through {copies} copies)"
                                if chain > 1 else "one step per CUDA graph replay",
                       "rotating_copies": copies,
                       "l2": f"inputs larger than L2: {copies} rotating weight copies of "
                             f"{weight_bytes_rank / 2**20:.0f} MiB per rank",
                       "seed": 0, "weights": "N(0, 1/sqrt(K)) fp16", "x": "N(0,1)", "bias": "N(0,0.02)"}
                      if args.fixture is None else
                      {"workload": f"SwiGLU FFN {H}->{I} batch 1 (captured layer)", "hidden": H, "intermediate": I,
                       "batch": 1, "parallelism": f"tp{world}", "gate_config": gcfg, "down_config": dcfg,
                       "layer_config": lcfg or None, "prefetch_weights": bool(flags),
                       "rotating_copies": copies, "fixture": str(args.fixture)},
            "roofline": roofline, "layer_roofline": layer_roofline, "cpu_baseline": cpu, "e2e": e2e,
            "cublas_baseline": cublas, "tp": tp, "clocks": clocks, "gpu_launches": launches_per_step * args.steps,
            "gpu_name": torch.cuda.get_device_name(device),
        }
        if tuned is not None:
            line["tuning_us"] = {"gate": {str(k): round(v, 3) for k, v in tuned["gate_times"].items()},
                                 "down": {str(k): round(v, 3) for k, v in tuned["down_times"].items()}}
        if pair_times:
            line.setdefault("tuning_us", {})["pairs"] = {f"{g}/{d}": round(v, 3) for (g, d), v in pair_times.items()}
        if layer_times:  # key 0 = the two-kernel step with the tuned gate/down pair
            line.setdefault("tuning_us", {})["layer"] = {str(k): round(v, 3) for k, v in layer_times.items()}
        print(json.dumps(line), flush=True)

    # Release every graph (some hold NCCL all-reduces) before the process group goes.
    torch.cuda.synchronize()
    for gr in graphs + chained:
        gr.reset()
    graphs.clear()
    chained.clear()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
        exchange.close()  # every rank is past its last fused call (barrier above)
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
