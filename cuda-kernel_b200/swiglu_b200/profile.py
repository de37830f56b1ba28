"""Run one fixed decode-layer workload for external profilers (ncu).

Allocates rotating weight copies whose total exceeds the L2 (so DRAM counters
mean something), runs ``--reps`` layers (or only the gate or down kernel) with
fixed registry geometries, synchronises and exits 0. No timing, no tuning: the
launch sequence is identical from run to run, so an ``ncu`` capture can select
launches by index.

    python -m swiglu_b200.profile --gate-config 69 --down-config 67 --reps 20
    python -m swiglu_b200.profile --only gate --gate-config 69 --reps 6
    python -m swiglu_b200.profile --tp-ranks 8 --gate-config 69 --down-config 87 --reps 12
    python -m swiglu_b200.profile --only gate --gate-config 68,69,79 --reps 4

A comma-separated list of ids runs ``--reps`` launches of each geometry in turn
(gate ids with ``--only gate``, down ids with ``--only down``); the plan is
printed first, one line per geometry, so a launch list can be split by geometry
in launch order (``ncu_summary traffic``).

``--tp-ranks n`` runs one tensor-parallel rank's layer (an intermediate shard
of I/n rows) through swb_ffn_tp_fused on a one-rank exchange: the fused down +
exchange kernel with all of its code (slot stores, waits, rank-ordered sum)
in one process on one GPU, which is what an ncu capture may profile.
"""
from __future__ import annotations

import argparse
import math


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--intermediate", type=int, default=14336)
    p.add_argument("--gate-config", type=str, default="69", help="registry id, or ids (comma-separated)")
    p.add_argument("--down-config", type=str, default="67", help="registry id, or ids (comma-separated)")
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--only", choices=("layer", "gate", "down"), default="layer")
    p.add_argument("--tp-ranks", type=int, default=0, help="profile one rank's fused layer at I / n rows")
    p.add_argument("--layer-config", type=int, default=0,
                   help="a whole-layer id (swb_ffn_fused): --only layer runs that kernel instead of the pair")
    p.add_argument("--min-bytes", type=float, default=300e6, help="total weight bytes across copies")
    a = p.parse_args()

    import torch
    from swiglu_b200 import _lib

    H, I = a.hidden, a.intermediate
    gate_ids = [int(v) for v in a.gate_config.split(",") if v]
    down_ids = [int(v) for v in a.down_config.split(",") if v]
    if a.only == "gate":
        plan = [(g, down_ids[0]) for g in gate_ids]
    elif a.only == "down":
        plan = [(gate_ids[0], d) for d in down_ids]
    else:
        if len(gate_ids) != len(down_ids):
            raise SystemExit("a layer plan needs as many gate ids as down ids")
        plan = list(zip(gate_ids, down_ids))
    if a.tp_ranks:
        if I % a.tp_ranks:
            raise SystemExit("intermediate size must divide by --tp-ranks")
        I //= a.tp_ranks
        a.only = "layer"
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    per_copy = (3 if a.only == "layer" else (2 if a.only == "gate" else 1)) * H * I * 2
    copies = max(2, math.ceil(a.min_bytes / per_copy))
    g = torch.Generator(device=dev).manual_seed(0)

    def normal(shape, scale):
        return (torch.randn(shape, generator=g, device=dev) * scale).half()

    sets = []
    for _ in range(copies):
        s = {}
        if a.only in ("layer", "gate"):
            s["wg"], s["wu"] = normal((I, H), H ** -0.5), normal((I, H), H ** -0.5)
        if a.only in ("layer", "down"):
            s["wd"] = normal((H, I), I ** -0.5)
        sets.append(s)
    x, bd = normal((H,), 1.0), normal((H,), 0.02)
    bg, bu = normal((I,), 0.02), normal((I,), 0.02)
    h = normal((I,), 0.5)
    y = torch.empty(H, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.synchronize()
    L = _lib.lib()
    sp = stream.cuda_stream
    ex = None
    if a.tp_ranks:
        from swiglu_b200.tp import Exchange
        ex = Exchange(0, 1, H, dev)
    ws = torch.zeros(_lib.SWB_LAYER_WORKSPACE_BYTES, dtype=torch.uint8, device=dev)
    for k, (gc, dc) in enumerate(plan):
        print(f"plan {k}: {a.reps} x {a.only} gate {gc} down {dc}", flush=True)
    with torch.cuda.stream(stream):
        for gc, dc in plan:
            for i in range(a.reps):
                s = sets[i % copies]
                if ex is not None:
                    rc = L.swb_ffn_tp_fused(ex.handle, a.layer_config or gc, dc, s["wg"].data_ptr(),
                                            s["wu"].data_ptr(), s["wd"].data_ptr(), x.data_ptr(), bg.data_ptr(),
                                            bu.data_ptr(), bd.data_ptr(), h.data_ptr(), y.data_ptr(), H, I, sp)
                elif a.only == "layer" and a.layer_config:
                    rc = L.swb_ffn_fused(a.layer_config, s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(),
                                         x.data_ptr(), bg.data_ptr(), bu.data_ptr(), bd.data_ptr(), h.data_ptr(),
                                         y.data_ptr(), H, I, ws.data_ptr(), sp)
                elif a.only == "layer":
                    rc = L.swb_ffn(gc, dc, s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(), x.data_ptr(),
                                   bg.data_ptr(), bu.data_ptr(), bd.data_ptr(), h.data_ptr(), y.data_ptr(), H, I, sp)
                elif a.only == "gate":
                    rc = L.swb_gate(gc, s["wg"].data_ptr(), s["wu"].data_ptr(), x.data_ptr(), bg.data_ptr(),
                                    bu.data_ptr(), h.data_ptr(), I, H, 0, sp)
                else:
                    rc = L.swb_project(dc, s["wd"].data_ptr(), h.data_ptr(), bd.data_ptr(), x.data_ptr(),
                                       y.data_ptr(), H, I, _lib.SWB_RESIDUAL, sp)
                _lib.check(rc)
    torch.cuda.synchronize()
    if ex is not None:
        ex.close()
    print(f"ran {a.reps} x {a.only} {H}->{I} for each of {len(plan)} geometries"
          f"{' (fused tensor-parallel rank)' if ex is not None else ''}, {copies} copies")


if __name__ == "__main__":
    main()
