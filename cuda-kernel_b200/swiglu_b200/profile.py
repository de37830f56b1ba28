"""Run one fixed decode-layer workload for external profilers (ncu).

Allocates rotating weight copies whose total exceeds the L2 (so DRAM counters
mean something), runs ``--reps`` layers (or only the gate or down kernel) with
fixed registry geometries, synchronises and exits 0. No timing, no tuning: the
launch sequence is identical from run to run, so an ``ncu`` capture can select
launches by index.

    python -m swiglu_b200.profile --gate-config 69 --down-config 67 --reps 20
    python -m swiglu_b200.profile --only gate --gate-config 69 --reps 6
    python -m swiglu_b200.profile --tp-ranks 8 --gate-config 69 --down-config 87 --reps 12

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
    p.add_argument("--gate-config", type=int, default=69)
    p.add_argument("--down-config", type=int, default=67)
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--only", choices=("layer", "gate", "down"), default="layer")
    p.add_argument("--tp-ranks", type=int, default=0, help="profile one rank's fused layer at I / n rows")
    p.add_argument("--min-bytes", type=float, default=300e6, help="total weight bytes across copies")
    a = p.parse_args()

    import torch
    from swiglu_b200 import _lib

    H, I = a.hidden, a.intermediate
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
    with torch.cuda.stream(stream):
        for i in range(a.reps):
            s = sets[i % copies]
            if ex is not None:
                rc = L.swb_ffn_tp_fused(ex.handle, a.gate_config, a.down_config, s["wg"].data_ptr(), s["wu"].data_ptr(),
                                        s["wd"].data_ptr(), x.data_ptr(), bg.data_ptr(), bu.data_ptr(), bd.data_ptr(),
                                        h.data_ptr(), y.data_ptr(), H, I, sp)
            elif a.only == "layer":
                rc = L.swb_ffn(a.gate_config, a.down_config, s["wg"].data_ptr(), s["wu"].data_ptr(),
                               s["wd"].data_ptr(), x.data_ptr(), bg.data_ptr(), bu.data_ptr(), bd.data_ptr(),
                               h.data_ptr(), y.data_ptr(), H, I, sp)
            elif a.only == "gate":
                rc = L.swb_gate(a.gate_config, s["wg"].data_ptr(), s["wu"].data_ptr(), x.data_ptr(), bg.data_ptr(),
                                bu.data_ptr(), h.data_ptr(), I, H, 0, sp)
            else:
                rc = L.swb_project(a.down_config, s["wd"].data_ptr(), h.data_ptr(), bd.data_ptr(), x.data_ptr(),
                                   y.data_ptr(), H, I, _lib.SWB_RESIDUAL, sp)
            _lib.check(rc)
    torch.cuda.synchronize()
    if ex is not None:
        ex.close()
    print(f"ran {a.reps} x {a.only} {H}->{I} (configs {a.gate_config}/{a.down_config}"
          f"{', fused tensor-parallel rank' if ex is not None else ''}), {copies} copies")


if __name__ == "__main__":
    main()
