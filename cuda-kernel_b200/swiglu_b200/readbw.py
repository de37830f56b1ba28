"""Sustained HBM read bandwidth of the gate kernels, against torch's copy and sum.

The layer's roofline uses the pool's measured copy bandwidth (read + write) as its
peak; a GEMV only reads. This measures what the gate kernels themselves read per
second when one launch streams much more than its ramp and tail cost: Wg and Wu of
`--rows` x 4096 fp16 each (1 GiB each at the default 131072 rows, two copies
alternating, so every launch comes from HBM), CUDA events around single launches,
median of `--reps`. The same kernels at the 14336-row layer shape are timed beside
it, so the difference is the per-launch cost. Prints one line per measurement.

    python -m swiglu_b200.readbw [--rows 131072] [--configs 68,69,83,96] [--reps 7]
"""
from __future__ import annotations

import argparse
import statistics


def _median_us(torch, fn, reps):
    fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        out.append(a.elapsed_time(b) * 1e3)
    return statistics.median(out)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--rows", type=int, default=131072)
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--configs", type=str, default="33,64,68,69,79,83,87,96")
    p.add_argument("--reps", type=int, default=7)
    a = p.parse_args(argv)

    import torch
    from . import _lib
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    H = a.hidden
    src = torch.empty(512 * 2 ** 20, dtype=torch.float16, device=dev).normal_()
    dst = torch.empty_like(src)
    us = _median_us(torch, lambda: dst.copy_(src), a.reps)
    print(f"torch copy 1 GiB -> 1 GiB: {2 * src.numel() * 2 / us / 1e3:.1f} GB/s (read + write)")
    us = _median_us(torch, lambda: src.sum(dtype=torch.float32), a.reps)
    print(f"torch sum of 1 GiB: {src.numel() * 2 / us / 1e3:.1f} GB/s (read)")
    del src, dst
    torch.cuda.empty_cache()
    s = torch.cuda.current_stream().cuda_stream
    ids = [int(v) for v in a.configs.split(",") if v]
    for rows in (14336, a.rows):
        mats = [torch.empty(rows, H, dtype=torch.float16, device=dev).normal_() for _ in range(4)]
        x = torch.randn(H, device=dev).half()
        h = torch.empty(rows, dtype=torch.float16, device=dev)
        for cfg in ids:
            k = [0]

            def launch(cfg=cfg):
                k[0] ^= 1
                wg, wu = mats[2 * k[0]], mats[2 * k[0] + 1]
                _lib.check(L.swb_gate(cfg, wg.data_ptr(), wu.data_ptr(), x.data_ptr(), None, None, h.data_ptr(),
                                      rows, H, 0, s))
            us = _median_us(torch, launch, a.reps)
            print(f"gate {cfg} rows {rows}: {us:.2f} us, {2 * rows * H * 2 / us / 1e3:.1f} GB/s (read)")
        del mats
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
