"""Per-CTA timeline of the streaming kernels: where a launch's time goes.

Loads the measurement build of the library (``make timeline`` ->
``lib/libswiglu_b200_timeline.so``, ``csrc/timeline.cuh``), in which every CTA of
the BULK, RBULK and SBULK kernels records the GPU's global timer at five points:
entry (0), first ring stage landed (1), last stage consumed (2), results written
(3) and the producer's last copy issued (4). Each run captures `--launches` calls
in one CUDA graph over rotating weight copies (more bytes than L2 holds), replays
it once with recording on, and reports per launch the spread of CTA starts, the
time to the first stage, the spread of CTA ends and the gap to the next launch,
then the steady period between launch starts. For fixed row -> CTA maps it also
ranks SMs by their mean end offset over the launches: an SM that ends late in
every launch streams slower, not later.

Runs: ``down:<id>`` (swb_project with bias and residual), ``gate:<id>``
(swb_gate), ``layer:<gate>/<down>`` (swb_ffn_ex chained with
SWB_PREFETCH_WEIGHTS) and ``plain:<gate>/<down>`` (swb_ffn_ex in plain stream
order).

    make -C cuda-kernel_b200 timeline
    python -m swiglu_b200.timeline --runs down:87,down:100,gate:69,layer:68/87 [--shape 4096x14336]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import statistics
from pathlib import Path

import numpy as np

WORDS = 8
POINTS = ("entry", "first stage", "last stage consumed", "written", "producer done")


def group_launches(rec: np.ndarray, by_time: bool, gap_ns: int = 3000):
    """Split CTA records (in ticket order) into launches. Fixed grids: consecutive
    runs of gridDim records (every CTA of a grid starts before any CTA of the next
    one, in plain stream order and under programmatic launch alike). Work stealing
    (cancelled CTAs never start): split where CTA starts pause for `gap_ns`."""
    if by_time:
        rec = rec[np.argsort(rec[:, 0], kind="stable")]
        t0 = rec[:, 0]
        cuts = [0] + [j for j in range(1, len(t0)) if t0[j] - t0[j - 1] > gap_ns] + [len(t0)]
        return rec, [(cuts[k], cuts[k + 1]) for k in range(len(cuts) - 1)]
    grid = (rec[:, 7] >> 16) & 0xFFFF
    out, i = [], 0
    while i < len(rec):
        g = int(grid[i])
        if g <= 0:
            break
        out.append((i, min(i + g, len(rec))))
        i += g
    return rec, out


def launch_rows(rec: np.ndarray, launches) -> list[dict]:
    base = int(rec[:, 0].min()) if len(rec) else 0
    rows = []
    for a, b in launches:
        r = rec[a:b]
        st = r[:, 0]
        end = np.where(r[:, 3] > 0, r[:, 3], r[:, 2])
        got = r[:, 1] > 0
        prod = r[:, 4] > 0
        rows.append({
            "ctas": int(b - a),
            "start_min": int(st.min() - base), "start_max": int(st.max() - base),
            "first_med": float(np.median(r[got, 1] - st[got])) if got.any() else float("nan"),
            "first_max": float((r[got, 1] - st[got]).max()) if got.any() else float("nan"),
            "end_min": int(end.min() - base), "end_med": float(np.median(end) - base),
            "end_p90": float(np.percentile(end, 90) - base), "end_max": int(end.max() - base),
            "producer_done_med": float(np.median(r[prod, 4] - st[prod])) if prod.any() else float("nan"),
        })
    return rows


def steady(rows: list[dict], rec: np.ndarray, launches) -> dict:
    """Medians over the middle half of the launches (first and last quarter dropped)."""
    n = len(rows)
    mid = range(n // 4, max(n // 4 + 1, 3 * n // 4))
    spans, med_end, tail = [], [], []
    for k in mid:
        a, b = launches[k]
        r = rec[a:b]
        end = np.where(r[:, 3] > 0, r[:, 3], r[:, 2])
        s0 = r[:, 0].min()
        spans.append(end.max() - s0)
        med_end.append(np.median(end) - s0)
        tail.append(end.max() - np.median(end))
    starts = [r["start_min"] for r in rows]
    per = np.diff(starts[2:]) if len(starts) > 4 else np.array([float("nan")])
    return {"span_us": float(np.median(spans)) / 1e3, "median_end_us": float(np.median(med_end)) / 1e3,
            "tail_us": float(np.median(tail)) / 1e3, "period_us": float(np.median(per)) / 1e3}


def sm_ranking(rec: np.ndarray, launches, top: int = 8) -> dict:
    """Mean end offset (from the launch's first start) per SM over the launches."""
    per_sm: dict[int, list[float]] = {}
    for a, b in launches:
        r = rec[a:b]
        end = np.where(r[:, 3] > 0, r[:, 3], r[:, 2])
        s0 = r[:, 0].min()
        for sm, e in zip(((r[:, 7] >> 32) & 0xFFFF).tolist(), (end - s0).tolist()):
            per_sm.setdefault(int(sm), []).append(e / 1e3)
    means = {sm: statistics.fmean(v) for sm, v in per_sm.items()}
    order = sorted(means, key=means.get)
    return {"fastest": [(sm, round(means[sm], 2)) for sm in order[:top]],
            "slowest": [(sm, round(means[sm], 2)) for sm in order[-top:]],
            "spread_us": round(means[order[-1]] - means[order[0]], 2) if order else float("nan")}


def summarise(name: str, rec: np.ndarray, by_time: bool) -> tuple[str, dict]:
    rec, launches = group_launches(rec, by_time)
    rows = launch_rows(rec, launches)
    st = steady(rows, rec, launches)
    lines = [f"== {name}: {len(rec)} CTA records, {len(rows)} launches"]
    lines.append("launch ctas | start min..max us | first stage med/max us | end min / med / p90 / max us "
                 "| producer done med us | gap to next start us")
    for j, r in enumerate(rows):
        gap = (rows[j + 1]["start_min"] - r["end_max"]) / 1e3 if j + 1 < len(rows) else float("nan")
        lines.append(f"{j:3d} {r['ctas']:4d} | {r['start_min'] / 1e3:8.2f}..{r['start_max'] / 1e3:8.2f} | "
                     f"{r['first_med'] / 1e3:5.2f}/{r['first_max'] / 1e3:5.2f} | {r['end_min'] / 1e3:8.2f} / "
                     f"{r['end_med'] / 1e3:8.2f} / {r['end_p90'] / 1e3:8.2f} / {r['end_max'] / 1e3:8.2f} | "
                     f"{r['producer_done_med'] / 1e3:6.2f} | {gap:6.2f}")
    lines.append(f"steady: period {st['period_us']:.2f} us between launch starts; span {st['span_us']:.2f} us; "
                 f"median CTA end {st['median_end_us']:.2f} us; last end - median end {st['tail_us']:.2f} us")
    out = {"name": name, "steady": st}
    if not by_time:
        sm = sm_ranking(rec, launches)
        lines.append(f"per-SM mean end: spread {sm['spread_us']} us; fastest {sm['fastest']}; slowest {sm['slowest']}")
        out["sm"] = sm
    return "\n".join(lines), out


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--runs", default="down:87,down:100,down:101,gate:68,gate:69,layer:68/87,layer:69/101")
    p.add_argument("--shape", default="4096x14336", help="hidden x intermediate (a tensor-parallel shard: "
                   "its intermediate slice)")
    p.add_argument("--launches", type=int, default=20)
    p.add_argument("--copies", type=int, default=0, help="rotating weight copies (default: above 2x L2)")
    p.add_argument("--lib", default=None, help="timeline library (default lib/libswiglu_b200_timeline.so)")
    p.add_argument("--output", default=None, help="write a JSON summary here")
    a = p.parse_args(argv)

    import torch
    from . import _lib
    L = _lib.timeline_lib(a.lib)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    H, I = (int(v) for v in a.shape.lower().split("x"))
    layer_bytes = 3 * H * I * 2
    copies = a.copies or max(2, -(-(2 * 126 * 2 ** 20) // layer_bytes))
    gen = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, scale=0.02):
        return (torch.randn(*shape, device=dev, generator=gen) * scale).half()

    sets = [{"wg": rnd(I, H), "wu": rnd(I, H), "wd": rnd(H, I)} for _ in range(copies)]
    v = {"x": rnd(H, scale=1.0), "bg": rnd(I), "bu": rnd(I), "bd": rnd(H),
         "h": torch.empty(I, dtype=torch.float16, device=dev), "y": torch.empty(H, dtype=torch.float32, device=dev)}

    def check(status):
        if status:
            raise RuntimeError((L.swb_last_error() or L.swb_status_string(status)).decode())

    def family(cid):
        info = _lib.SwbConfig()
        check(L.swb_config_info(cid, ctypes.byref(info)))
        return info.family

    def step_fn(kind, spec):
        if kind == "down":
            c = int(spec)
            return (lambda i, sp: L.swb_project(c, sets[i % copies]["wd"].data_ptr(), v["h"].data_ptr(),
                                                v["bd"].data_ptr(), v["x"].data_ptr(), v["y"].data_ptr(), H, I,
                                                _lib.SWB_RESIDUAL, sp)), family(c) == _lib.SWB_FAMILY_SBULK
        if kind == "gate":
            c = int(spec)
            return (lambda i, sp: L.swb_gate(c, sets[i % copies]["wg"].data_ptr(), sets[i % copies]["wu"].data_ptr(),
                                             v["x"].data_ptr(), v["bg"].data_ptr(), v["bu"].data_ptr(),
                                             v["h"].data_ptr(), I, H, 0, sp)), family(c) == _lib.SWB_FAMILY_SBULK
        g, d = (int(t) for t in spec.split("/"))
        flags = _lib.SWB_PREFETCH_WEIGHTS if kind == "layer" else 0

        def f(i, sp):
            s = sets[i % copies]
            return L.swb_ffn_ex(g, d, s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(), v["x"].data_ptr(),
                                v["bg"].data_ptr(), v["bu"].data_ptr(), v["bd"].data_ptr(), v["h"].data_ptr(),
                                v["y"].data_ptr(), H, I, flags, sp)
        return f, _lib.SWB_FAMILY_SBULK in (family(g), family(d))

    cap = L.swb_timeline_capacity()
    results = []
    stream = torch.cuda.Stream(dev)
    for run in [r for r in a.runs.split(",") if r]:
        kind, spec = run.split(":")
        fn, by_time = step_fn(kind, spec)
        sp = stream.cuda_stream
        with torch.cuda.stream(stream):
            for i in range(copies):
                check(fn(i, sp))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(a.launches):
                    check(fn(i, sp))
            g.replay()
        torch.cuda.synchronize()
        check(L.swb_timeline_reset())
        with torch.cuda.stream(stream):
            g.replay()
        buf = np.zeros(cap * WORDS, dtype=np.uint64)
        n = ctypes.c_uint(0)
        check(L.swb_timeline_read(buf.ctypes.data, ctypes.byref(n)))
        g.reset()
        rec = buf[: min(n.value, cap) * WORDS].reshape(-1, WORDS).astype(np.int64)
        text, summary = summarise(f"{run} at {H}x{I}", rec, by_time)
        print(text, flush=True)
        results.append(summary)
    if a.output:
        Path(a.output).write_text(json.dumps({"shape": [H, I], "copies": copies, "launches": a.launches,
                                              "runs": results}, indent=1))


if __name__ == "__main__":
    main()
