"""Summarise ncu output into the short text kept under profiles/.

    python -m swiglu_b200.ncu_summary launches <launches.csv>     # per-kernel launches, time, share
    python -m swiglu_b200.ncu_summary report <file.ncu-rep>       # key counters of each captured launch
    python -m swiglu_b200.ncu_summary traffic <metrics.csv> <reps> <id,id,...>
        # DRAM bytes per launch of each geometry of a `profile` plan (launches in plan order)

`launches` reads a `--metrics gpu__time_duration.sum --csv` log; `report` runs
`ncu -i <rep> --page raw --csv` (no GPU needed) and prints the DRAM, L2, SM and
stall counters used for the roofline and its `traffic` figure.
"""
from __future__ import annotations

import collections
import csv
import io
import statistics
import subprocess
import sys

_UNIT = {"ns": 1e-3, "nsecond": 1e-3, "us": 1.0, "usecond": 1.0, "ms": 1e3, "msecond": 1e3, "s": 1e6, "second": 1e6}

KEYS = [
    "gpu__time_duration.sum", "dram__bytes_read.sum", "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "dram__bytes_read.sum.per_second",
    "lts__t_sector_hit_rate.pct", "lts__throughput.avg.pct_of_peak_sustained_elapsed",
    "l1tex__throughput.avg.pct_of_peak_sustained_active", "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__warps_active.avg.pct_of_peak_sustained_active", "smsp__issue_active.avg.pct_of_peak_sustained_active",
    "launch__registers_per_thread", "launch__grid_size", "launch__block_size",
    "launch__shared_mem_per_block_dynamic", "sm__cycles_elapsed.avg.per_second",
]


def launches(path: str) -> str:
    text = open(path, encoding="utf-8", errors="replace").read()
    lines = text.splitlines()
    start = next(i for i, l in enumerate(lines) if "Kernel Name" in l and "Metric Name" in l)
    rows = list(csv.reader(io.StringIO("\n".join(lines[start:]))))
    hdr = rows[0]
    k, m, v, u = (hdr.index(x) for x in ("Kernel Name", "Metric Name", "Metric Value", "Metric Unit"))
    agg = collections.OrderedDict()
    for r in rows[1:]:
        if len(r) <= v or r[m] != "gpu__time_duration.sum":
            continue
        us = float(r[v].replace(",", "")) * _UNIT.get(r[u], 1.0)
        name = r[k].split("(")[0]
        c, t = agg.get(name, (0, 0.0))
        agg[name] = (c + 1, t + us)
    total = sum(t for _, t in agg.values())
    out = [f"{'launches':>8} {'total us':>10} {'mean us':>9} {'share':>6}  kernel"]
    for name, (c, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        out.append(f"{c:8d} {t:10.1f} {t / c:9.2f} {100 * t / total:5.1f}%  {name}")
    return "\n".join(out)


def report(path: str) -> str:
    raw = subprocess.run(["ncu", "-i", path, "--page", "raw", "--csv"], capture_output=True, text=True,
                         check=True).stdout
    rows = list(csv.reader(io.StringIO(raw)))
    hdr, units, data = rows[0], rows[1], rows[2:]
    out = []
    for n, d in enumerate(data):
        out.append(f"launch {n}: {d[hdr.index('Kernel Name')]}")
        for key in KEYS:
            if key in hdr:
                i = hdr.index(key)
                out.append(f"  {key} = {d[i]} {units[i]}")
        stalls = []
        for i, h in enumerate(hdr):
            if h.startswith("smsp__average_warps_issue_stalled_") and h.endswith("per_issue_active.ratio"):
                try:
                    val = float(d[i])
                except ValueError:
                    continue
                if val >= 0.1:
                    stalls.append((val, h[len("smsp__average_warps_issue_stalled_"):-len("_per_issue_active.ratio")]))
        out.append("  stalls per issue: " + ", ".join(f"{s} {v:.2f}" for v, s in sorted(stalls, reverse=True)))
        rd, wr = hdr.index("dram__bytes_read.sum"), hdr.index("dram__bytes_write.sum")
        scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
        traffic = float(d[rd]) * scale.get(units[rd], 1) + float(d[wr]) * scale.get(units[wr], 1)
        out.append(f"  traffic (dram read + write) = {traffic:.0f} bytes")
    return "\n".join(out)


def _per_launch(path: str) -> list[dict]:
    """Rows of a `--metrics ... --csv` log grouped by launch ID, in launch order."""
    text = open(path, encoding="utf-8", errors="replace").read()
    lines = text.splitlines()
    start = next(i for i, l in enumerate(lines) if "Kernel Name" in l and "Metric Name" in l)
    rows = list(csv.reader(io.StringIO("\n".join(lines[start:]))))
    hdr = rows[0]
    idc, k, m, v, u = (hdr.index(x) for x in ("ID", "Kernel Name", "Metric Name", "Metric Value", "Metric Unit"))
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "KB": 1e3, "MB": 1e6, "GB": 1e9}
    out = collections.OrderedDict()
    for r in rows[1:]:
        if len(r) <= v:
            continue
        d = out.setdefault(r[idc], {"kernel": r[k].split("(")[0]})
        val = float(r[v].replace(",", ""))
        if r[m] == "gpu__time_duration.sum":
            d["us"] = val * _UNIT.get(r[u], 1.0)
        else:
            d[r[m]] = val * scale.get(r[u], 1.0)
    return list(out.values())


def traffic(path: str, reps: int, ids: list[int]) -> str:
    """Per geometry of a profile plan (`reps` launches of each id, in order): mean DRAM read,
    write and duration per launch, and the `traffic_bytes_per_launch[<id>]` line bench.py reads."""
    launches_ = _per_launch(path)
    if len(launches_) != reps * len(ids):
        raise SystemExit(f"{len(launches_)} launches in the log, the plan has {reps} x {len(ids)}")
    out = []
    for n, cid in enumerate(ids):
        block = launches_[n * reps:(n + 1) * reps]
        rd = statistics.mean(b["dram__bytes_read.sum"] for b in block)
        wr = statistics.mean(b["dram__bytes_write.sum"] for b in block)
        us = statistics.mean(b["us"] for b in block) if all("us" in b for b in block) else float("nan")
        out.append(f"config {cid}: {block[0]['kernel']}, {reps} launches: read {rd / 1e6:.3f} MB, "
                   f"write {wr / 1e6:.3f} MB, {us:.2f} us (serialised)")
        out.append(f"traffic_bytes_per_launch[{cid}]: {rd + wr:.0f}")
    return "\n".join(out)


def main(argv=None):
    argv = argv or sys.argv[1:]
    if len(argv) == 4 and argv[0] == "traffic":
        print(traffic(argv[1], int(argv[2]), [int(v) for v in argv[3].split(",") if v]))
        return
    if len(argv) != 2 or argv[0] not in ("launches", "report"):
        raise SystemExit(__doc__)
    print(launches(argv[1]) if argv[0] == "launches" else report(argv[1]))


if __name__ == "__main__":
    main()
