"""Kernel evidence (schema v1): check every claim against its raw samples, then render it.

A tuner result (``swiglu_b200.tuner``) is accepted only when all of this holds,
and every violation found is listed in one error:

* header -- schema 1 with CUDA-graph event timing, a known data provenance, a
  GPU name, positive integer driver / runtime / cuBLAS versions and repeat and
  sample counts, at least three holdout samples per candidate;
* cases -- each (shape, operation) once, a known operation, positive integer
  dimensions;
* each side (custom and cuBLAS) -- marked correct, finite non-negative error
  figures with the scaled error within tolerance (<= 1), exactly ``samples``
  positive finite timings whose median is the recorded median;
* the recorded speedup equals baseline median / custom median, and any
  transfer-inclusive timings obey the same sample rules.

The verdict of a case is a "separated win" only when the median speedup is at
least 1.05 and the custom kernel's slowest sample beats the baseline's fastest
(the rule the reference's report states); "slower" below parity, otherwise
"inconclusive". Rendering adds the B200 roofline of each case: algorithmic
bytes, achieved GB/s and the fraction of the HBM copy peak.
"""
from __future__ import annotations

import argparse
import json
import math
import statistics
from pathlib import Path

from . import intensity

DATA = ("synthetic-fp16-model-shapes", "captured-model-fixture")
OPERATIONS = ("projection", "swiglu-ffn")
SIDES = ("custom", "baseline")
WIN_RATIO = 1.05


class EvidenceError(ValueError):
    """Raised with every problem found in a report."""


def positive(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(v) and v > 0


def _count(v) -> bool:
    return positive(v) and isinstance(v, int)


def _same(a, b) -> bool:
    return positive(a) and positive(b) and math.isclose(a, b, rel_tol=1e-7)


def _timings(where: str, block, n: int) -> list[str]:
    """Rules for one list of samples and its median."""
    if not isinstance(block, dict):
        return [f"{where}: no timing block"]
    xs = block.get("samples_us")
    if not isinstance(xs, list) or len(xs) != n:
        return [f"{where}: expected {n} samples"]
    if not all(positive(x) for x in xs):
        return [f"{where}: a sample is not a positive finite time"]
    if not _same(block.get("median_us"), statistics.median(xs)):
        return [f"{where}: recorded median is not the median of its samples"]
    return []


def _side(where: str, c, n: int) -> list[str]:
    if not isinstance(c, dict):
        return [f"{where}: missing"]
    out = [] if c.get("correct") is True else [f"{where}: not marked correct"]
    for key in ("max_abs_error", "max_scaled_error"):
        v = c.get(key)
        if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v) or v < 0:
            out.append(f"{where}: {key} is not a finite non-negative number")
        elif key == "max_scaled_error" and v > 1:
            out.append(f"{where}: outside the numeric tolerance (scaled error {v:g})")
    return out + _timings(where, c, n)


def problems(report: dict) -> list[str]:
    """Every rule the report breaks (empty when it is valid evidence)."""
    if not isinstance(report, dict):
        return ["not a JSON object"]
    out = []
    if report.get("schema_version") != 1:
        out.append("schema_version is not 1")
    if report.get("timing") != "cuda-graph-events":
        out.append("timing protocol is not cuda-graph-events")
    if report.get("data") not in DATA:
        out.append(f"data provenance {report.get('data')!r} is not one of {DATA}")
    if not report.get("gpu"):
        out.append("no GPU identity")
    for key in ("driver_version", "runtime_version", "cublas_version", "repeats", "samples"):
        if not _count(report.get(key)):
            out.append(f"{key} is not a positive integer")
    n = report.get("samples")
    if _count(n) and n < 3:
        out.append("fewer than 3 holdout samples")
    cases = report.get("cases")
    if not isinstance(cases, list) or not cases:
        return out + ["no cases"]
    idents = [(c.get("shape"), c.get("operation")) for c in cases if isinstance(c, dict)]
    if len(idents) != len(cases):
        out.append("a case is not an object")
    if len(set(idents)) != len(idents):
        out.append("the same (shape, operation) appears twice")
    for c in (c for c in cases if isinstance(c, dict)):
        tag = f"{c.get('shape')}/{c.get('operation')}"
        if c.get("operation") not in OPERATIONS:
            out.append(f"{tag}: unknown operation")
        if not (_count(c.get("hidden")) and _count(c.get("intermediate"))):
            out.append(f"{tag}: dimensions are not positive integers")
        for side in SIDES:
            out += _side(f"{tag} {side}", c.get(side), n)
        try:
            ratio = c["baseline"]["median_us"] / c["custom"]["median_us"]
            if not _same(ratio, c.get("speedup")):
                out.append(f"{tag}: speedup is not baseline median / custom median")
        except (KeyError, TypeError, ZeroDivisionError):
            out.append(f"{tag}: speedup cannot be recomputed")
        tr = c.get("transfer_inclusive")
        if tr is not None:
            for side in SIDES:
                out += _timings(f"{tag} transfer-inclusive {side}", tr.get(side) if isinstance(tr, dict) else None, n)
    return out


def validate(report: dict) -> dict:
    found = problems(report)
    if found:
        raise EvidenceError(f"{len(found)} problem(s) in the evidence: " + "; ".join(found))
    return report


def separated_win(case: dict) -> bool:
    return case["speedup"] >= WIN_RATIO and max(case["custom"]["samples_us"]) < min(case["baseline"]["samples_us"])


def verdict(case: dict) -> str:
    if separated_win(case):
        return "separated win"
    return "slower" if case["speedup"] < 1 else "inconclusive"


def p95(xs) -> float:
    """Nearest-rank 95th percentile."""
    ordered = sorted(xs)
    return ordered[max(0, math.ceil(0.95 * len(ordered)) - 1)]


def case_bytes(case: dict) -> int:
    h, i = case["hidden"], case["intermediate"]
    model = intensity.projection if case["operation"] == "projection" else intensity.layer
    return model(h, i)["bytes"]


def _table(header: list[str], align: str, rows: list[list[str]]) -> list[str]:
    rule = ["---:" if a == "r" else "---" for a in align]
    return ["| " + " | ".join(header) + " |", "| " + " | ".join(rule) + " |"] + \
           ["| " + " | ".join(r) + " |" for r in rows]


def render(report: dict, hbm_gbs: float | None = None) -> str:
    validate(report)
    peak = hbm_gbs or report.get("hbm_peak_gbs") or intensity.measured_peaks()["hbm_gbs"]
    cases = report["cases"]
    main_rows = []
    for c in cases:
        nbytes = case_bytes(c)
        gbs = nbytes / (c["custom"]["median_us"] * 1e-6) / 1e9
        main_rows.append([c["shape"], c["operation"], f"{c['custom']['median_us']:.3f}",
                          f"{c['baseline']['median_us']:.3f}", f"{c['speedup']:.3f}×", verdict(c), str(nbytes),
                          f"{gbs:.0f}", f"{100 * gbs / peak:.1f}"])
    tail_rows = [[c["shape"], c["operation"], f"{p95(c['custom']['samples_us']):.3f}",
                  f"{p95(c['baseline']['samples_us']):.3f}"] for c in cases]
    text = [f"Evidence from {report['gpu']} (compute capability {report.get('compute_capability', '?')}), "
            f"CUDA runtime {report['runtime_version']}, cuBLAS {report['cublas_version']}"
            + (f", result class `{report['result_class']}`." if report.get("result_class") else "."),
            "",
            f"Inputs: `{report['data']}`, weights rotated through copies larger than L2. Each candidate is a "
            f"warmed CUDA graph timed with GPU events, {report['samples']} holdout samples of {report['repeats']} "
            "replays after tuning; the correctness checks and the tuning itself are not in the times.",
            ""]
    text += _table(["Workload", "Operation", "Custom µs", "cuBLAS µs", "Ratio", "Verdict", "Bytes",
                    "Custom GB/s", f"% of {peak:.0f} GB/s"], "llrrrlrrr", main_rows)
    text += ["", "95th percentile (nearest rank) of the holdout samples:", ""]
    text += _table(["Workload", "Operation", "Custom p95 µs", "cuBLAS p95 µs"], "llrr", tail_rows)
    moved = [c for c in cases if c.get("transfer_inclusive")]
    if moved:
        rows = [[c["shape"], c["operation"]] + [f"{c['transfer_inclusive'][s]['median_us']:.3f}" for s in SIDES] +
                [f"{p95(c['transfer_inclusive'][s]['samples_us']):.3f}" for s in SIDES] for c in moved]
        text += ["", "Transfer-inclusive (the token input copied in from pinned host memory, the graph, the "
                 "output copied back; weights stay resident):", ""]
        text += _table(["Workload", "Operation", "Custom µs", "cuBLAS µs", "Custom p95 µs", "cuBLAS p95 µs"],
                       "llrrrr", rows)
    text += ["", f"Verdicts: a separated win needs a median ratio of at least {WIN_RATIO} and the slowest custom "
             "sample faster than the fastest cuBLAS sample. The baseline is cuBLAS GemmEx with the faster of its "
             "default algorithms plus two pointwise kernels; synthetic weights say nothing about a trained model."]
    return "\n".join(text) + "\n"


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("input", type=Path)
    p.add_argument("--output", type=Path)
    p.add_argument("--require-win", action="store_true", help="fail unless some case is a separated win")
    p.add_argument("--require-all-wins", action="store_true", help="fail unless every case is a separated win")
    a = p.parse_args(argv)
    report = json.loads(a.input.read_text())
    text = render(report)
    if a.output:
        a.output.write_text(text)
    else:
        print(text, end="")
    wins = [separated_win(c) for c in report["cases"]]
    if a.require_all_wins and not all(wins):
        raise SystemExit(f"{wins.count(False)} case(s) without a separated win")
    if a.require_win and not any(wins):
        raise SystemExit("no case has a separated win")


if __name__ == "__main__":
    main()
