"""Validate kernel-benchmark evidence (schema v1) and render a conservative comparison.

Same contract as tools/report.py of shubhxho/cuda-kernel (:9-111): a report is
rejected for an unknown schema or timing protocol, unknown data provenance,
missing GPU identity or versions, fewer than 3 holdout samples, duplicate or
unknown cases, non-positive timings, non-finite or failing correctness evidence,
medians that do not match their raw samples, or a speedup that does not match
the medians. A "separated win" needs a median speedup >= 1.05 and every custom
sample below every baseline sample (:82-84). Rendering adds the B200 roofline:
algorithmic bytes per case and the achieved fraction of the HBM peak.
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


def positive(v) -> bool:
    return isinstance(v, (float, int)) and not isinstance(v, bool) and math.isfinite(v) and v > 0


def validate(report: dict) -> dict:
    if report.get("schema_version") != 1 or report.get("timing") != "cuda-graph-events":
        raise ValueError("unsupported benchmark schema or timing protocol")
    if report.get("data") not in DATA:
        raise ValueError("unknown data provenance")
    if not report.get("gpu") or not report.get("cases"):
        raise ValueError("missing GPU identity or workload cases")
    for key in ("driver_version", "runtime_version", "cublas_version", "repeats", "samples"):
        if not positive(report.get(key)) or not isinstance(report[key], int):
            raise ValueError(f"missing or invalid {key}")
    if report["samples"] < 3:
        raise ValueError("insufficient holdout samples")
    seen = set()
    for case in report["cases"]:
        ident = (case.get("shape"), case.get("operation"))
        if ident in seen:
            raise ValueError("duplicate benchmark case")
        seen.add(ident)
        if case.get("operation") not in OPERATIONS:
            raise ValueError("unknown benchmark operation")
        for key in ("hidden", "intermediate"):
            if not positive(case.get(key)) or not isinstance(case[key], int):
                raise ValueError("invalid workload dimensions")
        for side in ("custom", "baseline"):
            c = case[side]
            values = c["samples_us"]
            if c.get("correct") is not True or len(values) != report["samples"]:
                raise ValueError("incorrect or incomplete candidate")
            if not all(positive(v) for v in values):
                raise ValueError("invalid GPU event timings")
            for key in ("max_abs_error", "max_scaled_error"):
                v = c.get(key)
                if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v) or v < 0:
                    raise ValueError("invalid correctness evidence")
            if c["max_scaled_error"] > 1:
                raise ValueError("numeric tolerance failed")
            if not math.isclose(c["median_us"], statistics.median(values), rel_tol=1e-7):
                raise ValueError("median does not match raw samples")
        ratio = case["baseline"]["median_us"] / case["custom"]["median_us"]
        if not math.isclose(ratio, case["speedup"], rel_tol=1e-7):
            raise ValueError("speedup does not match timings")
        transfer = case.get("transfer_inclusive")
        if transfer is not None:
            for side in ("custom", "baseline"):
                values = transfer[side]["samples_us"]
                if len(values) != report["samples"] or not all(positive(v) for v in values):
                    raise ValueError("invalid transfer-inclusive timings")
                if not math.isclose(transfer[side]["median_us"], statistics.median(values), rel_tol=1e-7):
                    raise ValueError("transfer median does not match raw samples")
    return report


def separated_win(case: dict) -> bool:
    return case["speedup"] >= 1.05 and max(case["custom"]["samples_us"]) < min(case["baseline"]["samples_us"])


def _p95(xs):
    xs = sorted(xs)
    return xs[math.ceil(0.95 * len(xs)) - 1]


def case_bytes(case: dict) -> int:
    h, i = case["hidden"], case["intermediate"]
    return intensity.projection(h, i)["bytes"] if case["operation"] == "projection" else intensity.layer(h, i)["bytes"]


def render(report: dict, hbm_gbs: float | None = None) -> str:
    validate(report)
    peak = hbm_gbs or report.get("hbm_peak_gbs") or intensity.measured_peaks()["hbm_gbs"]
    lines = [f"GPU: {report['gpu']} (SM {report.get('compute_capability', '?')}).",
             f"CUDA runtime {report['runtime_version']}; cuBLAS {report['cublas_version']}."]
    if report.get("result_class"):
        lines.append(f"Result class: `{report['result_class']}`.")
    lines += ["", f"Data: `{report['data']}`. Rotating weight copies larger than L2; warmed CUDA graphs; "
              "GPU event timing.", "Kernel-only holdout samples follow tuning. Reference checks and tuning are "
              "excluded from latency.", "",
              f"| Workload | Operation | Custom µs | cuBLAS µs | Ratio | Evidence | Bytes | Custom GB/s | % of {peak:.0f} GB/s |",
              "|---|---|---:|---:|---:|---|---:|---:|---:|"]
    for c in report["cases"]:
        a, b = c["custom"], c["baseline"]
        evidence = "separated win" if separated_win(c) else ("slower" if c["speedup"] < 1 else "inconclusive")
        nbytes = case_bytes(c)
        gbs = nbytes / (a["median_us"] * 1e-6) / 1e9
        lines.append(f"| {c['shape']} | {c['operation']} | {a['median_us']:.3f} | {b['median_us']:.3f} | "
                     f"{c['speedup']:.3f}× | {evidence} | {nbytes} | {gbs:.0f} | {100 * gbs / peak:.1f} |")
    lines += ["", "Tail latency (nearest-rank p95 of replay-batch averages):", "",
              "| Workload | Operation | Custom p95 µs | Baseline p95 µs |", "|---|---|---:|---:|"]
    for c in report["cases"]:
        lines.append(f"| {c['shape']} | {c['operation']} | {_p95(c['custom']['samples_us']):.3f} | "
                     f"{_p95(c['baseline']['samples_us']):.3f} |")
    if any("transfer_inclusive" in c for c in report["cases"]):
        lines += ["", "Transfer-inclusive (pinned H2D of the token input, kernel graph, D2H of the output; "
                  "weights resident):", "",
                  "| Workload | Operation | Custom µs | cuBLAS µs | Custom p95 µs | Baseline p95 µs |",
                  "|---|---|---:|---:|---:|---:|"]
        for c in report["cases"]:
            t = c.get("transfer_inclusive")
            if t:
                lines.append(f"| {c['shape']} | {c['operation']} | {t['custom']['median_us']:.3f} | "
                             f"{t['baseline']['median_us']:.3f} | {_p95(t['custom']['samples_us']):.3f} | "
                             f"{_p95(t['baseline']['samples_us']):.3f} |")
    lines += ["", "A separated win requires at least 5% median speedup and every custom sample below every "
              "baseline sample.", "This compares the selected cuBLAS GemmEx algorithms, not cuBLASLt or "
              "TensorRT-LLM. Synthetic shapes are not pretrained-model evidence."]
    return "\n".join(lines) + "\n"


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("input", type=Path)
    p.add_argument("--output", type=Path)
    p.add_argument("--require-win", action="store_true")
    p.add_argument("--require-all-wins", action="store_true")
    a = p.parse_args()
    report = validate(json.loads(a.input.read_text()))
    text = render(report)
    if a.output:
        a.output.write_text(text)
    else:
        print(text, end="")
    if a.require_all_wins and not all(separated_win(c) for c in report["cases"]):
        raise SystemExit("Not every benchmark has a separated win")
    if a.require_win and not any(separated_win(c) for c in report["cases"]):
        raise SystemExit("No separated win measured")


if __name__ == "__main__":
    main()
