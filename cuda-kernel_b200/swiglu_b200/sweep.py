"""Repeatable multi-seed GPU sweep (tools/sweep.py of shubhxho/cuda-kernel, :8-26).

Seeds {17, 101, 997} x suites {correctness, decode}: each run is the tuner with
its correctness gates; the sweep stops at the first failing gate and keeps the
command log. --model adds the decode-MLP replacement runner and its report.
"""
from __future__ import annotations

import argparse
import json
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--output", type=Path, default=Path("results/sweep"))
    p.add_argument("--seeds", default="17,101,997")
    p.add_argument("--suites", default="correctness,decode")
    p.add_argument("--model", action="store_true")
    a = p.parse_args(argv)
    a.output.mkdir(parents=True, exist_ok=True)
    logs = []
    for seed in (int(s) for s in a.seeds.split(",")):
        for suite in a.suites.split(","):
            out = (a.output / f"{suite}-{seed}.json").resolve()
            cmd = [sys.executable, "-m", "swiglu_b200.tuner", "--suite", suite, "--seed", str(seed),
                   "--output", str(out)]
            if suite == "correctness":
                cmd += ["--repeats", "5", "--samples", "3"]
            r = subprocess.run(cmd, text=True, capture_output=True, timeout=1800, cwd=PKG)
            logs.append({"command": cmd, "exit_code": r.returncode, "stderr": r.stderr})
            (a.output / "commands.json").write_text(json.dumps(logs, indent=2) + "\n")
            if r.returncode:
                raise SystemExit(f"GPU gate failed: {suite}, seed={seed}; see commands.json")
            subprocess.run([sys.executable, "-m", "swiglu_b200.report", str(out), "--output",
                            str(out.with_suffix(".md"))], check=True, cwd=PKG)
    if a.model:
        out = (a.output / "model.json").resolve()
        subprocess.run([sys.executable, "-m", "swiglu_b200.model_runner", "--output", str(out)], check=True,
                       timeout=1800, cwd=PKG)
        subprocess.run([sys.executable, "-m", "swiglu_b200.model_report", str(out), "--output",
                        str(out.with_suffix(".md"))], check=True, cwd=PKG)


if __name__ == "__main__":
    main()
