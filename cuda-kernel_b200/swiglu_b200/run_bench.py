"""Reproducible runner: environment probe, then the GPU suites only if a device exists.

Same flow as tools/run_bench.py of shubhxho/cuda-kernel (:52-145): record the
toolchain and GPU (clocks, power and throttle reasons are recorded, never set),
skip GPU work when there is no GPU or no nvcc, otherwise build, run the
correctness / smoke / tinyllama / decode suites with transfer-inclusive timing
(swiglu_b200.tuner), render each with the evidence validator, and with --model
run the decode-MLP replacement runner and its validator.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import shutil
import subprocess
import sys
from datetime import datetime, timezone
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]


def run(cmd, timeout=60, check=False, cwd=None):
    try:
        proc = subprocess.run(cmd, text=True, capture_output=True, timeout=timeout, cwd=cwd or PKG)
    except FileNotFoundError as exc:
        return {"command": cmd, "error": f"missing executable: {exc}", "exit_code": 127}
    except subprocess.TimeoutExpired:
        return {"command": cmd, "error": "timeout", "exit_code": 124}
    out = {"command": cmd, "exit_code": proc.returncode, "stdout": proc.stdout, "stderr": proc.stderr}
    if check and proc.returncode:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stderr}")
    return out


def nvidia_smi_query():
    if not shutil.which("nvidia-smi"):
        return {"available": False, "reason": "nvidia-smi not found"}
    query = ("name,uuid,driver_version,memory.total,memory.free,compute_cap,clocks.sm,clocks.mem,clocks.max.sm,"
             "clocks.max.mem,power.draw,power.limit,persistence_mode,pstate,clocks_event_reasons.active")
    raw = run(["nvidia-smi", f"--query-gpu={query}", "--format=csv"], timeout=30)
    return {"available": raw.get("exit_code") == 0, "query": raw}


def probe() -> dict:
    nvcc = shutil.which("nvcc") or (shutil.which("/usr/local/cuda/bin/nvcc"))
    info = {
        "schema_version": 1, "result_class": "environment-probe",
        "retrieved": datetime.now(timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ"),
        "platform": platform.platform(), "machine": platform.machine(), "python": sys.version,
        "executables": {"nvcc": nvcc, "g++": shutil.which("g++"), "nvidia-smi": shutil.which("nvidia-smi"),
                        "libswiglu_b200": str(PKG / "lib" / "libswiglu_b200.so")
                        if (PKG / "lib" / "libswiglu_b200.so").exists() else None},
        "nvcc_version": run([nvcc, "--version"]) if nvcc else {"available": False},
        "gxx_version": run(["g++", "--version"]) if shutil.which("g++") else {"available": False},
        "nvidia_smi": nvidia_smi_query(), "cuda_visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES"),
        "torch_cuda": None,
    }
    try:
        import torch
        avail = bool(torch.cuda.is_available())
        info["torch_cuda"] = {"torch": torch.__version__, "cuda_compiled": getattr(torch.version, "cuda", None),
                              "is_available": avail, "device_count": torch.cuda.device_count() if avail else 0,
                              "device_name": torch.cuda.get_device_name(0) if avail else None}
    except Exception as exc:  # a probe reports, it does not fail
        info["torch_cuda"] = {"available": False, "reason": str(exc)}
    info["gpu_present"] = bool(info["nvidia_smi"].get("available") or
                               (info["torch_cuda"] and info["torch_cuda"].get("is_available")))
    info["cuda_compiler_present"] = bool(nvcc)
    return info


def write_json(path: Path, data) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(data, indent=2) + "\n")


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--output-dir", type=Path, default=Path("results"))
    p.add_argument("--probe-only", action="store_true")
    p.add_argument("--model", action="store_true")
    p.add_argument("--skip-build", action="store_true")
    p.add_argument("--suites", default="correctness,smoke,tinyllama,decode")
    a = p.parse_args(argv)
    a.output_dir.mkdir(parents=True, exist_ok=True)
    env = probe()
    write_json(a.output_dir / "environment.json", env)
    print(f"GPU present: {env['gpu_present']}; nvcc: {env['cuda_compiler_present']}")
    if a.probe_only or not env["gpu_present"] or not env["cuda_compiler_present"]:
        if not env["gpu_present"] or not env["cuda_compiler_present"]:
            print("Skipping CUDA execution: no NVIDIA GPU and/or no nvcc in this environment.")
        return 0
    if not a.skip_build:
        run(["make", "-s", "-C", str(PKG)], timeout=900, check=True)
    for suite in a.suites.split(","):
        out = a.output_dir / f"kernels-{suite}.json"
        cmd = [sys.executable, "-m", "swiglu_b200.tuner", "--suite", suite, "--include-transfers",
               "--output", str(out.resolve())]
        if suite == "correctness":
            cmd += ["--repeats", "5", "--samples", "3"]
        run(cmd, timeout=1800, check=True)
        run([sys.executable, "-m", "swiglu_b200.report", str(out.resolve()), "--output",
             str(out.with_suffix(".md").resolve())], timeout=60, check=True)
        print(f"wrote {out}")
    if a.model:
        model_json = (a.output_dir / "model.json").resolve()
        run([sys.executable, "-m", "swiglu_b200.model_runner", "--output", str(model_json)], timeout=1800, check=True)
        run([sys.executable, "-m", "swiglu_b200.model_report", str(model_json), "--output",
             str(model_json.with_suffix(".md"))], timeout=60, check=True)
    print(f"Measured GPU evidence saved in {a.output_dir}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
