"""One-command evidence run: record the machine, then run the measured stages.

The run is a list of stages. Each stage is one subprocess (build, a tuner suite,
its rendered report, the model runner and its report) with a time limit; a
stage that fails stops the run. Before any stage the machine is described in
``environment.json`` (toolchain, GPU identity, clocks, power and throttle
reasons as nvidia-smi reports them -- read, never set). Without a GPU or nvcc
only that description is written and the run ends successfully, so the same
command is safe on a CPU-only machine. ``run.json`` lists every stage with its
command, exit code, duration and outputs.

    python -m swiglu_b200.run_bench --output-dir results [--model] [--suites decode,tinyllama]
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import platform
import shutil
import subprocess
import sys
import time
from datetime import datetime, timezone
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]
DEFAULT_SUITES = ("correctness", "smoke", "tinyllama", "decode")
# clocks, power and the active throttle reasons are recorded beside every result
SMI_FIELDS = ("name", "uuid", "driver_version", "memory.total", "compute_cap", "clocks.sm", "clocks.max.sm",
              "clocks.mem", "power.draw", "power.limit", "pstate", "clocks_event_reasons.active")


def _capture(cmd: list[str], timeout: float = 30) -> dict:
    """Run a short command; never raises (a description records what is missing)."""
    try:
        p = subprocess.run(cmd, text=True, capture_output=True, timeout=timeout)
    except (FileNotFoundError, PermissionError) as exc:
        return {"ok": False, "error": str(exc)}
    except subprocess.TimeoutExpired:
        return {"ok": False, "error": f"no answer within {timeout} s"}
    return {"ok": p.returncode == 0, "exit_code": p.returncode, "text": (p.stdout or p.stderr).strip()}


def _gpu_table() -> dict:
    smi = shutil.which("nvidia-smi")
    if not smi:
        return {"available": False, "error": "nvidia-smi not on PATH"}
    r = _capture([smi, "--query-gpu=" + ",".join(SMI_FIELDS), "--format=csv,noheader"])
    if not r["ok"]:
        return {"available": False, **r}
    gpus = [dict(zip(SMI_FIELDS, (v.strip() for v in line.split(",")))) for line in r["text"].splitlines()
            if line.strip()]
    return {"available": bool(gpus), "gpus": gpus}


def _torch_view() -> dict:
    try:
        import torch
    except Exception as exc:  # the description reports, it does not fail
        return {"importable": False, "error": str(exc)}
    view = {"importable": True, "torch": torch.__version__, "built_for_cuda": torch.version.cuda,
            "is_available": bool(torch.cuda.is_available())}
    if view["is_available"]:
        view["devices"] = [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())]
    return view


def probe() -> dict:
    """What this machine offers for the run (the ``environment-probe`` record)."""
    tools = {name: shutil.which(name) for name in ("nvcc", "g++", "make", "nvidia-smi", "ncu")}
    if not tools["nvcc"] and Path("/usr/local/cuda/bin/nvcc").exists():
        tools["nvcc"] = "/usr/local/cuda/bin/nvcc"
    lib = PKG / "lib" / "libswiglu_b200.so"
    tools["libswiglu_b200"] = str(lib) if lib.exists() else None
    versions = {name: _capture([path, "--version"])["text"].splitlines()[-1:]
                for name, path in tools.items() if path and name in ("nvcc", "g++")}
    gpu = _gpu_table()
    tv = _torch_view()
    return {"schema_version": 1, "result_class": "environment-probe",
            "retrieved": datetime.now(timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ"),
            "host": {"platform": platform.platform(), "machine": platform.machine(), "python": sys.version.split()[0],
                     "cpus": os.cpu_count()},
            "executables": tools, "versions": versions, "nvidia_smi": gpu, "torch_cuda": tv,
            "cuda_visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES"),
            "gpu_present": bool(gpu.get("available") or tv.get("is_available")),
            "cuda_compiler_present": bool(tools["nvcc"])}


def write_json(path: Path, data) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    tmp.write_text(json.dumps(data, indent=2) + "\n")
    tmp.replace(path)


@dataclasses.dataclass
class Stage:
    name: str
    cmd: list[str]
    limit_s: float
    outputs: list[Path] = dataclasses.field(default_factory=list)
    exit_code: int | None = None
    seconds: float | None = None
    tail: str = ""

    def run(self) -> bool:
        t0 = time.monotonic()
        try:
            p = subprocess.run(self.cmd, cwd=PKG, text=True, capture_output=True, timeout=self.limit_s)
            self.exit_code, self.tail = p.returncode, (p.stderr or p.stdout)[-2000:]
        except subprocess.TimeoutExpired:
            self.exit_code, self.tail = 124, f"stopped after {self.limit_s} s"
        self.seconds = round(time.monotonic() - t0, 1)
        return self.exit_code == 0

    def record(self) -> dict:
        return {"stage": self.name, "command": self.cmd, "exit_code": self.exit_code, "seconds": self.seconds,
                "outputs": [str(o) for o in self.outputs], "tail": self.tail if self.exit_code else ""}


def plan(out_dir: Path, suites: list[str], model: bool, build: bool) -> list[Stage]:
    py = sys.executable
    stages = [Stage("build", ["make", "-s", "-C", str(PKG)], 900)] if build else []
    for suite in suites:
        js, md = out_dir / f"kernels-{suite}.json", out_dir / f"kernels-{suite}.md"
        small = ["--repeats", "5", "--samples", "3"] if suite == "correctness" else []
        stages.append(Stage(f"tuner:{suite}", [py, "-m", "swiglu_b200.tuner", "--suite", suite,
                                               "--include-transfers", "--output", str(js), *small], 1800, [js]))
        stages.append(Stage(f"report:{suite}", [py, "-m", "swiglu_b200.report", str(js), "--output", str(md)],
                            60, [md]))
    if model:
        js = out_dir / "model.json"
        stages.append(Stage("model", [py, "-m", "swiglu_b200.model_runner", "--output", str(js)], 1800, [js]))
        stages.append(Stage("report:model", [py, "-m", "swiglu_b200.model_report", str(js), "--output",
                                             str(js.with_suffix(".md"))], 60, [js.with_suffix(".md")]))
    return stages


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--output-dir", type=Path, default=Path("results"))
    p.add_argument("--probe-only", action="store_true", help="describe the machine and stop")
    p.add_argument("--model", action="store_true", help="also run the decode-MLP replacement runner")
    p.add_argument("--skip-build", action="store_true")
    p.add_argument("--suites", default=",".join(DEFAULT_SUITES))
    a = p.parse_args(argv)
    out = a.output_dir.resolve()
    env = probe()
    write_json(out / "environment.json", env)
    if a.probe_only:
        return 0
    if not (env["gpu_present"] and env["cuda_compiler_present"]):
        missing = [n for n, ok in (("a GPU", env["gpu_present"]), ("nvcc", env["cuda_compiler_present"])) if not ok]
        print(f"described the machine only: no {' and no '.join(missing)} here")
        return 0
    stages = plan(out, [s for s in a.suites.split(",") if s], a.model, not a.skip_build)
    done = []
    for st in stages:
        ok = st.run()
        done.append(st.record())
        write_json(out / "run.json", {"schema_version": 1, "stages": done})
        print(f"{st.name}: {'ok' if ok else f'failed ({st.exit_code})'} in {st.seconds} s", flush=True)
        if not ok:
            print(st.tail, file=sys.stderr)
            return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
