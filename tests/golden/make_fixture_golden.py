"""Regenerate the captured-layer fixture goldens (run in a container that has the reference).

1. Writes a small seeded layer 16 -> 40 as a safetensors shard (fp32 tensors; the gate
   projection has a bias, up and down have none) and its input as a [1, 1, 16] .npy, under
   tests/golden/fixture_src/.
2. Runs the reference's own exporter (tools/export_ffn.py of shubhxho/cuda-kernel) on them,
   from the repository root with relative paths, into tests/golden/fixture_ref/: the raw fp16
   files and manifest.json that swiglu_b200.fixtures must reproduce byte for byte.

    python tests/golden/make_fixture_golden.py [--reference /path/to/cuda-kernel]
"""
import argparse
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
SRC = HERE / "fixture_src"
REF = HERE / "fixture_ref"
HIDDEN, INTER, PREFIX = 16, 40, "model.layers.0.mlp"


def write_sources():
    from safetensors.numpy import save_file
    rng = np.random.default_rng(23)
    SRC.mkdir(parents=True, exist_ok=True)
    tensors = {
        f"{PREFIX}.gate_proj.weight": (rng.standard_normal((INTER, HIDDEN)) / 4).astype(np.float32),
        f"{PREFIX}.gate_proj.bias": (rng.standard_normal(INTER) / 50).astype(np.float32),
        f"{PREFIX}.up_proj.weight": (rng.standard_normal((INTER, HIDDEN)) / 4).astype(np.float32),
        f"{PREFIX}.down_proj.weight": (rng.standard_normal((HIDDEN, INTER)) / 6).astype(np.float32),
        "model.layers.1.mlp.gate_proj.weight": np.zeros((2, 2), np.float32),  # another layer in the shard
    }
    save_file(tensors, str(SRC / "shard.safetensors"))
    np.save(SRC / "input.npy", rng.standard_normal((1, 1, HIDDEN)).astype(np.float32))


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--reference", type=Path, required=True, help="the reference checkout (read only)")
    a = p.parse_args()
    write_sources()
    exporter = a.reference / "tools" / "export_ffn.py"
    subprocess.run([sys.executable, str(exporter), "--weights", str(SRC.relative_to(ROOT) / "shard.safetensors"),
                    "--prefix", PREFIX, "--input", str(SRC.relative_to(ROOT) / "input.npy"),
                    "--output", str(REF.relative_to(ROOT))], check=True, cwd=ROOT)
    print("wrote", SRC, REF)


if __name__ == "__main__":
    main()
