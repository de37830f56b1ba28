"""Captured-layer fixtures: one real SwiGLU layer and its input, as raw fp16 files.

The format of shubhxho/cuda-kernel (written by tools/export_ffn.py, read by
src/benchmark.cu:95-105,122-127): a directory holding, for a layer H -> I,

    gate.f16 [I, H]   up.f16 [I, H]   down.f16 [H, I]   input.f16 [H]
    gate_bias.f16 [I] up_bias.f16 [I] down_bias.f16 [H]

each little-endian IEEE fp16 in C order, and ``manifest.json`` with the sizes,
the source checkpoint and prefix, the input file, one SHA-256 per file and the
precision label. ``export`` writes it from a local safetensors shard (absent
biases become zeros, as the reference's exporter does); ``load`` reads it with
the reference loader's checks and messages (exact size, every value finite),
optionally also checking the manifest's hashes.

    python -m swiglu_b200.fixtures --weights shard.safetensors \\
        --prefix model.layers.0.mlp --input x.npy --output fixture/
"""
from __future__ import annotations

import argparse
import hashlib
import json
from pathlib import Path

import numpy as np

NAMES = ("gate", "up", "down", "input", "gate_bias", "up_bias", "down_bias")
PRECISION = "fp16-storage-fp32-accumulation"


def shapes(hidden: int, intermediate: int) -> dict:
    """The shape of every fixture array of a layer hidden -> intermediate."""
    return {"gate": (intermediate, hidden), "up": (intermediate, hidden), "down": (hidden, intermediate),
            "input": (hidden,), "gate_bias": (intermediate,), "up_bias": (intermediate,),
            "down_bias": (hidden,)}


def export(weights: Path, prefix: str, input_npy: Path, output: Path) -> dict:
    """Write a layer's fixture directory (tools/export_ffn.py:8-47); returns the manifest.

    Reads the projections ``{prefix}.{gate,up,down}_proj.weight`` (and ``.bias`` when present)
    from a safetensors shard without executing pickle, and the captured FFN input from a
    ``.npy`` (one token). Raises ValueError on a wrong shape, a non-finite value, or a value
    that overflows fp16."""
    from safetensors import safe_open

    output = Path(output)
    output.mkdir(parents=True, exist_ok=True)
    arrays = {}
    with safe_open(str(weights), framework="numpy") as f:
        keys = set(f.keys())
        for short, key in (("gate", "gate_proj"), ("up", "up_proj"), ("down", "down_proj")):
            arrays[short] = f.get_tensor(f"{prefix}.{key}.weight")
            bias_key = f"{prefix}.{key}.bias"
            arrays[short + "_bias"] = f.get_tensor(bias_key) if bias_key in keys else np.zeros(arrays[short].shape[0])
    arrays["input"] = np.load(input_npy, allow_pickle=False).reshape(-1)
    intermediate, hidden = arrays["gate"].shape
    expected = shapes(hidden, intermediate)
    hashes = {}
    for name, array in arrays.items():
        if array.shape != expected[name] or not np.isfinite(array).all():
            raise ValueError(f"invalid {name} tensor: {array.shape}")
        with np.errstate(over="ignore"):  # an overflow is caught just below
            half = np.asarray(array, dtype="<f2", order="C")
        if not np.isfinite(half).all():
            raise ValueError(f"{name} overflows FP16")
        data = half.tobytes(order="C")
        (output / f"{name}.f16").write_bytes(data)
        hashes[name] = hashlib.sha256(data).hexdigest()
    manifest = {"hidden": hidden, "intermediate": intermediate, "weights": str(weights), "prefix": prefix,
                "input": str(input_npy), "sha256": hashes, "precision": PRECISION}
    (output / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def load(directory: Path, hidden: int, intermediate: int, verify: bool = False) -> dict:
    """Every array of a fixture directory as fp16 numpy (src/benchmark.cu:95-105).

    RuntimeError, with the reference's messages, when a file is missing or not exactly
    its size, or holds a non-finite value; with ``verify``, also when a file's SHA-256
    differs from the manifest's."""
    directory = Path(directory)
    manifest = None
    if verify:
        manifest = json.loads((directory / "manifest.json").read_text())
    out = {}
    for name, shape in shapes(hidden, intermediate).items():
        path = directory / f"{name}.f16"
        n = int(np.prod(shape))
        if not path.is_file() or path.stat().st_size != n * 2:
            raise RuntimeError(f"missing or incorrectly sized fixture: {name}.f16")
        data = path.read_bytes()
        if len(data) != n * 2:
            raise RuntimeError(f"fixture read failed: {name}.f16")
        array = np.frombuffer(data, dtype="<f2").reshape(shape).astype(np.float16)
        if not np.isfinite(array).all():
            raise RuntimeError(f"non-finite fixture: {name}.f16")
        if manifest is not None and manifest.get("sha256", {}).get(name) != hashlib.sha256(data).hexdigest():
            raise RuntimeError(f"fixture hash differs from its manifest: {name}.f16")
        out[name] = array
    return out


LAYER_KEYS = {"gate": "wg", "up": "wu", "down": "wd", "input": "x", "gate_bias": "bg", "up_bias": "bu",
              "down_bias": "bd"}


def as_layer(arrays: dict) -> dict:
    """A loaded fixture under the layer's argument names (wg, wu, wd, x, bg, bu, bd)."""
    return {LAYER_KEYS[name]: array for name, array in arrays.items()}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="Export one captured SwiGLU layer, without executing pickle.")
    p.add_argument("--weights", type=Path, required=True,
                   help="a safetensors file on disk that holds the layer's gate, up and down weights")
    p.add_argument("--prefix", required=True, help="tensor-name prefix of the layer, such as model.layers.0.mlp")
    p.add_argument("--input", type=Path, required=True,
                   help=".npy of one token's input to the MLP, taken after the layer norm")
    p.add_argument("--output", type=Path, required=True)
    a = p.parse_args(argv)
    m = export(a.weights, a.prefix, a.input, a.output)
    print(f"--fixture {a.output} --hidden {m['hidden']} --intermediate {m['intermediate']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
