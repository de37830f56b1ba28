"""Regenerate the golden fixtures from the reference's own host contract.

Runs ``oracle/_ref/libswiglu_ref.so`` -- the shim that compiles
``include/contract.hpp`` of shubhxho/cuda-kernel where it lies -- on the
reference's seeded workload (``src/benchmark.cu:89-94,116-121``, seed 17):

* ``reference_small.npz``: inputs and outputs (projection, fp16 activation, y)
  of the small correctness-suite shapes (``include/contract.hpp:12-13``);
* ``reference_digests.json``: SHA-256 of the inputs and outputs of every
  correctness, tinyllama and decode-suite shape, too large to store.

Usage (needs the reference tree at build time): ``make -C oracle ref && python tests/golden/make_golden.py``
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402

# include/contract.hpp:12-18 of the reference: (name, hidden, intermediate)
CORRECTNESS = [("tiny", 1, 1), ("odd", 37, 65), ("tail", 129, 257), ("aligned", 512, 1024),
               ("one-to-tail", 1, 9), ("half2-min", 2, 3), ("vector8-min", 8, 8), ("below-vector8", 7, 9),
               ("above-vector8", 9, 7), ("below-warp", 31, 33), ("exact-warp", 32, 32), ("above-warp", 33, 31),
               ("half2-warp", 64, 64), ("half2-tail", 66, 70), ("vector8-warp", 256, 256),
               ("vector8-loop", 264, 272), ("multiwarp-boundary", 1024, 256), ("long-odd", 1025, 513),
               ("long-even-tail", 1030, 514)]
SMOKE = [("smoke", 512, 1024)]
TINYLLAMA = [("tinyllama-1.1b", 2048, 5632)]
DECODE = [("decode-1b-shape", 2048, 8192), ("decode-7b-shape", 4096, 11008), ("decode-8b-shape", 4096, 14336)]
SMALL_LIMIT = 40_000  # hidden * intermediate stored in full below this
SEED = 17
KEYS = ("wg", "wu", "wd", "x", "bg", "bu", "bd")


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref/libswiglu_ref.so is not built (make -C oracle ref)")
    small = {}
    digests = {"seed": SEED, "generator": "reference contract.hpp via oracle/_ref", "shapes": {}}
    for name, hidden, inter in CORRECTNESS + SMOKE + TINYLLAMA + DECODE:
        w = oracle.ref_workload(SEED, hidden, inter)
        proj, act, y = oracle.ref_ffn(w, threads=8)
        entry = {"hidden": hidden, "intermediate": inter,
                 "inputs": {k: digest(w[k]) for k in KEYS},
                 "projection": digest(proj), "activation": digest(act), "y": digest(y)}
        digests["shapes"][name] = entry
        if hidden * inter <= SMALL_LIMIT:
            for k in KEYS:
                small[f"{name}/{k}"] = w[k].view(np.uint16)
            small[f"{name}/projection"] = proj
            small[f"{name}/activation"] = act.view(np.uint16)
            small[f"{name}/y"] = y
        print(f"{name}: {hidden}x{inter}", flush=True)
    np.savez_compressed(HERE / "reference_small.npz", **small)
    (HERE / "reference_digests.json").write_text(json.dumps(digests, indent=1) + "\n")


if __name__ == "__main__":
    main()
