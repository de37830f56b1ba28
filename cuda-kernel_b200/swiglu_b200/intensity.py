"""Algorithmic bytes and FLOPs of the decode kernels, and B200 HBM floors.

The byte model is the reference's (tools/intensity.py:50-99 of shubhxho/cuda-kernel):
each weight, input, bias and output element is counted once.

* projection (raw, fp32 out): I*H*2 + H*2 + I*4
* gate (fused, fp16 h):        2*I*H*2 + H*2 + I*2 + 2*I*2
* down (+bias +residual, fp32): H*I*2 + I*2 + H*4 + H*2 + H*2
* layer = gate + down; a tensor-parallel rank moves layer/N of the weight bytes.

Floors divide those bytes by an HBM bandwidth; they are analytical lower
bounds, not measurements.
"""
from __future__ import annotations

import json
from pathlib import Path

FP16 = 2
FP32 = 4
SILU_FLOPS = 4       # order-of-magnitude stand-in, as the reference counts it
GATE_MUL_FLOPS = 1

# Fallback HBM copy bandwidth of this pool's B200s when no measured file exists.
FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0


def gemv(rows: int, cols: int, out_bytes: int) -> dict:
    flops = 2 * rows * cols
    weight = rows * cols * FP16
    inp = cols * FP16
    total = weight + inp + out_bytes
    return {"flops": flops, "weight_bytes": weight, "input_bytes": inp, "output_bytes": out_bytes,
            "bytes": total, "flops_per_byte": flops / total}


def projection(hidden: int, inter: int) -> dict:
    return gemv(inter, hidden, inter * FP32)


def fused_gate(hidden: int, inter: int) -> dict:
    base = gemv(inter, hidden, inter * FP16)
    extra = inter * hidden * FP16
    bias = 2 * inter * FP16
    flops = 2 * base["flops"] + inter * (SILU_FLOPS + GATE_MUL_FLOPS)
    total = base["bytes"] + extra + bias
    return {"flops": flops, "weight_bytes": base["weight_bytes"] + extra, "input_bytes": base["input_bytes"],
            "output_bytes": base["output_bytes"], "bias_bytes": bias, "bytes": total,
            "flops_per_byte": flops / total}


def down_residual(hidden: int, inter: int) -> dict:
    base = gemv(hidden, inter, hidden * FP32)
    total = base["bytes"] + hidden * FP16 + hidden * FP16
    return {"flops": base["flops"], "weight_bytes": base["weight_bytes"], "input_bytes": base["input_bytes"],
            "output_bytes": base["output_bytes"], "residual_bytes": hidden * FP16, "bias_bytes": hidden * FP16,
            "bytes": total, "flops_per_byte": base["flops"] / total}


def layer(hidden: int, inter: int) -> dict:
    g, d = fused_gate(hidden, inter), down_residual(hidden, inter)
    return {"bytes": g["bytes"] + d["bytes"], "flops": g["flops"] + d["flops"],
            "weight_bytes": g["weight_bytes"] + d["weight_bytes"], "gate": g, "down": d}


def cublas_extra_bytes(hidden: int, inter: int) -> int:
    """fp32 g/u written and re-read by the gate epilogue, y re-read by the residual epilogue."""
    return 2 * inter * FP32 * 2 + hidden * FP32


def tp_rank(hidden: int, inter: int, n: int) -> dict:
    """Per-rank bytes of a tensor-parallel layer: gate rows and down columns split n ways."""
    if inter % n:
        raise ValueError("intermediate size must divide by the rank count")
    shard = inter // n
    g = fused_gate(hidden, shard)
    d = gemv(hidden, shard, hidden * FP32)  # partial y, no bias/residual before the all-reduce
    epilogue = hidden * FP32 * 2 + hidden * FP16 * 2
    return {"gate": g, "down": d, "epilogue_bytes": epilogue, "allreduce_bytes": hidden * FP32,
            "bytes": g["bytes"] + d["bytes"] + epilogue}


def floor_us(byte_count: int, gbs: float) -> float:
    return byte_count / (gbs * 1e9) * 1e6


def measured_peaks(path: Path | None = None) -> dict:
    """HBM peak for roofline fractions: the pool's measured copy bandwidth, else the fallback."""
    p = path or Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        data = json.loads(p.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured", "raw": data}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": FALLBACK_HBM_GBS, "source": "fallback", "raw": None}


SHAPES = (
    ("tinyllama-1.1b", 2048, 5632),
    ("decode-1b-shape", 2048, 8192),
    ("decode-7b-shape", 4096, 11008),
    ("decode-8b-shape", 4096, 14336),
    ("smoke", 512, 1024),
)


def table(gbs: float | None = None) -> list[dict]:
    peak = gbs or measured_peaks()["hbm_gbs"]
    rows = []
    for name, h, i in SHAPES:
        L = layer(h, i)
        rows.append({"shape": name, "hidden": h, "intermediate": i, "projection_bytes": projection(h, i)["bytes"],
                     "layer_bytes": L["bytes"], "layer_floor_us": floor_us(L["bytes"], peak),
                     "target_80pct_us": floor_us(L["bytes"], peak) / 0.8, "hbm_gbs": peak})
    return rows


if __name__ == "__main__":
    for r in table():
        print(json.dumps(r))
