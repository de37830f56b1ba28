"""CPU oracle for the batch-one SwiGLU decode layer -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline``
leg (and its ``--impl reference`` arm) may import this package, and only as the
checker or the timed CPU baseline. The CUDA product in ``cuda-kernel_b200/`` never
imports it.

Two libraries sit behind it:

* ``lib/libswiglu_oracle.so`` -- a plain-C restatement of the reference's host
  contract (``include/contract.hpp:21-71``) and FFN reference
  (``src/benchmark.cu:89-94,116-121,131-141``). Always built.
* ``_ref/libswiglu_ref.so`` -- a shim compiled against the reference's own
  ``contract.hpp`` (when the reference tree is present at build time). It pins
  the restatement bit-for-bit and is the ``"reference"`` CPU baseline.

Half-precision arrays travel as ``numpy.uint16`` bit patterns or ``numpy.float16``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "lib" / "libswiglu_oracle.so"
REF_PATH = HERE / "_ref" / "libswiglu_ref.so"
# The reference checkout: $SWIGLU_REFERENCE_TREE, else a `reference/` directory beside
# this repository's own directory (absent on machines that only run the prebuilt files).
REFERENCE_TREE = Path(os.environ.get("SWIGLU_REFERENCE_TREE") or (HERE.parents[1] / "reference"))

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_intp = ctypes.POINTER(ctypes.c_int)


def build(reference: bool = True) -> None:
    """Compile the oracle (and the reference shim when the reference tree exists)."""
    targets = ["all"]
    if reference and (REFERENCE_TREE / "include" / "contract.hpp").exists():
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REFERENCE_TREE}", *targets], check=True)


def _load(path: Path) -> ctypes.CDLL:
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built; run oracle.build()")
    return ctypes.CDLL(str(path))


_lib = None
_ref = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build(reference=False)
        L = _load(LIB_PATH)
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f32_to_f16_array.argtypes = [_f32p, _u16p, ctypes.c_size_t]
        L.orc_f16_to_f32_array.argtypes = [_u16p, _f32p, ctypes.c_size_t]
        L.orc_silu.argtypes = [ctypes.c_double]
        L.orc_silu.restype = ctypes.c_double
        L.orc_matvec.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_matvec_f16.argtypes = [_u16p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_compare.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_double, ctypes.c_double,
                                  _f64p, _f64p, _intp]
        L.orc_median.argtypes = [_f64p, ctypes.c_size_t, _f64p]
        L.orc_json_escape.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
        L.orc_json_escape.restype = ctypes.c_size_t
        L.orc_ffn.argtypes = [_u16p] * 7 + [ctypes.c_int, ctypes.c_int, _f32p, _u16p, _f32p]
        L.orc_ffn_model.argtypes = [_u16p] * 4 + [ctypes.c_int, ctypes.c_int, _u16p, _u16p]
        L.orc_gate.argtypes = [_u16p] * 5 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p]
        L.orc_project.argtypes = [_u16p] * 4 + [ctypes.c_int, ctypes.c_int, _f32p, _u16p]
        L.orc_reference_workload.argtypes = [ctypes.c_uint32, ctypes.c_int, ctypes.c_int] + [_u16p] * 7
        L.orc_mt_seed.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.orc_mt_next.argtypes = [ctypes.c_void_p]
        L.orc_mt_next.restype = ctypes.c_uint32
        _lib = L
    return _lib


def ref_available() -> bool:
    return REF_PATH.exists()


def ref() -> ctypes.CDLL:
    """The reference-contract shim (raises if it was never built)."""
    global _ref
    if _ref is None:
        R = _load(REF_PATH)
        R.ref_workload.argtypes = [ctypes.c_uint, ctypes.c_int, ctypes.c_int] + [_u16p] * 7
        R.ref_ffn.argtypes = [_u16p] * 7 + [ctypes.c_int, ctypes.c_int, _f32p, _u16p, _f32p, ctypes.c_int]
        R.ref_matvec.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        R.ref_silu.argtypes = [ctypes.c_double]
        R.ref_silu.restype = ctypes.c_double
        R.ref_compare.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_double, ctypes.c_double,
                                  _f64p, _f64p, _intp]
        R.ref_median.argtypes = [_f64p, ctypes.c_size_t, _f64p]
        R.ref_hardware_threads.restype = ctypes.c_int
        _ref = R
    return _ref


# ---------------------------------------------------------------- helpers

def _u16(a) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    if a.dtype != np.uint16:
        raise TypeError(f"expected float16/uint16 array, got {a.dtype}")
    return a


def _p16(a):
    return None if a is None else a.ctypes.data_as(_u16p)


def _p32(a):
    return None if a is None else a.ctypes.data_as(_f32p)


def f16_bits(values) -> np.ndarray:
    """float32 -> binary16 bits with round-to-nearest-even (C restatement)."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(v.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_array(_p32(v), _p16(out), v.size)
    return out


def f16_values(bits) -> np.ndarray:
    b = _u16(bits)
    out = np.empty(b.shape, dtype=np.float32)
    lib().orc_f16_to_f32_array(_p16(b), _p32(out), b.size)
    return out


def silu(x: float) -> float:
    return lib().orc_silu(float(x))


def matvec(w, x, rows: int) -> np.ndarray:
    """contract.hpp:23-34 on float32 inputs."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if rows <= 0 or x.size == 0 or w.size != rows * x.size:
        raise ValueError("invalid row-major matvec dimensions")
    y = np.empty(rows, dtype=np.float32)
    if lib().orc_matvec(_p32(w), _p32(x), rows, x.size, _p32(y)):
        raise ValueError("invalid row-major matvec dimensions")
    return y


def compare(actual, expected, atol: float = 0.003, rtol: float = 0.01):
    """contract.hpp:36-53 -> (passed, max_abs, max_scaled)."""
    a = np.ascontiguousarray(actual, dtype=np.float32).ravel()
    e = np.ascontiguousarray(expected, dtype=np.float32).ravel()
    if a.size != e.size or a.size == 0:
        raise ValueError("comparison sizes differ or are empty")
    ma, ms, ok = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
    if lib().orc_compare(_p32(a), _p32(e), a.size, atol, rtol, ctypes.byref(ma), ctypes.byref(ms), ctypes.byref(ok)):
        raise ValueError("invalid tolerance")
    return bool(ok.value), ma.value, ms.value


def median(xs) -> float:
    v = np.ascontiguousarray(xs, dtype=np.float64)
    out = ctypes.c_double()
    if lib().orc_median(v.ctypes.data_as(_f64p), v.size, ctypes.byref(out)):
        raise ValueError("invalid timing")
    return out.value


def json_escape(s: str) -> str:
    raw = s.encode()
    n = lib().orc_json_escape(raw, None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    lib().orc_json_escape(raw, buf, n + 1)
    return buf.value.decode()


def reference_workload(seed: int, hidden: int, inter: int) -> dict:
    """benchmark.cu:116-121 inputs (uniform, std::mt19937) as float16 arrays."""
    out = {
        "wg": np.empty((inter, hidden), np.uint16), "wu": np.empty((inter, hidden), np.uint16),
        "wd": np.empty((hidden, inter), np.uint16), "x": np.empty(hidden, np.uint16),
        "bg": np.empty(inter, np.uint16), "bu": np.empty(inter, np.uint16), "bd": np.empty(hidden, np.uint16),
    }
    rc = lib().orc_reference_workload(seed, hidden, inter, *(_p16(out[k]) for k in ("wg", "wu", "wd", "x", "bg", "bu", "bd")))
    if rc:
        raise ValueError("invalid workload shape")
    return {k: v.view(np.float16) for k, v in out.items()}


def normal_workload(seed: int, hidden: int, inter: int) -> dict:
    """Seeded normals: x~N(0,1), W~N(0, 1/sqrt(K)), b~N(0, 0.02), all fp16."""
    rng = np.random.default_rng(seed)

    def half(shape, scale):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(np.float16)

    return {
        "wg": half((inter, hidden), 1 / np.sqrt(hidden)), "wu": half((inter, hidden), 1 / np.sqrt(hidden)),
        "wd": half((hidden, inter), 1 / np.sqrt(inter)), "x": half(hidden, 1.0),
        "bg": half(inter, 0.02), "bu": half(inter, 0.02), "bd": half(hidden, 0.02),
    }


def ffn(w: dict):
    """benchmark.cu:131-141 -> (projection fp32 [I], activation fp16 [I], y fp32 [H])."""
    inter, hidden = w["wg"].shape
    proj = np.empty(inter, np.float32)
    act = np.empty(inter, np.uint16)
    y = np.empty(hidden, np.float32)
    args = [_p16(_u16(w[k])) for k in ("wg", "wu", "wd", "x", "bg", "bu", "bd")]
    if lib().orc_ffn(*args, hidden, inter, _p32(proj), _p16(act), _p32(y)):
        raise ValueError("invalid FFN inputs")
    return proj, act.view(np.float16), y


def ffn_model(w: dict):
    """Model-rounding path (torch binding): -> (h fp16 [I], y fp16 [H])."""
    inter, hidden = w["wg"].shape
    h = np.empty(inter, np.uint16)
    y = np.empty(hidden, np.uint16)
    args = [_p16(_u16(w[k])) for k in ("wg", "wu", "wd", "x")]
    if lib().orc_ffn_model(*args, hidden, inter, _p16(h), _p16(y)):
        raise ValueError("invalid FFN inputs")
    return h.view(np.float16), y.view(np.float16)


def gate(wg, wu, x, bg=None, bu=None, model_round=False) -> np.ndarray:
    rows, cols = wg.shape
    h = np.empty(rows, np.uint16)
    args = [_p16(_u16(wg)), _p16(_u16(wu)), _p16(_u16(x)),
            None if bg is None else _p16(_u16(bg)), None if bu is None else _p16(_u16(bu))]
    if lib().orc_gate(*args, rows, cols, int(bool(model_round)), _p16(h)):
        raise ValueError("invalid gate inputs")
    return h.view(np.float16)


def project(w, x, bias=None, residual=None, half_out=False) -> np.ndarray:
    rows, cols = w.shape
    args = [_p16(_u16(w)), _p16(_u16(x)), None if bias is None else _p16(_u16(bias)),
            None if residual is None else _p16(_u16(residual))]
    if half_out:
        yh = np.empty(rows, np.uint16)
        rc = lib().orc_project(*args, rows, cols, None, _p16(yh))
        out = yh.view(np.float16)
    else:
        y = np.empty(rows, np.float32)
        rc = lib().orc_project(*args, rows, cols, _p32(y), None)
        out = y
    if rc:
        raise ValueError("invalid projection inputs")
    return out


# ------------------------------------------------- reference shim (pinning)

def ref_workload(seed: int, hidden: int, inter: int) -> dict:
    out = {
        "wg": np.empty((inter, hidden), np.uint16), "wu": np.empty((inter, hidden), np.uint16),
        "wd": np.empty((hidden, inter), np.uint16), "x": np.empty(hidden, np.uint16),
        "bg": np.empty(inter, np.uint16), "bu": np.empty(inter, np.uint16), "bd": np.empty(hidden, np.uint16),
    }
    if ref().ref_workload(seed, hidden, inter, *(_p16(out[k]) for k in ("wg", "wu", "wd", "x", "bg", "bu", "bd"))):
        raise ValueError("invalid workload shape")
    return {k: v.view(np.float16) for k, v in out.items()}


def ref_ffn(w: dict, threads: int = 1):
    inter, hidden = w["wg"].shape
    proj = np.empty(inter, np.float32)
    act = np.empty(inter, np.uint16)
    y = np.empty(hidden, np.float32)
    args = [_p16(_u16(w[k])) for k in ("wg", "wu", "wd", "x", "bg", "bu", "bd")]
    if ref().ref_ffn(*args, hidden, inter, _p32(proj), _p16(act), _p32(y), int(threads)):
        raise ValueError("invalid FFN inputs")
    return proj, act.view(np.float16), y


def ref_compare(actual, expected, atol: float = 0.003, rtol: float = 0.01):
    a = np.ascontiguousarray(actual, dtype=np.float32).ravel()
    e = np.ascontiguousarray(expected, dtype=np.float32).ravel()
    ma, ms, ok = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
    if ref().ref_compare(_p32(a), _p32(e), a.size, atol, rtol, ctypes.byref(ma), ctypes.byref(ms), ctypes.byref(ok)):
        raise ValueError("invalid tolerance")
    return bool(ok.value), ma.value, ms.value
