"""The CPU oracle, pinned before it is trusted.

* known answers of the reference's host tests (tests/host_tests.cpp:9-39);
* the golden fixtures made by the reference's own contract.hpp (tests/golden);
* bit-exact agreement with the reference shim when it is built here.
"""
import ctypes
import hashlib
import json
import math
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
KEYS = ("wg", "wu", "wd", "x", "bg", "bu", "bd")


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---- host_tests.cpp known answers ------------------------------------------

def test_matvec_known_answer():  # host_tests.cpp:9
    assert O.matvec([1, 2, 3, 4, 5, 6], [2, -1, 3], 2).tolist() == [9, 21]


def test_silu_known_answers():  # host_tests.cpp:10-11,20-21
    assert O.silu(0) == 0
    assert abs(O.silu(2) - 1.7615941559557646) < 1e-12
    assert math.isfinite(O.silu(-1000)) and O.silu(-1000) == 0
    assert O.silu(1000) == 1000


def test_compare_contract():  # host_tests.cpp:12-14,22-25
    assert O.compare([1.001, 0], [1, 0])[0]
    assert not O.compare([1.2], [1])[0]
    assert not O.compare([float("nan")], [0])[0]
    assert not O.compare([float("inf")], [float("inf")])[0]
    for atol, rtol in ((0.003, -0.01), (0, 0), (float("nan"), 0.01)):
        with pytest.raises(ValueError):
            O.compare([1], [1], atol, rtol)
    with pytest.raises(ValueError):
        O.compare([], [])


def test_median_contract():  # host_tests.cpp:15-16,27-28,37
    assert O.median([4, 1, 2, 3]) == 2.5
    assert O.median([4, 1, 2]) == 2
    assert O.median([0.125]) == 0.125
    for bad in ([1, float("inf")], [0], []):
        with pytest.raises(ValueError):
            O.median(bad)


def test_matvec_cancellation_and_rejection():  # host_tests.cpp:26,35
    assert O.matvec([1000000, 1, -1000000], [1, 1, 1], 1)[0] == 1
    with pytest.raises(ValueError):
        O.matvec([1], [1, 2], 1)


def test_json_escape():  # host_tests.cpp:19
    assert O.json_escape('a"\n\\') == 'a\\"\\u000a\\\\'


# ---- arithmetic building blocks -------------------------------------------

def test_f16_to_f32_exhaustive():
    bits = np.arange(65536, dtype=np.uint16)
    ours = O.f16_values(bits)
    ref = bits.view(np.float16).astype(np.float32)
    same = (ours.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(ours) & np.isnan(ref))
    assert same.all()


def test_f32_to_f16_round_to_nearest_even():
    rng = np.random.default_rng(3)
    parts = [rng.standard_normal(200_000).astype(np.float32) * np.float32(s) for s in (1e-8, 1e-5, 1, 3e4)]
    raw = rng.integers(0, 2 ** 32, 500_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    edge = np.array([65504, 65519.99, 65520, -65520, 5.96e-8, 2.98e-8, 2.99e-8, -0.0, np.inf, -np.inf], np.float32)
    f = np.concatenate(parts + [raw[np.isfinite(raw)], edge])
    with np.errstate(over="ignore"):
        expected = f.astype(np.float16).view(np.uint16)
    assert np.array_equal(O.f16_bits(f), expected)


def test_mt19937_known_answer():
    # The 10000th draw of a default-seeded std::mt19937 is 4123659995 (C++ standard).
    state = ctypes.create_string_buffer(624 * 4 + 8)
    O.lib().orc_mt_seed(state, 5489)
    for _ in range(9999):
        O.lib().orc_mt_next(state)
    assert O.lib().orc_mt_next(state) == 4123659995


# ---- golden fixtures from the reference ------------------------------------

def _digests():
    return json.loads((GOLDEN / "reference_digests.json").read_text())


def test_golden_small_shapes_bit_exact():
    data = np.load(GOLDEN / "reference_small.npz")
    names = sorted({k.split("/")[0] for k in data.files})
    assert len(names) >= 10
    for name in names:
        w = {k: data[f"{name}/{k}"].view(np.float16) for k in KEYS}
        inter, hidden = w["wg"].shape
        gen = O.reference_workload(17, hidden, inter)
        for k in KEYS:
            assert np.array_equal(gen[k].view(np.uint16), w[k].view(np.uint16)), (name, k)
        proj, act, y = O.ffn(w)
        assert np.array_equal(proj.view(np.uint32), data[f"{name}/projection"].view(np.uint32)), name
        assert np.array_equal(act.view(np.uint16), data[f"{name}/activation"]), name
        assert np.array_equal(y.view(np.uint32), data[f"{name}/y"].view(np.uint32)), name


@pytest.mark.parametrize("name", ["aligned", "vector8-loop", "multiwarp-boundary", "long-odd",
                                  "long-even-tail", "smoke", "tinyllama-1.1b", "decode-1b-shape"])
def test_golden_digests_bit_exact(name):
    entry = _digests()["shapes"][name]
    w = O.reference_workload(17, entry["hidden"], entry["intermediate"])
    for k in KEYS:
        assert digest(w[k]) == entry["inputs"][k], k
    proj, act, y = O.ffn(w)
    assert digest(proj) == entry["projection"]
    assert digest(act) == entry["activation"]
    assert digest(y) == entry["y"]


@pytest.mark.slow
@pytest.mark.parametrize("name", ["decode-7b-shape", "decode-8b-shape"])
def test_golden_digests_large(name):
    test_golden_digests_bit_exact(name)


# ---- the reference itself, when built here ---------------------------------

ref_only = pytest.mark.skipif(not O.ref_available(), reason="reference shim not built in this environment")


@ref_only
@pytest.mark.parametrize("shape", [(1, 1), (17, 33), (37, 65), (2047, 5631)])
def test_oracle_matches_reference_shim(shape):
    hidden, inter = shape
    w = O.normal_workload(0, hidden, inter)
    a = O.ffn(w)
    b = O.ref_ffn(w, threads=4)
    assert np.array_equal(a[0].view(np.uint32), b[0].view(np.uint32))
    assert np.array_equal(a[1].view(np.uint16), b[1].view(np.uint16))
    assert np.array_equal(a[2].view(np.uint32), b[2].view(np.uint32))


@ref_only
def test_compare_matches_reference_shim():
    rng = np.random.default_rng(5)
    e = rng.standard_normal(1000).astype(np.float32)
    a = e + rng.standard_normal(1000).astype(np.float32) * 1e-3
    assert O.compare(a, e) == O.ref_compare(a, e)


@pytest.mark.skipif(not (O.HERE / "_ref" / "host_tests").exists(), reason="reference host tests not built")
def test_reference_host_tests_pass():
    for exe in ("host_tests", "mapping_tests"):
        out = subprocess.run([str(O.HERE / "_ref" / exe)], capture_output=True, text=True, timeout=120)
        assert out.returncode == 0, out.stderr


# ---- model-rounding path and per-kernel helpers ----------------------------

def test_model_path_matches_numpy_fp16_pipeline():
    w = O.normal_workload(1, 64, 96)
    h, y = O.ffn_model(w)
    x = w["x"].astype(np.float64)
    g = (w["wg"].astype(np.float64) @ x).astype(np.float32).astype(np.float16).astype(np.float32)
    u = (w["wu"].astype(np.float64) @ x).astype(np.float32).astype(np.float16).astype(np.float32)
    s = (g / (1 + np.exp(-g.astype(np.float64)))).astype(np.float32).astype(np.float16).astype(np.float32)
    hh = (s * u).astype(np.float16)
    assert np.array_equal(h.view(np.uint16), hh.view(np.uint16))
    yy = (w["wd"].astype(np.float64) @ hh.astype(np.float64)).astype(np.float32).astype(np.float16)
    assert np.array_equal(y.view(np.uint16), yy.view(np.uint16))


def test_gate_and_project_agree_with_ffn():
    w = O.normal_workload(2, 48, 80)
    proj, act, y = O.ffn(w)
    h = O.gate(w["wg"], w["wu"], w["x"], w["bg"], w["bu"])
    assert np.array_equal(h.view(np.uint16), act.view(np.uint16))
    assert np.array_equal(O.project(w["wg"], w["x"]).view(np.uint32), proj.view(np.uint32))
    yp = O.project(w["wd"], act, w["bd"], w["x"])
    assert np.allclose(yp, y, rtol=1e-6, atol=1e-6)  # association of the two adds differs
