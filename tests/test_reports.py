"""Evidence validators and the byte model (no GPU).

Mirrors the reference's report tests (tests/test_report.py, tests/test_model_report.py)
against this build's validators, and pins the byte model to the reference's
numbers (tests/test_intensity.py:20-27).
"""
import copy

import pytest

from swiglu_b200 import intensity, model_report, report


def kernel_fixture():
    def side(name, values):
        return {"name": name, "correct": True, "samples_us": values, "median_us": values[1],
                "max_abs_error": 0.0001, "max_scaled_error": 0.01}
    return {"schema_version": 1, "timing": "cuda-graph-events", "gpu": "test-only", "compute_capability": "10.0",
            "data": "synthetic-fp16-model-shapes", "driver_version": 12090, "runtime_version": 12090,
            "cublas_version": 120900, "repeats": 100, "samples": 3,
            "cases": [{"shape": "fixture", "operation": "projection", "hidden": 64, "intermediate": 128,
                       "custom": side("custom", [4, 5, 6]), "baseline": side("cublas", [9, 10, 11]), "speedup": 2}]}


def model_fixture():
    def side(times, calls):
        return {"samples": [{"wall_ms_per_token": t, "gpu_ms_per_token": t / 2, "calls": calls} for t in times],
                "wall_median_ms": times[1], "gpu_median_ms": times[1] / 2}
    return {"kind": "random-init-model-decode", "resolved_revision": "random-init-seed-0", "model": "fixture",
            "gpu": "test-only", "patched_layers": 2,
            "cases": [{"prompt": "test|prompt", "tokens": 4, "exact_greedy_match": True, "logits_close": True,
                       "max_logit_abs_error": .01, "max_logit_scaled_error": .1, "baseline": side([9, 10, 11], 0),
                       "custom": side([4, 5, 6], 8), "wall_speedup": 2}]}


def test_kernel_report_valid_and_separated_win():
    assert "separated win" in report.render(kernel_fixture(), hbm_gbs=6549.8)


@pytest.mark.parametrize("key,value", [("correct", False), ("median_us", 99), ("max_scaled_error", 1.1),
                                       ("max_abs_error", float("nan")), ("samples_us", [1, -1, 2]),
                                       ("max_scaled_error", True)])
def test_kernel_report_rejects_false_claims(key, value):
    bad = kernel_fixture()
    bad["cases"][0]["custom"][key] = value
    with pytest.raises(ValueError):
        report.validate(bad)


def test_kernel_report_rejects_structure_errors():
    for mutate in (lambda d: d["cases"].append(copy.deepcopy(d["cases"][0])),
                   lambda d: d["cases"][0].pop("hidden"),
                   lambda d: d.__setitem__("samples", 3.5),
                   lambda d: d["cases"][0].__setitem__("speedup", 100),
                   lambda d: d.__setitem__("timing", "wall-clock")):
        bad = kernel_fixture()
        mutate(bad)
        with pytest.raises(ValueError):
            report.validate(bad)


def test_kernel_report_noise_is_not_a_win_and_slower_is_reported():
    data = kernel_fixture()
    data["cases"][0]["custom"]["samples_us"] = [4, 5, 12]
    assert "| separated win |" not in report.render(data, hbm_gbs=6549.8)
    data = kernel_fixture()
    c = data["cases"][0]
    c["custom"], c["baseline"], c["speedup"] = c["baseline"], c["custom"], .5
    assert "| slower |" in report.render(data, hbm_gbs=6549.8)


def test_kernel_report_transfer_table_and_median_check():
    data = kernel_fixture()
    data["cases"][0]["transfer_inclusive"] = {"custom": {"samples_us": [7, 8, 9], "median_us": 8},
                                              "baseline": {"samples_us": [11, 12, 13], "median_us": 12}}
    assert "Transfer-inclusive" in report.render(data, hbm_gbs=6549.8)
    data["cases"][0]["transfer_inclusive"]["custom"]["median_us"] = 99
    with pytest.raises(ValueError):
        report.validate(data)


def test_model_report_gates():
    assert "| separated win |" in model_report.render(model_fixture())
    for mutate in (lambda d: d["cases"][0]["custom"]["samples"][0].__setitem__("calls", 1),
                   lambda d: d["cases"][0].__setitem__("exact_greedy_match", False),
                   lambda d: d["cases"][0].__setitem__("max_logit_scaled_error", 1.01),
                   lambda d: d["cases"][0].__setitem__("wall_speedup", 10),
                   lambda d: d.__setitem__("kind", "unknown")):
        bad = model_fixture()
        mutate(bad)
        with pytest.raises(ValueError):
            model_report.render(bad)


def test_byte_model_pinned_to_reference_values():
    g = intensity.gemv(8192, 2048, 8192 * 4)
    assert g["flops"] == 2 * 8192 * 2048 and g["bytes"] == 8192 * 2048 * 2 + 2048 * 2 + 8192 * 4
    assert 0.99 < g["flops_per_byte"] < 1.01
    assert intensity.projection(2048, 8192)["bytes"] == 33591296       # test_intensity.py:25
    assert intensity.layer(2048, 8192)["bytes"] == 100749312           # test_intensity.py:26
    assert intensity.layer(2048, 5632)["bytes"] == 69271552
    assert intensity.layer(4096, 11008)["bytes"] == 270661632
    assert intensity.layer(4096, 14336)["bytes"] == 352477184
    tp = intensity.tp_rank(4096, 14336, 8)
    assert tp["gate"]["weight_bytes"] * 8 == intensity.fused_gate(4096, 14336)["weight_bytes"]


def test_floors_are_bytes_over_bandwidth():
    rows = intensity.table(gbs=8000.0)
    r = next(x for x in rows if x["shape"] == "decode-8b-shape")
    assert abs(r["layer_floor_us"] - 352477184 / 8e12 * 1e6) < 1e-9
    assert abs(r["target_80pct_us"] - r["layer_floor_us"] / 0.8) < 1e-9


def test_run_bench_probe_records_missing_gpu(tmp_path):
    from swiglu_b200 import run_bench
    env = run_bench.probe()
    assert env["result_class"] == "environment-probe"
    for key in ("gpu_present", "cuda_compiler_present", "nvidia_smi", "executables"):
        assert key in env
    run_bench.write_json(tmp_path / "environment.json", env)
    assert "environment-probe" in (tmp_path / "environment.json").read_text()
    # without a GPU the runner stops after the probe and reports success
    if not env["gpu_present"]:
        assert run_bench.main(["--output-dir", str(tmp_path)]) == 0


def test_tuner_suites_cover_reference_and_baseline_shapes():
    from swiglu_b200 import tuner
    names = [s[0] for s in tuner.shapes("correctness")]
    assert names[:19][1] == "odd" and len(names) >= 19     # include/contract.hpp:12-13 order kept
    assert ("tinyllama-1.1b", 2048, 5632) in tuner.shapes("tinyllama")
    assert [s[1:] for s in tuner.shapes("decode")] == [(2048, 8192), (4096, 11008), (4096, 14336)]
    with pytest.raises(ValueError):
        tuner.shapes("typo")
