"""Captured-layer fixtures (tools/export_ffn.py, src/benchmark.cu:95-105 of the reference).

The exporter is pinned byte for byte to the reference's own exporter: tests/golden/fixture_ref
is what tools/export_ffn.py wrote for the shard and input in tests/golden/fixture_src
(tests/golden/make_fixture_golden.py). The loader keeps the reference loader's checks and
messages.
"""
import hashlib
import json
import shutil
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from swiglu_b200 import fixtures

ROOT = Path(__file__).resolve().parents[1]
SRC = Path("tests/golden/fixture_src")
REF = ROOT / "tests" / "golden" / "fixture_ref"
H, I = 16, 40


def test_export_reproduces_the_reference_exporter_byte_for_byte(tmp_path, monkeypatch):
    monkeypatch.chdir(ROOT)  # the golden manifest records the relative paths it was given
    out = tmp_path / "fx"
    m = fixtures.export(SRC / "shard.safetensors", "model.layers.0.mlp", SRC / "input.npy", out)
    assert (m["hidden"], m["intermediate"]) == (H, I)
    for name in fixtures.NAMES:
        assert (out / f"{name}.f16").read_bytes() == (REF / f"{name}.f16").read_bytes(), name
    assert (out / "manifest.json").read_text() == (REF / "manifest.json").read_text()


def test_cli_prints_the_reference_next_step(tmp_path, monkeypatch, capsys):
    monkeypatch.chdir(ROOT)
    assert fixtures.main(["--weights", str(SRC / "shard.safetensors"), "--prefix", "model.layers.0.mlp",
                          "--input", str(SRC / "input.npy"), "--output", str(tmp_path / "fx")]) == 0
    assert capsys.readouterr().out.strip() == f"--fixture {tmp_path / 'fx'} --hidden {H} --intermediate {I}"


def test_load_checks_and_oracle_runs_on_the_fixture():
    arrays = fixtures.load(REF, H, I, verify=True)
    assert {k: v.shape for k, v in arrays.items()} == fixtures.shapes(H, I)
    assert all(v.dtype == np.float16 for v in arrays.values())
    assert not arrays["up_bias"].any() and not arrays["down_bias"].any()  # absent biases export as zeros
    assert arrays["gate_bias"].any()
    layer = fixtures.as_layer(arrays)
    _, act, y = O.ffn(layer)
    assert np.isfinite(y).all() and act.shape == (I,)


def _copy(tmp_path):
    d = tmp_path / "fx"
    shutil.copytree(REF, d)
    return d


def test_load_rejects_like_the_reference_loader(tmp_path):
    d = _copy(tmp_path)
    (d / "up.f16").write_bytes((d / "up.f16").read_bytes()[:-2])
    with pytest.raises(RuntimeError, match=r"^missing or incorrectly sized fixture: up.f16$"):
        fixtures.load(d, H, I)
    d = _copy(tmp_path / "b")
    (d / "down_bias.f16").unlink()
    with pytest.raises(RuntimeError, match="missing or incorrectly sized fixture: down_bias.f16"):
        fixtures.load(d, H, I)
    with pytest.raises(RuntimeError, match="incorrectly sized fixture: gate.f16"):
        fixtures.load(REF, H + 1, I)  # the caller's dimensions decide the sizes
    d = _copy(tmp_path / "c")
    g = np.frombuffer((d / "gate.f16").read_bytes(), dtype="<f2").copy()
    g[7] = np.inf
    (d / "gate.f16").write_bytes(g.tobytes())
    with pytest.raises(RuntimeError, match="non-finite fixture: gate.f16"):
        fixtures.load(d, H, I)


def test_load_verify_catches_a_changed_file(tmp_path):
    d = _copy(tmp_path)
    x = np.frombuffer((d / "input.f16").read_bytes(), dtype="<f2").copy()
    x[0] = np.float16(0.5) if x[0] != np.float16(0.5) else np.float16(0.25)
    (d / "input.f16").write_bytes(x.tobytes())
    fixtures.load(d, H, I)  # the reference loader does not read the manifest
    with pytest.raises(RuntimeError, match="fixture hash differs from its manifest: input.f16"):
        fixtures.load(d, H, I, verify=True)


def test_export_rejects_bad_tensors(tmp_path):
    from safetensors.numpy import save_file
    p = "m.mlp"
    good = {f"{p}.gate_proj.weight": np.ones((8, 4), np.float32), f"{p}.up_proj.weight": np.ones((8, 4), np.float32),
            f"{p}.down_proj.weight": np.ones((4, 8), np.float32)}
    np.save(tmp_path / "x.npy", np.ones(4, np.float32))
    for key, value, message in ((f"{p}.up_proj.weight", np.full((8, 4), 1e6, np.float32), "up overflows FP16"),
                                (f"{p}.down_proj.weight", np.ones((8, 4), np.float32), r"invalid down tensor"),
                                (f"{p}.gate_proj.weight", np.full((8, 4), np.nan, np.float32), "invalid gate tensor")):
        bad = dict(good)
        bad[key] = value
        save_file(bad, str(tmp_path / "s.safetensors"))
        with pytest.raises(ValueError, match=message):
            fixtures.export(tmp_path / "s.safetensors", p, tmp_path / "x.npy", tmp_path / "out")
    save_file(good, str(tmp_path / "s.safetensors"))
    np.save(tmp_path / "x.npy", np.ones(5, np.float32))
    with pytest.raises(ValueError, match="invalid input tensor"):
        fixtures.export(tmp_path / "s.safetensors", p, tmp_path / "x.npy", tmp_path / "out")
    np.save(tmp_path / "x.npy", np.ones((1, 1, 4), np.float32))
    m = fixtures.export(tmp_path / "s.safetensors", p, tmp_path / "x.npy", tmp_path / "out")
    data = (tmp_path / "out" / "gate.f16").read_bytes()
    assert m["sha256"]["gate"] == hashlib.sha256(data).hexdigest()
    assert json.loads((tmp_path / "out" / "manifest.json").read_text())["precision"] == fixtures.PRECISION


def test_tuner_fixture_options_are_checked_like_decode_bench():
    from swiglu_b200 import tuner
    with pytest.raises(ValueError, match="fixture needs --hidden and --intermediate"):
        tuner.run(fixture=REF)
    with pytest.raises(ValueError, match="custom dimensions require --fixture"):
        tuner.run(hidden=16)


@pytest.mark.gpu
def test_captured_layer_runs_through_the_product_path():
    """The golden captured layer through swb_ffn (every family's fallback-safe ids) against the
    oracle with the reference's gate, and the tuner's fixture mode end to end."""
    import torch
    from swiglu_b200 import binding, tuner
    layer = fixtures.as_layer(fixtures.load(REF, H, I, verify=True))
    _, act, y_ref = O.ffn(layer)
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in layer.items()}
    for g, dn in ((33, 35), (1, 1), (69, 87), (82, 82)):
        h = torch.empty(I, dtype=torch.float16, device="cuda")
        y = torch.empty(H, dtype=torch.float32, device="cuda")
        binding.ffn(d["x"], d["wg"], d["wu"], d["wd"], d["bg"], d["bu"], d["bd"], h, y, g, dn)
        torch.cuda.synchronize()
        assert O.compare(y.cpu().numpy(), y_ref)[0], (g, dn)
    result = tuner.run(repeats=2, samples=3, ids=[33, 35, 69, 87], fixture=REF, hidden=H, intermediate=I)
    assert result["data"] == "captured-model-fixture"
    assert [c["shape"] for c in result["cases"]] == ["captured-model-ffn"] * 2
    assert all(c["custom"]["correct"] for c in result["cases"])
