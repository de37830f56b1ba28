"""TinyLlama-architecture decode with every decode MLP on the B200 kernels.

The gates of tools/model_bench.py:141-147: every decode MLP call took the custom
path (calls == tokens x layers), logits within atol .1 / rtol .02 of the stock
fp16 path, and greedy tokens identical. Random init (seed 0) and seeded token-id
prompts of length 16, 32 and 64 stand in for the pretrained model and its prompts.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_tinyllama_architecture_greedy_decode_identical():
    from swiglu_b200 import model_runner, model_report
    ids = [16, 33, 64, 69, 80, 87]
    pairs = [(g, d) for g in ids for d in ids]
    model = model_runner.build_model(seed=0, layers=22)
    import decode_swiglu as ext
    patched = model_runner.PatchedMLPs(model, ext)
    best, tuning = model_runner.tune_layer0(model, patched, ext, samples=3, replays=20, pairs=pairs)
    assert len(tuning) == len(pairs)
    del model, patched
    torch.cuda.empty_cache()
    result = model_runner.run(tokens=32, samples=3, layers=22, seed=0,
                              pair=(best["gate_config"], best["down_config"]))
    assert result["patched_layers"] == 22
    for case in result["cases"]:
        assert case["exact_greedy_match"] and case["logits_close"]
        assert all(s["calls"] == 32 * 22 for s in case["custom"]["samples"])
    text = model_report.render(result)  # re-validates routing, medians and the speedup
    assert "random-init-seed-0" in text
