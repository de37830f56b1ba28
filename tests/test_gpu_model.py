"""TinyLlama-architecture decode with every decode MLP on the B200 kernels, one GPU.

The gates of tools/model_bench.py:141-147, for four decodes of each of three seeded
prompts (16, 32, 64 token ids; random init, seed 0): the transformers loop with stock
and with replaced MLPs, and one CUDA graph per decode step with stock and with
replaced MLPs. Greedy tokens identical to the eager stock decode, logits within atol .1 /
rtol .02, every replaced decode routed through tokens x layers kernel calls; the graph
decode with stock MLPs reproduces the eager stock logits bit for bit (the slot cache
gives attention the shapes the growing cache gives it).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_tinyllama_architecture_greedy_decode_eager_and_graph():
    from swiglu_b200 import model_report, model_runner
    ids = [16, 33, 69, 80, 87, 96]
    cands = [(g, d) for g in ids for d in ids]
    result = model_runner.run(tokens=32, samples=3, layers=22, seed=0, candidates=cands)
    assert result["patched_layers"] == 22 and len(result["tuning"]) == len(cands)
    for case in result["cases"]:
        assert case["exact_greedy_match"] and case["logits_close"]
        assert all(s["calls"] == 32 * 22 for s in case["custom"]["samples"])
        assert all(s["calls"] == 32 * 22 for s in case["eager"]["custom"]["samples"])
        assert all(c["tokens_equal"] for c in case["checks"].values())
        assert case["checks"]["graph_stock"]["bit_identical_logits"]
    text = model_report.render(result)  # re-validates routing, medians and the speedups
    assert "random-init-seed-0" in text
    torch.cuda.empty_cache()
