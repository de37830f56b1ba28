"""TinyLlama-architecture greedy decode with every decode MLP on the B200 kernels.

Follows tools/model_bench.py of shubhxho/cuda-kernel (:48-171):

* each layer's ``mlp.forward`` is replaced by a closure that sends single-token
  batch-one inputs to ``swiglu_out`` with a per-layer workspace and output
  allocated once (allocation-free decode), and anything else to the stock MLP;
* the (gate, down) geometry pair is tuned on layer 0 with an independent random
  input, each pair checked against the stock MLP (atol .01, rtol .02) and timed
  as a CUDA graph (20 warm replays, 5 samples of 100 replays);
* gates before any timing: every decode MLP took the custom path
  (calls == tokens x layers), logits close (atol .1, rtol .02), greedy tokens
  identical to the stock path; then interleaved timed decodes.

No pretrained weights or tokenizer exist offline, so the model is the TinyLlama
1.1B architecture (22 layers, hidden 2048, FFN 5632 SwiGLU, 32 heads / 4 KV
heads, RMSNorm, RoPE, vocab 32000, fp16) with seeded N(0, 0.02) weights, and the
prompts are seeded random token ids of length 16, 32 and 64.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import statistics
import time
from pathlib import Path

PROMPT_LENGTHS = (16, 32, 64)


def build_model(seed: int = 0, layers: int = 22, device: str = "cuda"):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632, num_hidden_layers=layers,
                      num_attention_heads=32, num_key_value_heads=4, max_position_embeddings=2048,
                      hidden_act="silu", initializer_range=0.02, rms_norm_eps=1e-5, rope_theta=10000.0,
                      tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    torch.manual_seed(seed)
    with torch.device(device):
        model = LlamaForCausalLM(cfg)
    return model.half().eval()


def prompts(seed: int = 0, vocab: int = 32000):
    import torch
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (1, n), generator=g) for n in PROMPT_LENGTHS]


class PatchedMLPs:
    """Replaces every decode MLP forward; mirrors model_bench.py:48-71."""

    def __init__(self, model, ext):
        import torch
        self.enabled = False
        self.calls = 0
        self.gate_config = 1
        self.down_config = 1
        self.layers = []
        self.originals = []
        cfg = model.config
        for layer in model.model.layers:
            mlp = layer.mlp
            if any(p.bias is not None for p in (mlp.gate_proj, mlp.up_proj, mlp.down_proj)):
                raise SystemExit("the runner supports bias-free MLPs")
            original = mlp.forward
            weights = (mlp.gate_proj.weight.detach(), mlp.up_proj.weight.detach(), mlp.down_proj.weight.detach())
            scratch = torch.empty((cfg.intermediate_size,), device="cuda", dtype=torch.float16)
            output = torch.empty((1, 1, cfg.hidden_size), device="cuda", dtype=torch.float16)

            def forward(x, weights=weights, original=original, scratch=scratch, output=output):
                if self.enabled and x.numel() == x.shape[-1]:
                    self.calls += 1
                    ext.swiglu_out(x.contiguous(), *weights, scratch, output, self.gate_config, self.down_config)
                    return output
                return original(x)

            mlp.forward = forward
            self.layers.append(mlp)
            self.originals.append(original)


def tune_layer0(model, patched, ext, samples: int = 5, replays: int = 100, pairs=None):
    """model_bench.py:102-130: tune all (gate, down) pairs on layer 0 with an independent input."""
    import torch
    mlp = patched.layers[0]
    cfg = model.config
    tuning = []
    with torch.inference_mode():
        tx = torch.randn((1, 1, cfg.hidden_size), device="cuda", dtype=torch.float16)
        expected = patched.originals[0](tx)
        w = (mlp.gate_proj.weight.detach(), mlp.up_proj.weight.detach(), mlp.down_proj.weight.detach())
        th = torch.empty((cfg.intermediate_size,), device="cuda", dtype=torch.float16)
        ty = torch.empty_like(tx)
        ids = ext.config_ids()
        for g, d in (pairs or [(g, d) for g in ids for d in ids]):
            ext.swiglu_out(tx, *w, th, ty, g, d)
            torch.testing.assert_close(ty, expected, atol=0.01, rtol=0.02)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                ext.swiglu_out(tx, *w, th, ty, g, d)
            for _ in range(20):
                graph.replay()
            times = []
            for _ in range(samples):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(replays):
                    graph.replay()
                b.record()
                b.synchronize()
                times.append(a.elapsed_time(b) * 1e3 / replays)
            tuning.append({"gate_config": g, "down_config": d, "samples_us": times})
            del graph
    best = min(tuning, key=lambda c: statistics.median(c["samples_us"]))
    return best, tuning


def decode(model, patched, ids, tokens: int, collect: bool = False):
    """model_bench.py:73-100: stock prefill, then `tokens` greedy decode steps."""
    import torch
    with torch.inference_mode():
        initial = model(input_ids=ids, use_cache=True)
        past = initial.past_key_values
        next_token = initial.logits[:, -1:].argmax(-1)
        torch.cuda.synchronize()
        calls_before = patched.calls
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        logits, toks = [], []
        t0 = time.perf_counter()
        start.record()
        for _ in range(tokens):
            out = model(input_ids=next_token, past_key_values=past, use_cache=True)
            past = out.past_key_values
            next_token = out.logits[:, -1:].argmax(-1)
            if collect:
                logits.append(out.logits[:, -1].detach())
                toks.append(next_token)
        end.record()
        end.synchronize()
        wall = (time.perf_counter() - t0) * 1e3
    return {"gpu_ms_per_token": start.elapsed_time(end) / tokens, "wall_ms_per_token": wall / tokens,
            "calls": patched.calls - calls_before,
            "logits": torch.stack(logits) if collect else None,
            "tokens": torch.cat(toks, dim=1) if collect else None}


def run(tokens: int = 32, samples: int = 7, layers: int = 22, seed: int = 0, tune: bool = True,
        pair: tuple[int, int] | None = None) -> dict:
    import torch
    import transformers
    import decode_swiglu as ext

    if not torch.cuda.is_available():
        raise SystemExit("NVIDIA CUDA GPU required")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    model = build_model(seed, layers)
    patched = PatchedMLPs(model, ext)
    tuning = []
    if pair is not None:
        patched.gate_config, patched.down_config = pair
    elif tune:
        best, tuning = tune_layer0(model, patched, ext)
        patched.gate_config, patched.down_config = best["gate_config"], best["down_config"]
    torch.cuda.reset_peak_memory_stats()
    records = []
    for ids in prompts(seed):
        ids = ids.cuda()
        patched.enabled = False
        base = decode(model, patched, ids, tokens, collect=True)
        patched.enabled = True
        custom = decode(model, patched, ids, tokens, collect=True)
        if custom["calls"] != tokens * len(patched.layers):
            raise RuntimeError("not every decode MLP used the custom CUDA path")
        torch.testing.assert_close(custom["logits"], base["logits"], atol=0.1, rtol=0.02)
        if not torch.equal(custom["tokens"], base["tokens"]):
            raise RuntimeError("greedy generation differs; no performance claim allowed")
        errors = (custom["logits"].float() - base["logits"].float()).abs()
        scaled = errors / (0.1 + 0.02 * base["logits"].float().abs())
        for warm in (False, True):
            patched.enabled = warm
            decode(model, patched, ids, tokens)
        collected = {"baseline": [], "custom": []}
        for s in range(samples):
            for side in (("baseline", "custom") if s % 2 == 0 else ("custom", "baseline")):
                patched.enabled = side == "custom"
                r = decode(model, patched, ids, tokens)
                expected = tokens * len(patched.layers) if patched.enabled else 0
                if r["calls"] != expected:
                    raise RuntimeError("timed decode routing mismatch")
                collected[side].append({k: r[k] for k in ("gpu_ms_per_token", "wall_ms_per_token", "calls")})
        stats = {side: {"samples": v,
                        "gpu_median_ms": statistics.median(x["gpu_ms_per_token"] for x in v),
                        "wall_median_ms": statistics.median(x["wall_ms_per_token"] for x in v)}
                 for side, v in collected.items()}
        speedup = stats["baseline"]["wall_median_ms"] / stats["custom"]["wall_median_ms"]
        records.append({"prompt": f"seeded random token ids, length {ids.numel()}", "prompt_tokens": ids.numel(),
                        "tokens": tokens, "exact_greedy_match": True, "logits_close": True,
                        "max_logit_abs_error": errors.max().item(), "max_logit_scaled_error": scaled.max().item(),
                        "generated_tokens": custom["tokens"][0].tolist(), **stats, "wall_speedup": speedup})
    here = Path(__file__).resolve()
    sources = [here.parents[1] / "csrc" / n for n in ("kernels.cuh", "registry.h", "swiglu_b200.cu")] + [here]
    return {"schema_version": 1, "kind": "random-init-model-decode",
            "model": f"TinyLlama-1.1B architecture, random init N(0,0.02) seed {seed}",
            "resolved_revision": f"random-init-seed-{seed}", "gpu": torch.cuda.get_device_name(),
            "torch": torch.__version__, "cuda": torch.version.cuda, "transformers": transformers.__version__,
            "precision": "fp16", "attention": "sdpa", "batch": 1, "timing": "eager-decode-gpu-events-and-wall",
            "prefill_included": False, "patched_layers": len(patched.layers),
            "gate_config": patched.gate_config, "down_config": patched.down_config, "tuning": tuning,
            "source_sha256": {p.name: hashlib.sha256(p.read_bytes()).hexdigest() for p in sources},
            "peak_allocated_bytes": torch.cuda.max_memory_allocated(),
            "peak_reserved_bytes": torch.cuda.max_memory_reserved(), "cases": records}


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--tokens", type=int, default=32)
    p.add_argument("--samples", type=int, default=7)
    p.add_argument("--layers", type=int, default=22)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-tune", action="store_true")
    p.add_argument("--output", type=Path, default=Path("results/model.json"))
    a = p.parse_args()
    if not 1 <= a.tokens <= 256 or not 3 <= a.samples <= 31:
        raise SystemExit("tokens must be 1..256 and samples 3..31")
    result = run(a.tokens, a.samples, a.layers, a.seed, tune=not a.no_tune)
    a.output.parent.mkdir(parents=True, exist_ok=True)
    tmp = a.output.with_name(a.output.name + ".tmp")
    tmp.write_text(json.dumps(result, indent=2, allow_nan=False) + "\n")
    tmp.replace(a.output)
    for c in result["cases"]:
        print(f"{c['prompt']}: stock {c['baseline']['wall_median_ms']:.3f} ms/token, "
              f"custom {c['custom']['wall_median_ms']:.3f} ms/token, {c['wall_speedup']:.3f}x")


if __name__ == "__main__":
    main()
