"""Model-decode evidence: check the runner's result, then render one row per prompt.

A ``swiglu_b200.model_runner`` result is accepted only when every rule below
holds; all violations are listed in one error.

* identity -- a known kind (the reference's pretrained kind, or this runner's
  random-init kind, alone or tensor parallel), a resolved revision, at least one
  patched layer and at least one case;
* correctness gates (the runner's own, checked again here) -- greedy tokens
  identical to the stock path, logits marked close, a finite absolute error and
  a scaled logit error in [0, 1];
* routing -- every timed custom decode called the replaced MLP exactly
  tokens x layers times, every stock decode never;
* timing -- at least three samples per side, positive finite wall and GPU
  times, medians equal to the medians of the samples, and the wall speedup equal
  to stock median / custom median.

A prompt is a "separated win" when the speedup is at least 1.05 and every custom
sample is faster than every stock sample (the kernel report's rule, applied to
wall time per token).
"""
from __future__ import annotations

import argparse
import json
import math
import statistics
from pathlib import Path

KINDS = ("pretrained-model-decode", "random-init-model-decode", "random-init-model-decode-tp")
TIMES = (("wall_median_ms", "wall_ms_per_token"), ("gpu_median_ms", "gpu_ms_per_token"))


def _count(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and v > 0


def _finite(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(v)


def _case_problems(c: dict, layers: int) -> list[str]:
    tag = str(c.get("prompt", "?"))[:40]
    out = []
    if c.get("exact_greedy_match") is not True:
        out.append(f"{tag}: greedy tokens differ from the stock path")
    if c.get("logits_close") is not True or not _finite(c.get("max_logit_abs_error")):
        out.append(f"{tag}: logits not shown close")
    s = c.get("max_logit_scaled_error")
    if not _finite(s) or not 0 <= s <= 1:
        out.append(f"{tag}: scaled logit error {s!r} outside [0, 1]")
    if not _count(c.get("tokens")):
        out.append(f"{tag}: token count is not a positive integer")
        return out
    want = {"custom": c["tokens"] * layers, "baseline": 0}
    for side, calls in want.items():
        block = c.get(side) or {}
        samples = block.get("samples") or []
        if len(samples) < 3:
            out.append(f"{tag} {side}: fewer than 3 samples")
            continue
        if any(not (_finite(x.get(k)) and x[k] > 0) for x in samples for _, k in TIMES):
            out.append(f"{tag} {side}: a time is not a positive finite number")
            continue
        if any(x.get("calls") != calls for x in samples):
            out.append(f"{tag} {side}: a timed decode did not call the replaced MLP {calls} times")
        for med, k in TIMES:
            if not (_finite(block.get(med)) and math.isclose(block[med], statistics.median(x[k] for x in samples),
                                                             rel_tol=1e-7)):
                out.append(f"{tag} {side}: {med} is not the median of its samples")
    try:
        ratio = c["baseline"]["wall_median_ms"] / c["custom"]["wall_median_ms"]
        if not (_finite(c.get("wall_speedup")) and math.isclose(ratio, c["wall_speedup"], rel_tol=1e-7)):
            out.append(f"{tag}: wall_speedup is not stock median / custom median")
    except (KeyError, TypeError, ZeroDivisionError):
        out.append(f"{tag}: wall_speedup cannot be recomputed")
    return out


def problems(data: dict) -> list[str]:
    if not isinstance(data, dict):
        return ["not a JSON object"]
    out = []
    if data.get("kind") not in KINDS:
        out.append(f"kind {data.get('kind')!r} is not one of {KINDS}")
    if not data.get("resolved_revision"):
        out.append("no resolved model revision")
    layers = data.get("patched_layers")
    if not _count(layers):
        return out + ["patched_layers is not a positive integer"]
    cases = data.get("cases")
    if not isinstance(cases, list) or not cases:
        return out + ["no cases"]
    for c in cases:
        out += _case_problems(c, layers)
        if isinstance(c, dict) and c.get("eager") is not None:  # the runner's eager decodes, same rules
            e = dict(c["eager"], prompt=f"{c.get('prompt', '?')} (eager)", tokens=c.get("tokens"),
                     exact_greedy_match=c.get("exact_greedy_match"), logits_close=c.get("logits_close"),
                     max_logit_abs_error=c.get("max_logit_abs_error"),
                     max_logit_scaled_error=c.get("max_logit_scaled_error"))
            out += _case_problems(e, layers)
    return out


def verdict(c: dict) -> str:
    fast = max(x["wall_ms_per_token"] for x in c["custom"]["samples"])
    slow = min(x["wall_ms_per_token"] for x in c["baseline"]["samples"])
    if c["wall_speedup"] >= 1.05 and fast < slow:
        return "separated win"
    return "slower" if c["wall_speedup"] < 1 else "inconclusive"


def render(data: dict) -> str:
    found = problems(data)
    if found:
        raise ValueError(f"{len(found)} problem(s) in the model evidence: " + "; ".join(found))
    extra = [f"{data['ranks']} tensor-parallel ranks"] if (data.get("ranks") or 1) > 1 else []
    lines = [f"`{data['model']}` (revision `{data['resolved_revision']}`) on {data['gpu']}: fp16, batch 1, "
             f"{data['patched_layers']} decode MLPs replaced" + (f", {', '.join(extra)}" if extra else "") + ".",
             "Both sides prefill with the stock model and decode the same way ("
             + (data.get("decode") or "the transformers loop on its growing KV cache")
             + "); prefill, capture and set-up are not timed.", "",
             "| Prompt | Stock ms/token | Custom ms/token | Stock GPU ms | Custom GPU ms | Wall ratio | Verdict |",
             "|---|---:|---:|---:|---:|---:|---|"]
    for c in data["cases"]:
        prompt = str(c["prompt"]).replace("|", "\\|").replace("\n", " ")[:55]
        b, k = c["baseline"], c["custom"]
        lines.append(f"| {prompt} | {b['wall_median_ms']:.3f} | {k['wall_median_ms']:.3f} | {b['gpu_median_ms']:.3f} | "
                     f"{k['gpu_median_ms']:.3f} | {c['wall_speedup']:.3f}× | {verdict(c)} |")
    eager = [c for c in data["cases"] if c.get("eager")]
    if eager:
        lines += ["", "The same prompts through the transformers decode loop (one Python call per kernel, growing "
                  "cache), stock MLPs against replaced ones:", "",
                  "| Prompt | Stock ms/token | Custom ms/token | Wall ratio | Verdict |", "|---|---:|---:|---:|---|"]
        for c in eager:
            e = c["eager"]
            prompt = str(c["prompt"]).replace("|", "\\|").replace("\n", " ")[:55]
            lines.append(f"| {prompt} | {e['baseline']['wall_median_ms']:.3f} | {e['custom']['wall_median_ms']:.3f} | "
                         f"{e['wall_speedup']:.3f}× | {verdict(e)} |")
    lines += ["", "Accepted only with identical greedy tokens, logits within the runner's tolerance and every "
              "timed decode MLP on the replaced path. At model level attention, the KV cache and the host loop "
              "share the time with the MLPs, so a kernel win shrinks."]
    return "\n".join(lines) + "\n"


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("input", type=Path)
    p.add_argument("--output", type=Path)
    a = p.parse_args(argv)
    text = render(json.loads(a.input.read_text()))
    if a.output:
        a.output.write_text(text)
    else:
        print(text, end="")


if __name__ == "__main__":
    main()
