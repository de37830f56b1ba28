"""Greedy decode of a TinyLlama-architecture model with every decode MLP on the B200 kernels.

The integration surface is the reference's (tools/model_bench.py:48-71,133-171 of
shubhxho/cuda-kernel): each layer's ``mlp.forward`` is replaced by a router that
sends single-token batch-one inputs to ``swiglu_out`` with a per-layer workspace
and output allocated once, and anything else (the prefill) to the stock module.
The (gate, down) pair is tuned on layer 0 with an independent input, every pair
checked against the stock MLP (atol .01, rtol .02) and timed as a CUDA graph.

Each seeded prompt is decoded four ways:

* ``eager``: the transformers decode loop with its growing cache, one Python
  call per kernel, stock MLPs (the reference's baseline) and replaced MLPs (the
  reference's custom path);
* ``graph``: every decode step captured once as a CUDA graph and replayed,
  stock MLPs and replaced MLPs. The keys and values live in preallocated slot
  buffers (``SlotCache``) whose filled prefix each attention call reads, so
  attention sees exactly the shapes a growing cache gives it; a step's graph
  embeds the token, runs all 22 layers, takes the argmax and writes the next
  token where the next step's graph reads it, so a 32-token decode is 32 graph
  replays and no host synchronisation.

Gates before any timing: greedy tokens of the three replaced decodes identical
to the eager stock decode's, logits within atol .1 / rtol .02, every timed
custom decode routed through tokens x layers replaced MLP calls (eager: counted
per call; graph: counted at capture, ``layers`` per step graph).

Tensor parallel (``torchrun --nproc-per-node N -m swiglu_b200.model_runner``):
every rank holds the whole model (attention replicated) and its shard of each
MLP (rows of gate and up, the matching columns of down); a replaced MLP is one
``swb_swiglu_tp_out`` call -- the gate on the shard, the down projection with the
all-reduce over NVLink fused into it -- so every rank ends each layer with the
same fp16 output and decodes the same tokens. The stock side runs the full MLP
on every rank.

No pretrained weights or tokenizer exist offline: the model is the TinyLlama-1.1B
architecture (22 layers, hidden 2048, FFN 5632 SwiGLU, 32 heads / 4 KV heads,
RMSNorm, RoPE, vocab 32000, fp16) with seeded N(0, 0.02) weights, and the prompts
are seeded random token ids of length 16, 32 and 64.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import time
from pathlib import Path

PROMPT_LENGTHS = (16, 32, 64)
LOGIT_ATOL, LOGIT_RTOL = 0.1, 0.02      # tools/model_bench.py:143
PAIR_ATOL, PAIR_RTOL = 0.01, 0.02       # tools/model_bench.py:112


def build_model(seed: int = 0, layers: int = 22, device: str = "cuda"):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632, num_hidden_layers=layers,
                      num_attention_heads=32, num_key_value_heads=4, max_position_embeddings=2048,
                      hidden_act="silu", initializer_range=0.02, rms_norm_eps=1e-5, rope_theta=10000.0,
                      tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(device):
        model = LlamaForCausalLM(cfg)
    return model.half().eval() if device != "cpu" else model.eval()


def prompts(seed: int = 0, vocab: int = 32000):
    import torch
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (1, n), generator=g) for n in PROMPT_LENGTHS]


# ------------------------------------------------------------------ slot cache

def _slot_layer_class():
    from transformers.cache_utils import CacheLayerMixin

    class SlotLayer(CacheLayerMixin):
        """One layer's keys and values in preallocated [1, kv_heads, capacity, head_dim] buffers.

        ``length`` is a host integer. ``update`` copies the new positions into place and returns
        views of the filled prefix -- the sizes a growing cache returns -- so attention runs the
        same kernels on the same shapes. A captured step bakes its slice bounds into its graph."""

        def __init__(self, keys, values):
            super().__init__()
            self.keys, self.values = keys, values
            self.capacity = keys.shape[2]
            self.length = 0
            self.is_initialized = True
            self.dtype, self.device = keys.dtype, keys.device

        def lazy_initialization(self, key_states, value_states) -> None:
            pass

        def update(self, key_states, value_states, *args, **kwargs):
            a = self.length
            b = a + key_states.shape[-2]
            if b > self.capacity:
                raise RuntimeError(f"slot cache holds {self.capacity} positions, asked for {b}")
            self.keys[:, :, a:b].copy_(key_states)
            self.values[:, :, a:b].copy_(value_states)
            self.length = b
            return self.keys[:, :, :b], self.values[:, :, :b]

        def get_seq_length(self) -> int:
            return self.length

        def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
            return self.length + query_length, 0

        def get_max_cache_shape(self) -> int:
            return self.capacity

    return SlotLayer


class SlotCache:
    """A transformers ``Cache`` whose layers are ``SlotLayer``s of `capacity` positions."""

    def __init__(self, config, capacity: int, device, dtype):
        import torch
        from transformers.cache_utils import Cache
        layer_cls = _slot_layer_class()
        heads = config.num_key_value_heads
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        self.layers = [layer_cls(torch.zeros(1, heads, capacity, head_dim, device=device, dtype=dtype),
                                 torch.zeros(1, heads, capacity, head_dim, device=device, dtype=dtype))
                       for _ in range(config.num_hidden_layers)]
        self.cache = Cache(layers=self.layers)

    def seek(self, position: int) -> None:
        """Every layer's next write goes to `position` (the filled prefix is [0, position))."""
        for layer in self.layers:
            layer.length = position


# ------------------------------------------------------------------ MLP routing

class MLPRoutes:
    """Replaces every layer's ``mlp.forward`` by a router (tools/model_bench.py:60-71).

    While ``custom`` is set, a single-token input goes to ``call(layer, x, out)``, which writes
    the layer's output buffer (allocated once per layer); everything else, and every call while
    ``custom`` is clear, goes to the stock module. ``calls`` counts the replaced calls."""

    def __init__(self, model, call):
        import torch
        self.custom = False
        self.calls = 0
        self.stock = []
        cfg = model.config
        for idx, layer in enumerate(model.model.layers):
            mlp = layer.mlp
            if any(p.bias is not None for p in (mlp.gate_proj, mlp.up_proj, mlp.down_proj)):
                raise SystemExit("the runner replaces bias-free MLPs only")
            out = torch.empty((1, 1, cfg.hidden_size), device=mlp.gate_proj.weight.device, dtype=torch.float16)
            self.stock.append(mlp.forward)
            mlp.forward = self._router(idx, mlp.forward, out, call)

    def _router(self, idx, stock, out, call):
        def forward(x):
            if self.custom and x.numel() == x.shape[-1]:
                self.calls += 1
                call(idx, x.contiguous(), out)
                return out
            return stock(x)
        return forward


def single_gpu_call(model, ext, pair: list):
    """The replaced MLP on one GPU: ``swiglu_out`` with a per-layer workspace h; `pair` holds
    the (gate, down) ids and may be changed between calls."""
    import torch
    cfg = model.config
    weights = [(l.mlp.gate_proj.weight.detach(), l.mlp.up_proj.weight.detach(), l.mlp.down_proj.weight.detach())
               for l in model.model.layers]
    scratch = [torch.empty(cfg.intermediate_size, device=w[0].device, dtype=torch.float16) for w in weights]

    def call(idx, x, out):
        ext.swiglu_out(x, *weights[idx], scratch[idx], out, pair[0], pair[1])
    return call


def tensor_parallel_call(model, exchange, rank: int, world: int, pair: list):
    """The replaced MLP of rank `rank`: its shard of each layer through ``swb_swiglu_tp_out``."""
    import torch
    from . import tp as T
    shards, scratch = [], []
    for l in model.model.layers:
        m = l.mlp
        s = T.shard(m.gate_proj.weight.detach(), m.up_proj.weight.detach(), m.down_proj.weight.detach(), None,
                    None, rank, world)
        shards.append(s)
        scratch.append(torch.empty(s["wg"].shape[0], device=s["wg"].device, dtype=torch.float16))

    def call(idx, x, out):
        T.swiglu_tp_out(exchange, x, shards[idx], scratch[idx], out, pair[0], pair[1])
    return call


# ------------------------------------------------------------------ decoding

def eager_decode(model, routes, ids, tokens: int, custom: bool, collect: bool = False) -> dict:
    """The transformers loop: stock prefill, then `tokens` greedy steps on its growing cache."""
    import torch
    routes.custom = False
    with torch.inference_mode():
        first = model(input_ids=ids, use_cache=True)
        past, tok = first.past_key_values, first.logits[:, -1:].argmax(-1)
        torch.cuda.synchronize()
        routes.custom, c0 = custom, routes.calls
        logits, toks = [], []
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        t0 = time.perf_counter()
        ev[0].record()
        for _ in range(tokens):
            out = model(input_ids=tok, past_key_values=past, use_cache=True)
            past, tok = out.past_key_values, out.logits[:, -1:].argmax(-1)
            if collect:
                logits.append(out.logits[0, -1].detach().clone())
                toks.append(tok.clone())
        ev[1].record()
        ev[1].synchronize()
        wall = time.perf_counter() - t0
        routes.custom = False
    return {"gpu_ms_per_token": ev[0].elapsed_time(ev[1]) / tokens, "wall_ms_per_token": wall * 1e3 / tokens,
            "calls": routes.calls - c0, "logits": torch.stack(logits) if collect else None,
            "tokens": torch.cat(toks, dim=1) if collect else None}


class GraphDecoder:
    """Every decode step of one prompt length captured as a CUDA graph (stock or replaced MLPs).

    Static buffers: the slot cache, the current token, one position tensor per step, and the
    logits and tokens of every step. ``decode(ids)`` prefills eagerly (the stock MLPs run the
    prompt, as in the eager decode) and then replays the step graphs in order."""

    def __init__(self, model, routes, prompt_len: int, tokens: int, custom: bool, pool=None):
        import torch
        self.model, self.routes, self.custom = model, routes, custom
        self.P, self.T = prompt_len, tokens
        dev = model.model.embed_tokens.weight.device
        self.slots = SlotCache(model.config, prompt_len + tokens, dev, torch.float16)
        self.tok = torch.zeros((1, 1), dtype=torch.long, device=dev)
        self.pos = [torch.full((1, 1), prompt_len + t, dtype=torch.long, device=dev) for t in range(tokens)]
        self.logits = torch.empty((tokens, model.config.vocab_size), dtype=torch.float16, device=dev)
        self.out = torch.empty((1, tokens), dtype=torch.long, device=dev)
        self.graphs, self.captured_calls = [], []
        self.pool = pool

    def _prefill(self, ids):
        self.routes.custom = False
        self.slots.seek(0)
        out = self.model(input_ids=ids, past_key_values=self.slots.cache, use_cache=True)
        self.tok.copy_(out.logits[:, -1:].argmax(-1))

    def _step(self, t: int):
        out = self.model(input_ids=self.tok, past_key_values=self.slots.cache, position_ids=self.pos[t],
                         use_cache=True)
        last = out.logits[:, -1]
        self.logits[t].copy_(last[0])
        nxt = last.argmax(-1, keepdim=True)
        self.out[:, t:t + 1].copy_(nxt)
        self.tok.copy_(nxt)

    def capture(self, ids) -> None:
        """Warm every step eagerly (lazy library set-up happens outside capture), then capture."""
        import torch
        with torch.inference_mode():
            self._prefill(ids)
            self.routes.custom = self.custom
            for t in range(self.T):
                self._step(t)
            torch.cuda.synchronize()
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            for t in range(self.T):
                self.slots.seek(self.P + t)
                g = torch.cuda.CUDAGraph()
                c0 = self.routes.calls
                with torch.cuda.graph(g, pool=self.pool, stream=stream):
                    self._step(t)
                self.captured_calls.append(self.routes.calls - c0)
                self.graphs.append(g)
            self.routes.custom = False
            torch.cuda.current_stream().wait_stream(stream)
            torch.cuda.synchronize()

    def decode(self, ids, collect: bool = False) -> dict:
        import torch
        with torch.inference_mode():
            self._prefill(ids)
            torch.cuda.synchronize()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            t0 = time.perf_counter()
            ev[0].record()
            for g in self.graphs:
                g.replay()
            ev[1].record()
            ev[1].synchronize()
            wall = time.perf_counter() - t0
        return {"gpu_ms_per_token": ev[0].elapsed_time(ev[1]) / self.T, "wall_ms_per_token": wall * 1e3 / self.T,
                "calls": sum(self.captured_calls),
                "logits": self.logits.clone() if collect else None, "tokens": self.out.clone() if collect else None}

    def release(self):
        for g in self.graphs:
            g.reset()
        self.graphs = []


# ------------------------------------------------------------------ tuning

def tune_layer0(model, routes, call, pair: list, candidates, samples: int = 5, replays: int = 100,
                agree=None) -> tuple[tuple[int, int], list]:
    """tools/model_bench.py:102-130: every (gate, down) candidate on layer 0 with an independent
    random input, checked against the stock MLP and timed as a CUDA graph of the one call
    (20 warm replays, `samples` samples of `replays` replays). `agree` makes every rank take
    rank 0's choice."""
    import torch
    hidden = model.config.hidden_size
    results = []
    with torch.inference_mode():
        g = torch.Generator(device="cuda").manual_seed(1234)
        tx = torch.randn((1, 1, hidden), device="cuda", dtype=torch.float16, generator=g)
        expected = routes.stock[0](tx)
        ty = torch.empty_like(tx)
        for cand in candidates:
            pair[:] = list(cand)
            call(0, tx, ty)
            torch.testing.assert_close(ty, expected, atol=PAIR_ATOL, rtol=PAIR_RTOL)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                call(0, tx, ty)
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
            graph.reset()
            results.append({"gate_config": cand[0], "down_config": cand[1], "samples_us": times})
    best = min(results, key=lambda r: statistics.median(r["samples_us"]))
    choice = (best["gate_config"], best["down_config"])
    if agree is not None:
        choice = agree(choice)
    pair[:] = list(choice)
    return choice, results


# ------------------------------------------------------------------ the run

def _stats(samples: list) -> dict:
    return {"samples": samples, "gpu_median_ms": statistics.median(s["gpu_ms_per_token"] for s in samples),
            "wall_median_ms": statistics.median(s["wall_ms_per_token"] for s in samples)}


def _compare(torch, got: dict, ref: dict) -> dict:
    err = (got["logits"].float() - ref["logits"].float()).abs()
    scaled = err / (LOGIT_ATOL + LOGIT_RTOL * ref["logits"].float().abs())
    return {"tokens_equal": bool(torch.equal(got["tokens"].cpu(), ref["tokens"].cpu())),
            "max_abs": float(err.max()), "max_scaled": float(scaled.max()),
            "bit_identical_logits": bool(torch.equal(got["logits"], ref["logits"]))}


def run(tokens: int = 32, samples: int = 7, layers: int = 22, seed: int = 0, tune: bool = True,
        pair: tuple[int, int] | None = None, candidates=None) -> dict:
    import torch
    import transformers
    import decode_swiglu as ext
    from . import binding

    if not torch.cuda.is_available():
        raise SystemExit("an NVIDIA GPU is required")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = exchange = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    model = build_model(seed, layers)
    live = [1, 1]
    if world > 1:
        from .tp import Exchange
        exchange = Exchange(rank, world, model.config.hidden_size, torch.device("cuda", local))
        call = tensor_parallel_call(model, exchange, rank, world, live)
    else:
        call = single_gpu_call(model, ext, live)
    routes = MLPRoutes(model, call)

    def agree(choice):
        if world == 1:
            return choice
        t = torch.tensor(list(choice), dtype=torch.int64, device="cuda")
        dist.broadcast(t, 0)
        return int(t[0]), int(t[1])

    tuning = []
    if pair is not None:
        live[:] = list(pair)
    elif tune:
        ids_ = binding.config_ids()
        downs = ids_ if world == 1 else [c for c in ids_ if binding.config_info(c)["family"] == 2]
        cands = candidates or [(g, d) for g in ids_ for d in downs]
        _, tuning = tune_layer0(model, routes, call, live, cands, agree=agree)
    chosen = tuple(live)

    records = []
    for ids in prompts(seed):
        ids = ids.cuda()
        P = ids.shape[1]
        # correctness first: four decodes, each against the eager stock decode
        ref = eager_decode(model, routes, ids, tokens, custom=False, collect=True)
        eager_c = eager_decode(model, routes, ids, tokens, custom=True, collect=True)
        decoders = {}
        for name, custom in (("graph_stock", False), ("graph_custom", True)):
            d = GraphDecoder(model, routes, P, tokens, custom, pool=torch.cuda.graph_pool_handle())
            d.capture(ids)
            decoders[name] = d
        if any(c != layers for c in decoders["graph_custom"].captured_calls) or \
                any(decoders["graph_stock"].captured_calls):
            raise RuntimeError("a captured decode step does not route every MLP as asked")
        checks = {"eager_custom": _compare(torch, eager_c, ref)}
        for name, d in decoders.items():
            checks[name] = _compare(torch, d.decode(ids, collect=True), ref)
        if eager_c["calls"] != tokens * layers:
            raise RuntimeError("not every eager decode MLP used the custom path")
        for name, c in checks.items():
            if not c["tokens_equal"]:
                raise RuntimeError(f"{name}: greedy tokens differ from the stock decode; no performance claim")
            if c["max_scaled"] > 1:
                raise RuntimeError(f"{name}: logits outside atol {LOGIT_ATOL} / rtol {LOGIT_RTOL}")
        # timing: every side, interleaved, with its routing checked on every sample
        sides = {"eager_stock": lambda: eager_decode(model, routes, ids, tokens, custom=False),
                 "eager_custom": lambda: eager_decode(model, routes, ids, tokens, custom=True),
                 "graph_stock": lambda: decoders["graph_stock"].decode(ids),
                 "graph_custom": lambda: decoders["graph_custom"].decode(ids)}
        want = {"eager_stock": 0, "eager_custom": tokens * layers, "graph_stock": 0, "graph_custom": tokens * layers}
        for fn in sides.values():
            fn()  # warm
        got = {k: [] for k in sides}
        order = list(sides)
        for s in range(samples):
            for name in (order if s % 2 == 0 else order[::-1]):
                r = sides[name]()
                if r["calls"] != want[name]:
                    raise RuntimeError(f"timed {name} decode routing mismatch")
                got[name].append({k: r[k] for k in ("gpu_ms_per_token", "wall_ms_per_token", "calls")})
        for d in decoders.values():
            d.release()
        st = {k: _stats(v) for k, v in got.items()}
        wc = checks["graph_custom"]
        records.append({
            "prompt": f"seeded random token ids, length {P}", "prompt_tokens": P, "tokens": tokens,
            "exact_greedy_match": True, "logits_close": True,
            "max_logit_abs_error": max(c["max_abs"] for c in checks.values()),
            "max_logit_scaled_error": max(c["max_scaled"] for c in checks.values()),
            "generated_tokens": ref["tokens"][0].tolist(),
            "baseline": st["graph_stock"], "custom": st["graph_custom"],
            "wall_speedup": st["graph_stock"]["wall_median_ms"] / st["graph_custom"]["wall_median_ms"],
            "eager": {"baseline": st["eager_stock"], "custom": st["eager_custom"],
                      "wall_speedup": st["eager_stock"]["wall_median_ms"] / st["eager_custom"]["wall_median_ms"]},
            "graph_over_eager_custom": st["eager_custom"]["wall_median_ms"] / st["graph_custom"]["wall_median_ms"],
            "checks": checks, "graph_custom_max_logit_scaled_error": wc["max_scaled"]})
    here = Path(__file__).resolve()
    sources = [here.parents[1] / "csrc" / n for n in ("kernels.cuh", "registry.h", "swiglu_b200.cu")] + [here]
    result = {"schema_version": 1, "kind": "random-init-model-decode" + ("-tp" if world > 1 else ""),
              "model": f"TinyLlama-1.1B architecture, random init N(0,0.02) seed {seed}",
              "resolved_revision": f"random-init-seed-{seed}", "gpu": torch.cuda.get_device_name(),
              "torch": torch.__version__, "cuda": torch.version.cuda, "transformers": transformers.__version__,
              "precision": "fp16", "attention": "sdpa", "batch": 1, "ranks": world,
              "decode": "one CUDA graph per decode step (baseline/custom); eager transformers loop (eager)",
              "timing": "gpu-events-and-wall per decode of `tokens` steps", "prefill_included": False,
              "patched_layers": layers, "gate_config": chosen[0], "down_config": chosen[1], "tuning": tuning,
              "source_sha256": {p.name: hashlib.sha256(p.read_bytes()).hexdigest() for p in sources},
              "peak_allocated_bytes": torch.cuda.max_memory_allocated(), "cases": records}
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
        exchange.close()
        dist.barrier()
        dist.destroy_process_group()
    return result if rank == 0 else {}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--tokens", type=int, default=32)
    p.add_argument("--samples", type=int, default=7)
    p.add_argument("--layers", type=int, default=22)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-tune", action="store_true")
    p.add_argument("--pair", type=str, default="", help="gate,down ids (skips tuning)")
    p.add_argument("--output", type=Path, default=Path("results/model.json"))
    a = p.parse_args(argv)
    if not 1 <= a.tokens <= 256 or not 3 <= a.samples <= 31:
        raise SystemExit("tokens must be 1..256 and samples 3..31")
    pair = tuple(int(v) for v in a.pair.split(",")) if a.pair else None
    result = run(a.tokens, a.samples, a.layers, a.seed, tune=not a.no_tune, pair=pair)
    if not result:
        return
    a.output.parent.mkdir(parents=True, exist_ok=True)
    tmp = a.output.with_name(a.output.name + ".tmp")
    tmp.write_text(json.dumps(result, indent=2, allow_nan=False) + "\n")
    tmp.replace(a.output)
    for c in result["cases"]:
        print(f"{c['prompt']}: graph decode stock {c['baseline']['wall_median_ms']:.3f} ms/token, replaced "
              f"{c['custom']['wall_median_ms']:.3f} ({c['wall_speedup']:.3f}x); eager stock "
              f"{c['eager']['baseline']['wall_median_ms']:.3f}, replaced {c['eager']['custom']['wall_median_ms']:.3f}")


if __name__ == "__main__":
    main()
