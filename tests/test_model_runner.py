"""Decode runner pieces that need no GPU: the slot cache and the MLP router.

The slot cache must give the transformers decode loop exactly what its growing cache
gives: the same logits, bit for bit, step after step (a tiny fp32 Llama on CPU). The
router must send single-token calls to the replaced MLP only while asked, count them,
and leave the prefill and every stock call on the stock module.
"""
import pytest
import torch

from swiglu_b200 import model_runner as MR


def _tiny(layers=2):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=100, hidden_size=64, intermediate_size=96, num_hidden_layers=layers,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=128, hidden_act="silu")
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def test_slot_cache_matches_the_growing_cache_bit_for_bit():
    m = _tiny()
    ids = torch.randint(0, 100, (1, 7), generator=torch.Generator().manual_seed(3))
    steps = 6
    with torch.inference_mode():
        out = m(input_ids=ids, use_cache=True)
        past, tok = out.past_key_values, out.logits[:, -1:].argmax(-1)
        ref = []
        for _ in range(steps):
            o = m(input_ids=tok, past_key_values=past, use_cache=True)
            past, tok = o.past_key_values, o.logits[:, -1:].argmax(-1)
            ref.append(o.logits[0, -1])
        slots = MR.SlotCache(m.config, 7 + steps, "cpu", torch.float32)
        out = m(input_ids=ids, past_key_values=slots.cache, use_cache=True)
        tok = out.logits[:, -1:].argmax(-1)
        for t in range(steps):
            slots.seek(7 + t)  # a captured step's graph bakes exactly this position
            o = m(input_ids=tok, past_key_values=slots.cache, position_ids=torch.full((1, 1), 7 + t),
                  use_cache=True)
            tok = o.logits[:, -1:].argmax(-1)
            assert torch.equal(o.logits[0, -1], ref[t]), t
    with pytest.raises(RuntimeError, match="slot cache holds"):
        slots.layers[0].update(torch.zeros(1, 2, 1, 16), torch.zeros(1, 2, 1, 16))


def test_router_sends_only_single_token_calls_while_asked():
    m = _tiny()
    seen = []

    def call(idx, x, out):  # stands in for the kernels: the stock result, recorded
        seen.append(idx)
        out.copy_(routes.stock[idx](x).to(out.dtype))

    routes = MR.MLPRoutes(m, call)
    x1, x5 = torch.randn(1, 1, 64), torch.randn(1, 5, 64)
    mlp = m.model.layers[1].mlp
    stock = routes.stock[1](x1)
    assert torch.equal(mlp(x1), stock) and routes.calls == 0  # not asked: stock
    routes.custom = True
    assert mlp(x5).shape == (1, 5, 64) and routes.calls == 0  # prefill shape: stock
    y = mlp(x1)
    assert routes.calls == 1 and seen == [1] and y.shape == (1, 1, 64)
    assert torch.allclose(y.float(), stock.float(), atol=1e-2)


def test_prompts_are_seeded_and_sized():
    a, b = MR.prompts(0), MR.prompts(0)
    assert [p.shape[1] for p in a] == list(MR.PROMPT_LENGTHS)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
