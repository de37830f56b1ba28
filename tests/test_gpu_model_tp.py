"""TinyLlama-architecture decode with tensor-parallel MLPs: two ranks, one GPU each.

Each rank holds the whole model and its shard of every MLP; a replaced MLP is one
swb_swiglu_tp_out call (gate on the shard, down projection with the all-reduce over
NVLink fused in). The runner's gates must hold on every rank: greedy tokens of the eager
and graph-captured replaced decodes identical to the eager stock decode, logits within
atol .1 / rtol .02, every replaced decode routed through tokens x layers calls. Skipped
with fewer than two GPUs.
"""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "cuda-kernel_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), LOCAL_RANK=str(rank),
                      WORLD_SIZE=str(world), NCCL_NVLS_ENABLE="0")
    try:
        from swiglu_b200 import model_runner
        res = model_runner.run(tokens=32, samples=3, layers=22, seed=0, pair=(69, 87))
        q.put((rank, res))
    except BaseException as exc:  # report at once instead of letting the parent wait
        import traceback
        q.put((rank, "error: " + "".join(traceback.format_exception(exc))))
        raise


def test_tinyllama_architecture_decode_tensor_parallel_two_ranks():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from swiglu_b200 import model_report
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, res = q.get(timeout=900)
        assert not isinstance(res, str), res
        out[rank] = res
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    result = out[0]
    assert result["kind"] == "random-init-model-decode-tp" and result["ranks"] == 2
    for case in result["cases"]:
        assert case["exact_greedy_match"] and case["logits_close"]
        assert all(c["tokens_equal"] for c in case["checks"].values())
    assert "random-init-seed-0" in model_report.render(result)
