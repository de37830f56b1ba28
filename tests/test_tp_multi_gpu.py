"""Tensor-parallel layer on real GPUs: one process per GPU, NCCL all-reduce.

Each rank runs swb_ffn_tp on its shard (rows of Wg/Wu, columns of Wd), the fp32
partial y is summed with an NCCL all-reduce, and bias + residual are applied once
(swb_residual_epilogue); then the fused paths (swb_ffn_tp_fused: the down kernel
or the whole-layer kernel sums the partials over NVLink peer memory), including
calls of different geometries issued back to back and the exchange's call count
after them. Every rank's y is compared with the unsharded CPU oracle at the
parity tests' tolerance, and the ranks' y must be bit-identical. Runs at 2, 4 and
8 ranks, each skipped when the process sees fewer GPUs.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, hidden, inter, q):
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "cuda-kernel_b200")]
    import torch
    import torch.distributed as dist
    import oracle as O
    from swiglu_b200 import binding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        _rank_body(rank, world, hidden, inter, q, dev, dist, torch, O, binding)
    except BaseException as exc:  # report to the parent at once instead of letting it wait
        import traceback
        q.put((rank, "error: " + "".join(traceback.format_exception(exc))))
        raise
    finally:
        dist.destroy_process_group()


def _rank_body(rank, world, hidden, inter, q, dev, dist, torch, O, binding):
    w = O.normal_workload(0, hidden, inter)
    a, b = rank * inter // world, (rank + 1) * inter // world
    t = lambda v: torch.from_numpy(np.ascontiguousarray(v)).to(dev)  # noqa: E731
    wg, wu, wd = t(w["wg"][a:b]), t(w["wu"][a:b]), t(w["wd"][:, a:b])
    bg, bu, x, bd = t(w["bg"][a:b]), t(w["bu"][a:b]), t(w["x"]), t(w["bd"])
    h = torch.empty(b - a, dtype=torch.float16, device=dev)
    y = torch.empty(hidden, dtype=torch.float32, device=dev)
    out = []
    for cfg in (33, 69, 87):
        binding.ffn_tp(x, wg, wu, wd, bg, bu, h, y, cfg, cfg)
        dist.all_reduce(y)
        binding.residual_epilogue(y, bd, x)
        torch.cuda.synchronize()
        out.append(y.cpu().numpy().copy())
    # the fused path: down projection + all-reduce over peer memory + epilogue in one kernel
    from swiglu_b200 import tp as T
    ex = T.Exchange(rank, world, hidden, dev)
    s = {"wg": wg, "wu": wu, "wd": wd, "bg": bg, "bu": bu}
    for gate, down in ((69, 80), (69, 83), (69, 87), (69, 87), (69, 102), (103, 102), (69, 100), (200, 0), (201, 0),
                       (200, 0), (220, 0), (223, 0), (221, 0)):
        y.zero_()
        T.ffn_tp_fused(ex, x, s, bd, h, y, gate, down)  # 200+: the rank's whole layer in one kernel
        torch.cuda.synchronize()
        out.append(y.cpu().numpy().copy())
    # from pinned host x to pinned host y (swb_ffn_tp_host_ex): the same reduced y on every rank
    x_host = x.cpu().pin_memory()
    xd = torch.empty_like(x)
    for gate, down in ((69, 102), (220, 0)):
        y_host = torch.empty(hidden, dtype=torch.float32).pin_memory()
        T.ffn_tp_host(ex, x_host, s, bd, xd, h, y, y_host, gate, down)
        torch.cuda.synchronize()
        out.append(y_host.numpy().copy())
    # geometries switched back to back with no host synchronisation: every call keeps its own y
    seq = [(69, 80), (200, 0), (69, 87), (220, 0), (201, 0), (69, 83), (223, 0), (103, 102), (69, 80)] * 3
    ys = [torch.empty_like(y) for _ in seq]
    for (gate, down), yk in zip(seq, ys):
        T.ffn_tp_fused(ex, x, s, bd, h, yk, gate, down)
    torch.cuda.synchronize()
    out.extend(yk.cpu().numpy().copy() for yk in ys)
    # layers chained with SWB_PREFETCH_WEIGHTS in one CUDA graph: bit-identical to plain calls
    # (69/102: the next layer's gate CTAs fit beside the down CTAs that wait on the exchange)
    stream = torch.cuda.Stream(dev)
    for gate, down in ((69, 87), (69, 102)):
        plain = torch.empty_like(y)
        T.ffn_tp_fused(ex, x, s, bd, h, plain, gate, down)
        torch.cuda.synchronize()  # calls on one exchange must not overlap (the chain runs on another stream)
        chain_ys = [torch.empty_like(y) for _ in range(4)]
        with torch.cuda.stream(stream):
            for yk in chain_ys:  # warm (and NCCL-free): eager chain first
                T.ffn_tp_fused(ex, x, s, bd, h, yk, gate, down, stream=stream.cuda_stream, prefetch_weights=True)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for yk in chain_ys:
                    T.ffn_tp_fused(ex, x, s, bd, h, yk, gate, down, stream=stream.cuda_stream, prefetch_weights=True)
            for yk in chain_ys:
                yk.zero_()
            g.replay()
            stream.synchronize()
            g.reset()
        torch.cuda.synchronize()
        assert all(torch.equal(yk, plain) for yk in chain_ys)
    # the model path (swiglu_out of a rank: model-rounding gate, fp16 y summed over the ranks)
    s_model = {"wg": wg, "wu": wu, "wd": wd}
    xm = x.view(1, 1, hidden)
    ym = torch.empty_like(xm)
    for gate, down in ((69, 87), (96, 80)):
        T.swiglu_tp_out(ex, xm, s_model, h, ym, gate, down)
        torch.cuda.synchronize()
        q.put((rank, ("model", gate, down, ym.cpu().numpy().ravel().copy())))
    # every call advanced the exchange's epoch once on every rank, whichever gate ran it
    # (SBULK work stealing included): 100 back-to-back calls, no host synchronisation
    before = ex.epoch()
    for k in range(100):
        T.ffn_tp_fused(ex, x, s, bd, h, y, (96, 69, 92, 200)[k % 4], 87)
    assert ex.epoch() - before == 100
    torch.cuda.synchronize()
    out.append(y.cpu().numpy().copy())
    dist.barrier()
    assert binding.device_error() == 0
    ex.close()
    q.put((rank, out))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_nccl_matches_oracle(world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    import oracle as O
    hidden, inter = 4096, 14336
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, hidden, inter, q)) for r in range(world)]
    for p in procs:
        p.start()
    results, model = {}, {}
    while len(results) < world:
        rank, out = q.get(timeout=300)
        assert not isinstance(out, str), out
        if isinstance(out, tuple) and out[0] == "model":
            model.setdefault(rank, []).append(out[1:])
        else:
            results[rank] = out
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = O.normal_workload(0, hidden, inter)
    _, act, y_ref = O.ffn(w)
    atol = 2.0 ** -11 * (np.abs(w["wd"].astype(np.float32)) @ np.abs(act.astype(np.float32)))
    for rank in range(world):
        for y in results[rank]:
            assert np.max(np.abs(y - y_ref) / (np.abs(y_ref) + atol)) <= 2e-3
            assert O.compare(y, y_ref)[0]
    for rank in range(1, world):
        for y0, yr in zip(results[0], results[rank]):
            assert np.array_equal(y0, yr)  # every rank holds the same reduced y
    # model path: fp16 y against the oracle's eager-fp16 pipeline at the binding's tolerance
    _, ym_ref = O.ffn_model(w)
    e = ym_ref.astype(np.float64)
    for rank in range(world):
        assert len(model[rank]) == 2
        for (g, d, ym), (_, _, ym0) in zip(model[rank], model[0]):
            assert np.max(np.abs(ym.astype(np.float64) - e) / (np.abs(e) + 1e-3 * np.abs(e).max())) <= 1e-2, (g, d)
            assert np.array_equal(ym.view(np.uint16), ym0.view(np.uint16))
