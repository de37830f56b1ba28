"""Tensor-parallel layer: sharding arithmetic on CPU ranks (gloo), and the rank
entry point on one GPU with the ranks emulated as shards.

Partitioning (rank r of n): Wg, Wu rows [r*I/n, (r+1)*I/n); Wd columns of the same
range, stored contiguously; y = sum_r Wd_r h_r, then + bd + x once.
"""
import os
import socket

import numpy as np
import pytest
import torch

import oracle as O


def shard(w, r, n):
    inter = w["wg"].shape[0]
    a, b = r * inter // n, (r + 1) * inter // n
    return {"wg": np.ascontiguousarray(w["wg"][a:b]), "wu": np.ascontiguousarray(w["wu"][a:b]),
            "wd": np.ascontiguousarray(w["wd"][:, a:b]), "bg": w["bg"][a:b], "bu": w["bu"][a:b],
            "x": w["x"]}


def rank_partial(w, r, n):
    """One rank's work in the oracle's arithmetic: h_r (fp16) and the fp32 partial Wd_r h_r."""
    s = shard(w, r, n)
    h = O.gate(s["wg"], s["wu"], s["x"], s["bg"], s["bu"])
    return h, O.project(s["wd"], h)


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, hidden, inter, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = O.normal_workload(0, hidden, inter)
        h, part = rank_partial(w, rank, world)
        y = torch.from_numpy(part.astype(np.float64))
        dist.all_reduce(y)  # the exchange step of the layer
        if rank == 0:
            q.put(y.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_partition_matches_unsharded_oracle_gloo(world):
    import torch.multiprocessing as mp
    hidden, inter = 96, 352
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, hidden, inter, q)) for r in range(world)]
    for p in procs:
        p.start()
    y = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = O.normal_workload(0, hidden, inter)
    _, act, y_ref = O.ffn(w)
    y_tp = (y + O.f16_values(w["x"]).astype(np.float64) + O.f16_values(w["bd"]).astype(np.float64))
    # every h element is computed by exactly one rank with the same arithmetic: only the
    # order of the final K-sum differs from the unsharded oracle
    assert np.allclose(y_tp, y_ref, rtol=1e-5, atol=1e-5)


def test_tp_gate_shards_are_bit_identical_to_unsharded():
    w = O.normal_workload(1, 64, 240)
    full = O.gate(w["wg"], w["wu"], w["x"], w["bg"], w["bu"])
    parts = [rank_partial(w, r, 4)[0] for r in range(4)]
    assert np.array_equal(np.concatenate(parts).view(np.uint16), full.view(np.uint16))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [2, 4, 8])
def test_ffn_tp_ranks_emulated_on_one_gpu(n):
    from swiglu_b200 import binding
    hidden, inter = 4096, 14336
    w = O.normal_workload(0, hidden, inter)
    _, act, y_ref = O.ffn(w)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    x, bd = dev(w["x"]), dev(w["bd"])
    y = torch.zeros(hidden, dtype=torch.float32, device="cuda")
    for cfg in (33, 64, 69):
        parts = []
        for r in range(n):
            s = {k: dev(v) for k, v in shard(w, r, n).items()}
            h = torch.empty(inter // n, dtype=torch.float16, device="cuda")
            yp = torch.empty(hidden, dtype=torch.float32, device="cuda")
            binding.ffn_tp(x, s["wg"], s["wu"], s["wd"], s["bg"], s["bu"], h, yp, cfg, cfg)
            parts.append(yp)
        y.copy_(torch.stack(parts).sum(0))  # stands in for the all-reduce
        binding.residual_epilogue(y, bd, x)
        yc = y.cpu().numpy()
        atol = 2.0 ** -11 * (np.abs(w["wd"].astype(np.float32)) @ np.abs(act.astype(np.float32)))
        assert np.max(np.abs(yc - y_ref) / (np.abs(y_ref) + atol)) <= 2e-3
        assert O.compare(yc, y_ref)[0]


@pytest.mark.gpu
def test_fused_tp_single_rank_eager_and_graph_replays():
    """World size 1 runs the whole fused epilogue (push, flag, wait, rank-ordered sum) on one GPU."""
    from swiglu_b200 import tp as T
    hidden, inter = 4096, 14336
    w = O.normal_workload(0, hidden, inter)
    _, act, y_ref = O.ffn(w)
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    s = T.shard(t(w["wg"]), t(w["wu"]), t(w["wd"]), t(w["bg"]), t(w["bu"]), 0, 1)
    x, bd = t(w["x"]), t(w["bd"])
    h = torch.empty(inter, dtype=torch.float16, device=dev)
    y = torch.empty(hidden, dtype=torch.float32, device=dev)
    ex = T.Exchange(0, 1, hidden, dev)
    atol = 2.0 ** -11 * (np.abs(w["wd"].astype(np.float32)) @ np.abs(act.astype(np.float32)))

    def ok():
        # y against the oracle's down projection of the kernel's own h (one rank holds all of h)
        yc, hc = y.cpu().numpy(), h.cpu().numpy()
        y_own = O.project(w["wd"], hc, w["bd"], w["x"])
        a_own = 2.0 ** -11 * (np.abs(w["wd"].astype(np.float32)) @ np.abs(hc.astype(np.float32)))
        return np.max(np.abs(yc - y_own) / (np.abs(y_own) + a_own)) <= 2e-3 and O.compare(yc, y_ref)[0]

    from swiglu_b200 import binding
    for down in (80, 83, 87):
        for _ in range(3):  # epochs advance call after call
            y.zero_()
            T.ffn_tp_fused(ex, x, s, bd, h, y, 69, down)
            torch.cuda.synchronize()
            assert ok(), down
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            T.ffn_tp_fused(ex, x, s, bd, h, y, 69, 87, stream=stream.cuda_stream)
        for _ in range(5):  # the captured epoch counters live in device memory: replays keep working
            y.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert ok()
        g.reset()
    for layer in binding.layer_config_ids()[:3]:  # the whole rank's layer as one persistent kernel
        for _ in range(2):
            y.zero_()
            T.ffn_tp_fused(ex, x, s, bd, h, y, layer, 0)
            torch.cuda.synchronize()
            assert ok(), layer
    assert binding.device_error() == 0
    with pytest.raises(RuntimeError, match="RBULK"):
        T.ffn_tp_fused(ex, x, s, bd, h, y, 69, 33)
    ex.close()


@pytest.mark.gpu
@pytest.mark.parametrize("gcfg", [69, 33, 82, 96])
def test_fused_tp_prefetch_chain_matches_plain(gcfg):
    """A rank's fused layers chained with SWB_PREFETCH_WEIGHTS (each gate starts streaming while
    the previous layer's down + exchange runs; the epoch advance waits for it) are bit-identical
    to plain calls, eagerly and in one CUDA graph (one-rank exchange)."""
    from swiglu_b200 import binding
    from swiglu_b200 import tp as T
    H, I, n = 4096, 14336, 8
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    shards, xs = [], []
    for seed in (0, 1):
        w = O.normal_workload(seed, H, I)
        shards.append(T.shard(t(w["wg"]), t(w["wu"]), t(w["wd"]), t(w["bg"]), t(w["bu"]), 3, n))
        xs.append((t(w["x"]), t(w["bd"])))
    ex = T.Exchange(0, 1, H, dev)
    h = torch.empty(I // n, dtype=torch.float16, device=dev)
    ref = []
    for k in range(2):
        y = torch.empty(H, dtype=torch.float32, device=dev)
        T.ffn_tp_fused(ex, xs[k][0], shards[k], xs[k][1], h, y, gcfg, 87)
        torch.cuda.synchronize()
        ref.append(y.clone())
    ys = [torch.empty(H, dtype=torch.float32, device=dev) for _ in range(6)]
    stream = torch.cuda.Stream(dev)

    def chain():
        for k in range(6):
            T.ffn_tp_fused(ex, xs[k % 2][0], shards[k % 2], xs[k % 2][1], h, ys[k], gcfg, 87,
                           stream=stream.cuda_stream, prefetch_weights=True)

    with torch.cuda.stream(stream):
        chain()
        stream.synchronize()
        assert all(torch.equal(ys[k], ref[k % 2]) for k in range(6))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            chain()
        for _ in range(3):
            for yk in ys:
                yk.zero_()
            g.replay()
            stream.synchronize()
            assert all(torch.equal(ys[k], ref[k % 2]) for k in range(6))
        g.reset()
    assert binding.device_error() == 0
    ex.close()
