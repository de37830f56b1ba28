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
    for layer in binding.layer_config_ids():  # the whole rank's layer as one persistent kernel
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


@pytest.mark.gpu
@pytest.mark.parametrize("gcfg,dcfg", [(69, 102), (69, 87), (220, 0), (200, 0)])
def test_fused_tp_host_buffers_match_device_calls(gcfg, dcfg):
    """swb_ffn_tp_host_ex (pinned host x in, the rank's fused layer, pinned host y out) gives
    bit-identically the y of swb_ffn_tp_fused, one call at a time and chained with
    SWB_PREFETCH_WEIGHTS in one CUDA graph, each step with its own host buffers (one-rank
    exchange); pageable host memory is refused before any launch."""
    from swiglu_b200 import _lib, binding
    from swiglu_b200 import tp as T
    H, I, n = 4096, 14336, 8
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    w = O.normal_workload(4, H, I)
    s = T.shard(t(w["wg"]), t(w["wu"]), t(w["wd"]), t(w["bg"]), t(w["bu"]), 5, n)
    bd = t(w["bd"])
    ex = T.Exchange(0, 1, H, dev)
    h = torch.empty(I // n, dtype=torch.float16, device=dev)
    x = torch.empty(H, dtype=torch.float16, device=dev)
    y = torch.empty(H, dtype=torch.float32, device=dev)
    steps = 5
    xs = [(torch.from_numpy(w["x"]).float() * (1 + 0.25 * k)).half().pin_memory() for k in range(steps)]
    ys = [torch.empty(H, dtype=torch.float32).pin_memory() for _ in range(steps)]
    ref = []
    for k in range(steps):
        T.ffn_tp_fused(ex, xs[k].to(dev), s, bd, h, y, gcfg, dcfg)
        torch.cuda.synchronize()
        ref.append(y.cpu().clone())
    for k in range(steps):
        T.ffn_tp_host(ex, xs[k], s, bd, x, h, y, ys[k], gcfg, dcfg)
    torch.cuda.synchronize()
    assert all(torch.equal(ys[k], ref[k]) for k in range(steps))
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for k in range(steps):
                T.ffn_tp_host(ex, xs[k], s, bd, x, h, y, ys[k], gcfg, dcfg, stream=stream.cuda_stream,
                              prefetch_weights=True)
        for _ in range(3):
            for yk in ys:
                yk.fill_(float("nan"))
            g.replay()
            stream.synchronize()
            assert all(torch.equal(ys[k], ref[k]) for k in range(steps))
        g.reset()
    pageable = torch.from_numpy(w["x"].copy())
    rc = _lib.lib().swb_ffn_tp_host_ex(ex.handle, gcfg, dcfg, s["wg"].data_ptr(), s["wu"].data_ptr(),
                                       s["wd"].data_ptr(), pageable.data_ptr(), s["bg"].data_ptr(),
                                       s["bu"].data_ptr(), bd.data_ptr(), x.data_ptr(), h.data_ptr(), y.data_ptr(),
                                       ys[0].data_ptr(), H, I // n, 0, None)
    assert rc == _lib.SWB_E_INPUT
    torch.cuda.synchronize()
    assert binding.device_error() == 0
    ex.close()


@pytest.mark.gpu
def test_model_path_rank_matches_swiglu_out_and_oracle():
    """swb_swiglu_tp_out on a one-rank exchange is the binding's swiglu_out (model rounding,
    fp16 y, no bias or residual) with the down projection's rows summed through the exchange:
    bit-identical to swiglu_out with the same geometries, within the binding's tolerance of
    the oracle's fp16 pipeline; its guards reject what swiglu_out rejects."""
    from swiglu_b200 import binding
    from swiglu_b200 import tp as T
    H, I = 2048, 5632
    w = O.normal_workload(4, H, I)
    h_ref, y_ref = O.ffn_model(w)
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    s = {"wg": t(w["wg"]), "wu": t(w["wu"]), "wd": t(w["wd"])}
    x = t(w["x"]).view(1, 1, H)
    h, h1 = torch.empty(I, dtype=torch.float16, device=dev), torch.empty(I, dtype=torch.float16, device=dev)
    y, y1 = torch.empty_like(x), torch.empty_like(x)
    ex = T.Exchange(0, 1, H, dev)
    for g, d in ((69, 87), (33, 85), (96, 82), (79, 80)):
        binding.swiglu_out(x, s["wg"], s["wu"], s["wd"], h1, y1, g, d)
        T.swiglu_tp_out(ex, x, s, h, y, g, d)
        torch.cuda.synchronize()
        assert torch.equal(h, h1) and torch.equal(y, y1), (g, d)
        yc = y.cpu().numpy().ravel().astype(np.float64)
        e = y_ref.astype(np.float64)
        assert np.max(np.abs(yc - e) / (np.abs(e) + 1e-3 * np.abs(e).max())) <= 1e-2
    with pytest.raises(RuntimeError, match="workspace overlaps input storage"):
        T.swiglu_tp_out(ex, x, s, h, x, 69, 87)
    with pytest.raises(RuntimeError, match="configuration out of range"):
        T.swiglu_tp_out(ex, x, s, h, y, 1001, 87)
    with pytest.raises(RuntimeError, match="invalid configuration"):
        T.swiglu_tp_out(ex, x, s, h, y, 69, 999)
    with pytest.raises(RuntimeError, match="RBULK"):
        T.swiglu_tp_out(ex, x, s, h, y, 69, 33)
    assert binding.device_error() == 0
    ex.close()


@pytest.mark.gpu
def test_every_call_advances_the_exchange_epoch_once():
    """Each fused tensor-parallel call advances the exchange's call epoch exactly once,
    whichever gate family runs it. Under work stealing (SBULK ids) the CTA that owns row 0
    does it, not CTA 0 (which the hardware may cancel before it starts): 200 back-to-back
    calls per gate, no host synchronisation between them, must count 200."""
    from swiglu_b200 import binding
    from swiglu_b200 import tp as T
    H, I, n = 4096, 14336, 8
    dev = torch.device("cuda", 0)
    w = O.normal_workload(0, H, I)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    s = T.shard(t(w["wg"]), t(w["wu"]), t(w["wd"]), t(w["bg"]), t(w["bu"]), 2, n)
    x, bd = t(w["x"]), t(w["bd"])
    h = torch.empty(I // n, dtype=torch.float16, device=dev)
    y = torch.empty(H, dtype=torch.float32, device=dev)
    ex = T.Exchange(0, 1, H, dev)
    for gate in (96, 92, 99, 69, 33, 87, 200):
        before = ex.epoch()
        for _ in range(200):
            T.ffn_tp_fused(ex, x, s, bd, h, y, gate, 87)
        assert ex.epoch() - before == 200, gate
    assert binding.device_error() == 0
    ex.close()


def _handles_worker(rank, world, port, mode, q):
    import datetime
    import time
    import torch.distributed as dist
    from swiglu_b200 import tp as T
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    mine = bytes([rank + 1]) * 64
    t0 = time.monotonic()
    try:
        if rank == 1 and mode == "absent":
            q.put((rank, "left", 0.0))
            q.close()
            q.join_thread()  # the message is out before the process vanishes
            os._exit(0)  # leaves without joining the exchange (and without shutting the group down)
        if rank == 1 and mode == "malformed":
            dist.all_gather_object([None] * world, b"short")  # bypasses its own check
            q.put((rank, "sent", 0.0))
            return
        handles = T.share_handles(mine, world)
        q.put((rank, [h[0] for h in handles], time.monotonic() - t0))
    except Exception as exc:  # noqa: BLE001 -- reported to the parent
        q.put((rank, f"{type(exc).__name__}: {exc}"[:200], time.monotonic() - t0))
    finally:
        if not (rank == 1 and mode == "absent"):
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


@pytest.mark.parametrize("mode", ["ok", "absent", "malformed"])
def test_exchange_handle_sharing_fails_cleanly_gloo(mode):
    """Set-up of the fused exchange on CPU ranks: every rank gets every handle in rank order;
    a rank that never joins makes the other's set-up raise within the group's timeout (no
    hang); a malformed handle raises on the rank that receives it."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_handles_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, out, dt = q.get(timeout=120)
        got[rank] = (out, dt)
    for p in procs:
        p.join(timeout=60)
    if mode == "ok":
        assert got[0][0] == [1, 2] and got[1][0] == [1, 2]
    elif mode == "absent":
        assert got[1][0] == "left"
        assert isinstance(got[0][0], str) and got[0][1] < 60  # an error, within the timeout scale
    else:
        assert isinstance(got[0][0], str) and got[0][0].startswith("ValueError")


def _idle_peer_proc(role, H, hq, tq, rq, done):
    """One rank of a two-rank exchange on GPU 0 (see test_peer_wait_times_out_and_reports)."""
    import ctypes
    import sys
    import time
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "cuda-kernel_b200")]
    import torch
    from swiglu_b200 import _lib, binding
    torch.cuda.set_device(0)
    L = _lib.lib()
    tp = ctypes.c_void_p()
    _lib.check(L.swb_tp_create(role, 2, H, ctypes.byref(tp)))
    mine = (ctypes.c_uint8 * _lib.SWB_TP_HANDLE_BYTES)()
    _lib.check(L.swb_tp_ipc_handle(tp, mine))
    hq.put((role, bytes(mine)))
    table = tq.get(timeout=120)
    buf = (ctypes.c_uint8 * len(table)).from_buffer_copy(table)
    _lib.check(L.swb_tp_connect(tp, buf))
    if role == 1:
        # holds its buffer mapped and never calls: nothing writes rank 1's slots in rank 0's buffer
        rq.put((1, "ready", 0.0))
        done.wait(120)
        L.swb_tp_destroy(tp)
        return
    I = 256
    dev = torch.device("cuda", 0)
    wg = (torch.randn(I, H, device=dev) * 0.05).half()
    wu = (torch.randn(I, H, device=dev) * 0.05).half()
    wd = (torch.randn(H, I, device=dev) * 0.05).half()
    x = torch.randn(H, device=dev).half()
    h = torch.empty(I, dtype=torch.float16, device=dev)
    y = torch.full((H,), 7.0, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    binding.device_error(clear=True)
    t0 = time.monotonic()
    _lib.check(L.swb_ffn_tp_fused(tp, 69, 87, wg.data_ptr(), wu.data_ptr(), wd.data_ptr(), x.data_ptr(), None, None,
                                  None, h.data_ptr(), y.data_ptr(), H, I, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    err = binding.device_error(clear=True)
    untouched = bool(torch.all(y == 7.0).item())  # rows whose peer did not deliver are not written
    usable = float(torch.ones(8, device=dev).sum().item()) == 8.0
    L.swb_tp_destroy(tp)
    rq.put((0, (err, elapsed, untouched, usable), elapsed))
    done.set()


@pytest.mark.gpu
def test_peer_wait_times_out_and_reports():
    """Failure detection without a GPU fault: rank 1 of a two-rank exchange (a second process
    on the same GPU) maps its buffer but never runs the layer -- a flag nothing sets. Rank 0's
    fused layer stores its partials, waits (bounded, 1 s) for rank 1's, gives up, returns
    without writing y and reports SWB_DEVERR_PEER_TIMEOUT; the context stays usable. Only one
    kernel ever waits, and every store lands in memory that stays mapped."""
    import torch.multiprocessing as mp
    H = 512
    ctx = mp.get_context("spawn")
    hq, rq = ctx.Queue(), ctx.Queue()
    tqs = [ctx.Queue(), ctx.Queue()]
    done = ctx.Event()
    procs = [ctx.Process(target=_idle_peer_proc, args=(r, H, hq, tqs[r], rq, done)) for r in range(2)]
    for p in procs:
        p.start()
    handles = dict(hq.get(timeout=180) for _ in range(2))
    table = handles[0] + handles[1]
    for q in tqs:
        q.put(table)
    results = {}
    for _ in range(2):
        rank, out, _ = rq.get(timeout=180)
        results[rank] = out
    done.set()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    err, elapsed, untouched, usable = results[0]
    assert err & 2, err  # SWB_DEVERR_PEER_TIMEOUT
    assert 0.9 < elapsed < 30, elapsed
    assert untouched and usable
