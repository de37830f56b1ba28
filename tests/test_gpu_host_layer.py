"""GPU: the layer from pinned host x to pinned host y (swb_ffn_host_ex).

y_host must be bit-identical to y of the device-buffer layer (swb_ffn_ex) with the same
geometries -- the transfers move bytes and nothing else -- and within the oracle's y
tolerance (atol 0.003, rtol 0.01, include/contract.hpp:36-53). A chain of calls captured in
one CUDA graph with SWB_PREFETCH_WEIGHTS (each step its own pinned buffers) must give every
step the result of that step's plain call. Host memory that is not page-locked, and device
memory passed as host memory, are refused on the host before any launch.
"""
import numpy as np
import pytest
import torch

import oracle as O
from swiglu_b200 import _lib, binding

pytestmark = pytest.mark.gpu

PAIRS = [(69, 101), (68, 87), (69, 100), (33, 83), (96, 92), (69, 33)]  # 33: LDG down, y out by a transfer kernel


def _layer(hidden, inter, seed, dev):
    w = O.normal_workload(seed, hidden, inter)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in w.items()}
    return w, t


@pytest.mark.parametrize("hidden,inter", [(4096, 14336), (2048, 5632), (1030, 514), (64, 96)])
def test_host_layer_matches_device_layer_and_oracle(hidden, inter):
    dev = torch.device("cuda", 0)
    w, t = _layer(hidden, inter, 5, dev)
    x_host = t["x"].cpu().pin_memory()
    y_host = torch.empty(hidden, dtype=torch.float32).pin_memory()
    x = torch.empty(hidden, dtype=torch.float16, device=dev)
    h = torch.empty(inter, dtype=torch.float16, device=dev)
    y = torch.empty(hidden, dtype=torch.float32, device=dev)
    h_ref = torch.empty_like(h)
    y_ref = torch.empty_like(y)
    _, _, y_oracle = O.ffn(w)
    for g, d in PAIRS:
        binding.ffn(t["x"], t["wg"], t["wu"], t["wd"], t["bg"], t["bu"], t["bd"], h_ref, y_ref, g, d)
        y_host.fill_(float("nan"))
        binding.ffn_host(x_host, t["wg"], t["wu"], t["wd"], t["bg"], t["bu"], t["bd"], x, h, y, y_host, g, d)
        torch.cuda.synchronize()
        assert torch.equal(y_host, y_ref.cpu()), (g, d)
        assert torch.equal(y.cpu(), y_ref.cpu()), (g, d)
        assert O.compare(y_host.numpy(), y_oracle)[0], (g, d)
    assert binding.device_error() == 0


def test_host_layer_chain_in_one_graph_matches_plain_calls():
    dev = torch.device("cuda", 0)
    hidden, inter, steps = 4096, 14336, 6
    w, t = _layer(hidden, inter, 11, dev)
    xs = [(torch.randn(hidden) * (1 + k)).half().pin_memory() for k in range(steps)]
    ys = [torch.empty(hidden, dtype=torch.float32).pin_memory() for _ in range(steps)]
    x = torch.empty(hidden, dtype=torch.float16, device=dev)
    h = torch.empty(inter, dtype=torch.float16, device=dev)
    y = torch.empty(hidden, dtype=torch.float32, device=dev)
    expect = []
    for k in range(steps):
        binding.ffn(xs[k].to(dev), t["wg"], t["wu"], t["wd"], t["bg"], t["bu"], t["bd"], h, y, 69, 101)
        expect.append(y.cpu().clone())
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for k in range(steps):
                binding.ffn_host(xs[k], t["wg"], t["wu"], t["wd"], t["bg"], t["bu"], t["bd"], x, h, y, ys[k], 69, 101,
                                 stream=stream.cuda_stream, prefetch_weights=True)
        for r in range(3):  # the host rewrites nothing; each replay must reproduce every step
            for yk in ys:
                yk.fill_(float("nan"))
            g.replay()
            stream.synchronize()
            for k in range(steps):
                assert torch.equal(ys[k], expect[k]), (r, k)
        g.reset()
    # eager chain on the default stream as well
    for k in range(steps):
        binding.ffn_host(xs[k], t["wg"], t["wu"], t["wd"], t["bg"], t["bu"], t["bd"], x, h, y, ys[k], 69, 101,
                         prefetch_weights=True)
    torch.cuda.synchronize()
    assert all(torch.equal(ys[k], expect[k]) for k in range(steps))
    assert binding.device_error() == 0


def test_host_layer_refuses_pageable_and_device_memory_before_launch():
    dev = torch.device("cuda", 0)
    hidden, inter = 256, 512
    _, t = _layer(hidden, inter, 3, dev)
    x = torch.empty(hidden, dtype=torch.float16, device=dev)
    h = torch.empty(inter, dtype=torch.float16, device=dev)
    y = torch.empty(hidden, dtype=torch.float32, device=dev)
    pinned_x = t["x"].cpu().pin_memory()
    pinned_y = torch.empty(hidden, dtype=torch.float32).pin_memory()
    pageable_x = t["x"].cpu()
    L = _lib.lib()

    def call(xh, yh):
        return L.swb_ffn_host_ex(69, 101, t["wg"].data_ptr(), t["wu"].data_ptr(), t["wd"].data_ptr(), xh,
                                 t["bg"].data_ptr(), t["bu"].data_ptr(), t["bd"].data_ptr(), x.data_ptr(),
                                 h.data_ptr(), y.data_ptr(), yh, hidden, inter, 0, None)

    assert call(pageable_x.data_ptr(), pinned_y.data_ptr()) == _lib.SWB_E_INPUT
    assert b"page-locked" in L.swb_last_error()
    assert call(t["x"].data_ptr(), pinned_y.data_ptr()) == _lib.SWB_E_INPUT       # device memory as x_host
    assert call(pinned_x.data_ptr(), y.data_ptr()) == _lib.SWB_E_INPUT            # device memory as y_host
    with pytest.raises(RuntimeError, match="pinned"):
        binding.ffn_host(pageable_x, t["wg"], t["wu"], t["wd"], t["bg"], t["bu"], t["bd"], x, h, y, pinned_y, 69, 101)
    assert call(pinned_x.data_ptr(), pinned_y.data_ptr()) == 0
    torch.cuda.synchronize()
    assert binding.device_error() == 0
