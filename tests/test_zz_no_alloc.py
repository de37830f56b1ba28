"""swb_ffn_noalloc: the layer entry point for callers that cannot allocate.

Such callers (a foreign-function boundary with only raw pointers, a serving
runtime that owns all device memory, a loop that must never allocate) get h from
a fixed array inside the library instead of a workspace argument. This file is
named to be collected last; it must pass alone in a fresh process and after the
other tests.

Checked through the C ABI on two calls in a row with different inputs:
* against swb_ffn (the entry point that takes a caller workspace): bit-identical,
  the same kernels in the same order;
* against the CPU oracle: y within the parity tests' tolerance of the oracle's
  down projection of the kernels' h (relative error |a - e| / (|e| + atol_j) <= 2e-3,
  atol_j = 2^-11 sum_i |Wd[j,i] h[i]|), and within the reference's own gate
  (atol .003, rtol .01) of the oracle's whole layer.
Sizes beyond the array are rejected with a clear error before anything runs.
"""
import numpy as np
import pytest
import torch

import oracle as O
from swiglu_b200 import _lib

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _y_tol_ok(y, y_ref, wd, h):
    atol = 2.0 ** -11 * (np.abs(wd.astype(np.float32)) @ np.abs(h.astype(np.float32))).astype(np.float64)
    err = np.abs(y.astype(np.float64) - y_ref.astype(np.float64)) / (np.abs(y_ref.astype(np.float64)) + atol)
    return float(err.max()) <= 2e-3


def _run(fn_name, cfg, d, hidden, inter, h=None):
    L = _lib.lib()
    y = torch.empty(hidden, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    common = [d["wg"].data_ptr(), d["wu"].data_ptr(), d["wd"].data_ptr(), d["x"].data_ptr(), d["bg"].data_ptr(),
              d["bu"].data_ptr(), d["bd"].data_ptr()]
    if fn_name == "swb_ffn":
        rc = L.swb_ffn(cfg[0], cfg[1], *common, h.data_ptr(), y.data_ptr(), hidden, inter, s)
    else:
        rc = L.swb_ffn_noalloc(cfg[0], cfg[1], *common, y.data_ptr(), hidden, inter, s)
    _lib.check(rc)
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("shape", [(2048, 5632), (4096, 14336), (2047, 5631)])
def test_noalloc_matches_workspace_entry_point_twice(shape):
    hidden, inter = shape
    cfgs = [(80, 82), (33, 33), (64, 64)]
    for seed in (0, 1):  # two calls in a row with different inputs: nothing stale survives
        w = O.normal_workload(seed, hidden, inter)
        d = {k: _dev(v) for k, v in w.items()}
        h = torch.empty(inter, dtype=torch.float16, device="cuda")
        _, _, y_ref = O.ffn(w)
        for cfg in cfgs:
            y_ws = _run("swb_ffn", cfg, d, hidden, inter, h)
            h_k = h.cpu().numpy()  # the kernels' h (the no-alloc call writes the same into its array)
            y_na = _run("swb_ffn_noalloc", cfg, d, hidden, inter)
            assert np.array_equal(y_na.view(np.uint32), y_ws.view(np.uint32)), (shape, seed, cfg)
            y_own = O.project(w["wd"], h_k, w["bd"], w["x"])
            assert _y_tol_ok(y_na, y_own, w["wd"], h_k), (shape, seed, cfg)
            assert O.compare(y_na, y_ref)[0], (shape, seed, cfg)


def test_noalloc_rejects_sizes_beyond_its_array():
    """inter one past the array: rejected before any launch. Real buffers of that size are
    passed, so a regression in the guard fails the assertion instead of reading bad memory."""
    L = _lib.lib()
    hidden, inter = 64, _lib.SWB_NOALLOC_MAX_INTER + 1
    wg = torch.zeros(inter, hidden, dtype=torch.float16, device="cuda")
    wu = torch.zeros_like(wg)
    wd = torch.zeros(hidden, inter, dtype=torch.float16, device="cuda")
    x = torch.zeros(hidden, dtype=torch.float16, device="cuda")
    y = torch.full((hidden,), 3.0, dtype=torch.float32, device="cuda")
    rc = L.swb_ffn_noalloc(33, 33, wg.data_ptr(), wu.data_ptr(), wd.data_ptr(), x.data_ptr(), None, None, None,
                           y.data_ptr(), hidden, inter, None)
    assert rc == _lib.SWB_E_WORKSPACE
    assert "65536" in _lib.last_error()
    torch.cuda.synchronize()
    assert bool(torch.all(y == 3.0))  # nothing ran
