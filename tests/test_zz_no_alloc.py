"""swb_ffn_noalloc: the layer entry point for callers that cannot allocate.

Such callers (a foreign-function boundary with only raw pointers, a serving
runtime that owns all device memory, a loop that must never allocate) get h from
a fixed array inside the library instead of a workspace argument. This file is
named to be collected last; it must pass alone in a fresh process and after the
other tests.

Checked through the C ABI: two calls in a row, each against swb_ffn (the entry
point that takes a caller workspace) with the y tolerance the parity tests use
(relative error |a - e| / (|e| + atol_j) <= 2e-3, atol_j = 2^-11 sum_i |Wd[j,i] h[i]|);
sizes beyond the array are rejected with a clear error before anything runs.
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
        _, act, _ = O.ffn(w)
        for cfg in cfgs:
            y_ws = _run("swb_ffn", cfg, d, hidden, inter, h)
            y_na = _run("swb_ffn_noalloc", cfg, d, hidden, inter)
            assert _y_tol_ok(y_na, y_ws, w["wd"], act), (shape, seed, cfg)
            assert np.array_equal(y_na.view(np.uint32), y_ws.view(np.uint32))  # same kernels, same order


def test_noalloc_rejects_sizes_beyond_its_array():
    L = _lib.lib()
    fake = 0x7F0000000000
    rc = L.swb_ffn_noalloc(33, 33, fake, fake, fake, fake, None, None, None, fake, 64,
                           _lib.SWB_NOALLOC_MAX_INTER + 1, None)
    assert rc == _lib.SWB_E_WORKSPACE
    assert "65536" in _lib.last_error()
