"""PyTorch-facing surface of the decode layer, drop-in for the reference binding.

``swiglu_out``, ``swiglu`` and ``config_ids`` keep the names, arguments,
checks (in the same order), messages and error type (``RuntimeError``) of
``src/torch_extension.cu`` in shubhxho/cuda-kernel, so callers written against
``torch.utils.cpp_extension.load(name="decode_swiglu", ...)`` work unchanged
(``cuda-kernel_b200/decode_swiglu.py`` re-exports them under that module name).

Torch supplies device memory and the current stream only; every launch goes
through the C ABI of ``libswiglu_b200.so``. Calls are asynchronous on the
current CUDA stream, allocate nothing (``swiglu`` allocates its outputs, as the
reference's does), and overwrite the caller's workspace and output.
"""
from __future__ import annotations

import operator

import torch

from . import _lib

_INT64_MIN, _INT64_MAX = -(2 ** 63), 2 ** 63 - 1


def _check(cond: bool, message: str) -> None:
    if not cond:
        raise RuntimeError(message)


def _as_int64(value) -> int:
    v = operator.index(value)
    if not _INT64_MIN <= v <= _INT64_MAX:
        raise TypeError("configuration id does not fit in int64")
    return v


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def config_ids() -> list[int]:
    """Registry ids in order (torch_extension.cu:52; config.hpp:7-11)."""
    L = _lib.lib()
    n = L.swb_config_count()
    buf = (_lib.ctypes.c_int * n)()
    L.swb_config_ids(buf, n)
    return list(buf)


def config_info(config_id: int) -> dict:
    info = _lib.SwbConfig()
    _lib.check(_lib.lib().swb_config_info(_as_int64(config_id), _lib.ctypes.byref(info)))
    return info.as_dict()


def valid_config(config_id: int) -> bool:
    return bool(_lib.lib().swb_valid_config(_as_int64(config_id)))


def swiglu_out(x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
               h: torch.Tensor, y: torch.Tensor, gate_config: int, down_config: int) -> None:
    """Batch-one SwiGLU MLP into caller-owned buffers (torch_extension.cu:7-40).

    x: [..., H] single token; gate, up: [I, H]; down: [H, I]; h: [I] workspace;
    y: same shape as x. All contiguous CUDA fp16 on one device, no grad.
    Computes y = fp16(down @ fp16(fp16(SiLU(fp16(gate@x))) * fp16(up@x))),
    rounding where eager fp16 PyTorch rounds.
    """
    gate_config = _as_int64(gate_config)
    down_config = _as_int64(down_config)
    for t in (x, gate, up, down, h, y):
        _check(t.is_cuda and t.dtype == torch.float16 and t.is_contiguous(),
               "all buffers must be contiguous CUDA FP16 tensors")
        _check(t.device == x.device, "buffers must share a device")
        _check(not t.requires_grad, "inference only: disable gradients")
    _check(gate.dim() == 2 and up.dim() == 2 and down.dim() == 2 and x.dim() >= 1, "invalid dimensions")
    hidden, intermediate = gate.size(1), gate.size(0)
    _check(0 < hidden <= 100000 and 0 < intermediate <= 100000, "invalid shape")
    _check(x.numel() == hidden and x.size(-1) == hidden, "single-token batch-one decode required")
    _check(up.shape == gate.shape and down.size(0) == hidden and down.size(1) == intermediate,
           "incompatible weights")
    _check(h.numel() == intermediate and y.shape == x.shape, "invalid workspace shape")
    # Config range / validity and the alias guards run in the C ABI, in the
    # binding's order (torch_extension.cu:21-30), before anything launches.
    with torch.cuda.device(x.device):
        status = _lib.lib().swb_swiglu_out(
            x.data_ptr(), gate.data_ptr(), up.data_ptr(), down.data_ptr(), h.data_ptr(), y.data_ptr(),
            hidden, intermediate, gate_config, down_config, _stream(x.device))
    _lib.check(status)


def swiglu(x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
           gate_config: int, down_config: int = -1) -> torch.Tensor:
    """Allocating wrapper (torch_extension.cu:41-47): down_config < 0 reuses gate_config."""
    _check(gate.dim() == 2, "gate must be a matrix")
    h = torch.empty((gate.size(0),), dtype=x.dtype, device=x.device)
    y = torch.empty_like(x)
    swiglu_out(x, gate, up, down, h, y, gate_config, gate_config if _as_int64(down_config) < 0 else down_config)
    return y


# ------------------------------------------------------------ lower level

def _ptr(t):
    return None if t is None else t.data_ptr()


def gate(wg: torch.Tensor, wu: torch.Tensor, x: torch.Tensor, h: torch.Tensor, config: int,
         bg: torch.Tensor | None = None, bu: torch.Tensor | None = None, model_round: bool = False,
         stream: int | None = None) -> None:
    """h[i] = fp16(SiLU(Wg[i].x + bg[i]) * (Wu[i].x + bu[i])) -- decode::launch<true,false>."""
    rows, cols = wg.shape
    s = _stream(x.device) if stream is None else stream
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_gate(int(config), wg.data_ptr(), wu.data_ptr(), x.data_ptr(), _ptr(bg), _ptr(bu),
                                       h.data_ptr(), rows, cols, int(bool(model_round)), s))


def project(w: torch.Tensor, x: torch.Tensor, out: torch.Tensor, config: int,
            bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
            stream: int | None = None) -> None:
    """out[r] = W[r].x (+bias) (+residual); fp32 out, or fp16 when ``out`` is fp16."""
    rows, cols = w.shape
    flags = (_lib.SWB_RESIDUAL if residual is not None else 0) | \
            (_lib.SWB_HALF_OUT if out.dtype == torch.float16 else 0)
    s = _stream(x.device) if stream is None else stream
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_project(int(config), w.data_ptr(), x.data_ptr(), _ptr(bias), _ptr(residual),
                                          out.data_ptr(), rows, cols, flags, s))


def ffn(x: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor, bg: torch.Tensor,
        bu: torch.Tensor, bd: torch.Tensor, h: torch.Tensor, y: torch.Tensor, gate_config: int,
        down_config: int, stream: int | None = None, prefetch_weights: bool = False) -> None:
    """Whole layer with biases and residual (benchmark.cu:161-165): y fp32 [H].

    ``prefetch_weights``: SWB_PREFETCH_WEIGHTS -- the gate may start streaming Wg/Wu
    before the previous kernel in the stream finishes (no kernel before the call may
    write them)."""
    inter, hidden = wg.shape
    s = _stream(x.device) if stream is None else stream
    flags = _lib.SWB_PREFETCH_WEIGHTS if prefetch_weights else 0
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_ffn_ex(int(gate_config), int(down_config), wg.data_ptr(), wu.data_ptr(),
                                         wd.data_ptr(), x.data_ptr(), _ptr(bg), _ptr(bu), _ptr(bd), h.data_ptr(),
                                         y.data_ptr(), hidden, inter, flags, s))


def ffn_host(x_host: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor, bg: torch.Tensor,
             bu: torch.Tensor, bd: torch.Tensor, x: torch.Tensor, h: torch.Tensor, y: torch.Tensor,
             y_host: torch.Tensor, gate_config: int, down_config: int, stream: int | None = None,
             prefetch_weights: bool = False) -> None:
    """The layer from pinned host ``x_host`` (fp16 [H]) to pinned host ``y_host`` (fp32 [H])
    (swb_ffn_host_ex): x in, gate, down, y out as one programmatic chain on the GPU. ``x``,
    ``h`` and ``y`` are device buffers the call overwrites. ``y_host`` holds the result once
    the stream has passed the call. ``prefetch_weights``: consecutive calls form one chain."""
    inter, hidden = wg.shape
    _check(x_host.device.type == "cpu" and y_host.device.type == "cpu", "x_host and y_host must be host tensors")
    _check(x_host.is_pinned() and y_host.is_pinned(), "x_host and y_host must be pinned (page-locked)")
    _check(x_host.dtype == torch.float16 and y_host.dtype == torch.float32, "x_host fp16, y_host fp32")
    _check(x_host.numel() == hidden and y_host.numel() == hidden and x_host.is_contiguous()
           and y_host.is_contiguous(), "x_host and y_host must be contiguous [hidden]")
    s = _stream(x.device) if stream is None else stream
    flags = _lib.SWB_PREFETCH_WEIGHTS if prefetch_weights else 0
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_ffn_host_ex(int(gate_config), int(down_config), wg.data_ptr(), wu.data_ptr(),
                                              wd.data_ptr(), x_host.data_ptr(), _ptr(bg), _ptr(bu), _ptr(bd),
                                              x.data_ptr(), h.data_ptr(), y.data_ptr(), y_host.data_ptr(), hidden,
                                              inter, flags, s))


def layer_config_ids() -> list[int]:
    """Ids of the fused whole-layer kernels (swb_ffn_fused)."""
    L = _lib.lib()
    n = L.swb_layer_config_count()
    buf = (_lib.ctypes.c_int * n)()
    L.swb_layer_config_ids(buf, n)
    return list(buf)


def layer_workspace(device: torch.device | int | None = None) -> torch.Tensor:
    """A zeroed workspace for swb_ffn_fused (one per stream of calls)."""
    return torch.zeros(_lib.SWB_LAYER_WORKSPACE_BYTES, dtype=torch.uint8, device=device or "cuda")


def ffn_fused(x: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor, bg: torch.Tensor,
              bu: torch.Tensor, bd: torch.Tensor, h: torch.Tensor, y: torch.Tensor, layer_config: int,
              workspace: torch.Tensor, stream: int | None = None, prefetch_weights: bool = False) -> None:
    """The whole layer as one persistent kernel: y fp32 [H]. Ids 200-219 run the gate, a grid
    barrier, then the down rows; ids 220+ stream the down rows block by block as h fills.
    ``prefetch_weights`` (ids 220+): launched programmatically after the kernel before it."""
    inter, hidden = wg.shape
    s = _stream(x.device) if stream is None else stream
    flags = _lib.SWB_PREFETCH_WEIGHTS if prefetch_weights else 0
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_ffn_fused_ex(int(layer_config), wg.data_ptr(), wu.data_ptr(), wd.data_ptr(),
                                               x.data_ptr(), _ptr(bg), _ptr(bu), _ptr(bd), h.data_ptr(),
                                               y.data_ptr(), hidden, inter, workspace.data_ptr(), flags, s))


def ffn_tp(x: torch.Tensor, wg_shard: torch.Tensor, wu_shard: torch.Tensor, wd_shard: torch.Tensor,
           bg_shard: torch.Tensor | None, bu_shard: torch.Tensor | None, h_shard: torch.Tensor,
           y_partial: torch.Tensor, gate_config: int, down_config: int, stream: int | None = None) -> None:
    """One tensor-parallel rank: h_r = gate(shard rows), y_partial = Wd[:, shard] h_r (fp32, no bias)."""
    shard, hidden = wg_shard.shape
    s = _stream(x.device) if stream is None else stream
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_ffn_tp(int(gate_config), int(down_config), wg_shard.data_ptr(),
                                         wu_shard.data_ptr(), wd_shard.data_ptr(), x.data_ptr(), _ptr(bg_shard),
                                         _ptr(bu_shard), h_shard.data_ptr(), y_partial.data_ptr(), hidden, shard, s))


def residual_epilogue(y: torch.Tensor, bias: torch.Tensor, x: torch.Tensor, stream: int | None = None) -> None:
    """y += bias + x (kernels.cuh:142-145); closes a tensor-parallel layer."""
    s = _stream(y.device) if stream is None else stream
    with torch.cuda.device(y.device):
        _lib.check(_lib.lib().swb_residual_epilogue(y.data_ptr(), bias.data_ptr(), x.data_ptr(), y.numel(), s))


def cuda_versions() -> tuple[int, int]:
    """(driver, runtime) versions seen by the native library."""
    d, r = _lib.ctypes.c_int(), _lib.ctypes.c_int()
    _lib.check(_lib.lib().swb_cuda_versions(_lib.ctypes.byref(d), _lib.ctypes.byref(r)))
    return d.value, r.value


def device_error(clear: bool = True) -> int:
    """OR of device-side error codes on the current device (synchronises)."""
    out = _lib.ctypes.c_int()
    _lib.check(_lib.lib().swb_device_error(int(bool(clear)), _lib.ctypes.byref(out)))
    return out.value


class CublasBaseline:
    """cuBLAS GemmEx + pointwise baseline (benchmark.cu:143-160) on one device."""

    def __init__(self, device: torch.device | int | None = None):
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   (device if isinstance(device, int) else device.index))
        self._L = _lib.cublas_lib()
        handle = _lib.ctypes.c_void_p()
        with torch.cuda.device(self.device):
            self._check(self._L.swbl_create(_lib.ctypes.byref(handle)))
        self.handle = handle

    def _check(self, status: int) -> None:
        if status:
            raise RuntimeError(self._L.swbl_last_error().decode() or f"cuBLAS baseline status {status}")

    def gemv(self, w, x, y, algo: int = 0, stream: int | None = None) -> None:
        rows, cols = w.shape
        s = _stream(self.device) if stream is None else stream
        with torch.cuda.device(self.device):
            self._check(self._L.swbl_gemv(self.handle, algo, w.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, s))

    def ffn(self, x, wg, wu, wd, bg, bu, bd, g, u, h, y, algo: int = 0, stream: int | None = None) -> None:
        inter, hidden = wg.shape
        s = _stream(self.device) if stream is None else stream
        with torch.cuda.device(self.device):
            self._check(self._L.swbl_ffn(self.handle, algo, wg.data_ptr(), wu.data_ptr(), wd.data_ptr(),
                                         x.data_ptr(), bg.data_ptr(), bu.data_ptr(), bd.data_ptr(), g.data_ptr(),
                                         u.data_ptr(), h.data_ptr(), y.data_ptr(), hidden, inter, s))

    def version(self) -> int:
        out = _lib.ctypes.c_int()
        self._check(self._L.swbl_version(self.handle, _lib.ctypes.byref(out)))
        return out.value

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            with torch.cuda.device(self.device):
                self._L.swbl_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
