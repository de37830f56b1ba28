"""Tensor-parallel layer: one process per GPU, fused all-reduce over peer memory.

Rank r of n holds rows [r*I/n, (r+1)*I/n) of Wg and Wu and the same columns of Wd
(stored contiguously). ``Exchange`` sets up the rank's exchange buffer once:
it allocates it (C ABI ``swb_tp_create``), shares its CUDA IPC handle with every
rank through ``torch.distributed`` and maps the peers' buffers
(``swb_tp_connect``). ``ffn_tp_fused`` then runs a rank's layer as two kernels:
the gate on the shard, and the down projection whose epilogue stores its partial
rows into every rank's buffer over NVLink (each value with the call's epoch in one
64-bit word), waits until the peers' words carry the epoch and writes
y = sum of partials + bias + residual (identical on every rank); or, with a
fused-layer id, the whole rank's layer in one kernel. ``shard`` cuts
the weights for a rank. The NCCL alternative (``swb_ffn_tp`` + all-reduce +
``swb_residual_epilogue``) stays available as the baseline.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def shard(wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor, bg, bu, rank: int, world: int) -> dict:
    """Rank `rank`'s contiguous shards of the layer's weights (and gate biases)."""
    inter = wg.shape[0]
    if inter % world:
        raise ValueError("intermediate size must divide by the rank count")
    a, b = rank * inter // world, (rank + 1) * inter // world
    out = {"wg": wg[a:b].contiguous(), "wu": wu[a:b].contiguous(), "wd": wd[:, a:b].contiguous()}
    out["bg"] = None if bg is None else bg[a:b].contiguous()
    out["bu"] = None if bu is None else bu[a:b].contiguous()
    return out


def share_handles(mine: bytes, world: int, group=None) -> list[bytes]:
    """Every rank's exchange IPC handle, in rank order (one all_gather over the process group).

    A rank that never joins makes the others' call fail with the process group's timeout
    instead of hanging; a malformed handle from any rank raises ValueError on every rank
    (all of them see the same gathered list)."""
    import torch.distributed as dist
    if len(mine) != _lib.SWB_TP_HANDLE_BYTES:
        raise ValueError(f"exchange handle must be {_lib.SWB_TP_HANDLE_BYTES} bytes, got {len(mine)}")
    if world == 1:
        return [bytes(mine)]
    gathered = [None] * world
    dist.all_gather_object(gathered, bytes(mine), group=group)
    bad = [r for r, h in enumerate(gathered) if not isinstance(h, bytes) or len(h) != _lib.SWB_TP_HANDLE_BYTES]
    if bad:
        raise ValueError(f"malformed exchange handle from rank(s) {bad}")
    return gathered


class Exchange:
    """This rank's fused-all-reduce exchange buffer, mapped into every rank."""

    def __init__(self, rank: int, world: int, rows: int, device: torch.device, group=None):
        self.rank, self.world, self.rows, self.device = rank, world, rows, device
        L = _lib.lib()
        self._ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(L.swb_tp_create(rank, world, rows, ctypes.byref(self._ptr)))
            mine = (ctypes.c_uint8 * _lib.SWB_TP_HANDLE_BYTES)()
            _lib.check(L.swb_tp_ipc_handle(self._ptr, mine))
            gathered = share_handles(bytes(mine), world, group)
            table = (ctypes.c_uint8 * (_lib.SWB_TP_HANDLE_BYTES * world)).from_buffer_copy(b"".join(gathered))
            _lib.check(L.swb_tp_connect(self._ptr, table))

    @property
    def handle(self):
        return self._ptr

    def epoch(self) -> int:
        """Calls this rank's exchange has counted (synchronises the device)."""
        out = ctypes.c_uint32()
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().swb_tp_epoch(self._ptr, ctypes.byref(out)))
        return out.value

    def close(self) -> None:
        if self._ptr is not None and self._ptr.value:
            with torch.cuda.device(self.device):
                _lib.lib().swb_tp_destroy(self._ptr)
            self._ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ffn_tp_fused(ex: Exchange, x: torch.Tensor, s: dict, bd: torch.Tensor | None, h: torch.Tensor,
                 y: torch.Tensor, gate_config: int, down_config: int, stream: int | None = None,
                 prefetch_weights: bool = False) -> None:
    """One rank's layer with the fused all-reduce; y (fp32 [hidden]) ends identical on every rank.

    ``prefetch_weights``: SWB_PREFETCH_WEIGHTS (see binding.ffn)."""
    shard_rows, hidden = s["wg"].shape
    sp = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    flags = _lib.SWB_PREFETCH_WEIGHTS if prefetch_weights else 0
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_ffn_tp_fused_ex(ex.handle, int(gate_config), int(down_config),
                                                  s["wg"].data_ptr(), s["wu"].data_ptr(), s["wd"].data_ptr(),
                                                  x.data_ptr(), ptr(s["bg"]), ptr(s["bu"]), ptr(bd), h.data_ptr(),
                                                  y.data_ptr(), hidden, shard_rows, flags, sp))


def ffn_tp_host(ex: Exchange, x_host: torch.Tensor, s: dict, bd: torch.Tensor | None, x: torch.Tensor,
                h: torch.Tensor, y: torch.Tensor, y_host: torch.Tensor, gate_config: int, down_config: int,
                stream: int | None = None, prefetch_weights: bool = False) -> None:
    """ffn_tp_fused from pinned host ``x_host`` (fp16 [hidden], the same on every rank) to pinned
    host ``y_host`` (fp32 [hidden], the reduced y, the same on every rank) (swb_ffn_tp_host_ex):
    x in, the rank's gate and fused down + exchange, y out as one programmatic chain. ``x``,
    ``h`` and ``y`` are device buffers the call overwrites."""
    shard_rows, hidden = s["wg"].shape
    if not (x_host.is_pinned() and y_host.is_pinned()):
        raise RuntimeError("x_host and y_host must be pinned (page-locked) host tensors")
    sp = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    flags = _lib.SWB_PREFETCH_WEIGHTS if prefetch_weights else 0
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_ffn_tp_host_ex(ex.handle, int(gate_config), int(down_config), s["wg"].data_ptr(),
                                                 s["wu"].data_ptr(), s["wd"].data_ptr(), x_host.data_ptr(),
                                                 ptr(s["bg"]), ptr(s["bu"]), ptr(bd), x.data_ptr(), h.data_ptr(),
                                                 y.data_ptr(), y_host.data_ptr(), hidden, shard_rows, flags, sp))


def swiglu_tp_out(ex: Exchange, x: torch.Tensor, s: dict, h: torch.Tensor, y: torch.Tensor, gate_config: int,
                  down_config: int, stream: int | None = None, prefetch_weights: bool = False) -> None:
    """``swiglu_out`` for one tensor-parallel rank (the model path): eager-fp16 rounding in the
    gate on the rank's shard, the fused down projection + exchange, y = fp16 of the ranks' summed
    partials (no bias, no residual), identical on every rank. x, y: [..., hidden] fp16; h: [shard]."""
    shard_rows, hidden = s["wg"].shape
    sp = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
    flags = _lib.SWB_PREFETCH_WEIGHTS if prefetch_weights else 0
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().swb_swiglu_tp_out(ex.handle, x.data_ptr(), s["wg"].data_ptr(), s["wu"].data_ptr(),
                                                s["wd"].data_ptr(), h.data_ptr(), y.data_ptr(), hidden, shard_rows,
                                                int(gate_config), int(down_config), flags, sp))
