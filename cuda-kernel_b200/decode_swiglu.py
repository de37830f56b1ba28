"""Drop-in module for callers of the reference's ``decode_swiglu`` torch extension.

The reference builds ``src/torch_extension.cu`` with
``torch.utils.cpp_extension.load(name="decode_swiglu", ...)`` and calls
``ext.swiglu_out``, ``ext.swiglu`` and ``ext.config_ids``. With
``cuda-kernel_b200/`` on ``sys.path``, ``import decode_swiglu as ext`` gives the
same three functions backed by the B200 kernels.
"""
from swiglu_b200.binding import config_ids, swiglu, swiglu_out

__all__ = ["swiglu_out", "swiglu", "config_ids"]
