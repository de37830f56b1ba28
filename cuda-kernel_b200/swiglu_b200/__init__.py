"""B200-native batch-one SwiGLU decode layer (sm_100a).

Host-side mirror of shubhxho/cuda-kernel's operator surface over the C ABI of
``libswiglu_b200.so``:

* ``swiglu_out`` / ``swiglu`` / ``config_ids`` -- the torch binding
  (``src/torch_extension.cu``), same names, checks and errors;
* ``gate`` / ``project`` / ``ffn`` -- the kernel launches of
  ``decode::launch`` (``include/kernels.cuh:115-133``);
* ``CublasBaseline`` -- the cuBLAS GemmEx + pointwise comparison path.

Importing this package does not need a GPU; calling a kernel does.
"""
from .binding import (CublasBaseline, config_ids, config_info, device_error, ffn, ffn_fused, ffn_tp, gate,
                      layer_config_ids, layer_workspace, project,
                      residual_epilogue, swiglu, swiglu_out, valid_config)
from ._lib import build, lib

__all__ = ["swiglu_out", "swiglu", "config_ids", "config_info", "valid_config", "gate", "project", "ffn", "ffn_fused", "ffn_tp",
           "layer_config_ids", "layer_workspace",
           "residual_epilogue", "device_error", "CublasBaseline", "build", "lib"]
