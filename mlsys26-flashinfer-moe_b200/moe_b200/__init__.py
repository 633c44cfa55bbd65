"""B200-native (sm_100a) fused FP8 block-scale DeepSeek-V3 MoE forward.

``moe_b200.run`` is a drop-in for ``run()`` of nikhilnd/mlsys26-flashinfer-moe
(``kernel.py:562``); the kernels live in ``libmoe_b200.so`` (C ABI in
``include/moe_b200.h``).
"""
from .api import (run, build_args, forward_args, workspace_views, device_error,  # noqa: F401
                  quantize_1x128, prepare_gemm2_weights, check_workspace, describe_error,
                  raise_device_error, router_logits)
from .graph import LayerGraph  # noqa: F401
from . import workloads  # noqa: F401

__all__ = ["run", "build_args", "forward_args", "workspace_views", "device_error", "quantize_1x128",
           "prepare_gemm2_weights", "check_workspace", "describe_error", "raise_device_error",
           "router_logits", "LayerGraph", "workloads"]
