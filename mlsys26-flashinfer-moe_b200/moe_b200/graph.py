"""CUDA-graph capture of one MoE layer forward, for decode-sized batches.

A forward is one memset and five kernel launches with no host synchronisation
(``moe_fp8_forward``).  At decode sizes the launch gaps between them are a
sizeable share of the step, so ``LayerGraph`` captures the whole forward once
for a fixed set of device buffers and ``replay()`` re-issues it as one graph
launch.  This is the reference's ``run()`` (``kernel.py:562``) frozen to one set
of tensors: a graph bakes in every device address, so per-step inputs are
written into the captured tensors (``copy_``) rather than passed anew.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import api

_STEP_INPUTS = ("routing_logits", "hidden_states", "hidden_states_scale")


class LayerGraph:
    """Captured forward over caller-owned CUDA tensors.

    All tensors must already be contiguous CUDA tensors of the reference's
    dtypes on one device (no implicit copies are allowed, since a copy made at
    capture time would never see later updates).  They stay borrowed for the
    graph's lifetime.  ``replay()`` runs on ``stream`` (default: the current
    stream at replay time) and writes ``output``.  ``deterministic`` and
    ``n_shared_experts`` are those of ``run()``.
    """

    def __init__(self, routing_logits: torch.Tensor, routing_bias: torch.Tensor,
                 hidden_states: torch.Tensor, hidden_states_scale: torch.Tensor,
                 gemm1_weights: torch.Tensor, gemm1_weights_scale: torch.Tensor,
                 gemm2_weights: torch.Tensor, gemm2_weights_scale: torch.Tensor,
                 local_expert_offset: int, routed_scaling_factor: float, output: torch.Tensor,
                 *, n_group: int = 8, topk_group: int = 4, top_k: int = 8,
                 deterministic: bool = False, n_shared_experts: int = 0):
        given = dict(routing_logits=routing_logits, routing_bias=routing_bias,
                     hidden_states=hidden_states, hidden_states_scale=hidden_states_scale,
                     gemm1_weights=gemm1_weights, gemm1_weights_scale=gemm1_weights_scale,
                     gemm2_weights=gemm2_weights, gemm2_weights_scale=gemm2_weights_scale)
        args, keep, out_dev = api.build_args(*given.values(), local_expert_offset,
                                             routed_scaling_factor, output, n_group, topk_group,
                                             top_k, deterministic=deterministic,
                                             n_shared_experts=n_shared_experts)
        for (name, t), k in zip(given.items(), keep):
            if k.data_ptr() != t.data_ptr():
                raise ValueError(f"{name} must be a contiguous tensor on the output's CUDA device")
        if out_dev is not output:
            raise ValueError("output must be a contiguous bf16 CUDA tensor")
        if args.T == 0:
            raise ValueError("a graph of an empty batch has nothing to run")
        self.args, self._keep, self.output = args, keep, output
        self.inputs = given
        self.device = output.device
        lay = api.workspace_layout(args)
        self.workspace = torch.empty(lay.total_bytes, dtype=torch.uint8, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            # Warm-up outside capture: per-device kernel attributes and the
            # tensor-map cache are set up on the first call.
            api.forward_args(args, self.workspace, self.device)
        side.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            api.forward_args(args, self.workspace, self.device)
        torch.cuda.current_stream(self.device).wait_stream(side)

    def set_inputs(self, routing_logits: Optional[torch.Tensor] = None,
                   hidden_states: Optional[torch.Tensor] = None,
                   hidden_states_scale: Optional[torch.Tensor] = None) -> None:
        """Copy a new step's inputs into the captured tensors (same shapes)."""
        for name, t in zip(_STEP_INPUTS, (routing_logits, hidden_states, hidden_states_scale)):
            if t is not None:
                self.inputs[name].copy_(t, non_blocking=True)

    def replay(self) -> torch.Tensor:
        """Run the captured forward; returns ``output``."""
        self.graph.replay()
        return self.output
