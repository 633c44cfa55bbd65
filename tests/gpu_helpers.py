"""Helpers shared by the GPU tests: run the CUDA path through the C ABI with an
explicit workspace, and run the CPU oracle on the same inputs."""
from __future__ import annotations

import numpy as np
import torch

import moe_oracle as mo
from moe_b200 import api


def run_cuda(inp: dict, shape, output=None, workspace=None):
    """One forward through ``moe_fp8_forward``; returns (output, stage views, args)."""
    dev = torch.device("cuda", 0)
    t, h = shape.t, shape.hidden
    if output is None:
        output = torch.full((t, h), float("nan"), dtype=torch.bfloat16, device=dev)
    args, keep, out_dev = api.build_args(
        inp["routing_logits"], inp["routing_bias"], inp["hidden_states"],
        inp["hidden_states_scale"], inp["gemm1_weights"], inp["gemm1_weights_scale"],
        inp["gemm2_weights"], inp["gemm2_weights_scale"], inp["local_expert_offset"],
        inp["routed_scaling_factor"], output, shape.n_group, shape.topk_group, shape.top_k)
    lay = api.workspace_layout(args)
    if workspace is None:
        workspace = torch.empty(lay.total_bytes, dtype=torch.uint8, device=dev)
    if t > 0:
        api.forward_args(args, workspace, dev)
    if out_dev is not output:
        output.copy_(out_dev)
    torch.cuda.synchronize()
    views = api.workspace_views(args, workspace) if t > 0 else None
    return output, views, args


def lazy_expert_getter(inp: dict):
    """Copy one expert's weights to the host only when the oracle needs it."""
    cache = {}

    def get(e):
        if e not in cache:
            cache[e] = (inp["gemm1_weights"][e].view(torch.uint8).cpu().numpy(),
                        inp["gemm1_weights_scale"][e].cpu().numpy(),
                        inp["gemm2_weights"][e].view(torch.uint8).cpu().numpy(),
                        inp["gemm2_weights_scale"][e].cpu().numpy())
        return cache[e]
    return get


def host_inputs(inp: dict, shape) -> dict:
    """Non-weight inputs as numpy (the oracle's form)."""
    out = {}
    for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale"):
        v = inp[k].detach().cpu()
        if v.dtype == torch.float8_e4m3fn:
            v = v.view(torch.uint8)
        elif v.dtype != torch.float32:
            v = v.float()
        out[k] = v.numpy()
    out["local_expert_offset"] = inp["local_expert_offset"]
    out["routed_scaling_factor"] = inp["routed_scaling_factor"]
    out["e_local"] = shape.e_local
    return out


def oracle_output(inp: dict, shape, tokens=None, requant=True, n_shared=0):
    hi = host_inputs(inp, shape)
    return mo.moe_forward(hi, shape.n_group, shape.topk_group, shape.top_k, requant=requant,
                          tokens=tokens, get_expert=lazy_expert_getter(inp), n_shared=n_shared)


def check_routing_and_dispatch(views, inp, shape):
    """Routing indices and the permutation must equal the oracle's bit for bit."""
    hi = host_inputs(inp, shape)
    idx, w = mo.route(hi["routing_logits"], hi["routing_bias"], shape.n_group, shape.topk_group,
                      shape.top_k, shape.routed_scaling_factor)
    got_idx = views["topk_idx"].cpu().numpy()
    mism = np.nonzero((got_idx != idx).any(axis=1))[0]
    assert len(mism) == 0, f"routing differs on tokens {mism[:8]}"
    np.testing.assert_allclose(views["topk_weights"].cpu().numpy(), w, rtol=2e-6, atol=0)
    counts, starts, tok, wt = mo.dispatch(idx, w, shape.local_expert_offset, shape.e_local)
    np.testing.assert_array_equal(views["counts"].cpu().numpy(), counts)
    tstart = views["tile_start"].cpu().numpy()
    tiles = (counts.astype(np.int64) + 127) // 128
    np.testing.assert_array_equal(tstart, np.concatenate([[0], np.cumsum(tiles)]))
    row_tok = views["row_token"].cpu().numpy()
    row_w = views["row_weight"].cpu().numpy()
    for e in range(shape.e_local):
        seg = slice(128 * tstart[e], 128 * tstart[e] + counts[e])
        np.testing.assert_array_equal(row_tok[seg], tok[starts[e]:starts[e + 1]])
        np.testing.assert_allclose(row_w[seg], wt[starts[e]:starts[e + 1]], rtol=2e-6, atol=0)
    return idx, w, counts, starts, tok


def bf16_np(x: torch.Tensor) -> np.ndarray:
    return x.float().cpu().numpy()
