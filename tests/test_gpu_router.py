"""Router logits (``moe_router_logits_bf16``): bf16 x [T, H] . w_gate [E, H]^T in
fp32, against the exact float64 product of the same bf16 values.

Batches of at most 128 tokens (and shapes with E not a multiple of 256) take
the CUDA-core kernel, larger ones the tensor-core GEMM.  Both sum exact fp32
products in fp32.  The CUDA-core kernel rounds every addition to nearest and
sits within a few fp32 rounding steps of the float64 sum, as torch's own fp32
matmul does.  The tensor core's fp32 accumulator does not round each addition
to nearest (as in any bf16 tensor-core GEMM with an fp32 result); measured at
H=7168 its error is about 7e-6 of the largest logit, so its bound is 2e-5 of it.
"""
import pytest
import torch

import moe_oracle as mo
from moe_b200 import api, workloads

pytestmark = pytest.mark.gpu


def make(t, h, e, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(t, h, generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn(e, h, generator=g, device="cuda")).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("t,h,e", [
    (1, 7168, 256), (7, 7168, 256), (64, 7168, 256), (128, 7168, 256),   # CUDA cores
    (129, 7168, 256), (1000, 7168, 256), (4096, 7168, 256),             # tensor cores
    (13, 7168, 250),                                                     # ragged expert block
    (300, 512, 16), (2048, 512, 16),                                     # E % 256 != 0
    (2048, 512, 512),                                                    # two N tiles
])
def test_router_logits_match_the_exact_product(cuda_device, t, h, e):
    x, w = make(t, h, e, seed=900 + t + e)
    got = api.router_logits(x, w)
    torch.cuda.synchronize()
    exact = x.double() @ w.double().T
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        torch_f32 = x.float() @ w.float().T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    err = (got.double() - exact).abs().max().item()
    err_torch = (torch_f32.double() - exact).abs().max().item()
    scale = exact.abs().max().item()
    tensor_cores = t > 128 and e % 256 == 0 and h % 64 == 0
    bound = 2e-5 * scale if tensor_cores else max(4 * err_torch, 2e-6 * scale)
    assert err <= bound, (err, err_torch, scale)
    # fixed summation order: the same bits on a second run
    again = api.router_logits(x, w)
    assert torch.equal(again, got)


def test_router_logits_feed_the_layer(cuda_device):
    """The logits drive run(): the layer routes them exactly as the oracle
    routes the same fp32 values."""
    shape = workloads.tiny_shape(700)
    inp = workloads.make_inputs(shape, seed=950, device="cuda")
    x, w = make(shape.t, shape.hidden, shape.e_global, seed=951)
    logits = api.router_logits(x, w)
    inp["routing_logits"] = logits
    out = torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16, device="cuda")
    args, keep, _ = api.build_args(*workloads.run_args(inp), out, shape.n_group,
                                   shape.topk_group, shape.top_k)
    ws = api.forward_args(args, None, torch.device("cuda", 0))
    torch.cuda.synchronize()
    assert api.device_error(args) == (0, 0)
    idx = api.workspace_views(args, ws)["topk_idx"]
    ref_idx, _ = mo.route(logits.cpu().numpy(), inp["routing_bias"].cpu().numpy(), shape.n_group,
                          shape.topk_group, shape.top_k, shape.routed_scaling_factor)
    assert (idx.cpu().numpy() == ref_idx).all()
