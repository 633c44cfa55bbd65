"""Shared expert (``n_shared_experts=1``): DeepSeek-V3's always-on expert fused
into the routed layer as one more dispatch bucket, against the oracle's
y = sum_k w_k E_k(x) + S(x).

The shared expert's weights are appended to the routed experts' tensors
([E_local + 1, ...]), as serving stacks that fuse it lay them out; every token
fills one more row of the permuted buffers with weight 1.
"""
import numpy as np
import pytest
import torch

import moe_oracle as mo
from gpu_helpers import oracle_output
from moe_b200 import _lib, api, workloads

pytestmark = pytest.mark.gpu


def add_shared_expert(inp, shape, seed):
    """The inputs with one more expert (same weight recipe) after the routed ones."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    h, i = shape.hidden, shape.inter
    w1 = (0.02 * torch.randn(1, 2 * i, h, generator=g, device="cuda")).to(torch.bfloat16)
    w2 = (0.02 * torch.randn(1, h, i, generator=g, device="cuda")).to(torch.bfloat16)
    q1, s1 = workloads.quantize_weight_blocks(w1)
    q2, s2 = workloads.quantize_weight_blocks(w2)
    out = dict(inp)
    out["gemm1_weights"] = torch.cat([inp["gemm1_weights"], q1])
    out["gemm1_weights_scale"] = torch.cat([inp["gemm1_weights_scale"], s1])
    out["gemm2_weights"] = torch.cat([inp["gemm2_weights"], q2])
    out["gemm2_weights_scale"] = torch.cat([inp["gemm2_weights_scale"], s2])
    return out


def forward(inp, shape, flags=0):
    out = torch.full((shape.t, shape.hidden), float("nan"), dtype=torch.bfloat16, device="cuda")
    args, keep, _ = api.build_args(*workloads.run_args(inp), out, shape.n_group,
                                   shape.topk_group, shape.top_k, n_shared_experts=1)
    args.flags = flags
    ws = api.forward_args(args, None, torch.device("cuda", 0))
    torch.cuda.synchronize()
    assert api.device_error(args) == (0, 0)
    return out, args, ws


@pytest.mark.parametrize("t", [1, 2, 3, 4, 17, 300])
@pytest.mark.parametrize("det", [False, True])
def test_shared_expert_tiny_matches_oracle(cuda_device, t, det):
    """T=1/2 fused bf16 output, T<=4 one-block routing, decode GEMMs at 17,
    prefill GEMMs at 300; atomic and fixed-order combine."""
    shape = workloads.tiny_shape(t)
    inp = add_shared_expert(workloads.make_inputs(shape, seed=1000 + t, device="cuda"), shape,
                            seed=1100 + t)
    out, args, ws = forward(inp, shape, _lib.MOE_FLAG_DETERMINISTIC if det else 0)
    ref = mo.moe_forward(mo.to_numpy_inputs({k: (v.cpu() if isinstance(v, torch.Tensor) else v)
                                             for k, v in inp.items()}),
                         shape.n_group, shape.topk_group, shape.top_k, n_shared=1)
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, ref, atol=1e-2, rtol=2e-2)
    assert mo.cosine(got, ref) >= 0.9999
    # the shared bucket holds every token in order, weight 1
    v = api.workspace_views(args, ws)
    el = shape.e_local
    assert int(v["counts"][el]) == t
    base = 128 * int(v["tile_start"][el])
    assert torch.equal(v["row_token"][base:base + t].cpu(), torch.arange(t, dtype=torch.int32))
    assert bool((v["row_weight"][base:base + t] == 1.0).all())
    # and the debug checker accepts the tables
    assert api.check_workspace(args) == (0, 0)


@pytest.mark.parametrize("t,e_local,offset", [(7, 32, 96), (901, 32, 224), (1, 256, 0),
                                              (600, 256, 0)])
def test_shared_expert_dsv3(cuda_device, t, e_local, offset):
    """DeepSeek-V3 layer with the shared expert: the contest's 32 local
    experts, and all 256 (257 dispatch buckets) on the decode and prefill
    paths; sampled tokens against the oracle."""
    shape = workloads.dsv3_shape(t, e_local=e_local, local_expert_offset=offset)
    inp = add_shared_expert(workloads.make_inputs(shape, seed=1200 + t, device="cuda"), shape,
                            seed=1300 + t)
    out, args, _ = forward(inp, shape)
    tokens = sorted({0, t // 3, t // 2, t - 1})
    ref = oracle_output(inp, shape, tokens=tokens, n_shared=1)
    got = out.float().cpu().numpy()[tokens]
    np.testing.assert_allclose(got, ref, atol=1e-2, rtol=2e-2)
    assert mo.cosine(got, ref) >= 0.9999
    assert api.check_workspace(args) == (0, 0)


def test_shared_expert_is_added_once(cuda_device):
    """With a shared expert whose weights are all zero the layer equals the
    routed layer bit for bit (fixed-order combine), so the extra bucket adds
    exactly its own rows."""
    shape = workloads.tiny_shape(57)
    base = workloads.make_inputs(shape, seed=1400, device="cuda")
    inp = add_shared_expert(base, shape, seed=1401)
    el = shape.e_local
    for k in ("gemm1_weights", "gemm2_weights"):
        inp[k] = inp[k].clone()
        inp[k][el].view(torch.uint8).zero_()
    out, _, _ = forward(inp, shape, _lib.MOE_FLAG_DETERMINISTIC)
    ref = torch.empty_like(out)
    api.run(*workloads.run_args(base), ref, n_group=shape.n_group, topk_group=shape.topk_group,
            top_k=shape.top_k, deterministic=True)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_shared_expert_rejects_prepared_w2(cuda_device):
    shape = workloads.tiny_shape(8)
    inp = add_shared_expert(workloads.make_inputs(shape, seed=1500, device="cuda"), shape, 1501)
    out = torch.empty(8, shape.hidden, dtype=torch.bfloat16, device="cuda")
    w2b = torch.zeros(shape.e_local, shape.hidden, shape.inter, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(AssertionError):
        api.run(*workloads.run_args(inp), out, n_group=shape.n_group, topk_group=shape.topk_group,
                top_k=shape.top_k, n_shared_experts=1, gemm2_weights_bf16=w2b)
