"""Debug bounds checks (``MOE_FLAG_DEBUG``, ``moe_fp8_check_workspace``) and the
router on NaN inputs, on the GPU.

The corruption tests write wrong values into the tables that a finished forward
left in its workspace, then run only the checker on them.  The checker reads a
table entry as an index only after checking its range, so nothing reads or
writes outside the workspace; no forward runs on a corrupted table.

A check kernel reports the first failure it finds (the reporting is an atomic
compare-and-swap across threads), so where one corruption breaks two checks the
tests accept either report.
"""
import numpy as np
import pytest
import torch

import moe_oracle as mo
from gpu_helpers import oracle_output
from moe_b200 import _lib, api, workloads

pytestmark = pytest.mark.gpu

DEBUG, DET = _lib.MOE_FLAG_DEBUG, _lib.MOE_FLAG_DETERMINISTIC
BOUNDS = _lib.MOE_ERR_BOUNDS
SITE = {v: k for k, v in _lib.CHECK_SITES.items()}


def forward(inp, shape, flags=0, ws=None):
    out = torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16, device="cuda")
    args, keep, _ = api.build_args(*workloads.run_args(inp), out, shape.n_group,
                                   shape.topk_group, shape.top_k)
    args.flags = flags
    if ws is None:
        ws = torch.empty(api.workspace_layout(args).total_bytes, dtype=torch.uint8, device="cuda")
    api.forward_args(args, ws, torch.device("cuda", 0))
    torch.cuda.synchronize()
    return out, args, ws, keep


def decode(info):
    return (info >> 24) & 0xFF, info & 0xFFFFFF


def bf16_bits(x):
    return x.contiguous().view(torch.int16)


@pytest.mark.parametrize("t", [1, 2, 3, 4, 17, 300])
def test_debug_forward_is_clean_and_identical(cuda_device, t):
    shape = workloads.tiny_shape(t)
    inp = workloads.make_inputs(shape, seed=700 + t, device="cuda")
    ref, _, _, _ = forward(inp, shape, DET)
    out, args, ws, _ = forward(inp, shape, DET | DEBUG)
    assert api.device_error(args) == (0, 0)
    assert torch.equal(bf16_bits(out), bf16_bits(ref))
    # the standalone checker on the same workspace, guards included
    assert api.check_workspace(args) == (0, 0)
    # the atomic combine under debug: within one bf16 rounding of the fixed order
    out2, args2, _, _ = forward(inp, shape, DEBUG)
    assert api.device_error(args2) == (0, 0)
    torch.testing.assert_close(out2.float(), ref.float(), rtol=2 ** -7, atol=2 ** -14)


@pytest.mark.parametrize("t", [80, 901])
def test_debug_forward_contest_shape(cuda_device, t):
    """DeepSeek-V3 layer with 32 local experts: T=80 takes the decode GEMMs,
    T=901 the prefill GEMMs."""
    shape = workloads.dsv3_shape(t, e_local=32, local_expert_offset=96)
    inp = workloads.make_inputs(shape, seed=710 + t, device="cuda")
    ref, _, _, _ = forward(inp, shape, DET)
    out, args, _, _ = forward(inp, shape, DET | DEBUG)
    assert api.device_error(args) == (0, 0)
    assert torch.equal(bf16_bits(out), bf16_bits(ref))
    assert api.check_workspace(args) == (0, 0)


def _expect(args, allowed):
    code, info = api.check_workspace(args)
    assert code == BOUNDS, (code, info)
    assert decode(info) in allowed, (decode(info), allowed)


def test_checker_finds_each_corruption(cuda_device):
    shape = workloads.tiny_shape(300)
    k = shape.top_k
    inp = workloads.make_inputs(shape, seed=720, device="cuda")
    _, args, ws, _ = forward(inp, shape, DEBUG)
    assert api.check_workspace(args) == (0, 0)
    v = api.workspace_views(args, ws)
    lay = v["layout"]
    assign = v["assign_row"].cpu()

    # a live row's token out of range (both the row's and its assignment's checks see it)
    t0 = next(t for t in range(shape.t) if assign[t, 0] >= 0)
    r = int(assign[t0, 0])
    keep = v["row_token"][r].clone()
    v["row_token"][r] = shape.t + 5
    _expect(args, {(SITE["row_token"], r), (SITE["assign_row"], t0 * k)})
    v["row_token"][r] = keep

    # a routed expert id out of range
    t1 = next(t for t in range(7, shape.t) if assign[t, 1] >= 0)
    j = t1 * k + 1
    keep = v["topk_idx"][t1, 1].clone()
    v["topk_idx"][t1, 1] = shape.e_global + 3
    _expect(args, {(SITE["topk_idx"], j), (SITE["row_expert"], int(assign[t1, 1]))})
    v["topk_idx"][t1, 1] = keep

    # a repeated expert within one token
    keep = v["topk_idx"][t1, 2].clone()
    v["topk_idx"][t1, 2] = v["topk_idx"][t1, 1]
    allowed = {(SITE["topk_idx"], t1 * k + 2), (SITE["assign_row"], t1 * k + 2)}
    if assign[t1, 2] >= 0:
        allowed.add((SITE["row_expert"], int(assign[t1, 2])))
    _expect(args, allowed)
    v["topk_idx"][t1, 2] = keep

    # a negative count (its assignments then have no live row)
    counts = v["counts"].cpu()
    e = int(torch.nonzero(counts > 0)[0, 0])
    g = e + shape.local_expert_offset
    keep = v["counts"][e].clone()
    v["counts"][e] = -1
    idx = v["topk_idx"].cpu().flatten()
    allowed = {(SITE["counts"], e)} | {(SITE["assign_row"], int(jj))
                                       for jj in torch.nonzero(idx == g).flatten()}
    _expect(args, allowed)
    v["counts"][e] = keep

    # the tile prefix running past the row capacity
    el = shape.e_local
    keep = v["tile_start"][el].clone()
    v["tile_start"][el] = lay.npad // 128 + 1
    _expect(args, {(SITE["tile_start"], el)})
    v["tile_start"][el] = keep

    # a routing weight that is not finite (the rows' copies then differ too)
    keep = v["topk_weights"][t0, 0].clone()
    v["topk_weights"][t0, 0] = float("inf")
    _expect(args, {(SITE["topk_weights"], t0 * k), (SITE["row_weight"], r)})
    v["topk_weights"][t0, 0] = keep

    # an overwritten guard: the one after row_token (buffer number 6)
    g_off = (lay.row_token + 4 * lay.npad + 15) // 16 * 16
    keep = ws[g_off:g_off + 16].clone()
    ws[g_off + 3] ^= 0x5A
    _expect(args, {(SITE["guard"], 6)})
    ws[g_off:g_off + 16] = keep

    assert api.check_workspace(args) == (0, 0)


def test_nan_logits_route_distinct_experts_and_debug_stops_the_gemms(cuda_device):
    """NaN logits rank below every number: a token's experts stay distinct and
    in range (the permute relies on it), the other tokens are unaffected, and a
    debug forward reports the NaN routing weights before any GEMM runs."""
    shape = workloads.tiny_shape(40)
    k = shape.top_k
    inp = workloads.make_inputs(shape, seed=730, device="cuda")
    inp["routing_logits"][3] = float("nan")        # every score of token 3
    inp["routing_logits"][9, :5] = float("nan")    # experts 0-4 of token 9
    out, args, ws, _ = forward(inp, shape)
    v = api.workspace_views(args, ws)
    idx = v["topk_idx"].cpu()
    assert bool(((idx >= 0) & (idx < shape.e_global)).all())
    for t in range(shape.t):
        assert len(set(idx[t].tolist())) == k, (t, idx[t])
    # token 9 keeps away from its NaN experts; token 3 takes the lowest ids of
    # the lowest groups (all its scores rank equal)
    assert not set(idx[9].tolist()) & {0, 1, 2, 3, 4}
    assert sorted(idx[3].tolist()) == list(range(k))
    code, info = api.check_workspace(args)
    assert code == BOUNDS and decode(info) in {(SITE["topk_weights"], 3 * k + i) for i in range(k)}

    # every token without NaN inputs matches the oracle
    tokens = [t for t in range(shape.t) if t not in (3, 9)]
    ref = oracle_output(inp, shape, tokens=tokens)
    got = out.float().cpu().numpy()[tokens]
    np.testing.assert_allclose(got, ref, atol=1e-2, rtol=2e-2)

    # debug: the check fails before GEMM1, the GEMMs schedule no units, run() raises
    dev_out = torch.full((shape.t, shape.hidden), 7.0, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="topk_weights"):
        api.run(*workloads.run_args(inp), dev_out, n_group=shape.n_group,
                topk_group=shape.topk_group, top_k=shape.top_k, debug=True)
    assert dev_out.float().abs().max().item() == 0.0   # the zeroed accumulator, nothing added
