"""Parity of the sm_100a path (through the C ABI) with the reference and the oracle.

Bars:
* routing indices and the expert permutation: bit-exact;
* routing weights: within 2e-6 relative (fp32, same operation order);
* bf16 output: ``allclose(atol=1e-2, rtol=2e-2)`` and cosine >= 0.9999
  against the dequantised fp32 math of the reference algorithm, which includes
  its FP8 re-quantisation of the SwiGLU output at 1x64 granularity
  (kernel.py:131-135);
* against the fp32 math *without* that re-quantisation, the output must be no
  less accurate than the reference algorithm itself: at DeepSeek-V3
  magnitudes (outputs ~1) the FP8 intermediate alone moves outputs by up to
  ~0.08, beyond atol 1e-2, so the bar is the requantising oracle's own error.
"""
import ast
import os

import numpy as np
import pytest
import torch

import cases
import moe_oracle as mo
from gpu_helpers import (bf16_np, check_routing_and_dispatch, oracle_output, run_cuda)
from moe_b200 import workloads

pytestmark = pytest.mark.gpu

ATOL, RTOL, COS = 1e-2, 2e-2, 0.9999


def assert_as_accurate_as_reference(got, ref_requant, ref_fp32):
    """Error vs the un-requantised fp32 math no larger than the reference
    algorithm's (within 10% in norm, 25% in max)."""
    e_ours = got.astype(np.float64) - ref_fp32
    e_ref = ref_requant.astype(np.float64) - ref_fp32
    assert np.linalg.norm(e_ours) <= 1.1 * np.linalg.norm(e_ref) + 1e-3
    assert np.abs(e_ours).max() <= 1.25 * np.abs(e_ref).max() + 1e-2


def to_cuda(inp):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}


# ---------------------------------------------------------------- golden fixtures

@pytest.mark.parametrize("name", list(cases.CASES))
def test_golden_case(cuda_device, name):
    g = np.load(f"{cases.HERE}/{name}.npz")
    inp, shape, _ = cases.case_inputs(name)
    meta = ast.literal_eval(str(g["meta"]))
    assert workloads.tensor_digest(inp) == meta["digest"]
    out, views, _ = run_cuda(to_cuda(inp), shape)
    np.testing.assert_array_equal(views["topk_idx"].cpu().numpy(), g["topk_idx"])
    np.testing.assert_allclose(views["topk_weights"].cpu().numpy(), g["topk_weights"], rtol=2e-6)
    np.testing.assert_array_equal(views["counts"].cpu().numpy(), g["counts"])
    tstart = views["tile_start"].cpu().numpy()
    row_tok = views["row_token"].cpu().numpy()
    st = g["starts"]
    for e in range(shape.e_local):
        ours = row_tok[128 * tstart[e]: 128 * tstart[e] + g["counts"][e]]
        np.testing.assert_array_equal(ours, np.sort(g["sorted_tokens"][st[e]:st[e + 1]]))
    ref = mo.bf16_to_f32(g["output_bf16"])
    got = bf16_np(out)
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)
    assert mo.cosine(got, g["out_f32"]) >= COS


@pytest.mark.parametrize("name", ["tiny_t16_seed0", "tiny_t300_seed4"])
def test_golden_intermediate(cuda_device, name):
    """FP8 SwiGLU output and its 1x64 scales vs the reference kernel's, per row."""
    g = np.load(f"{cases.HERE}/{name}.npz")
    inp, shape, _ = cases.case_inputs(name)
    out, views, _ = run_cuda(to_cuda(inp), shape)
    tstart = views["tile_start"].cpu().numpy()
    inter = views["inter"].cpu().numpy()
    isc = views["inter_scale"].cpu().numpy()
    st = g["starts"]
    for e in range(shape.e_local):
        a, b = st[e], st[e + 1]
        if a == b:
            continue
        order = np.argsort(g["sorted_tokens"][a:b], kind="stable")
        ref_codes = g["gemm1_out"][a:b][order]
        ref_sc = g["gemm1_scale"][:, a:b][:, order]
        r0 = 128 * tstart[e]
        np.testing.assert_allclose(isc[:, r0:r0 + (b - a)], ref_sc, rtol=1e-5)
        assert np.mean(inter[r0:r0 + (b - a)] == ref_codes) > 0.999


# ---------------------------------------------------------------- DeepSeek-V3 shapes

def dsv3_inputs(t, seed, **kw):
    shape = workloads.dsv3_shape(t, **{k: v for k, v in kw.items() if k != "zipf"})
    inp = workloads.make_inputs(shape, seed=seed, device="cuda", zipf=kw.get("zipf"))
    return inp, shape


@pytest.mark.parametrize("t,offset", [(1, 0), (2, 128), (4, 64), (7, 96), (80, 224), (901, 32)])
def test_contest_shape_32_local_experts(cuda_device, t, offset):
    """The FlashInfer-Bench definition: 32 local experts of 256 (kernel.py:581).
    T <= 2 exercises the GEMM2 that writes the bf16 output itself, T <= 4 the
    one-launch route/pack, T=7, 80 and 901 the separate route and permute
    kernels."""
    inp, shape = dsv3_inputs(t, seed=10 + t, e_local=32, local_expert_offset=offset)
    out, views, _ = run_cuda(inp, shape)
    check_routing_and_dispatch(views, inp, shape)
    toks = np.arange(t) if t <= 80 else np.random.default_rng(t).choice(t, 48, replace=False)
    ref = oracle_output(inp, shape, tokens=toks)
    got = bf16_np(out)[toks]
    assert mo.cosine(got, ref) >= COS
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)
    ref32 = oracle_output(inp, shape, tokens=toks, requant=False)
    assert_as_accurate_as_reference(got, ref, ref32)


@pytest.mark.parametrize("t", [1, 8, 64])
def test_decode_all_256_experts(cuda_device, t):
    inp, shape = dsv3_inputs(t, seed=100 + t)
    out, views, _ = run_cuda(inp, shape)
    check_routing_and_dispatch(views, inp, shape)
    toks = np.arange(t) if t <= 8 else np.random.default_rng(t).choice(t, 12, replace=False)
    ref = oracle_output(inp, shape, tokens=toks)
    got = bf16_np(out)[toks]
    assert mo.cosine(got, ref) >= COS
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("t,zipf", [(2048, None), (4096, 1.2)])
def test_prefill_routing_permutation_and_sampled_output(cuda_device, t, zipf):
    """Full-size routing and permutation are checked bit-exactly for every
    token; the output is checked on sampled tokens (each token's output depends
    only on its own routing)."""
    inp, shape = dsv3_inputs(t, seed=7, zipf=zipf)
    out, views, _ = run_cuda(inp, shape)
    idx, w, counts, starts, tok = check_routing_and_dispatch(views, inp, shape)
    if zipf is not None:
        assert counts.max() > 5 * counts.mean() and (counts == 0).any()
    toks = np.random.default_rng(1).choice(t, 6, replace=False)
    ref = oracle_output(inp, shape, tokens=toks)
    got = bf16_np(out)[toks]
    assert mo.cosine(got, ref) >= COS
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)
    assert np.isfinite(bf16_np(out)).all()


@pytest.mark.parametrize("t,e_local,zipf", [(100, 256, 1.2), (60, 256, 2.0)])
def test_decode_path_skewed_routing(cuda_device, t, e_local, zipf):
    """Decode-sized batches take the swapped-operand kernels (rows per expert on
    average <= 4); skewed routing gives some experts several 16-row token tiles."""
    inp, shape = dsv3_inputs(t, seed=21 + t, e_local=e_local, zipf=zipf)
    out, views, _ = run_cuda(inp, shape)
    _, _, counts, _, _ = check_routing_and_dispatch(views, inp, shape)
    assert counts.max() > 16
    toks = np.random.default_rng(t).choice(t, 10, replace=False)
    ref = oracle_output(inp, shape, tokens=toks)
    got = bf16_np(out)[toks]
    assert mo.cosine(got, ref) >= COS
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("t", [1, 8])
def test_layer_graph_replay(cuda_device, t):
    """A captured forward equals the eager one, also after new step inputs are
    copied into the captured tensors."""
    from moe_b200 import LayerGraph, run
    inp, shape = dsv3_inputs(t, seed=40 + t, e_local=32)
    out_g = torch.empty(t, shape.hidden, dtype=torch.bfloat16, device="cuda")
    graph = LayerGraph(*workloads.run_args(inp), out_g, n_group=8, topk_group=4, top_k=8)
    for step in range(2):
        nxt = workloads.make_inputs(shape, seed=80 + 10 * step + t, device="cuda", weights=False)
        graph.set_inputs(nxt["routing_logits"], nxt["hidden_states"], nxt["hidden_states_scale"])
        graph.replay()
        eager_args = workloads.run_args(inp)
        eager_args[0], eager_args[2], eager_args[3] = (nxt["routing_logits"], nxt["hidden_states"],
                                                       nxt["hidden_states_scale"])
        out_e = torch.empty_like(out_g)
        run(*eager_args, out_e)
        torch.cuda.synchronize()
        assert (out_g.float() - out_e.float()).abs().max().item() <= 2e-3


@pytest.mark.parametrize("t", [5, 700])
def test_odd_layer_shape(cuda_device, t):
    """H=1024, I=384 (three 128-feature tiles, odd), 64 experts in 8 groups of 8,
    top-2 groups / top-6: both GEMM paths (t=5 decode-sized, t=700 prefill) against
    the oracle."""
    shape = workloads.MoeShape(t=t, hidden=1024, inter=384, e_global=64, e_local=64, n_group=8,
                               topk_group=2, top_k=6)
    inp = workloads.make_inputs(shape, seed=300 + t, device="cuda")
    out, views, _ = run_cuda(inp, shape)
    check_routing_and_dispatch(views, inp, shape)
    toks = np.arange(t) if t <= 16 else np.random.default_rng(t).choice(t, 24, replace=False)
    ref = oracle_output(inp, shape, tokens=toks)
    got = bf16_np(out)[toks]
    assert mo.cosine(got, ref) >= COS
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)


def test_zero_tokens_is_a_noop(cuda_device):
    inp, shape = dsv3_inputs(0, seed=1, e_local=32)
    out, _, _ = run_cuda(inp, shape)
    assert out.shape == (0, 7168)


def test_bias_dtypes_and_cpu_inputs(cuda_device):
    """run() accepts bf16/fp16 bias and CPU tensors (kernel.py:544-549, 595, 616)."""
    from moe_b200 import run
    shape = workloads.tiny_shape(33)
    inp = workloads.make_inputs(shape, seed=5, device="cpu")
    outs = []
    for dt in (torch.float32, torch.bfloat16, torch.float16):
        args = workloads.run_args(inp)
        args[1] = inp["routing_bias"].to(dt)
        o = torch.empty(33, shape.hidden, dtype=torch.bfloat16)          # CPU output
        run(*args, o, n_group=shape.n_group, topk_group=shape.topk_group, top_k=shape.top_k)
        outs.append(o)
        ni = mo.to_numpy_inputs(inp)
        ni["routing_bias"] = args[1].float().numpy()
        ref = mo.moe_forward(ni, shape.n_group, shape.topk_group, shape.top_k)
        np.testing.assert_allclose(o.float().numpy(), ref, atol=ATOL, rtol=RTOL)


def test_repeated_calls_and_error_word(cuda_device):
    from moe_b200 import api
    inp, shape = dsv3_inputs(256, seed=3, e_local=64, local_expert_offset=64)
    o1, v1, args = run_cuda(inp, shape)
    ws = torch.empty(api.workspace_layout(args).total_bytes, dtype=torch.uint8, device="cuda")
    o2, v2, args2 = run_cuda(inp, shape, workspace=ws)
    o3, v3, _ = run_cuda(inp, shape, workspace=ws)
    assert torch.equal(v2["topk_idx"], v3["topk_idx"])
    assert torch.equal(v2["row_token"][:v2["counts"].sum()], v3["row_token"][:v3["counts"].sum()])
    # fp32 atomics make the summation order vary; bf16 results agree closely
    assert (o2.float() - o3.float()).abs().max().item() <= 2e-3
    assert api.device_error(args2) == (0, 0)


def test_tokens_routed_elsewhere_get_zeros(cuda_device):
    """An expert-parallel shard only adds its own experts' contributions."""
    inp, shape = dsv3_inputs(64, seed=9, e_local=32, local_expert_offset=0)
    out, views, _ = run_cuda(inp, shape)
    idx = views["topk_idx"].cpu().numpy()
    none_local = ~((idx >= 0) & (idx < 32)).any(axis=1)
    assert none_local.any()
    assert (bf16_np(out)[none_local] == 0).all()


@pytest.mark.parametrize("t,e_local", [(2, 32), (8, 256), (300, 32), (901, 32)])
def test_deterministic_combine_is_bit_identical(cuda_device, t, e_local):
    """MOE_FLAG_DETERMINISTIC: three runs give the same bits, and the result
    agrees with the default (fp32 atomics) path and the oracle.  T=2 and 8 take
    the decode GEMMs (no split units, no fused bf16 output), 300 and 901 the
    prefill GEMMs."""
    from moe_b200 import run
    inp, shape = dsv3_inputs(t, seed=700 + t, e_local=e_local, local_expert_offset=0)
    outs = []
    for _ in range(3):
        o = torch.empty(t, shape.hidden, dtype=torch.bfloat16, device="cuda")
        run(*workloads.run_args(inp), o, deterministic=True)
        outs.append(o)
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    o_def = torch.empty_like(outs[0])
    run(*workloads.run_args(inp), o_def)
    torch.cuda.synchronize()
    # the two paths add the same fp32 terms in different orders: at most one
    # bf16 rounding step apart (2^-7 relative)
    torch.testing.assert_close(o_def.float(), outs[0].float(), rtol=2.0 ** -7, atol=1e-4)
    toks = np.arange(t) if t <= 8 else np.random.default_rng(t).choice(t, 8, replace=False)
    ref = oracle_output(inp, shape, tokens=toks)
    got = bf16_np(outs[0])[toks]
    assert mo.cosine(got, ref) >= COS
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)


# ---------------------------------------------------------------- contest-shape fixtures

CONTEST_FIXTURES = [n for n in cases.CONTEST_CASES if os.path.exists(f"{cases.HERE}/{n}.npz")]


@pytest.mark.parametrize("name", CONTEST_FIXTURES)
def test_contest_fixture_from_reference_kernels(cuda_device, name):
    """DeepSeek-V3 contest shape (H=7168, I=2048, experts 0..31 of 256) against
    the reference's own kernels (Triton interpreter, tests/golden/make_golden.py
    --contest): routing and the per-expert token lists bit-exact, the sampled
    FP8 intermediate rows and scales, and the sampled output tokens within the
    tests' tolerance."""
    g = np.load(f"{cases.HERE}/{name}.npz")
    meta = ast.literal_eval(str(g["meta"]))
    inp, shape, _ = cases.contest_case_inputs(name)
    assert workloads.tensor_digest(inp) == meta["digest"]
    out, views, _ = run_cuda(to_cuda(inp), shape)
    np.testing.assert_array_equal(views["topk_idx"].cpu().numpy(), g["topk_idx"])
    np.testing.assert_allclose(views["topk_weights"].cpu().numpy(), g["topk_weights"], rtol=2e-6)
    np.testing.assert_array_equal(views["counts"].cpu().numpy(), g["counts"])
    tstart = views["tile_start"].cpu().numpy()
    row_tok = views["row_token"].cpu().numpy()
    st, stok = g["starts"], g["sorted_tokens"]
    for e in range(shape.e_local):
        ours = row_tok[128 * tstart[e]: 128 * tstart[e] + g["counts"][e]]
        np.testing.assert_array_equal(ours, np.sort(stok[st[e]:st[e + 1]]))
    # sampled intermediate rows: fixture row p (bucket position in the
    # reference's order) -> our row of the same (expert, token)
    inter = views["inter"].cpu().numpy()
    isc = views["inter_scale"].cpu().numpy()
    same = total = 0
    for j, p in enumerate(g["inter_rows"]):
        e = int(np.searchsorted(st, p, side="right") - 1)
        tok = stok[p]
        ours_row = 128 * tstart[e] + int(np.searchsorted(np.sort(stok[st[e]:st[e + 1]]), tok))
        np.testing.assert_allclose(isc[:, ours_row], g["gemm1_scale"][:, j], rtol=1e-5)
        same += int((inter[ours_row] == g["gemm1_out"][j]).sum())
        total += inter.shape[1]
    assert total == 0 or same / total > 0.999
    toks = g["sample_tokens"]
    got = bf16_np(out)[toks]
    ref = mo.bf16_to_f32(g["output_bf16"])
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)
    assert mo.cosine(got, ref) >= COS


def torch_fp32_layer(inp, shape, topk_idx, topk_w):
    """The layer in fp32 PyTorch on the GPU for every token, given the routing:
    dequantised operands, fp32 GEMMs (TF32 off), SwiGLU, the reference's 1x64
    FP8 requant of the intermediate (kernel.py:128-135, torch's RNE cast) and
    the routing-weighted sum (kernel.py:236-250)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    t, h, i = shape.t, shape.hidden, shape.inter
    a = inp["hidden_states"].float().view(t, h // 128, 128) * \
        inp["hidden_states_scale"].t().reshape(t, h // 128, 1)
    a = a.view(t, h)
    out = torch.zeros(t, h, dtype=torch.float32, device="cuda")
    loc = topk_idx.long() - shape.local_expert_offset
    for e in range(shape.e_local):
        sel = (loc == e).nonzero()
        if sel.numel() == 0:
            continue
        tok, kk = sel[:, 0], sel[:, 1]
        w1 = inp["gemm1_weights"][e].float().view(2 * i // 128, 128, h // 128, 128) * \
            inp["gemm1_weights_scale"][e].view(2 * i // 128, 1, h // 128, 1)
        g = a[tok] @ w1.view(2 * i, h).t()
        c = torch.nn.functional.silu(g[:, i:]) * g[:, :i]
        cb = c.view(-1, i // 64, 64)
        sc = torch.clamp(cb.abs().amax(dim=2, keepdim=True) / 448.0, min=1e-12)
        cq = (cb / sc).to(torch.float8_e4m3fn).float() * sc
        w2 = inp["gemm2_weights"][e].float().view(h // 128, 128, i // 128, 128) * \
            inp["gemm2_weights_scale"][e].view(h // 128, 1, i // 128, 1)
        d = cq.view(-1, i) @ w2.view(h, i).t()
        out.index_add_(0, tok, d * topk_w[tok, kk].unsqueeze(1))
    return out


def test_prefill_full_output_against_torch_fp32(cuda_device):
    """Every output element of a T=2048, 256-expert prefill (all 56 K blocks of
    GEMM1, the persistent multi-wave schedule) against the fp32 PyTorch layer;
    that reference is itself checked against the numpy oracle on sampled
    tokens."""
    inp, shape = dsv3_inputs(2048, seed=17)
    out, views, _ = run_cuda(inp, shape)
    check_routing_and_dispatch(views, inp, shape)
    ref = torch_fp32_layer(inp, shape, views["topk_idx"], views["topk_weights"])
    toks = np.random.default_rng(17).choice(2048, 4, replace=False)
    ora = oracle_output(inp, shape, tokens=toks)
    assert mo.cosine(ref[toks].cpu().numpy(), ora) >= 0.99999
    np.testing.assert_allclose(ref[toks].cpu().numpy(), ora, atol=1e-2, rtol=2e-2)
    got = out.float()
    # The FP8 requant of the intermediate rounds sums that both sides compute
    # in fp32 in different orders; where a sum sits on a rounding boundary the
    # two pick neighbouring codes, and one such code moves an output element
    # by up to ~0.02.  Observed: 32 of 14.7 M elements outside allclose.  The
    # bar: cosine (global and per token), at most 0.001% of the elements
    # outside allclose(1e-2, 2e-2), and none further off than 0.05.
    diff = (got - ref).abs()
    outside = diff > ATOL + RTOL * ref.abs()
    assert outside.float().mean().item() <= 1e-5, int(outside.sum())
    assert diff.max().item() <= 0.05
    cos = torch.dot(got.flatten(), ref.flatten()) / (got.norm() * ref.norm())
    assert cos.item() >= COS
    # per-token cosine, so that no single token hides in the global figure
    tc = (got * ref).sum(1) / (got.norm(dim=1) * ref.norm(dim=1) + 1e-30)
    assert tc.min().item() >= 0.999


def test_routing_exact_ties_match_the_oracle(cuda_device):
    """Routing with exact ties, bit-exact against the oracle (lowest group and
    expert id win, kernel.py:497-499, 524-525): all-equal scores; a few values
    repeated across groups and inside a lane's experts; a bias that makes every
    group's top-2 sum equal; and one-hot scores that tie the rest."""
    e, t = 256, 6
    rng = np.random.default_rng(5)
    logits = np.zeros((t, e), np.float32)
    logits[1] = rng.choice(np.array([-1.0, 0.0, 0.5, 2.0], np.float32), e)
    logits[2] = np.repeat(np.arange(32, dtype=np.float32) * 0.25, 8)[::-1]
    logits[3] = np.tile(np.array([0.0, 1.0, 1.0, 0.0, 2.0, 2.0, 2.0, 0.0], np.float32), 32)
    logits[4, ::37] = 3.0
    logits[5] = rng.standard_normal(e).astype(np.float32).round(1)
    bias = np.zeros(e, np.float32)
    bias[::32] = 0.5           # every group gets the same head
    full = workloads.make_inputs(workloads.dsv3_shape(t), seed=9, device="cuda")
    for tt in (t, 3):          # the routing kernel, and the one-block route+pack
        shape = workloads.dsv3_shape(tt)
        inp = dict(full)
        inp["routing_logits"] = torch.from_numpy(logits[:tt]).cuda()
        inp["hidden_states"] = full["hidden_states"][:tt].contiguous()
        inp["hidden_states_scale"] = full["hidden_states_scale"][:, :tt].contiguous()
        for b in (np.zeros(e, np.float32), bias):
            inp["routing_bias"] = torch.from_numpy(b).cuda()
            _, views, _ = run_cuda(inp, shape)
            check_routing_and_dispatch(views, inp, shape)


# ---------------------------------------------------------------- prepared bf16 W2

def test_prepare_gemm2_weights_is_bf16_of_the_dequantised_weight(cuda_device):
    from moe_b200 import prepare_gemm2_weights
    shape = workloads.MoeShape(t=1, hidden=1024, inter=384, e_global=64, e_local=8, n_group=8,
                               topk_group=2, top_k=6)
    inp = workloads.make_inputs(shape, seed=801, device="cuda")
    w, s = inp["gemm2_weights"], inp["gemm2_weights_scale"]
    got = prepare_gemm2_weights(w, s)
    e, h, i = w.shape
    ref = (w.float().view(e, h // 128, 128, i // 128, 128) *
           s.view(e, h // 128, 1, i // 128, 1)).view(e, h, i).to(torch.bfloat16)
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("case", ["dsv3_2048", "odd_700", "contest_901"])
def test_prepared_bf16_gemm2_prefill(cuda_device, case):
    """GEMM2 on bf16 operands (prepared W2, dequantised intermediate): routing
    unchanged; output against the oracle and, at DeepSeek-V3 size, every element
    against the fp32 PyTorch layer.  bf16 rounds each GEMM2 operand once more
    (2^-9 relative), so the bar is the north star's cosine >= 0.9999 with at
    most 0.1% of the elements outside allclose(1e-2, 2e-2) (observed: 0.014% of
    a sample, the largest 0.015 off) and none further off than 0.05."""
    from moe_b200 import prepare_gemm2_weights, run
    if case == "dsv3_2048":
        inp, shape = dsv3_inputs(2048, seed=17)
    elif case == "contest_901":
        inp, shape = dsv3_inputs(901, seed=32, e_local=32, local_expert_offset=32)
    else:
        shape = workloads.MoeShape(t=700, hidden=1024, inter=384, e_global=64, e_local=64,
                                   n_group=8, topk_group=2, top_k=6)
        inp = workloads.make_inputs(shape, seed=1000, device="cuda")
    wb = prepare_gemm2_weights(inp["gemm2_weights"], inp["gemm2_weights_scale"])
    out = torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16, device="cuda")
    run(*workloads.run_args(inp), out, n_group=shape.n_group, topk_group=shape.topk_group,
        top_k=shape.top_k, gemm2_weights_bf16=wb)
    out_fp8, views, _ = run_cuda(inp, shape)
    torch.cuda.synchronize()
    check_routing_and_dispatch(views, inp, shape)
    toks = np.random.default_rng(shape.t).choice(shape.t, 6, replace=False)
    ref = oracle_output(inp, shape, tokens=toks)
    got = bf16_np(out)[toks]
    assert mo.cosine(got, ref) >= COS
    d = np.abs(got.astype(np.float64) - ref)
    assert np.mean(d > ATOL + RTOL * np.abs(ref)) <= 1e-3 and d.max() <= 0.05
    g, f = out.float(), out_fp8.float()
    assert (torch.dot(g.flatten(), f.flatten()) / (g.norm() * f.norm())).item() >= 0.99999
    if case == "dsv3_2048":
        ref_t = torch_fp32_layer(inp, shape, views["topk_idx"], views["topk_weights"])
        diff = (g - ref_t).abs()
        outside = diff > ATOL + RTOL * ref_t.abs()
        assert outside.float().mean().item() <= 1e-3, int(outside.sum())
        assert diff.max().item() <= 0.05
        cos = torch.dot(g.flatten(), ref_t.flatten()) / (g.norm() * ref_t.norm())
        assert cos.item() >= COS


def test_prepared_bf16_gemm2_deterministic_and_decode(cuda_device):
    """The bf16 GEMM2 with the deterministic combine gives the same bits twice;
    a decode-sized batch ignores the prepared weights (FP8 decode GEMMs)."""
    from moe_b200 import prepare_gemm2_weights, run
    inp, shape = dsv3_inputs(600, seed=33, e_local=64, local_expert_offset=0)
    wb = prepare_gemm2_weights(inp["gemm2_weights"], inp["gemm2_weights_scale"])
    outs = []
    for _ in range(2):
        o = torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16, device="cuda")
        run(*workloads.run_args(inp), o, deterministic=True, gemm2_weights_bf16=wb)
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    inp8, shape8 = dsv3_inputs(8, seed=34, e_local=64, local_expert_offset=0)
    wb8 = prepare_gemm2_weights(inp8["gemm2_weights"], inp8["gemm2_weights_scale"])
    a = torch.empty(8, shape8.hidden, dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    run(*workloads.run_args(inp8), a, deterministic=True, gemm2_weights_bf16=wb8)
    run(*workloads.run_args(inp8), b, deterministic=True)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
