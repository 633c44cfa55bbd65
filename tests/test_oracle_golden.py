"""The CPU oracle against the reference's own outputs (golden fixtures).

The fixtures in ``tests/golden`` come from the reference's Triton kernels run
under the Triton interpreter (``tests/golden/make_golden.py``).  These tests pin
the oracle that the GPU parity tests rely on.  CPU only.
"""
import ast
import os

import numpy as np
import pytest
import torch

import cases
import moe_oracle as mo
from moe_b200 import workloads

CASE_NAMES = list(cases.CASES)


def load_case(name):
    g = np.load(f"{cases.HERE}/{name}.npz")
    meta = ast.literal_eval(str(g["meta"]))
    inp, shape, _ = cases.case_inputs(name)
    return g, meta, inp, shape


@pytest.mark.parametrize("name", CASE_NAMES)
def test_inputs_match_fixture_digest(name):
    g, meta, inp, _ = load_case(name)
    assert workloads.tensor_digest(inp) == meta["digest"], \
        "input generator drifted from the one that produced the fixture"


@pytest.mark.parametrize("name", CASE_NAMES)
def test_routing_bit_exact(name):
    g, meta, inp, s = load_case(name)
    ni = mo.to_numpy_inputs(inp)
    idx, w = mo.route(ni["routing_logits"], ni["routing_bias"], s.n_group, s.topk_group, s.top_k,
                      s.routed_scaling_factor)
    np.testing.assert_array_equal(idx, g["topk_idx"])
    np.testing.assert_allclose(w, g["topk_weights"], rtol=2e-6, atol=0)


@pytest.mark.parametrize("name", CASE_NAMES)
def test_dispatch_matches_reference(name):
    g, meta, inp, s = load_case(name)
    counts, starts, tok, wt = mo.dispatch(g["topk_idx"], g["topk_weights"],
                                          s.local_expert_offset, s.e_local)
    np.testing.assert_array_equal(counts, g["counts"])
    np.testing.assert_array_equal(starts, g["starts"])
    # the reference orders a bucket by atomics; compare bucket contents sorted
    for e in range(s.e_local):
        a, b = starts[e], starts[e + 1]
        ref_order = np.argsort(g["sorted_tokens"][a:b], kind="stable")
        np.testing.assert_array_equal(tok[a:b], g["sorted_tokens"][a:b][ref_order])
        np.testing.assert_array_equal(wt[a:b], g["sorted_weights"][a:b][ref_order])
    te, tm, _ = mo.tile_schedule(counts, 64)
    np.testing.assert_array_equal(te, g["tile_expert"])
    np.testing.assert_array_equal(tm, g["tile_local_m"])


@pytest.mark.parametrize("name", CASE_NAMES)
def test_intermediate_matches_reference(name):
    """GEMM1 + SwiGLU + 1x64 requant of the oracle vs the reference kernel's
    FP8 intermediate, row by row in bucket order."""
    g, meta, inp, s = load_case(name)
    ni = mo.to_numpy_inputs(inp)
    starts, stok = g["starts"], g["sorted_tokens"]
    for e in range(s.e_local):
        a, b = starts[e], starts[e + 1]
        if a == b:
            continue
        rows = stok[a:b]
        ad = mo.dequant_act(ni["hidden_states"][rows], ni["hidden_states_scale"][:, rows])
        gm = ad @ mo.dequant_weight(ni["gemm1_weights"][e], ni["gemm1_weights_scale"][e]).T
        codes, sc, _ = mo.swiglu_requant(gm, s.inter)
        ref_codes = g["gemm1_out"][a:b]
        ref_sc = g["gemm1_scale"][:, a:b]
        np.testing.assert_allclose(sc, ref_sc, rtol=1e-5)
        # fp32 summation order differs; allow a rare one-step rounding flip
        assert np.mean(codes == ref_codes) > 0.999
        dv = np.abs(mo.e4m3_decode(codes).astype(np.float64) -
                    mo.e4m3_decode(ref_codes).astype(np.float64))
        assert dv.max() <= 32.0   # one e4m3 step at the top of the range


@pytest.mark.parametrize("name", CASE_NAMES)
def test_output_matches_reference(name):
    g, meta, inp, s = load_case(name)
    ni = mo.to_numpy_inputs(inp)
    out = mo.moe_forward(ni, s.n_group, s.topk_group, s.top_k)
    ref = mo.bf16_to_f32(g["output_bf16"])
    ours = mo.bf16_to_f32(mo.bf16_bits(out))
    np.testing.assert_allclose(ours, ref, atol=1e-2, rtol=2e-2)
    assert mo.cosine(out, g["out_f32"]) >= 0.9999
    assert np.mean(ours == ref) > 0.99


def test_fp32_oracle_within_tolerance_of_reference():
    """Without the FP8 requant of the intermediate the oracle is the
    dequantised fp32 math the tolerance atol 1e-2 / rtol 2e-2 is stated on."""
    g, meta, inp, s = load_case("tiny_t300_seed4")
    ni = mo.to_numpy_inputs(inp)
    out = mo.moe_forward(ni, s.n_group, s.topk_group, s.top_k, requant=False)
    ref = mo.bf16_to_f32(g["output_bf16"])
    np.testing.assert_allclose(ref, out, atol=1e-2, rtol=2e-2)


def test_e4m3_encoder_is_rne_and_saturating():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200_000).astype(np.float32) * sc
                        for sc in (1e-3, 0.3, 30, 200)])
    x = np.concatenate([x, np.float32([0.0, -0.0, 448.0, 448.0001, 464.0, 1.0625, 1.1875,
                                       2.0 ** -10, 3 * 2.0 ** -10])])
    codes = mo.e4m3_encode(x)
    back = mo.e4m3_decode(codes).astype(np.float64)
    xc = np.clip(x.astype(np.float64), -448, 448)
    # nearest representable value
    vals = np.sort(mo.E4M3_VALUES[np.isfinite(mo.E4M3_VALUES)].astype(np.float64))
    pos = np.clip(np.searchsorted(vals, xc), 1, len(vals) - 1)
    best = np.minimum(np.abs(vals[pos] - xc), np.abs(vals[pos - 1] - xc))
    assert np.all(np.abs(back - xc) <= best + 1e-30)
    # ties go to even mantissa: 1.0625 is halfway between 1.0 and 1.125
    assert mo.e4m3_decode(mo.e4m3_encode(np.float32([1.0625, 1.1875])))[0] == 1.0
    assert mo.e4m3_decode(mo.e4m3_encode(np.float32([1.1875])))[0] == 1.25


def test_routing_ties_go_to_lowest_index():
    """All-equal logits and zero bias: every score ties, so the reference's
    max-and-mask picks the lowest group and expert ids (kernel.py:497-499,
    524-525)."""
    t, e = 3, 256
    idx, w = mo.route(np.zeros((t, e), np.float32), np.zeros(e, np.float32), 8, 4, 8, 2.5)
    np.testing.assert_array_equal(idx, np.tile(np.arange(8, dtype=np.int32), (t, 1)))
    np.testing.assert_allclose(w, np.full((t, 8), 2.5 / 8, np.float32), rtol=1e-7)


def test_routing_bias_only_selects():
    """The bias steers selection, the unbiased sigmoid sets the weights
    (kernel.py:467, 530, 537-538)."""
    e = 256
    logits = np.zeros((1, e), np.float32)
    bias = np.zeros(e, np.float32)
    chosen = [3, 40, 77, 100, 130, 161, 200, 250]
    bias[chosen] = 1.0
    idx, w = mo.route(logits, bias, 8, 4, 8, 1.0)
    # groups 0..7 hold one chosen expert each -> the top-4 groups are tied on
    # score 1.5+0.5; lowest groups win, then the 4 chosen experts in them plus
    # the 4 lowest unchosen experts of those groups.
    assert set(idx[0][:4]) == {3, 40, 77, 100}
    np.testing.assert_allclose(w.sum(), 1.0, rtol=1e-6)


# ---------------------------------------------------------------- contest shape

CONTEST_NAMES = [n for n in cases.CONTEST_CASES if os.path.exists(f"{cases.HERE}/{n}.npz")]
_expert_cache = {}


def load_contest(name):
    g = np.load(f"{cases.HERE}/{name}.npz")
    meta = ast.literal_eval(str(g["meta"]))
    inp, shape, _ = cases.contest_case_inputs(name)
    return g, meta, inp, shape


def contest_expert(inp, e):
    if e not in _expert_cache:
        _expert_cache[e] = tuple(inp[k][e].view(torch.uint8).numpy() if inp[k].dtype ==
                                 torch.float8_e4m3fn else inp[k][e].numpy()
                                 for k in cases.WEIGHT_KEYS)
    return _expert_cache[e]


@pytest.mark.parametrize("name", CONTEST_NAMES)
def test_contest_routing_dispatch_and_output(name):
    """DeepSeek-V3 contest shape (H=7168, I=2048, 32 of 256 experts): the
    oracle's routing and dispatch equal the reference kernels' bit for bit, and
    its output matches theirs on the fixture's first sampled tokens."""
    g, meta, inp, s = load_contest(name)
    assert workloads.tensor_digest(inp) == meta["digest"]
    ni = {k: v for k, v in mo.to_numpy_inputs({k: v for k, v in inp.items()
                                               if k not in cases.WEIGHT_KEYS}).items()}
    idx, w = mo.route(ni["routing_logits"], ni["routing_bias"], s.n_group, s.topk_group, s.top_k,
                      s.routed_scaling_factor)
    np.testing.assert_array_equal(idx, g["topk_idx"])
    np.testing.assert_allclose(w, g["topk_weights"], rtol=2e-6, atol=0)
    counts, starts, tok, wt = mo.dispatch(idx, w, s.local_expert_offset, s.e_local)
    np.testing.assert_array_equal(counts, g["counts"])
    np.testing.assert_array_equal(starts, g["starts"])
    for e in range(s.e_local):
        a, b = starts[e], starts[e + 1]
        np.testing.assert_array_equal(tok[a:b], np.sort(g["sorted_tokens"][a:b]))
    toks = g["sample_tokens"][:4]
    hi = dict(ni, local_expert_offset=0, routed_scaling_factor=s.routed_scaling_factor,
              e_local=s.e_local)
    ref = mo.moe_forward(hi, s.n_group, s.topk_group, s.top_k, tokens=toks,
                         get_expert=lambda e: contest_expert(inp, e))
    got = mo.bf16_to_f32(g["output_bf16"][:4])
    np.testing.assert_allclose(ref, got, atol=1e-2, rtol=2e-2)
    assert mo.cosine(ref, got) >= 0.9999
