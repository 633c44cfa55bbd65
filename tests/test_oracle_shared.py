"""The oracle's shared-expert extension (``moe_forward(..., n_shared=1)``) on the
CPU: the layer with a shared expert equals the routed layer plus that expert's
``expert_forward`` on every token, and an all-zero shared expert changes nothing."""
import numpy as np
import torch

import moe_oracle as mo
from moe_b200 import workloads


def _inputs(t, seed):
    shape = workloads.tiny_shape(t)
    inp = workloads.make_inputs(shape, seed=seed, device="cpu")
    g = torch.Generator(device="cpu")
    g.manual_seed(seed + 1)
    h, i = shape.hidden, shape.inter
    w1 = (0.02 * torch.randn(1, 2 * i, h, generator=g)).to(torch.bfloat16)
    w2 = (0.02 * torch.randn(1, h, i, generator=g)).to(torch.bfloat16)
    (q1, s1), (q2, s2) = workloads.quantize_weight_blocks(w1), workloads.quantize_weight_blocks(w2)
    with_shared = dict(inp)
    for k, v in (("gemm1_weights", q1), ("gemm1_weights_scale", s1), ("gemm2_weights", q2),
                 ("gemm2_weights_scale", s2)):
        with_shared[k] = torch.cat([inp[k], v])
    return shape, mo.to_numpy_inputs(inp), mo.to_numpy_inputs(with_shared)


def test_shared_expert_adds_its_own_output():
    shape, routed, shared = _inputs(24, seed=300)
    args = (shape.n_group, shape.topk_group, shape.top_k)
    y_routed = mo.moe_forward(routed, *args)
    y = mo.moe_forward(shared, *args, n_shared=1)
    el = shape.e_local
    s = mo.expert_forward(shared["hidden_states"], shared["hidden_states_scale"],
                          shared["gemm1_weights"][el], shared["gemm1_weights_scale"][el],
                          shared["gemm2_weights"][el], shared["gemm2_weights_scale"][el],
                          shape.inter)
    np.testing.assert_array_equal(y, y_routed + s.astype(np.float32))
    # restricted to a token subset it is the same rows (to fp32 rounding: BLAS sums
    # a different number of rows in a different blocked order)
    tok = np.array([3, 11, 23])
    np.testing.assert_allclose(mo.moe_forward(shared, *args, tokens=tok, n_shared=1), y[tok],
                               rtol=1e-5, atol=1e-6)


def test_zero_shared_expert_changes_nothing():
    shape, routed, shared = _inputs(9, seed=301)
    el = shape.e_local
    shared["gemm1_weights"][el] = 0
    shared["gemm2_weights"][el] = 0
    args = (shape.n_group, shape.topk_group, shape.top_k)
    np.testing.assert_array_equal(mo.moe_forward(shared, *args, n_shared=1),
                                  mo.moe_forward(routed, *args))
