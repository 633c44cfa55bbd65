"""Seeded input cases behind the golden fixtures in this directory.

``make_golden.py`` runs the reference on these inputs; the tests rebuild the
same inputs from the same seeds and check the stored digest first, so a change
in the generator shows up as a digest mismatch rather than as a parity failure.
"""
from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                "mlsys26-flashinfer-moe_b200"))

from moe_b200 import workloads  # noqa: E402

CASES = {
    # tiny MoE, all 16 experts local.
    "tiny_t16_seed0": dict(shape=workloads.tiny_shape(16), seed=0),
    # the same layer as an expert-parallel shard: experts 4..11 of 16.
    "tiny_t16_seed1_ep": dict(shape=workloads.MoeShape(
        t=16, **dict(workloads.TINY, e_local=8, local_expert_offset=4)), seed=1),
    # ragged token count with a bf16 router bias (run() accepts bf16/fp16 bias)
    "tiny_t7_seed2_bf16bias": dict(shape=workloads.tiny_shape(7), seed=2,
                                   dtype_bias=torch.bfloat16),
    # a single token
    "tiny_t1_seed3": dict(shape=workloads.tiny_shape(1), seed=3),
    # enough tokens that experts span several 64- and 128-row tiles
    "tiny_t300_seed4": dict(shape=workloads.tiny_shape(300), seed=4),
}


def case_inputs(name: str):
    """Inputs of case ``name``: weights for all ``e_global`` experts are drawn,
    then the local slice is kept, so an EP shard sees the same experts as the
    full layer does."""
    spec = CASES[name]
    shape = spec["shape"]
    full = workloads.MoeShape(**{**shape.__dict__, "e_local": shape.e_global,
                                 "local_expert_offset": 0})
    inp = workloads.make_inputs(full, seed=spec["seed"], device="cpu",
                                dtype_bias=spec.get("dtype_bias", torch.float32))
    if shape.e_local != shape.e_global:
        lo, el = shape.local_expert_offset, shape.e_local
        for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights",
                  "gemm2_weights_scale"):
            inp[k] = inp[k][lo:lo + el].contiguous()
    inp["local_expert_offset"] = shape.local_expert_offset
    return inp, shape, spec


# The contest shape (FlashInfer-Bench definition, kernel.py:577-588): DeepSeek-V3
# H=7168, I=2048, experts 0..31 of 256 local.  One set of 32 experts' weights
# (CPU generator, seed CONTEST_WEIGHT_SEED) is shared by the cases; each case
# draws its own tokens.  The fixtures keep routing and dispatch in full and a
# sample of intermediate rows and output tokens (make_golden.py --contest).
CONTEST_WEIGHT_SEED = 50
CONTEST_CASES = {
    "dsv3_e32_t7": dict(t=7, seed=51),
    "dsv3_e32_t80": dict(t=80, seed=52),
    "dsv3_e32_t901": dict(t=901, seed=53),
}
WEIGHT_KEYS = ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")
_contest_weights = {}


def contest_weights():
    if not _contest_weights:
        w = workloads.make_inputs(workloads.dsv3_shape(1, e_local=32), seed=CONTEST_WEIGHT_SEED,
                                  device="cpu")
        _contest_weights.update({k: w[k] for k in WEIGHT_KEYS})
    return _contest_weights


def contest_case_inputs(name: str):
    spec = CONTEST_CASES[name]
    shape = workloads.dsv3_shape(spec["t"], e_local=32, local_expert_offset=0)
    inp = workloads.make_inputs(shape, seed=spec["seed"], device="cpu", weights=False)
    inp.update(contest_weights())
    return inp, shape, spec


def contest_sample_tokens(t: int):
    """Tokens whose output rows a contest fixture keeps."""
    import numpy as np
    return np.arange(t) if t <= 16 else np.sort(np.random.default_rng(t).choice(t, 16, replace=False))
