"""Seeded synthetic workloads for the fused FP8 block-scale MoE forward.

The reference is scored on FlashInfer-Bench workloads (real router logits) that
are not available offline, so every benchmark and test here uses seeded
synthetic inputs with the shapes and value distributions of the benchmark
definition ``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``:

* weights: bf16 N(0, 0.02), quantised to e4m3 with one fp32 scale per 128x128
  block, ``scale = amax / 448`` (layout ``[E, N/128, K/128]``);
* activations: bf16 N(0, 1), quantised per token per 128 columns, scale stored
  transposed as ``[H/128, T]`` (the layout ``run()`` asserts, reference
  ``kernel.py:603``);
* router logits fp32 N(0, 1), router bias fp32 N(0, 0.1);
* optional Zipf(s) expert popularity, realised through the router bias.

Generation runs on any torch device; the DeepSeek-V3 shapes (11 GB of FP8
weights for 256 experts) are generated directly on the GPU.  This module is
input generation only: it never computes the MoE.
"""
from __future__ import annotations

import dataclasses
import hashlib
import math
from typing import Optional

import torch

FP8_MAX = 448.0
BLOCK = 128


@dataclasses.dataclass(frozen=True)
class MoeShape:
    """Layer shape. ``e_global`` experts are routed; ``e_local`` of them (starting at
    ``local_expert_offset``) have weights on this device."""
    t: int
    hidden: int = 7168
    inter: int = 2048
    e_global: int = 256
    e_local: int = 256
    n_group: int = 8
    topk_group: int = 4
    top_k: int = 8
    local_expert_offset: int = 0
    routed_scaling_factor: float = 2.5


# BASELINE configs. Config 0 is the tiny CPU-runnable case; the others use the
# DeepSeek-V3 layer (H=7168, I=2048, 256 experts, 8 groups / top-4, top-8).
TINY = dict(hidden=512, inter=256, e_global=16, e_local=16, n_group=4, topk_group=2,
            top_k=4, routed_scaling_factor=2.5)
DSV3 = dict(hidden=7168, inter=2048, e_global=256, e_local=256, n_group=8, topk_group=4,
            top_k=8, routed_scaling_factor=2.5)
# The FlashInfer-Bench contest definition: 32 local experts out of 256.
CONTEST = dict(DSV3, e_local=32)


def tiny_shape(t: int = 16) -> MoeShape:
    return MoeShape(t=t, **TINY)


def dsv3_shape(t: int, **kw) -> MoeShape:
    d = dict(DSV3)
    d.update(kw)
    return MoeShape(t=t, **d)


def quantize_weight_blocks(w: torch.Tensor):
    """Quantise ``[E, N, K]`` weights to e4m3 with one scale per 128x128 block.

    Returns ``(q [E,N,K] float8_e4m3fn, s [E,N/128,K/128] fp32)`` with
    ``w ~= q * s`` blockwise, ``s = amax/448``.
    """
    e, n, k = w.shape
    assert n % BLOCK == 0 and k % BLOCK == 0
    wf = w.float().view(e, n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    amax = wf.abs().amax(dim=(2, 4))
    s = torch.clamp(amax / FP8_MAX, min=1e-12)
    q = (wf / s[:, :, None, :, None]).to(torch.float8_e4m3fn)
    return q.view(e, n, k), s.contiguous()


def quantize_act_1x128(x: torch.Tensor):
    """Quantise ``[T, H]`` activations per token per 128 columns.

    Returns ``(q [T,H] e4m3, s [H/128, T] fp32)``; the scale tensor is stored
    transposed, as the reference's ``hidden_states_scale`` is.
    """
    t, h = x.shape
    assert h % BLOCK == 0
    xf = x.float().view(t, h // BLOCK, BLOCK)
    amax = xf.abs().amax(dim=2)
    s = torch.clamp(amax / FP8_MAX, min=1e-12)
    q = (xf / s[:, :, None]).to(torch.float8_e4m3fn).view(t, h)
    return q, s.t().contiguous()


def zipf_bias(shape: MoeShape, s: float, g: torch.Generator, device) -> torch.Tensor:
    """Router bias that makes expert popularity roughly Zipf(``s``) over a random
    permutation of the experts (the skewed-routing stress config)."""
    e = shape.e_global
    ranks = torch.randperm(e, generator=g, device="cpu").to(torch.float64) + 1.0
    pop = ranks.pow(-s)
    pop = pop / pop.mean()
    # Sigmoid scores live in (0,1); a log-popularity bias tilts them towards the
    # head of the distribution.  The factor 0.1 gives what the benchmark
    # configuration describes at s=1.2, T=8192 (DeepSeek-V3 routing, measured
    # with the oracle's router): the hottest expert ~21x the mean count, 43 of
    # 256 experts never chosen.
    bias = 0.1 * torch.log(pop)
    return bias.to(torch.float32).to(device)


def make_inputs(shape: MoeShape, seed: int = 0, device="cpu", zipf: Optional[float] = None,
                weights: bool = True, dtype_bias=torch.float32):
    """Build the positional inputs of ``run()`` for ``shape``.

    Returns a dict with keys ``routing_logits, routing_bias, hidden_states,
    hidden_states_scale, gemm1_weights, gemm1_weights_scale, gemm2_weights,
    gemm2_weights_scale`` plus ``local_expert_offset`` and
    ``routed_scaling_factor``.  With ``weights=False`` the weight tensors are
    omitted (routing-only tests).
    """
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    gc = torch.Generator(device="cpu")
    gc.manual_seed(seed + 1)
    t, h, i = shape.t, shape.hidden, shape.inter
    out = {}
    out["routing_logits"] = torch.randn(t, shape.e_global, generator=g, device=device,
                                        dtype=torch.float32)
    if zipf is None:
        bias = 0.1 * torch.randn(shape.e_global, generator=g, device=device, dtype=torch.float32)
    else:
        bias = zipf_bias(shape, zipf, gc, device)
    out["routing_bias"] = bias.to(dtype_bias)
    x = torch.randn(t, h, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    out["hidden_states"], out["hidden_states_scale"] = quantize_act_1x128(x)
    if weights:
        el = shape.e_local
        # Generate one expert at a time to bound the fp32 temporaries.
        w1q = torch.empty(el, 2 * i, h, dtype=torch.float8_e4m3fn, device=device)
        w1s = torch.empty(el, 2 * i // BLOCK, h // BLOCK, dtype=torch.float32, device=device)
        w2q = torch.empty(el, h, i, dtype=torch.float8_e4m3fn, device=device)
        w2s = torch.empty(el, h // BLOCK, i // BLOCK, dtype=torch.float32, device=device)
        for e in range(el):
            w1 = (0.02 * torch.randn(1, 2 * i, h, generator=g, device=device,
                                     dtype=torch.float32)).to(torch.bfloat16)
            q, s = quantize_weight_blocks(w1)
            w1q[e] = q[0]
            w1s[e] = s[0]
            w2 = (0.02 * torch.randn(1, h, i, generator=g, device=device,
                                     dtype=torch.float32)).to(torch.bfloat16)
            q, s = quantize_weight_blocks(w2)
            w2q[e] = q[0]
            w2s[e] = s[0]
        out["gemm1_weights"], out["gemm1_weights_scale"] = w1q, w1s
        out["gemm2_weights"], out["gemm2_weights_scale"] = w2q, w2s
    out["local_expert_offset"] = shape.local_expert_offset
    out["routed_scaling_factor"] = shape.routed_scaling_factor
    return out


POSITIONAL = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
              "gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale",
              "local_expert_offset", "routed_scaling_factor")


def run_args(inp: dict):
    """The inputs of ``make_inputs`` as the positional argument list of ``run()``
    (without ``output``)."""
    return [inp[k] for k in POSITIONAL]


def tensor_digest(inp: dict) -> str:
    """sha256 over every tensor input, used to pin committed fixtures to the
    generator that made them."""
    hsh = hashlib.sha256()
    for k in POSITIONAL:
        v = inp.get(k)
        if isinstance(v, torch.Tensor):
            t = v.detach().cpu().contiguous()
            if t.dtype in (torch.float8_e4m3fn, torch.bfloat16):
                t = t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t.view(torch.int16)
            hsh.update(k.encode())
            hsh.update(t.numpy().tobytes())
        elif v is not None:
            hsh.update(f"{k}={v}".encode())
    return hsh.hexdigest()


def flops_per_assignment(shape: MoeShape) -> int:
    """GEMM1 (2*H*2I) + GEMM2 (2*I*H) flops for one (token, expert) pair."""
    return 6 * shape.hidden * shape.inter


def weight_bytes_per_expert(shape: MoeShape) -> int:
    h, i = shape.hidden, shape.inter
    return 2 * i * h + h * i + 4 * ((2 * i // BLOCK) * (h // BLOCK) + (h // BLOCK) * (i // BLOCK))


def expected_active_experts(shape: MoeShape) -> float:
    return shape.e_global * (1.0 - (1.0 - shape.top_k / shape.e_global) ** shape.t)


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def ilog2(x: int) -> int:
    return int(math.log2(x))
