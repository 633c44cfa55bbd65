"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference solution's own Triton kernels (``kernel.py`` of
nikhilnd/mlsys26-flashinfer-moe) under ``TRITON_INTERPRET=1`` on the CPU, on
seeded inputs from ``moe_b200.workloads``, and stores every stage's result in
``tests/golden/<name>.npz``.  The reference sources are imported read-only from
``--ref`` and never copied.

``run()`` itself cannot run here: it requires CUDA (kernel.py:552-559) and
hard-codes the DeepSeek-V3 shapes (kernel.py:577-607).  ``drive_reference``
below therefore replays the launch sequence of ``run()`` (kernel.py:624-729)
with the shapes taken from the inputs, calling the reference's unmodified
kernels and host helpers.  Two things differ from a verbatim replay:

* the router is given ``GROUP_SIZE = E_global // N_GROUP``; ``run()`` passes
  ``E_local`` (kernel.py:638), which only coincides with the group size at the
  contest shape (32 of 256 experts, 8 groups);
* ``build_expert_dispatch`` asserts CUDA tensors (kernel.py:336), so its host
  logic (kernel.py:341-382) is replayed around the two unmodified kernels.

The Triton 3.6 interpreter's fp32->fp8e4nv cast rounds half-up and lets a
mantissa carry corrupt the exponent (``triton/runtime/interpreter.py``
``_convert_float``).  That cast is replaced here by torch's round-to-nearest-
even conversion, which is what the compiled GPU kernel does; everything else in
the interpreter is left as is.

Usage: ``python tests/golden/make_golden.py --ref DIR [--contest]`` (DIR: a
checkout of the reference; the committed .npz files are what the tests read).
``--contest`` makes the DeepSeek-V3 contest-shape cases (H=7168, I=2048, 32
of 256 experts local), which keep routing and dispatch in full and a sample
of intermediate rows and output tokens.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402
from triton.runtime import interpreter as _interp  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "mlsys26-flashinfer-moe_b200"))

from moe_b200 import workloads  # noqa: E402

sys.path.insert(0, HERE)
import cases  # noqa: E402

_orig_convert = _interp._convert_float


def _convert_float_fixed(inp, input_dtype, output_dtype, rounding_mode):
    if output_dtype == tl.float8e4nv and input_dtype == tl.float32:
        x = torch.from_numpy(np.ascontiguousarray(inp).view(np.float32).copy())
        x = torch.clamp(x, -448.0, 448.0)
        return x.to(torch.float8_e4m3fn).view(torch.uint8).numpy().reshape(np.shape(inp))
    return _orig_convert(inp, input_dtype, output_dtype, rounding_mode)


_interp._convert_float = _convert_float_fixed


def load_reference(ref_dir: str):
    spec = importlib.util.spec_from_file_location("reference_kernel",
                                                  os.path.join(ref_dir, "kernel.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def drive_reference(ref, inp: dict, shape: workloads.MoeShape):
    """Replay of ``run()`` (kernel.py:624-729) with parametrised shapes."""
    logits = inp["routing_logits"].float().contiguous()
    bias = inp["routing_bias"].float().reshape(-1).contiguous()
    hs = inp["hidden_states"].contiguous()
    hss = inp["hidden_states_scale"].contiguous()
    w1, w1s = inp["gemm1_weights"].contiguous(), inp["gemm1_weights_scale"].contiguous()
    w2, w2s = inp["gemm2_weights"].contiguous(), inp["gemm2_weights_scale"].contiguous()
    t = logits.shape[0]
    h, i = shape.hidden, shape.inter
    e_global, e_local = shape.e_global, shape.e_local
    top_k, n_group, topk_group = shape.top_k, shape.n_group, shape.topk_group
    lo = shape.local_expert_offset

    topk_idx = torch.empty((t, top_k), dtype=torch.int32)
    topk_w = torch.empty((t, top_k), dtype=torch.float32)
    ref.moe_routing_kernel[(t,)](logits, bias, topk_idx, topk_w, logits.stride(0),
                                 shape.routed_scaling_factor, e_global, n_group,
                                 e_global // n_group, topk_group, top_k)

    # build_expert_dispatch host logic (kernel.py:341-382) around the kernels
    m = t * top_k
    flat_e = topk_idx.reshape(-1).contiguous()
    flat_w = topk_w.reshape(-1).contiguous().to(torch.float32)
    bs = 1024
    nb = triton.cdiv(m, bs)
    partial = torch.zeros((nb, e_local), dtype=torch.int32)
    ref._count_kernel[(nb,)](flat_e, partial, m, lo, e_local, BLOCK_SIZE=bs)
    counts = partial.sum(dim=0).to(torch.int32)
    starts = torch.empty(e_local + 1, dtype=torch.int32)
    starts[0] = 0
    torch.cumsum(counts, dim=0, out=starts[1:])
    n = int(starts[-1].item())
    sorted_tok = torch.empty(n, dtype=torch.int32)
    sorted_w = torch.empty(n, dtype=torch.float32)
    cursor = starts[:e_local].clone()
    ref._scatter_kernel[(nb,)](flat_e, flat_w, cursor, sorted_tok, sorted_w, m, TOP_K=top_k,
                               lo=lo, E_local=e_local, BLOCK_SIZE=bs)

    bm1, bn1, bk1, gsm1 = 64, 64, 128, 4
    tile_e, tile_m, total = ref.build_tile_schedule(counts, bm1, e_local)
    total = int(total.item())
    a_packed = torch.index_select(hs, 0, sorted_tok.long()).contiguous()
    a_scale_packed = torch.index_select(hss, 1, sorted_tok.long()).contiguous()
    g1 = torch.zeros((n, i), dtype=torch.float8_e4m3fn)
    g1s = torch.zeros((triton.cdiv(i, bn1), n), dtype=torch.float32)
    ref.moe_gemm1_kernel[(total * triton.cdiv(i, bn1),)](
        a_packed, a_scale_packed, a_packed.stride(0), a_packed.stride(1),
        a_scale_packed.stride(0), a_scale_packed.stride(1),
        w1, w1s, w1.stride(0), w1.stride(1), w1.stride(2),
        w1s.stride(0), w1s.stride(1), w1s.stride(2),
        g1, g1s, g1.stride(0), g1.stride(1), g1s.stride(0), g1s.stride(1),
        sorted_tok, starts, tile_e, tile_m,
        t, h, i, 2 * i, bm1, bn1, bk1, gsm1, total)
    # GEMM2's A-scale load is unmasked (kernel.py:218-220); pad the scale
    # tensor so the replay never reads past the end of a CPU allocation.
    g1s_pad = torch.zeros((g1s.shape[0], n + 64), dtype=torch.float32)
    g1s_pad[:, :n] = g1s
    g1s_view = g1s_pad[:, :n]
    out32 = torch.zeros((t, h), dtype=torch.float32)
    bm2, bn2, bk2, gsm2 = 64, 64, 64, 4
    ref.moe_gemm2_kernel[(total * triton.cdiv(h, bn2),)](
        g1, g1s_view, g1.stride(0), g1.stride(1), g1s_view.stride(0), g1s_view.stride(1),
        w2, w2s, w2.stride(0), w2.stride(1), w2.stride(2),
        w2s.stride(0), w2s.stride(1), w2s.stride(2),
        sorted_w, out32, out32.stride(0), out32.stride(1),
        sorted_tok, starts, tile_e, tile_m,
        t, h, i, bm2, bn2, bk2, bn1, gsm2, total)
    out = out32.to(torch.bfloat16)
    return dict(topk_idx=topk_idx.numpy(), topk_weights=topk_w.numpy(),
                counts=counts.numpy(), starts=starts.numpy(),
                sorted_tokens=sorted_tok.numpy(), sorted_weights=sorted_w.numpy(),
                tile_expert=tile_e.numpy(), tile_local_m=tile_m.numpy(),
                gemm1_out=g1.view(torch.uint8).numpy(), gemm1_scale=g1s.numpy(),
                out_f32=out32.numpy(), output_bf16=out.view(torch.int16).numpy().view(np.uint16))


def make_case(ref, name: str):
    inp, shape, spec = cases.case_inputs(name)
    res = drive_reference(ref, inp, shape)
    meta = dict(name=name, seed=spec["seed"], digest=workloads.tensor_digest(inp),
                **{k: v for k, v in shape.__dict__.items()},
                bias_dtype=str(inp["routing_bias"].dtype),
                generator="tests/golden/cases.py case_inputs",
                reference="kernel.py kernels under TRITON_INTERPRET=1 (fp8 cast fixed)")
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"),
                        meta=np.array(repr(meta)), **res)
    print(name, "tokens", shape.t, "assignments", int(res["starts"][-1]), "digest",
          meta["digest"][:16])


def make_contest_case(ref, name: str, inter_rows: int = 24):
    """A contest-shape case (DeepSeek-V3, 32 of 256 experts local).  Routing and
    dispatch are kept in full; the intermediate for the first ``inter_rows``
    rows in bucket order and the output for ``cases.contest_sample_tokens``."""
    import time
    inp, shape, spec = cases.contest_case_inputs(name)
    t0 = time.time()
    res = drive_reference(ref, inp, shape)
    n = int(res["starts"][-1])
    k = min(n, inter_rows)
    toks = cases.contest_sample_tokens(shape.t)
    keep = dict(topk_idx=res["topk_idx"], topk_weights=res["topk_weights"], counts=res["counts"],
                starts=res["starts"], sorted_tokens=res["sorted_tokens"],
                sorted_weights=res["sorted_weights"], tile_expert=res["tile_expert"],
                tile_local_m=res["tile_local_m"], inter_rows=np.arange(k),
                gemm1_out=res["gemm1_out"][:k], gemm1_scale=res["gemm1_scale"][:, :k],
                sample_tokens=toks, output_bf16=res["output_bf16"][toks])
    meta = dict(name=name, seed=spec["seed"], weight_seed=cases.CONTEST_WEIGHT_SEED,
                digest=workloads.tensor_digest(inp),
                **{kk: v for kk, v in shape.__dict__.items()},
                generator="tests/golden/cases.py contest_case_inputs",
                reference="kernel.py kernels under TRITON_INTERPRET=1 (fp8 cast fixed)")
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), meta=np.array(repr(meta)), **keep)
    print(name, "tokens", shape.t, "local assignments", n, "digest", meta["digest"][:16],
          f"{time.time() - t0:.0f} s")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference solution (read-only)")
    ap.add_argument("--case", default=None)
    ap.add_argument("--contest", action="store_true",
                    help="the DeepSeek-V3 contest-shape cases (cases.CONTEST_CASES)")
    a = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    ref = load_reference(a.ref)
    names = cases.CONTEST_CASES if a.contest else cases.CASES
    for name in names:
        if a.case and a.case != name:
            continue
        (make_contest_case if a.contest else make_case)(ref, name)


if __name__ == "__main__":
    main()
