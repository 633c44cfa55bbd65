"""Failure detection on the GPU without a GPU fault.

Every wait inside the GEMM kernels is bounded (``MoeFwdArgs.wait_limit_ns``);
when one runs out, the CTA raises its abort flag, lets the copies and MMAs it
has in flight land, frees its TMEM and exits, and the workspace's error word
records ``MOE_ERR_TIMEOUT`` with the wait site.  ``MOE_FLAG_TEST_STALL`` makes
that happen on purpose: the first MMA issuer of every GEMM1 CTA waits on a
barrier that nothing completes.  The device must keep answering, and the next
normal forward on the same workspace must be correct.
"""
import numpy as np
import pytest
import torch

import moe_oracle as mo
from gpu_helpers import run_cuda
from moe_b200 import _lib, api, workloads

pytestmark = pytest.mark.gpu

# wait sites of the prefill GEMMs (moe_gemm.cu) and of the decode GEMMs
# (moe_gemm_small.cu), as recorded in the error word's info
PREFILL_SITES = {1, 2, 3, 4, 5, 9}
DECODE_SITES = {11, 12, 13, 14, 15, 16, 19}


def forward_with(inp, shape, workspace, flags=0, wait_limit_ns=0):
    dev = torch.device("cuda", 0)
    out = torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16, device=dev)
    args, keep, out_dev = api.build_args(*workloads.run_args(inp), out, shape.n_group,
                                         shape.topk_group, shape.top_k)
    args.flags = flags
    args.wait_limit_ns = wait_limit_ns
    api.forward_args(args, workspace, dev)
    torch.cuda.synchronize()
    return out, args


@pytest.mark.parametrize("t,sites", [(48, PREFILL_SITES), (4, DECODE_SITES)])
def test_stalled_wait_times_out_and_the_next_forward_is_correct(cuda_device, t, sites):
    shape = workloads.tiny_shape(t)
    inp = workloads.make_inputs(shape, seed=600 + t, device="cuda")
    args0, _, _ = api.build_args(*workloads.run_args(inp),
                                 torch.empty(t, shape.hidden, dtype=torch.bfloat16, device="cuda"),
                                 shape.n_group, shape.topk_group, shape.top_k)
    ws = torch.empty(api.workspace_layout(args0).total_bytes, dtype=torch.uint8, device="cuda")

    _, args = forward_with(inp, shape, ws, flags=_lib.MOE_FLAG_TEST_STALL, wait_limit_ns=50_000)
    code, info = api.device_error(args)
    assert code == _lib.MOE_ERR_TIMEOUT, (code, info)
    assert info in sites, info

    # the device still answers, and the same workspace gives a correct layer
    out, args = forward_with(inp, shape, ws)
    assert api.device_error(args) == (0, 0)
    ref = mo.moe_forward(mo.to_numpy_inputs({k: (v.cpu() if isinstance(v, torch.Tensor) else v)
                                             for k, v in inp.items()}),
                         shape.n_group, shape.topk_group, shape.top_k)
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, ref, atol=1e-2, rtol=2e-2)
    assert mo.cosine(got, ref) >= 0.9999


def test_wait_limit_alone_changes_nothing(cuda_device):
    """A short but sufficient limit (5 ms) leaves a normal forward untouched."""
    shape = workloads.tiny_shape(300)
    inp = workloads.make_inputs(shape, seed=611, device="cuda")
    out_ref, _, _ = run_cuda(inp, shape)
    args0, _, _ = api.build_args(*workloads.run_args(inp), out_ref, shape.n_group,
                                 shape.topk_group, shape.top_k)
    ws = torch.empty(api.workspace_layout(args0).total_bytes, dtype=torch.uint8, device="cuda")
    out, args = forward_with(inp, shape, ws, wait_limit_ns=5_000_000)
    assert api.device_error(args) == (0, 0)
    assert (out.float() - out_ref.float()).abs().max().item() <= 2e-3


def test_unknown_flags_are_rejected(cuda_device):
    shape = workloads.tiny_shape(8)
    inp = workloads.make_inputs(shape, seed=612, device="cuda")
    out = torch.empty(8, shape.hidden, dtype=torch.bfloat16, device="cuda")
    args, _, _ = api.build_args(*workloads.run_args(inp), out, shape.n_group, shape.topk_group,
                                shape.top_k)
    args.flags = 0x80
    with pytest.raises(AssertionError):
        api.forward_args(args, None, torch.device("cuda", 0))
