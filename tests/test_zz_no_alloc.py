"""The zero-allocation routing entry point, checked against the workspace path.

``moe_fp8_route_noalloc`` exists for callers that cannot allocate device
memory while the layer runs (a plugin callback in an inference engine where
allocation is forbidden, a serving loop whose memory belongs to another pool, a
foreign-language host with no device allocator).  It keeps its scratch in a
fixed array inside the library instead of a caller workspace.

Two calls in a row with different shapes must each reproduce what the existing
``moe_fp8_forward`` writes into its workspace: the array keeps the previous
call's contents, so the second call also shows that nothing leaks between
calls.  This file sorts last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import run_cuda
from moe_b200 import _lib, workloads

pytestmark = pytest.mark.gpu


def route_noalloc(inp, shape):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    t, k = shape.t, shape.top_k
    idx = torch.full((t, k), -1, dtype=torch.int32, device=dev)
    w = torch.full((t, k), float("nan"), dtype=torch.float32, device=dev)
    counts = torch.full((shape.e_local,), -1, dtype=torch.int32, device=dev)
    bias = inp["routing_bias"]
    bias_dtype = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[bias.dtype]
    code = lib.moe_fp8_route_noalloc(
        inp["routing_logits"].data_ptr(), bias.data_ptr(), bias_dtype, t, shape.e_global,
        shape.n_group, shape.topk_group, k, shape.e_local, shape.local_expert_offset,
        shape.routed_scaling_factor, idx.data_ptr(), w.data_ptr(), counts.data_ptr(),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code == 0, _lib.status_string(code)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy(), counts.cpu().numpy()


def test_noalloc_route_matches_workspace_route_twice(cuda_device):
    calls = [
        (workloads.dsv3_shape(300, e_local=32, local_expert_offset=64), 21, None),
        (workloads.dsv3_shape(4096, e_local=256), 22, torch.bfloat16),
    ]
    for shape, seed, bias_dtype in calls:
        inp = workloads.make_inputs(shape, seed=seed, device="cuda",
                                    dtype_bias=bias_dtype or torch.float32)
        _, views, _ = run_cuda(inp, shape)
        idx, w, counts = route_noalloc(inp, shape)
        np.testing.assert_array_equal(idx, views["topk_idx"].cpu().numpy())
        np.testing.assert_allclose(w, views["topk_weights"].cpu().numpy(), rtol=2e-6, atol=0)
        np.testing.assert_array_equal(counts, views["counts"].cpu().numpy())


def test_noalloc_route_rejects_sizes_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    code = lib.moe_fp8_route_noalloc(None, None, 0, 65537, 256, 8, 4, 8, 256, 0, 2.5, None,
                                     None, None, None)
    assert code == _lib.MOE_ERR_TOO_LARGE
    assert "scratch" in _lib.status_string(code)
