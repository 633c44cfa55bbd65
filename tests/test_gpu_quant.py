"""bf16 -> FP8 1x128 activation quantisation on the GPU, bit-exact against the
quantisation the reference's workloads apply (``moe_b200.workloads``:
``scale = max(amax/448, 1e-12)``, ``q = e4m3(x / scale)`` round-to-nearest-even)."""
import pytest
import torch

from moe_b200 import quantize_1x128, workloads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t,h", [(1, 512), (3, 7168), (257, 7168), (4097, 1024)])
def test_quantize_matches_reference_recipe(cuda_device, t, h):
    g = torch.Generator(device="cuda")
    g.manual_seed(t * 31 + h)
    x = torch.randn(t, h, generator=g, device="cuda").to(torch.bfloat16)
    # edge blocks: all zero, one huge value, tiny values
    x[0, :128] = 0
    if h >= 256:
        x[-1, 128:256] = 0
        x[-1, 130] = 3.0e38
    if h >= 384:
        x[t // 2, 256:384] *= 1e-30
    q, s = quantize_1x128(x)
    q_ref, s_ref = workloads.quantize_act_1x128(x)
    assert torch.equal(s, s_ref)
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))


def test_quantize_empty_and_shape_checks(cuda_device):
    q, s = quantize_1x128(torch.empty(0, 256, dtype=torch.bfloat16, device="cuda"))
    assert q.shape == (0, 256) and s.shape == (2, 0)
    with pytest.raises(AssertionError):
        quantize_1x128(torch.zeros(4, 200, dtype=torch.bfloat16, device="cuda"))


def test_quantize_then_forward_equals_workload_path(cuda_device):
    """A layer fed from bf16 through the quantiser computes what the workload
    path (torch quantisation) computes, bit for bit."""
    from moe_b200 import run
    shape = workloads.tiny_shape(40)
    inp = workloads.make_inputs(shape, seed=3, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = torch.randn(shape.t, shape.hidden, generator=g, device="cuda").to(torch.bfloat16)
    outs = []
    for q, s in (quantize_1x128(x), workloads.quantize_act_1x128(x)):
        args = workloads.run_args(inp)
        args[2], args[3] = q, s
        o = torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16, device="cuda")
        run(*args, o, n_group=shape.n_group, topk_group=shape.topk_group, top_k=shape.top_k)
        outs.append(o)
    torch.cuda.synchronize()
    assert (outs[0].float() - outs[1].float()).abs().max().item() <= 2e-3
