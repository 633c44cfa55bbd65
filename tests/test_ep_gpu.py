"""Expert parallelism over NCCL: one rank (any GPU box) and two ranks (skipped
with fewer GPUs).

Each rank holds 256/W of the experts and its own tokens; the layer output of
every rank's tokens must match the single-GPU kernel with all experts on that
GPU, within the output tolerance (partials travel as bf16).  The bf16 variants
start from bf16 activations (``ep_forward_bf16``, config 4) and compare with the
same activations quantised by ``quantize_1x128`` and run on one GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir, bf16=False, fused=False, steps=1):
    import datetime
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(repo, "mlsys26-flashinfer-moe_b200"))
    import torch.distributed as dist
    from moe_b200 import ep, quantize_1x128, run, workloads
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    # DeepSeek-V3 routing (256 experts, 8 groups / top-4, top-8) on a narrow layer
    full = workloads.MoeShape(t=1, hidden=512, inter=256)
    wts = workloads.make_inputs(full, seed=3, device="cuda")
    t = 300 + 57 * rank
    tok = workloads.make_inputs(workloads.MoeShape(t=t, hidden=512, inter=256), seed=40 + rank,
                                device="cuda", weights=False)
    tok["routing_bias"] = wts["routing_bias"]
    lo, per = ep.expert_range(rank, world, 256)
    sl = slice(lo, lo + per)
    out = torch.empty(t, 512, dtype=torch.bfloat16, device="cuda")
    shard = (wts["gemm1_weights"][sl].contiguous(), wts["gemm1_weights_scale"][sl].contiguous(),
             wts["gemm2_weights"][sl].contiguous(), wts["gemm2_weights_scale"][sl].contiguous())
    if fused:
        layer = ep.FusedEP(400, 512, 256, 256)
        for _ in range(steps):     # repeated steps reuse every exchange buffer
            out.fill_(float("nan"))
            if bf16:
                g = torch.Generator(device="cuda")
                g.manual_seed(70 + rank)
                x = torch.randn(t, 512, generator=g, device="cuda").to(torch.bfloat16)
                layer.forward_bf16(tok["routing_logits"], tok["routing_bias"], x, *shard, 2.5, out)
                tok["hidden_states"], tok["hidden_states_scale"] = quantize_1x128(x)
            else:
                layer.forward(tok["routing_logits"], tok["routing_bias"], tok["hidden_states"],
                              tok["hidden_states_scale"], *shard, 2.5, out)
        torch.cuda.synchronize()
        assert layer.device_error() == (0, 0)
    elif bf16:
        g = torch.Generator(device="cuda")
        g.manual_seed(70 + rank)
        x = torch.randn(t, 512, generator=g, device="cuda").to(torch.bfloat16)
        ep.ep_forward_bf16(tok["routing_logits"], tok["routing_bias"], x, *shard, 2.5, out)
        tok["hidden_states"], tok["hidden_states_scale"] = quantize_1x128(x)
    else:
        ep.ep_forward(tok["routing_logits"], tok["routing_bias"], tok["hidden_states"],
                      tok["hidden_states_scale"], *shard, 2.5, out)
    ref = torch.empty_like(out)
    run(tok["routing_logits"], tok["routing_bias"], tok["hidden_states"],
        tok["hidden_states_scale"], wts["gemm1_weights"], wts["gemm1_weights_scale"],
        wts["gemm2_weights"], wts["gemm2_weights_scale"], 0, 2.5, ref)
    torch.cuda.synchronize()
    np.savez(os.path.join(out_dir, f"gpu_rank{rank}.npz"), out=out.float().cpu().numpy(),
             ref=ref.float().cpu().numpy())
    dist.barrier()
    if fused:
        layer.close()
    dist.destroy_process_group()


def _check(tmp_path, world):
    for r in range(world):
        d = np.load(tmp_path / f"gpu_rank{r}.npz")
        assert np.isfinite(d["out"]).all()
        np.testing.assert_allclose(d["out"], d["ref"], atol=1e-2, rtol=2e-2)
        cos = float((d["out"] * d["ref"]).sum() /
                    (np.linalg.norm(d["out"]) * np.linalg.norm(d["ref"])))
        assert cos >= 0.9999


def test_ep_one_gpu_from_bf16(tmp_path, cuda_device):
    mp.spawn(_worker, args=(1, _free_port(), str(tmp_path), True), nprocs=1, join=True)
    _check(tmp_path, 1)


@pytest.mark.parametrize("bf16", [False, True])
def test_fused_ep_one_gpu(tmp_path, cuda_device, bf16):
    """The NVLink dispatch/combine path with one rank (its own peer)."""
    mp.spawn(_worker, args=(1, _free_port(), str(tmp_path), bf16, True, 3), nprocs=1, join=True)
    _check(tmp_path, 1)


@pytest.mark.parametrize("bf16,fused", [(False, False), (True, False), (False, True),
                                        (True, True)])
def test_ep_two_gpus_match_single_gpu(tmp_path, bf16, fused):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), bf16, fused, 3), nprocs=2, join=True)
    _check(tmp_path, 2)
