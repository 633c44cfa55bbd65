"""Worker for the CPU expert-parallel tests (spawned as gloo ranks).

The exchange logic of ``moe_b200.ep.ep_forward`` runs unchanged; routing and
the per-rank expert compute are the CPU oracle (test doubles standing in for
the CUDA kernels, which need a GPU).
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (os.path.join(REPO, "mlsys26-flashinfer-moe_b200"), os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import moe_oracle as mo  # noqa: E402
from moe_b200 import ep, workloads  # noqa: E402


def oracle_route(logits, bias, hs, hss, w1, w1s, w2, w2s, lo, rsf, n_group, topk_group, top_k):
    idx, _ = mo.route(logits.numpy(), bias.float().numpy(), n_group, topk_group, top_k, rsf)
    return torch.from_numpy(idx)


def oracle_expert(logits, bias, x, xs_t, w1, w1s, w2, w2s, lo, rsf, out, n_group, topk_group,
                  top_k):
    inp = dict(routing_logits=logits.numpy(), routing_bias=bias.float().numpy(),
               hidden_states=x.view(torch.uint8).numpy(), hidden_states_scale=xs_t.numpy(),
               local_expert_offset=lo, routed_scaling_factor=rsf, e_local=w1.shape[0])
    w1u, w2u = w1.view(torch.uint8).numpy(), w2.view(torch.uint8).numpy()

    def get(e):
        return w1u[e], w1s[e].numpy(), w2u[e], w2s[e].numpy()
    res = mo.moe_forward(inp, n_group, topk_group, top_k, get_expert=get)
    out.copy_(torch.from_numpy(res).to(torch.bfloat16))


def rank_inputs(shape_full, rank, tokens):
    """Weights of the whole layer (same on every rank) and this rank's tokens."""
    wts = workloads.make_inputs(shape_full, seed=77, device="cpu")
    tok = workloads.make_inputs(workloads.MoeShape(**{**shape_full.__dict__, "t": tokens}),
                                seed=500 + rank, device="cpu", weights=False)
    tok["routing_bias"] = wts["routing_bias"]       # a model parameter, shared by all ranks
    return wts, tok


def worker(rank, world, port, tokens_per_rank, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    shape = workloads.tiny_shape(1)
    t = tokens_per_rank[rank]
    wts, tok = rank_inputs(shape, rank, t)
    lo, per = ep.expert_range(rank, world, shape.e_global)
    sl = slice(lo, lo + per)
    out = torch.full((t, shape.hidden), float("nan"), dtype=torch.bfloat16)
    tim = {}
    ep.ep_forward(tok["routing_logits"], tok["routing_bias"], tok["hidden_states"],
                  tok["hidden_states_scale"], wts["gemm1_weights"][sl], wts["gemm1_weights_scale"][sl],
                  wts["gemm2_weights"][sl], wts["gemm2_weights_scale"][sl],
                  shape.routed_scaling_factor, out, n_group=shape.n_group,
                  topk_group=shape.topk_group, top_k=shape.top_k, route_fn=oracle_route,
                  expert_fn=oracle_expert, timings=tim)
    # reference: the whole layer on one process, all experts, this rank's tokens
    full = dict(mo.to_numpy_inputs(tok))
    full.update(gemm1_weights=wts["gemm1_weights"].view(torch.uint8).numpy(),
                gemm1_weights_scale=wts["gemm1_weights_scale"].numpy(),
                gemm2_weights=wts["gemm2_weights"].view(torch.uint8).numpy(),
                gemm2_weights_scale=wts["gemm2_weights_scale"].numpy(), local_expert_offset=0)
    ref = mo.moe_forward(full, shape.n_group, shape.topk_group, shape.top_k) if t else \
        np.zeros((0, shape.hidden), np.float32)
    np.savez(os.path.join(result_dir, f"rank{rank}.npz"), out=out.float().numpy(), ref=ref,
             sent=tim["rows_sent"], recv=tim["rows_received"])
    dist.destroy_process_group()


def failing_worker(rank, world, port, fail_rank, result_dir):
    """Two expert-parallel steps; rank ``fail_rank`` raises between them.

    The surviving ranks' second step must end with an error (their collective
    loses its peer, or the process group's short timeout expires) instead of
    waiting for ever; each rank writes what happened to ``result_dir``.
    """
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    torch.set_num_threads(1)
    shape = workloads.tiny_shape(1)
    wts, tok = rank_inputs(shape, rank, 6)
    lo, per = ep.expert_range(rank, world, shape.e_global)
    sl = slice(lo, lo + per)

    def step():
        out = torch.empty(6, shape.hidden, dtype=torch.bfloat16)
        ep.ep_forward(tok["routing_logits"], tok["routing_bias"], tok["hidden_states"],
                      tok["hidden_states_scale"], wts["gemm1_weights"][sl],
                      wts["gemm1_weights_scale"][sl], wts["gemm2_weights"][sl],
                      wts["gemm2_weights_scale"][sl], shape.routed_scaling_factor, out,
                      n_group=shape.n_group, topk_group=shape.topk_group, top_k=shape.top_k,
                      route_fn=oracle_route, expert_fn=oracle_expert)
        return out

    step()
    path = os.path.join(result_dir, f"rank{rank}.txt")
    if rank == fail_rank:
        with open(path, "w") as f:
            f.write("raised")
        raise RuntimeError(f"injected failure on rank {rank} between steps")
    t0 = time.time()
    try:
        step()
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - the test inspects the outcome
        outcome = f"error {type(e).__name__}"
    with open(path, "w") as f:
        f.write(f"{outcome}\n{time.time() - t0:.2f}")
    os._exit(0)   # the group is broken: no destroy_process_group
