"""Expert-parallel exchange (``moe_b200.ep``) on CPU gloo ranks.

The dispatch / combine logic runs exactly as on GPUs; routing and expert
compute are the CPU oracle.  Each rank's result must equal the single-process
layer over all experts for that rank's tokens, within the output tolerance
(the partial sums travel as bf16, as on the GPU path).
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import ep_worker


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,tokens", [(2, [24, 17]), (4, [9, 0, 13, 5])])
def test_ep_matches_single_process(tmp_path, world, tokens):
    mp.spawn(ep_worker.worker, args=(world, free_port(), tokens, str(tmp_path)), nprocs=world,
             join=True)
    sent_total = recv_total = 0
    for r in range(world):
        d = np.load(tmp_path / f"rank{r}.npz")
        assert d["out"].shape == d["ref"].shape
        assert np.isfinite(d["out"]).all()
        np.testing.assert_allclose(d["out"], d["ref"], atol=1e-2, rtol=2e-2)
        sent_total += int(d["sent"])
        recv_total += int(d["recv"])
    assert sent_total == recv_total          # every dispatched row arrived once


def test_rank_failure_between_steps_ends_in_an_error_not_a_hang(tmp_path):
    """Failure detection on the host: rank 1 raises after the first step; rank
    0's second step must raise within the process group's timeout (20 s) rather
    than wait for ever."""
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=ep_worker.failing_worker, args=(r, 2, port, 1, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    assert not alive, "a rank was still waiting after 90 s"
    assert procs[1].exitcode != 0
    assert (tmp_path / "rank1.txt").read_text() == "raised"
    outcome, secs = (tmp_path / "rank0.txt").read_text().split("\n")
    assert outcome.startswith("error"), outcome
    assert float(secs) < 60
