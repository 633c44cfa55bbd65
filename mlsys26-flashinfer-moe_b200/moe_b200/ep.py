"""Expert parallelism for the fused FP8 MoE layer: one process per GPU.

The reference already expresses an expert shard in its API
(``local_expert_offset`` + a contiguous weight slice, kernel.py:572, 271-272)
but leaves the exchange of tokens to the caller.  This module provides it:
rank ``r`` of ``W`` owns experts ``[r*E/W, (r+1)*E/W)`` and its own tokens, and
one forward is

1. route the rank's tokens (``moe_fp8_route``) to find, per token, the ranks
   that own at least one of its experts;
2. exchange per-destination row counts (all-to-all of ``W`` ints, the only
   host synchronisation: NCCL needs split sizes on the host);
3. dispatch each token's FP8 row, its 1x128 scales and its router logits once
   per destination rank (deduplicated), all-to-all-v over NCCL;
4. run the fused layer (``moe_fp8_forward``) on the received rows with the
   local expert slice; re-routing the received logits on the destination gives
   exactly the source's expert choice (routing is a pure function of logits and
   bias), and the kernel keeps only local experts;
5. send the bf16 partial outputs back (all-to-all-v) and add them per token in
   fixed rank order in fp32.

Steps 1 and 4 are pluggable (``route_fn``, ``expert_fn``) so that the exchange
logic runs on CPU ``gloo`` ranks in tests with the oracle as the expert
compute; the product path uses the CUDA kernels and NCCL.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib, api


def expert_range(rank: int, world: int, e_global: int):
    assert e_global % world == 0, "experts must split evenly over ranks"
    per = e_global // world
    return rank * per, per


def cuda_route(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
               gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
               routed_scaling_factor, n_group, topk_group, top_k):
    """topk_idx [T, top_k] int32 of the rank's own tokens via ``moe_fp8_route``."""
    t, h = hidden_states.shape
    dummy = torch.empty(t, h, dtype=torch.bfloat16, device=hidden_states.device)
    args, keep, _ = api.build_args(routing_logits, routing_bias, hidden_states,
                                   hidden_states_scale, gemm1_weights, gemm1_weights_scale,
                                   gemm2_weights, gemm2_weights_scale, local_expert_offset,
                                   routed_scaling_factor, dummy, n_group, topk_group, top_k)
    lay = api.workspace_layout(args)
    stream = torch.cuda.current_stream()
    ws = api.get_workspace(lay.total_bytes, hidden_states.device, stream)
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    code = _lib.load().moe_fp8_route(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream))
    if code:
        raise _lib.MoeError(code, "moe_fp8_route")
    return api.workspace_views(args, ws)["topk_idx"].clone()


def cuda_expert(logits, bias, x, xs_t, w1, w1s, w2, w2s, offset, rsf, out, n_group, topk_group,
                top_k):
    api.run(logits, bias, x, xs_t, w1, w1s, w2, w2s, offset, rsf, out, n_group=n_group,
            topk_group=topk_group, top_k=top_k)


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group):
    """all_to_all_single on byte views (NCCL has no fp8 type)."""
    o = out.view(torch.uint8) if out.dtype in (torch.float8_e4m3fn,) else out
    i = inp.view(torch.uint8) if inp.dtype in (torch.float8_e4m3fn,) else inp
    dist.all_to_all_single(o, i, out_splits, in_splits, group=group)


@torch.no_grad()
def ep_forward(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
               gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor,
               output, *, group=None, n_group=8, topk_group=4, top_k=8,
               route_fn: Optional[Callable] = None, expert_fn: Optional[Callable] = None,
               timings: Optional[dict] = None):
    """Expert-parallel forward of this rank's tokens; writes bf16 ``output``.

    ``gemm*_weights`` are this rank's contiguous expert slice (``E/W`` experts
    starting at ``rank*E/W``); ``routing_bias`` is the layer's bias and must be
    the same on every rank (destinations re-route the rows they receive).  All
    ranks must call together (collectives).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    t, h = hidden_states.shape
    e_global = routing_logits.shape[1]
    lo, per = expert_range(rank, world, e_global)
    assert gemm1_weights.shape[0] == per, "weights must be this rank's expert slice"
    dev = hidden_states.device
    route_fn = route_fn or cuda_route
    expert_fn = expert_fn or cuda_expert

    # 1. destinations of every token
    idx = route_fn(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                   gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, lo,
                   routed_scaling_factor, n_group, topk_group, top_k)
    dest = (idx.long() // per)                                   # [T, top_k]
    mask = torch.zeros(t, world, dtype=torch.bool, device=dev)
    if t:
        mask.scatter_(1, dest, True)
    pairs = mask.t().nonzero()                                   # (rank, token), rank-major
    send_tok = pairs[:, 1].contiguous()
    send_counts = mask.sum(0).to(torch.int64)

    # 2. counts exchange (host sync for the NCCL split sizes)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    sc = send_counts.tolist()
    rc = recv_counts.tolist()
    n_recv = int(sum(rc))

    # 3. dispatch FP8 rows, scales (row-major) and logits, once per destination
    send_x = hidden_states.index_select(0, send_tok)
    send_s = hidden_states_scale.index_select(1, send_tok).t().contiguous()
    send_l = routing_logits.index_select(0, send_tok)
    recv_x = torch.empty(n_recv, h, dtype=hidden_states.dtype, device=dev)
    recv_s = torch.empty(n_recv, h // 128, dtype=torch.float32, device=dev)
    recv_l = torch.empty(n_recv, e_global, dtype=torch.float32, device=dev)
    _a2a(recv_x, send_x, rc, sc, group)
    _a2a(recv_s, send_s, rc, sc, group)
    _a2a(recv_l, send_l, rc, sc, group)

    # 4. local experts on the received rows
    part = torch.empty(n_recv, h, dtype=torch.bfloat16, device=dev)
    if n_recv:
        expert_fn(recv_l, routing_bias, recv_x, recv_s.t().contiguous(), gemm1_weights,
                  gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, lo,
                  routed_scaling_factor, part, n_group, topk_group, top_k)

    # 5. combine: partial rows back to their source, fixed-order fp32 sum
    back = torch.empty(len(send_tok), h, dtype=torch.bfloat16, device=dev)
    _a2a(back, part, sc, rc, group)
    acc = torch.zeros(t, h, dtype=torch.float32, device=dev)
    start = 0
    for d in range(world):
        n = sc[d]
        if n:
            acc.index_add_(0, send_tok[start:start + n], back[start:start + n].float())
        start += n
    output.copy_(acc.to(torch.bfloat16))
    if timings is not None:
        timings["rows_sent"] = len(send_tok)
        timings["rows_received"] = n_recv
    return output


def ep_forward_bf16(routing_logits, routing_bias, hidden_states_bf16, gemm1_weights,
                    gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                    routed_scaling_factor, output, **kw):
    """``ep_forward`` for a layer that starts from bf16 activations: this rank's
    tokens are quantised to e4m3 with 1x128 scales on the GPU
    (``moe_bf16_to_fp8_1x128``) before routing, so only FP8 rows and their scales
    cross NVLink in the dispatch."""
    hs, hss = api.quantize_1x128(hidden_states_bf16)
    return ep_forward(routing_logits, routing_bias, hs, hss, gemm1_weights, gemm1_weights_scale,
                      gemm2_weights, gemm2_weights_scale, routed_scaling_factor, output, **kw)


class FusedEP:
    """Expert-parallel layer whose dispatch and combine are this library's own
    kernels storing over NVLink into peer ranks' buffers (``moe_ep_*`` in
    ``include/moe_b200.h``); NCCL only all-gathers the per-rank row counts
    (``world*world`` ints, on the device) and orders the phases.

    Build once per process group and layer shape (collective: every rank calls
    it together), then call ``forward`` on every rank with its own tokens.
    """

    def __init__(self, t_max: int, hidden: int, inter: int, e_global: int = 256, *,
                 n_group: int = 8, topk_group: int = 4, top_k: int = 8, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.t_max, self.hidden, self.inter, self.e_global = t_max, hidden, inter, e_global
        self.n_group, self.topk_group, self.top_k = n_group, topk_group, top_k
        self.lo, self.per = expert_range(self.rank, self.world, e_global)
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        cfg = _lib.MoeEpConfig(self.world, self.rank, t_max, hidden, inter, e_global, n_group,
                               topk_group, top_k)
        h = ctypes.c_void_p()
        code = lib.moe_ep_create(ctypes.byref(cfg), ctypes.byref(h))
        if code:
            api._raise(code, "moe_ep_create")
        self._h = h
        handle = (ctypes.c_ubyte * 64)()
        code = lib.moe_ep_ipc_handle(self._h, ctypes.cast(handle, ctypes.c_void_p))
        if code:
            api._raise(code, "moe_ep_ipc_handle")
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        allh = torch.empty(self.world * 64, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allh, mine, group=group)
        code = lib.moe_ep_connect(self._h, bytes(allh.cpu().tolist()))
        if code:
            api._raise(code, "moe_ep_connect")
        dist.barrier(group=group)
        self.send_cnt = torch.zeros(self.world, dtype=torch.int32, device=self.device)
        self.cnt_all = torch.zeros(self.world * self.world, dtype=torch.int32, device=self.device)
        self._bar = torch.zeros(1, dtype=torch.int32, device=self.device)

    def _barrier(self):
        dist.all_reduce(self._bar, group=self.group)

    @torch.no_grad()
    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                routed_scaling_factor, output, events: Optional[list] = None):
        """Same arguments as ``ep_forward`` (this rank's tokens and expert slice,
        the layer's bias); writes bf16 ``output`` [T, H].  ``events``: optional
        list of 8 timing-enabled CUDA events recorded at the stage boundaries
        (start, send plan, count all-gather, dispatch, barrier, experts + combine,
        barrier, finalize)."""
        t, h = hidden_states.shape
        assert t <= self.t_max and h == self.hidden, "tokens exceed T_max or hidden mismatch"
        assert gemm1_weights.shape == (self.per, 2 * self.inter, h), "weights must be this rank's slice"
        assert routing_logits.shape == (t, self.e_global) and routing_logits.dtype == torch.float32
        assert hidden_states.dtype == torch.float8_e4m3fn and output.dtype == torch.bfloat16
        assert routing_bias.dtype in api._BIAS_DTYPES
        for x in (routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                  gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, output):
            assert x.is_cuda and x.is_contiguous(), "tensors must be contiguous CUDA tensors"
        lib = _lib.load()
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        bdt = api._BIAS_DTYPES[routing_bias.dtype]
        rsf = float(routed_scaling_factor)

        def chk(code, where):
            if code:
                api._raise(code, where)

        def mark(i):
            if events is not None:
                events[i].record()
        mark(0)
        chk(lib.moe_ep_send_plan(self._h, routing_logits.data_ptr(), routing_bias.data_ptr(), bdt,
                                 t, rsf, self.send_cnt.data_ptr(), st), "moe_ep_send_plan")
        mark(1)
        dist.all_gather_into_tensor(self.cnt_all, self.send_cnt, group=self.group)
        mark(2)
        chk(lib.moe_ep_dispatch(self._h, hidden_states.data_ptr(), hidden_states_scale.data_ptr(),
                                routing_logits.data_ptr(), t, self.cnt_all.data_ptr(), st),
            "moe_ep_dispatch")
        mark(3)
        self._barrier()
        mark(4)
        chk(lib.moe_ep_experts(self._h, routing_bias.data_ptr(), bdt, rsf,
                               gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr(),
                               gemm2_weights.data_ptr(), gemm2_weights_scale.data_ptr(),
                               self.cnt_all.data_ptr(), st), "moe_ep_experts")
        mark(5)
        self._barrier()
        mark(6)
        chk(lib.moe_ep_finalize(self._h, t, output.data_ptr(), st), "moe_ep_finalize")
        mark(7)
        return output

    def forward_bf16(self, routing_logits, routing_bias, hidden_states_bf16, *weights_and_rest,
                     events: Optional[list] = None):
        """``forward`` from bf16 activations, quantised 1x128 on the GPU first."""
        hs, hss = api.quantize_1x128(hidden_states_bf16)
        return self.forward(routing_logits, routing_bias, hs, hss, *weights_and_rest,
                            events=events)

    def device_error(self):
        code, info = ctypes.c_int32(0), ctypes.c_int32(0)
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        if _lib.load().moe_ep_device_error(self._h, st, ctypes.byref(code), ctypes.byref(info)):
            raise RuntimeError("moe_ep_device_error failed")
        return code.value, info.value

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().moe_ep_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
