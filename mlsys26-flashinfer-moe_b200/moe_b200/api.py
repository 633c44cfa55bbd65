"""Host side of the drop-in: the reference's ``run()`` entry point over the C ABI.

``run`` keeps the reference's positional signature, destination-passing style
and error behaviour (``kernel.py:562-729``):

* dtype and shape violations raise ``AssertionError`` (kernel.py:591-607);
* a missing CUDA device raises ``RuntimeError`` (kernel.py:552-559);
* CPU inputs are moved to the GPU (kernel.py:544-549);
* the bf16 result is written into ``output`` and ``None`` is returned.

Differences, all additive: shapes are taken from the tensors instead of being
hard-coded to 32 of 256 experts (kernel.py:577-588), the routing
hyper-parameters are keyword-only arguments with the DeepSeek-V3 defaults, and
the whole layer runs without a single device-to-host synchronisation (the
reference blocks three times, kernel.py:361, 394, 661).

All arithmetic happens in ``libmoe_b200.so``; this module only validates,
allocates the workspace through the torch caching allocator and passes raw
pointers.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_F8 = torch.float8_e4m3fn
_BIAS_DTYPES = {torch.float32: _lib.MOE_BIAS_F32, torch.bfloat16: _lib.MOE_BIAS_BF16,
                torch.float16: _lib.MOE_BIAS_F16}

# One workspace per (device, stream): calls on different streams must not share
# scratch.  Grown on demand, never shrunk.
_workspaces: dict = {}


def _ensure_cuda(*tensors) -> torch.device:
    """kernel.py:552-559."""
    if not torch.cuda.is_available():
        for t in tensors:
            if isinstance(t, torch.Tensor) and t.is_cuda:
                raise RuntimeError("CUDA inputs provided but CUDA is reported unavailable.")
        raise RuntimeError("CUDA is required to run this kernel; no CUDA device available.")
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return t.device
    return torch.device("cuda", torch.cuda.current_device())


def _to_device(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    """kernel.py:544-549, plus ``.contiguous()`` (615-622)."""
    if t.device != device:
        t = t.to(device, non_blocking=True)
    return t.contiguous()


def build_args(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
               gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
               local_expert_offset: int, routed_scaling_factor: float, output: torch.Tensor,
               n_group: int = 8, topk_group: int = 4, top_k: int = 8,
               deterministic: bool = False, gemm2_weights_bf16: Optional[torch.Tensor] = None,
               debug: bool = False, n_shared_experts: int = 0):
    """Validate like the reference and fill a ``MoeFwdArgs`` (no workspace yet).

    ``deterministic`` selects the fixed-order combine (``MOE_FLAG_DETERMINISTIC``):
    bit-identical output from run to run, at the cost of one fp32 row per
    (token, expert) assignment in the workspace.  ``gemm2_weights_bf16``: the
    same down-projection weights prepared by ``prepare_gemm2_weights`` (bf16
    GEMM2 without block-scale promotion on the prefill path).  ``debug`` sets
    ``MOE_FLAG_DEBUG`` (device checks of the dispatch tables and workspace
    guards).  ``n_shared_experts=1``: the weight tensors hold the local routed
    experts followed by DeepSeek-V3's shared expert (``[E_local + 1, ...]``),
    which every token also goes through with weight 1.

    Returns ``(args, keepalive, out_dev)``: ``keepalive`` holds the device
    copies the pointers refer to; ``out_dev`` is where the kernel writes (the
    caller's ``output`` itself whenever it is a contiguous bf16 CUDA tensor).
    """
    assert hidden_states.dtype == _F8, "hidden_states must be FLOAT8_E4M3FN"
    assert gemm1_weights.dtype == _F8, "gemm1_weights must be FLOAT8_E4M3FN"
    assert gemm2_weights.dtype == _F8, "gemm2_weights must be FLOAT8_E4M3FN"
    assert routing_logits.dtype == torch.float32, "routing_logits must be float32"
    assert routing_bias.dtype in _BIAS_DTYPES, "routing_bias must be float or bf16/fp16"
    assert hidden_states_scale.dtype == torch.float32, "hidden_states_scale must be float32"
    assert gemm1_weights_scale.dtype == torch.float32, "gemm1_weights_scale must be float32"
    assert gemm2_weights_scale.dtype == torch.float32, "gemm2_weights_scale must be float32"
    assert routing_logits.dim() == 2, "routing_logits must be [T, E_global]"
    t, e_global = int(routing_logits.shape[0]), int(routing_logits.shape[1])
    assert gemm1_weights.dim() == 3, "gemm1_weights must be [E_local, 2I, H]"
    assert n_shared_experts in (0, 1), "n_shared_experts must be 0 or 1"
    e_all, i2, h = (int(x) for x in gemm1_weights.shape)
    e_local = e_all - int(n_shared_experts)   # routed experts; the shared one follows them
    assert e_local >= 1, "gemm1_weights must hold at least one routed expert"
    i = i2 // 2
    assert i2 == 2 * i, "gemm1_weights second dim must be 2*I"
    assert routing_bias.numel() == e_global, f"routing_bias must have {e_global} entries"
    assert hidden_states.shape == (t, h), f"hidden_states must be [{t}, {h}]"
    assert hidden_states_scale.shape == (h // 128, t), f"hidden_states_scale must be [{h // 128}, {t}]"
    assert gemm1_weights_scale.shape == (e_all, i2 // 128, h // 128), \
        f"gemm1_weights_scale must be [{e_all}, {i2 // 128}, {h // 128}]"
    assert gemm2_weights.shape == (e_all, h, i), f"gemm2_weights must be [{e_all}, {h}, {i}]"
    assert gemm2_weights_scale.shape == (e_all, h // 128, i // 128), \
        f"gemm2_weights_scale must be [{e_all}, {h // 128}, {i // 128}]"
    assert output.shape == (t, h), f"output must be [{t}, {h}]"
    assert 0 <= int(local_expert_offset) and int(local_expert_offset) + e_local <= e_global, \
        "local experts must lie inside [0, E_global)"

    device = _ensure_cuda(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                          gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                          output)
    tensors = [_to_device(x, device) for x in
               (routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)]
    if output.is_cuda and output.device == device and output.dtype == torch.bfloat16 and \
            output.is_contiguous():
        out_dev = output
    else:
        out_dev = torch.empty((t, h), dtype=torch.bfloat16, device=device)
    a = _lib.MoeFwdArgs()
    (a.routing_logits, a.routing_bias, a.hidden_states, a.hidden_states_scale, a.gemm1_weights,
     a.gemm1_weights_scale, a.gemm2_weights, a.gemm2_weights_scale) = (x.data_ptr()
                                                                       for x in tensors)
    a.output = out_dev.data_ptr()
    a.T, a.H, a.I, a.E_global, a.E_local = t, h, i, e_global, e_local
    a.local_expert_offset = int(local_expert_offset)
    a.n_group, a.topk_group, a.top_k = int(n_group), int(topk_group), int(top_k)
    a.routed_scaling_factor = float(routed_scaling_factor)
    a.bias_dtype = _BIAS_DTYPES[routing_bias.dtype]
    a.flags = (_lib.MOE_FLAG_DETERMINISTIC if deterministic else 0) | \
        (_lib.MOE_FLAG_DEBUG if debug else 0)
    a.n_shared_experts = int(n_shared_experts)
    if gemm2_weights_bf16 is not None:
        assert gemm2_weights_bf16.dtype == torch.bfloat16 and \
            gemm2_weights_bf16.shape == (e_local, h, i), \
            f"gemm2_weights_bf16 must be bf16 [{e_local}, {h}, {i}] (prepare_gemm2_weights)"
        wb = _to_device(gemm2_weights_bf16, device)
        tensors.append(wb)
        a.gemm2_weights_bf16 = wb.data_ptr()
    return a, tensors, out_dev


def _raise(code: int, where: str):
    if code in (_lib.MOE_ERR_SHAPE, _lib.MOE_ERR_INVALID_ARG):
        raise AssertionError(f"{where}: {_lib.status_string(code)}")
    raise _lib.MoeError(code, where)


def workspace_layout(args: _lib.MoeFwdArgs) -> _lib.MoeWorkspaceLayout:
    lay = _lib.MoeWorkspaceLayout()
    code = _lib.load().moe_fp8_workspace_layout(ctypes.byref(args), ctypes.byref(lay))
    if code:
        _raise(code, "moe_fp8_workspace_layout")
    return lay


def get_workspace(nbytes: int, device: torch.device, stream: torch.cuda.Stream) -> torch.Tensor:
    key = (device.index, stream.cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def forward_args(args: _lib.MoeFwdArgs, workspace: Optional[torch.Tensor], device: torch.device):
    """Run ``moe_fp8_forward`` on the current stream; returns the workspace."""
    lib = _lib.load()
    stream = torch.cuda.current_stream(device)
    lay = workspace_layout(args)
    if workspace is None:
        workspace = get_workspace(lay.total_bytes, device, stream)
    args.workspace = workspace.data_ptr()
    args.workspace_bytes = workspace.numel() * workspace.element_size()
    code = lib.moe_fp8_forward(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream))
    if code:
        _raise(code, "moe_fp8_forward")
    return workspace


@torch.no_grad()
def run(routing_logits: torch.Tensor, routing_bias: torch.Tensor, hidden_states: torch.Tensor,
        hidden_states_scale: torch.Tensor, gemm1_weights: torch.Tensor,
        gemm1_weights_scale: torch.Tensor, gemm2_weights: torch.Tensor,
        gemm2_weights_scale: torch.Tensor, local_expert_offset: int,
        routed_scaling_factor: float, output: torch.Tensor, *, n_group: int = 8,
        topk_group: int = 4, top_k: int = 8, workspace: Optional[torch.Tensor] = None,
        deterministic: bool = False,
        gemm2_weights_bf16: Optional[torch.Tensor] = None, debug: bool = False,
        n_shared_experts: int = 0) -> None:
    """Fused FP8 block-scale DeepSeek-V3 MoE forward (reference ``kernel.py:562``).

    Writes the bf16 ``[T, H]`` layer output into ``output``.  Only the experts
    ``[local_expert_offset, local_expert_offset + E_local)`` whose weights are
    passed contribute.  ``workspace`` (uint8 CUDA tensor) may be supplied to
    avoid the internal per-stream cache.  ``deterministic=True`` adds each
    token's expert rows in a fixed order (bit-identical runs) instead of with
    fp32 atomics as the reference does (kernel.py:246-250).
    ``gemm2_weights_bf16`` (from ``prepare_gemm2_weights(gemm2_weights,
    gemm2_weights_scale)``, made once for a layer's weights) runs the prefill
    GEMM2 on bf16 operands; decode-sized batches ignore it.  ``debug=True``
    checks the routing and dispatch tables on the device before the GEMMs use
    them and guards every workspace buffer; it then waits for the forward and
    raises ``MoeError`` (a ``RuntimeError``) naming the failed check.
    ``n_shared_experts=1`` adds DeepSeek-V3's shared expert, passed as the last
    slice of each weight tensor (``[E_local + 1, ...]``), with weight 1; the
    reference computes the routed sum only.
    """
    args, keep, out_dev = build_args(routing_logits, routing_bias, hidden_states,
                                     hidden_states_scale, gemm1_weights, gemm1_weights_scale,
                                     gemm2_weights, gemm2_weights_scale, local_expert_offset,
                                     routed_scaling_factor, output, n_group, topk_group, top_k,
                                     deterministic, gemm2_weights_bf16, debug,
                                     n_shared_experts)
    device = keep[0].device
    if args.T > 0:
        forward_args(args, workspace, device)
        if debug:
            raise_device_error(args, "moe_fp8_forward (debug)")
    if out_dev is not output:
        output.copy_(out_dev)
    return None


def prepare_gemm2_weights(gemm2_weights: torch.Tensor, gemm2_weights_scale: torch.Tensor,
                          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One-time relayout of a layer's down-projection weights for the bf16
    GEMM2: ``bf16(W2 * block scale)`` as ``[E_local, H, I]`` (twice the bytes of
    the FP8 weights).  Pass the result to ``run(..., gemm2_weights_bf16=...)``
    for every forward with these weights."""
    assert gemm2_weights.dtype == _F8 and gemm2_weights.dim() == 3, "gemm2_weights must be e4m3 [E, H, I]"
    assert gemm2_weights.is_cuda, "gemm2_weights must be a CUDA tensor"
    e, h, i = (int(x) for x in gemm2_weights.shape)
    assert gemm2_weights_scale.dtype == torch.float32 and \
        gemm2_weights_scale.shape == (e, h // 128, i // 128)
    w = gemm2_weights.contiguous()
    s = gemm2_weights_scale.to(w.device).contiguous()
    if out is None:
        out = torch.empty(e, h, i, dtype=torch.bfloat16, device=w.device)
    stream = torch.cuda.current_stream(w.device)
    code = _lib.load().moe_fp8_prepare_gemm2_bf16(w.data_ptr(), s.data_ptr(), e, h, i,
                                                 out.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
    if code:
        _raise(code, "moe_fp8_prepare_gemm2_bf16")
    return out


_router_ws: dict = {}


def router_logits(x: torch.Tensor, w_gate: torch.Tensor, out: Optional[torch.Tensor] = None,
                  workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Router logits ``x @ w_gate.T`` for bf16 ``x [T, H]`` and ``w_gate [E, H]`` (CUDA),
    fp32 ``[T, E]`` on the current stream: the ``routing_logits`` input of ``run()``.
    Products of the bf16 values are exact in fp32 and summed in fp32; large
    batches run on the tensor cores and use ``workspace`` (an internal cached
    buffer per stream when omitted)."""
    assert x.dtype == torch.bfloat16 and x.dim() == 2, "x must be a bf16 [T, H] tensor"
    assert w_gate.dtype == torch.bfloat16 and w_gate.dim() == 2, "w_gate must be a bf16 [E, H] tensor"
    assert x.is_cuda and w_gate.is_cuda, "x and w_gate must be CUDA tensors"
    t, h = (int(v) for v in x.shape)
    e = int(w_gate.shape[0])
    assert int(w_gate.shape[1]) == h, f"w_gate must be [E, {h}]"
    x, w_gate = x.contiguous(), w_gate.contiguous()
    if out is None:
        out = torch.empty(t, e, dtype=torch.float32, device=x.device)
    assert out.shape == (t, e) and out.dtype == torch.float32 and out.is_contiguous()
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    code = lib.moe_router_workspace_size(t, h, e, ctypes.byref(nbytes))
    if code:
        _raise(code, "moe_router_workspace_size")
    stream = torch.cuda.current_stream(x.device)
    ws_ptr, ws_bytes = None, 0
    if nbytes.value:
        if workspace is None:
            key = (x.device.index, stream.cuda_stream)
            workspace = _router_ws.get(key)
            if workspace is None or workspace.numel() < nbytes.value:
                workspace = torch.empty(nbytes.value, dtype=torch.uint8, device=x.device)
                _router_ws[key] = workspace
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel()
    code = lib.moe_router_logits_bf16(x.data_ptr(), w_gate.data_ptr(), t, h, e, out.data_ptr(),
                                      ws_ptr, ws_bytes, ctypes.c_void_p(stream.cuda_stream))
    if code:
        _raise(code, "moe_router_logits_bf16")
    return out


def quantize_1x128(x: torch.Tensor, q: Optional[torch.Tensor] = None,
                   scale: Optional[torch.Tensor] = None):
    """bf16 ``[T, H]`` CUDA activations -> (e4m3 ``[T, H]``, fp32 ``[H/128, T]``) on the
    current stream: ``scale = max(amax/448, 1e-12)`` per token and 128 columns and
    ``q = e4m3(x / scale)``, the layout ``run()`` takes as ``hidden_states`` /
    ``hidden_states_scale`` (reference ``kernel.py:603``)."""
    assert x.dtype == torch.bfloat16 and x.dim() == 2, "x must be a bf16 [T, H] tensor"
    assert x.is_cuda, "x must be a CUDA tensor"
    x = x.contiguous()
    t, h = x.shape
    assert h % 128 == 0, "H must be a multiple of 128"
    if q is None:
        q = torch.empty(t, h, dtype=_F8, device=x.device)
    if scale is None:
        scale = torch.empty(h // 128, t, dtype=torch.float32, device=x.device)
    assert q.shape == (t, h) and q.dtype == _F8 and q.is_contiguous()
    assert scale.shape == (h // 128, t) and scale.dtype == torch.float32 and scale.is_contiguous()
    stream = torch.cuda.current_stream(x.device)
    code = _lib.load().moe_bf16_to_fp8_1x128(x.data_ptr(), t, h, q.data_ptr(), scale.data_ptr(),
                                            ctypes.c_void_p(stream.cuda_stream))
    if code:
        _raise(code, "moe_bf16_to_fp8_1x128")
    return q, scale


def device_error(args: _lib.MoeFwdArgs, stream: Optional[torch.cuda.Stream] = None):
    """(code, info) of the device-side error word of the last forward on the
    workspace in ``args``; blocks on the stream."""
    stream = stream or torch.cuda.current_stream()
    code, info = ctypes.c_int32(0), ctypes.c_int32(0)
    st = _lib.load().moe_fp8_device_error(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream),
                                          ctypes.byref(code), ctypes.byref(info))
    if st:
        _raise(st, "moe_fp8_device_error")
    return code.value, info.value


def describe_error(code: int, info: int) -> str:
    """Text for a device error word: the failed check and index of
    ``MOE_ERR_BOUNDS``, the wait site of ``MOE_ERR_TIMEOUT``."""
    if code == _lib.MOE_ERR_BOUNDS:
        site = _lib.CHECK_SITES.get((info >> 24) & 0xFF, "unknown")
        return f"{_lib.status_string(code)}: check '{site}' at index {info & 0xFFFFFF}"
    if code == _lib.MOE_ERR_TIMEOUT:
        return f"{_lib.status_string(code)} at wait site {info}"
    return f"{_lib.status_string(code)} (info {info})"


def raise_device_error(args: _lib.MoeFwdArgs, where: str,
                       stream: Optional[torch.cuda.Stream] = None) -> None:
    """Waits for the stream and raises ``MoeError`` if the device error word
    of the workspace in ``args`` is set."""
    code, info = device_error(args, stream)
    if code:
        err = _lib.MoeError(code, where)
        err.args = (f"{where}: {describe_error(code, info)}",)
        err.info = info
        raise err


def check_workspace(args: _lib.MoeFwdArgs, stream: Optional[torch.cuda.Stream] = None):
    """Runs ``moe_fp8_check_workspace`` on the tables the last forward left
    in ``args.workspace`` (and its guards when ``args.flags`` has
    ``MOE_FLAG_DEBUG``); returns the resulting (code, info)."""
    stream = stream or torch.cuda.current_stream()
    st = _lib.load().moe_fp8_check_workspace(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream))
    if st:
        _raise(st, "moe_fp8_check_workspace")
    return device_error(args, stream)


def workspace_views(args: _lib.MoeFwdArgs, workspace: torch.Tensor) -> dict:
    """Typed views of the per-stage buffers a forward leaves in ``workspace``."""
    lay = workspace_layout(args)
    t, k, el, h, i = args.T, args.top_k, args.E_local, args.H, args.I
    nb = el + args.n_shared_experts   # dispatch buckets
    npad = lay.npad

    def view(off, n, dtype):
        nb = n * torch.empty((), dtype=dtype).element_size()
        return workspace[off:off + nb].view(dtype)

    return dict(
        layout=lay,
        topk_idx=view(lay.topk_idx, t * k, torch.int32).view(t, k),
        topk_weights=view(lay.topk_weights, t * k, torch.float32).view(t, k),
        counts=view(lay.counts, nb, torch.int32),
        tile_start=view(lay.tile_start, nb + 1, torch.int32),
        row_token=view(lay.row_token, npad, torch.int32),
        row_weight=view(lay.row_weight, npad, torch.float32),
        a_perm=view(lay.a_perm, npad * h, torch.uint8).view(npad, h),
        a_scale_perm=view(lay.a_scale_perm, (h // 128) * npad, torch.float32).view(h // 128, npad),
        inter=view(lay.inter, npad * i, torch.uint8).view(npad, i),
        inter_scale=view(lay.inter_scale, (i // 64) * npad, torch.float32).view(i // 64, npad),
        out_f32=view(lay.out_f32, t * h, torch.float32).view(t, h),
        assign_row=view(lay.assign_row, t * k, torch.int32).view(t, k),
    )
