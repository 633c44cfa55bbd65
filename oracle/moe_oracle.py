"""CPU oracle for the fused FP8 block-scale DeepSeek-V3 MoE forward.

TEST INFRASTRUCTURE ONLY.  This module restates, in numpy on the CPU, the
algorithm of the reference solution (nikhilnd/mlsys26-flashinfer-moe,
``kernel.py``) so that the CUDA implementation can be checked against it.  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it.  The product path never calls it and has no CPU
fallback.

Every function cites the reference lines it follows.  The restatement is pinned
by ``tests/golden/`` fixtures produced by running the reference's own Triton
kernels under ``TRITON_INTERPRET=1`` (see ``tests/golden/make_golden.py``).

Arithmetic conventions (chosen to be reproducible bit-for-bit by the CUDA
kernels where the reference leaves them open):

* sigmoid is evaluated in float64 and rounded once to float32; the CUDA router
  does the same, so routing indices agree bit for bit;
* e4m3 rounding is round-to-nearest-even with saturation to +-448 (the
  reference casts with ``.to(tl.float8e4nv)``; ``kernel.py:135``);
* GEMMs are computed as fp32 matmuls of the dequantised operands, which equals
  the reference's blockwise ``dot * sa * sw`` accumulation up to fp32 summation
  order.
"""
from __future__ import annotations

import numpy as np

FP8_MAX = 448.0


# ----------------------------------------------------------------------------
# number formats
# ----------------------------------------------------------------------------

def _e4m3_table() -> np.ndarray:
    """float32 value of every e4m3fn code (0x7f / 0xff are NaN)."""
    vals = np.zeros(256, dtype=np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        exp = (code >> 3) & 0xF
        man = code & 0x7
        if exp == 0xF and man == 0x7:
            vals[code] = np.nan
        elif exp == 0:
            vals[code] = sign * (man / 8.0) * 2.0 ** -6
        else:
            vals[code] = sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)
    return vals


E4M3_VALUES = _e4m3_table()


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    return E4M3_VALUES[np.asarray(codes, dtype=np.uint8)]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn code, round-to-nearest-even, saturating at +-448."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    sign = np.signbit(x)
    # exponent of the quantisation step: normals have 3 mantissa bits, the
    # subnormal range (below 2^-6) has a fixed step of 2^-9.
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)
    step = np.exp2(e - 3.0)
    q = np.round(a / step) * step          # np.round is half-to-even
    q = np.minimum(q, FP8_MAX)
    # encode q exactly
    qe = np.where(q >= 2.0 ** -6, np.floor(np.log2(np.where(q > 0, q, 1.0))), -7.0)
    biased = np.where(q >= 2.0 ** -6, qe + 7, 0).astype(np.int64)
    man = np.where(q >= 2.0 ** -6,
                   np.round((q / np.exp2(qe) - 1.0) * 8.0),
                   np.round(q / 2.0 ** -9)).astype(np.int64)
    code = (biased << 3) | man
    code = np.where(q == 0, 0, code)
    code = code | np.where(sign, 0x80, 0)     # -0 keeps its sign, as the cast does
    return code.astype(np.uint8)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern (uint16), round-to-nearest-even (as
    ``Tensor.copy_`` does in ``kernel.py:729``)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    return np.where(nan, np.uint16(0x7FC0), out)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------
# routing  (reference kernel.py:428-542)
# ----------------------------------------------------------------------------

def sigmoid_f32(x: np.ndarray) -> np.ndarray:
    """``tl.sigmoid`` (kernel.py:466): 1/(1+exp(-x)), evaluated in float64 and
    rounded once to float32."""
    xd = np.asarray(x, dtype=np.float32).astype(np.float64)
    return (1.0 / (1.0 + np.exp(-xd))).astype(np.float32)


def route(logits: np.ndarray, bias: np.ndarray, n_group: int, topk_group: int, top_k: int,
          routed_scaling_factor: float):
    """DeepSeek-V3 no-aux group-limited top-k routing.

    Follows ``moe_routing_kernel`` (kernel.py:428-542):
      s = sigmoid(logits); sb = s + bias                      (466-467)
      group score = top-2 sum of sb within each group         (479-488)
      keep top ``topk_group`` groups, ties -> lowest index    (495-501)
      top ``top_k`` experts by sb inside them, ties -> lowest (522-534)
      weights = s / (sum s + 1e-20) * routed_scaling_factor   (537-538)
    Indices are returned in selection (descending sb) order.
    Returns ``(idx int32 [T,top_k], weights float32 [T,top_k])``.
    """
    logits = np.asarray(logits, dtype=np.float32)
    t, e = logits.shape
    g = e // n_group
    s = sigmoid_f32(logits)
    sb = (s + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    sbg = sb.reshape(t, n_group, g)
    # top-2 sum per group: max, then max with the first occurrence masked.
    order = np.argsort(-sbg, axis=2, kind="stable")
    m1 = np.take_along_axis(sbg, order[:, :, 0:1], axis=2)[:, :, 0]
    m2 = (np.take_along_axis(sbg, order[:, :, 1:2], axis=2)[:, :, 0] if g > 1
          else np.full_like(m1, -np.inf))
    gscore = (m1 + m2).astype(np.float32)
    # stable argsort on -score gives lowest index first among equal scores
    gsel = np.argsort(-gscore, axis=1, kind="stable")[:, :topk_group]
    gmask = np.zeros((t, n_group), dtype=bool)
    np.put_along_axis(gmask, gsel, True, axis=1)
    emask = np.repeat(gmask, g, axis=1)
    pruned = np.where(emask, sb, np.float32(-np.inf)).astype(np.float32)
    idx = np.argsort(-pruned, axis=1, kind="stable")[:, :top_k].astype(np.int32)
    sv = np.take_along_axis(s, idx, axis=1).astype(np.float32)
    ssum = _sum_like_kernel(sv) + np.float32(1e-20)
    w = ((sv / ssum[:, None]).astype(np.float32) * np.float32(routed_scaling_factor)).astype(
        np.float32)
    return idx, w


def _sum_like_kernel(v: np.ndarray) -> np.ndarray:
    """Row sum of a ``[T,k]`` fp32 array in the fixed order the CUDA router
    uses: pairwise tree for k a power of two, else left to right."""
    v = np.asarray(v, dtype=np.float32)
    k = v.shape[1]
    if k & (k - 1) == 0:
        cur = v
        while cur.shape[1] > 1:
            cur = (cur[:, 0::2] + cur[:, 1::2]).astype(np.float32)
        return cur[:, 0]
    acc = v[:, 0].copy()
    for j in range(1, k):
        acc = (acc + v[:, j]).astype(np.float32)
    return acc


# ----------------------------------------------------------------------------
# dispatch  (reference kernel.py:252-407)
# ----------------------------------------------------------------------------

def dispatch(idx: np.ndarray, weights: np.ndarray, local_expert_offset: int, e_local: int):
    """Filter assignments to local experts and bucket them by expert.

    Follows ``_count_kernel`` / ``_scatter_kernel`` / ``build_expert_dispatch``
    (kernel.py:252-382): ``token = flat // top_k`` (317), local expert
    ``e - lo`` in ``[0, E_local)`` (271-272, 313-314).  The reference's order
    inside a bucket is decided by atomics (321) and is not reproducible; this
    restatement orders each bucket by token index, which is the canonical form
    parity is defined on.
    Returns ``counts [E_local] int32``, ``starts [E_local+1] int32`` and the
    bucketed ``tokens [N] int32`` / ``weights [N] float32``.
    """
    t, k = idx.shape
    flat_e = idx.reshape(-1).astype(np.int64) - local_expert_offset
    flat_w = np.asarray(weights, dtype=np.float32).reshape(-1)
    tok = np.arange(t * k, dtype=np.int64) // k
    keep = (flat_e >= 0) & (flat_e < e_local)
    le, tk, wv = flat_e[keep], tok[keep], flat_w[keep]
    order = np.lexsort((tk, le))   # by expert, then token
    counts = np.bincount(le, minlength=e_local).astype(np.int32)
    starts = np.zeros(e_local + 1, dtype=np.int32)
    np.cumsum(counts, out=starts[1:])
    return counts, starts, tk[order].astype(np.int32), wv[order].astype(np.float32)


def tile_schedule(counts: np.ndarray, block_m: int):
    """``build_tile_schedule`` (kernel.py:384-407): per-tile expert id and
    tile index inside the expert, tiles of ``block_m`` rows."""
    tiles = (np.asarray(counts, dtype=np.int64) + block_m - 1) // block_m
    tstart = np.zeros(len(counts) + 1, dtype=np.int64)
    np.cumsum(tiles, out=tstart[1:])
    total = int(tstart[-1])
    tile_idx = np.arange(total, dtype=np.int64)
    tile_expert = np.searchsorted(tstart[1:], tile_idx, side="right").astype(np.int32)
    tile_local_m = (tile_idx - tstart[tile_expert]).astype(np.int32)
    return tile_expert, tile_local_m, tstart.astype(np.int32)


# ----------------------------------------------------------------------------
# expert GEMMs  (reference kernel.py:7-250)
# ----------------------------------------------------------------------------

def dequant_weight(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """``[N,K]`` e4m3 codes with ``[N/128,K/128]`` scales -> fp32."""
    w = e4m3_decode(q)
    n, k = w.shape
    return (w.reshape(n // 128, 128, k // 128, 128) * s[:, None, :, None]).reshape(n, k).astype(
        np.float32)


def dequant_act(q: np.ndarray, s_t: np.ndarray) -> np.ndarray:
    """``[R,H]`` e4m3 codes with the transposed ``[H/128, R]`` scales -> fp32."""
    a = e4m3_decode(q)
    r, h = a.shape
    return (a.reshape(r, h // 128, 128) * s_t.T[:, :, None]).reshape(r, h).astype(np.float32)


def swiglu_requant(g: np.ndarray, inter: int, block: int = 64, requant: bool = True):
    """GEMM1 epilogue (kernel.py:126-135): ``C = silu(X2) * X1`` with
    ``X1 = G[:, :I]``, ``X2 = G[:, I:]``; then per row, per ``block`` columns,
    ``scale = max(amax/448, 1e-12)`` and ``Cq = e4m3(C/scale)``.
    Returns ``(codes [R,I] uint8, scales [I/block, R] fp32, C fp32)``; with
    ``requant=False`` codes/scales are None."""
    g = np.asarray(g, dtype=np.float32)
    x1 = g[:, :inter]
    x2 = g[:, inter:]
    silu = (x2 / (np.float32(1.0) + np.exp(-x2.astype(np.float32)))).astype(np.float32)
    c = (silu * x1).astype(np.float32)
    if not requant:
        return None, None, c
    r = c.shape[0]
    cb = c.reshape(r, inter // block, block)
    amax = np.abs(cb).max(axis=2)
    sc = np.maximum((amax / np.float32(FP8_MAX)).astype(np.float32), np.float32(1e-12))
    codes = e4m3_encode((cb / sc[:, :, None]).astype(np.float32)).reshape(r, inter)
    return codes, sc.T.copy().astype(np.float32), c


def expert_forward(a_codes, a_scale_t, w1q, w1s, w2q, w2s, inter: int, requant: bool = True,
                   block: int = 64):
    """One expert over the rows routed to it: GEMM1 -> SwiGLU (+requant) -> GEMM2.

    ``a_codes [R,H]`` e4m3 rows, ``a_scale_t [H/128,R]``; returns the fp32
    ``[R,H]`` expert output before routing weights (kernel.py:7-250)."""
    a = dequant_act(a_codes, a_scale_t)
    w1 = dequant_weight(w1q, w1s)
    g = a @ w1.T
    codes, sc, c = swiglu_requant(g, inter, block, requant)
    if requant:
        r = codes.shape[0]
        cd = (e4m3_decode(codes).reshape(r, inter // block, block) *
              sc.T[:, :, None]).reshape(r, inter).astype(np.float32)
    else:
        cd = c
    w2 = dequant_weight(w2q, w2s)
    return (cd @ w2.T).astype(np.float32)


def moe_forward(inp: dict, n_group: int, topk_group: int, top_k: int, requant: bool = True,
                block: int = 64, tokens: np.ndarray | None = None, return_parts: bool = False,
                get_expert=None, n_shared: int = 0):
    """Whole layer, as ``run()`` computes it (kernel.py:562-729).

    ``inp`` holds numpy arrays: ``routing_logits [T,E]``, ``routing_bias [E]``,
    ``hidden_states [T,H]`` (uint8 e4m3 codes), ``hidden_states_scale [H/128,T]``,
    ``gemm1_weights [El,2I,H]`` / ``gemm2_weights [El,H,I]`` (uint8 codes) and
    their scales, ``local_expert_offset`` and ``routed_scaling_factor``.
    ``tokens`` restricts the output to a subset of token rows (each token's
    output depends only on its own routing), which keeps DeepSeek-V3-size
    checks cheap.  ``get_expert(e)`` may supply ``(w1q, w1s, w2q, w2s)`` of
    local expert ``e`` lazily instead of the four weight arrays in ``inp``.  Returns the fp32 ``[T or len(tokens), H]`` sum before the
    bf16 cast; ``bf16_bits`` of it is the reference's ``output``.

    ``n_shared=1`` adds DeepSeek-V3's shared expert, which the reference does
    not have: the weight arrays then hold the routed experts followed by the
    shared one (index ``e_local``), and every token's output gains that
    expert's output with weight 1 after its routed sum (y = sum_k w_k E_k(x) +
    S(x)), computed by the same ``expert_forward`` (1x64 requant included).
    """
    logits = inp["routing_logits"]
    t = logits.shape[0]
    idx, w = route(logits, inp["routing_bias"], n_group, topk_group, top_k,
                   inp["routed_scaling_factor"])
    if get_expert is None:
        def get_expert(e):
            return (inp["gemm1_weights"][e], inp["gemm1_weights_scale"][e],
                    inp["gemm2_weights"][e], inp["gemm2_weights_scale"][e])
        e_local = inp["gemm1_weights"].shape[0] - n_shared
    else:
        e_local = int(inp["e_local"])
    h = inp["hidden_states"].shape[1]
    lo = int(inp["local_expert_offset"])
    counts, starts, btok, bw = dispatch(idx, w, lo, e_local)
    sel = np.arange(t) if tokens is None else np.asarray(tokens)
    pos = {int(tok): j for j, tok in enumerate(sel)}
    out = np.zeros((len(sel), h), dtype=np.float32)
    hs, hss = inp["hidden_states"], inp["hidden_states_scale"]
    parts = {}
    for e in range(e_local):
        rows_tok = btok[starts[e]:starts[e + 1]]
        rows_w = bw[starts[e]:starts[e + 1]]
        keep = np.array([int(x) in pos for x in rows_tok], dtype=bool)
        if not keep.any():
            continue
        rows_tok, rows_w = rows_tok[keep], rows_w[keep]
        w1q, w1s, w2q, w2s = get_expert(e)
        inter = w1q.shape[0] // 2
        y = expert_forward(hs[rows_tok], hss[:, rows_tok], w1q, w1s, w2q, w2s, inter, requant,
                           block)
        if return_parts:
            parts[e] = (rows_tok, y)
        # weighted scatter-add (kernel.py:236-250), fp32
        for r, tok in enumerate(rows_tok):
            out[pos[int(tok)]] += (y[r] * rows_w[r]).astype(np.float32)
    if n_shared:
        w1q, w1s, w2q, w2s = get_expert(e_local)
        y = expert_forward(hs[sel], hss[:, sel], w1q, w1s, w2q, w2s, w1q.shape[0] // 2, requant,
                           block)
        out += y.astype(np.float32)
    if return_parts:
        return out, dict(idx=idx, w=w, counts=counts, starts=starts, tokens=btok, weights=bw,
                         parts=parts)
    return out


def to_numpy_inputs(inp: dict) -> dict:
    """Convert a dict of torch tensors (as made by ``moe_b200.workloads``) to the
    numpy form ``moe_forward`` takes (e4m3 tensors as uint8 codes)."""
    import torch
    out = {}
    for k, v in inp.items():
        if isinstance(v, torch.Tensor):
            v = v.detach().cpu()
            if v.dtype == torch.float8_e4m3fn:
                v = v.view(torch.uint8)
            elif v.dtype in (torch.bfloat16, torch.float16):
                v = v.float()
            out[k] = v.numpy()
        else:
            out[k] = v
    return out


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))
