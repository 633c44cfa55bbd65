#!/usr/bin/env python
"""Benchmark of the B200 fused FP8 block-scale DeepSeek-V3 MoE forward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (N=1): one DeepSeek-V3 MoE layer (H=7168, I=2048, 256 routed experts,
8 groups / top-4 groups, top-8, routed_scaling_factor 2.5) with all 256 experts
on the GPU and T=8192 tokens -- the prefill point BASELINE.json's north star
quotes (config 2).  Inputs are seeded synthetic tensors with the benchmark
definition's shapes and distributions (``moe_b200.workloads``); the weights
(11.3 GB of FP8) exceed L2, so no flush is needed between steps.

A step is one full ``moe_fp8_forward``: routing, dispatch, GEMM1 + SwiGLU +
requant, GEMM2 + weighted scatter-add, bf16 cast.  ``value`` is tokens/s with
all inputs resident in HBM (K plain forwards between two events); the per-stage
times come from K more forwards with events recorded by the library between
its kernels.  ``e2e`` is the same metric through the public ``run()`` with
every step's activations copied from pinned host memory and its bf16 output
copied back, the copies on their own streams so that they overlap the
neighbouring steps' compute (double-buffered, as a serving loop would).

Extra keys: the other prefill sizes of config 2 (T=1024/4096/16384), config 3
(Zipf-skewed routing, T=8192) with its realised expert histogram, config 4 on
one GPU (4096 bf16 tokens quantised on the GPU, uniform routing), decode
latency (config 1, T=1..64), the reference's contest shape (32 of 256 experts)
next to its published latencies and to FlashInfer's
``trtllm_fp8_block_scale_moe`` timed as a black box on the same GPU and inputs.

``--impl reference`` times the CPU restatement of the reference algorithm
(``oracle/``) on the host cores, on a bounded sample of the same workload.

Under ``torchrun`` (N>1) every rank runs the expert-parallel layer (config 4:
256 experts sharded contiguously, 4096 bf16 tokens per rank, uniform routing)
with dispatch and combine by the library's NVLink kernels; value = all ranks'
tokens / max over ranks of the step time.  Before timing, a sample of every
rank's output rows is checked against the single-GPU layer (``parity``).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "mlsys26-flashinfer-moe_b200"))

METRIC = "MoE-layer tokens/s (DeepSeek-V3 FP8 block-scale layer, 256 experts)"
NOMINAL_FP8_TFLOPS = 4500.0
# Published latencies of the reference at the contest shape (32 local experts),
# writeup.pdf p3 Table 1, ms.
REF_PUBLISHED_MS = {1: 0.636, 7: 0.668, 80: 0.968, 901: 1.046, 11984: 2.579, 14107: 3.440}
# The FlashInfer baseline of the writeup's speed-up column, derived from the
# same table (reference ms x its published speed-up over FlashInfer).
FLASHINFER_IMPLIED_MS = {1: 0.064, 7: 0.094, 80: 0.271, 901: 0.701, 11984: 4.977, 14107: 6.364}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per GPU (default 8192 at N=1, 4096 per GPU under EP)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the extra configurations, e2e and the cpu baseline")
    ap.add_argument("--cpu-sample-tokens", type=int, default=4)
    ap.add_argument("--e-local", type=int, default=256,
                    help="local experts (0..e_local-1 of 256); < 256 gives the small "
                         "same-density case used for ncu captures")
    ap.add_argument("--zipf", type=float, default=None,
                    help="headline run with Zipf(s)-skewed routing (config 3) instead")
    ap.add_argument("--concentrate", action="store_true",
                    help="router bias +10 on the local experts, so every token's experts are "
                         "local: T=1 with --e-local 8 does the work of a 256-expert decode step "
                         "with 0.35 GB of weights resident (for ncu captures)")
    ap.add_argument("--router-bias", action="store_true",
                    help="headline with config 1's router bias N(0, 0.1) instead of config 2's "
                         "uniform routing (zero bias)")
    ap.add_argument("--prepared-w2", action="store_true",
                    help="headline run with the one-time bf16 relayout of W2 (bf16 GEMM2)")
    ap.add_argument("--flashinfer-contest", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--build-flashinfer", action="store_true",
                    help="compile FlashInfer's MoE launcher (the comparator) and exit")
    return ap.parse_args()


# DRAM bytes (read + write) of one GEMM1 launch, ncu dram__bytes_read.sum +
# dram__bytes_write.sum, measured on the same-density 32-local-expert case
# (T=8192 tokens routed over 256 experts, experts 0-31 local); weights
# dominate, so a launch over more experts moves that many times more.
GEMM1_E32_DRAM_BYTES = (1043.3 + 20.0) * 1e6
GEMM1_E32_ACTIVE = 32


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, \
            "fallback"


# ----------------------------------------------------------------------------
# clocks during the timed region (NVML reads only)
# ----------------------------------------------------------------------------

class ClockSampler:
    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period_s: float = 0.005):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self.max_mhz = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.nvml = None

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------

def fp8_cublas_peak_tflops(torch):
    """Dense FP8 throughput of cuBLAS (torch._scaled_mm, 8192^3) on this GPU:
    the measured denominator for the tensor-bound roofline."""
    n = 8192
    a = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn).t()
    one = torch.ones((), device="cuda")
    for _ in range(3):
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def algorithmic_bytes(shape, counts_active, t):
    """Weights of active experts (+ scales) plus activations in and bf16 out."""
    from moe_b200.workloads import weight_bytes_per_expert
    h = shape.hidden
    return (counts_active * weight_bytes_per_expert(shape) +
            t * (h + 4 * (h // 128) + 4 * shape.e_global + 2 * h))


WEIGHT_KEYS = ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")


def layer_inputs(weights, shape, seed, zipf=None, zero_bias=False):
    """Token-side inputs for ``shape`` (seeded) combined with shared weights; the
    weights' first ``shape.e_local`` experts are the local ones."""
    from moe_b200 import workloads
    inp = workloads.make_inputs(shape, seed=seed, device="cuda", zipf=zipf, weights=False)
    for k in WEIGHT_KEYS:
        inp[k] = weights[k][:shape.e_local]
    if zero_bias:
        inp["routing_bias"] = inp["routing_bias"].zero_()
    return inp


class Runner:
    """Holds inputs, workspace and events for repeated forwards of one shape."""

    def __init__(self, torch, shape, inp, gemm2_weights_bf16=None, n_shared=0):
        from moe_b200 import api, _lib
        self.torch, self.api, self._lib, self.shape = torch, api, _lib, shape
        self.inp = inp
        self.out = torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16, device="cuda")
        from moe_b200 import workloads
        self.args, self.keep, _ = api.build_args(*workloads.run_args(self.inp), self.out,
                                                 shape.n_group, shape.topk_group, shape.top_k,
                                                 gemm2_weights_bf16=gemm2_weights_bf16,
                                                 n_shared_experts=n_shared)
        lay = api.workspace_layout(self.args)
        self.ws = torch.empty(lay.total_bytes, dtype=torch.uint8, device="cuda")
        self.args.workspace = self.ws.data_ptr()
        self.args.workspace_bytes = lay.total_bytes
        self.lib = _lib.load()
        self.stream = torch.cuda.current_stream()

    def forward(self, events=None):
        import ctypes
        if events is None:
            code = self.lib.moe_fp8_forward(ctypes.byref(self.args),
                                            ctypes.c_void_p(self.stream.cuda_stream))
        else:
            arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in events])
            code = self.lib.moe_fp8_forward_profiled(ctypes.byref(self.args),
                                                     ctypes.c_void_p(self.stream.cuda_stream),
                                                     arr, 6)
        if code:
            raise RuntimeError(f"moe_fp8_forward failed: {self._lib.status_string(code)}")

    def make_events(self, n):
        torch = self.torch
        evs = []
        for _ in range(n):
            row = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            for e in row:
                e.record(self.stream)   # creates the underlying cudaEvent_t
            evs.append(row)
        torch.cuda.synchronize()
        return evs

    def views(self):
        return self.api.workspace_views(self.args, self.ws)

    def active_experts(self):
        return int((self.views()["counts"] > 0).sum().item())

    def assignments(self):
        return int(self.views()["counts"].sum().item())


STAGES = ["route", "permute", "gemm1", "gemm2", "finalize"]


def time_plain(torch, runner, steps, warmup):
    """ms per forward over ``steps`` back-to-back forwards (no per-stage events)."""
    for _ in range(warmup):
        runner.forward()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        runner.forward()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def time_stages(torch, runner, steps, flush=None):
    """Mean per-stage ms from the library's stage events (one event row per step)."""
    evs = runner.make_events(steps)
    for i in range(steps):
        if flush is not None:
            flush()
        runner.forward(evs[i])
    torch.cuda.synchronize()
    return {n: statistics.mean(row[j].elapsed_time(row[j + 1]) for row in evs)
            for j, n in enumerate(STAGES)}


def prefill_point(torch, runner, steps, warmup, fp8_peak):
    from moe_b200 import workloads
    ms = time_plain(torch, runner, steps, warmup)
    st = time_stages(torch, runner, max(3, steps // 2))
    n_assign = runner.assignments()
    flops = n_assign * workloads.flops_per_assignment(runner.shape)
    tf = flops / (ms * 1e-3) / 1e12
    g1 = n_assign * 4 * runner.shape.hidden * runner.shape.inter / (st["gemm1"] * 1e-3) / 1e12
    g2 = n_assign * 2 * runner.shape.hidden * runner.shape.inter / (st["gemm2"] * 1e-3) / 1e12
    return {"ms": round(ms, 4), "tokens_per_s": round(runner.shape.t / (ms * 1e-3), 1),
            "tflops": round(tf, 1), "fp8_frac_measured": round(tf / fp8_peak, 3),
            "fp8_frac_nominal": round(tf / NOMINAL_FP8_TFLOPS, 3),
            "gemm1_tflops": round(g1, 1), "gemm2_tflops": round(g2, 1),
            "stage_ms": {k: round(v, 4) for k, v in st.items()},
            "active_experts": runner.active_experts()}


# ----------------------------------------------------------------------------
# CPU baseline (the oracle port)
# ----------------------------------------------------------------------------

def cpu_baseline(shape, inp_gpu, sample_tokens, torch):
    """The CPU oracle (the reference algorithm restated in numpy) on the first
    ``sample_tokens`` tokens of the batch; returns tokens/s and the thread count."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import moe_oracle as mo
    t = min(sample_tokens, shape.t)
    hi = {}
    for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale"):
        v = inp_gpu[k]
        v = v[:t] if k in ("routing_logits", "hidden_states") else v
        if k == "hidden_states_scale":
            v = v[:, :t]
        v = v.detach().contiguous().cpu()
        hi[k] = (v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else v.float()).numpy()
    hi.update(local_expert_offset=shape.local_expert_offset,
              routed_scaling_factor=shape.routed_scaling_factor, e_local=shape.e_local)
    cache = {}

    def get(e):   # weight transfer is outside the timed region
        return cache[e]
    idx, _ = mo.route(hi["routing_logits"], hi["routing_bias"], shape.n_group, shape.topk_group,
                      shape.top_k, shape.routed_scaling_factor)
    for e in np.unique(idx):
        le = int(e) - shape.local_expert_offset
        if 0 <= le < shape.e_local:
            cache[le] = (inp_gpu["gemm1_weights"][le].view(torch.uint8).cpu().numpy(),
                         inp_gpu["gemm1_weights_scale"][le].cpu().numpy(),
                         inp_gpu["gemm2_weights"][le].view(torch.uint8).cpu().numpy(),
                         inp_gpu["gemm2_weights_scale"][le].cpu().numpy())
    t0 = time.perf_counter()
    mo.moe_forward(hi, shape.n_group, shape.topk_group, shape.top_k, get_expert=get)
    dt = time.perf_counter() - t0
    threads = os.cpu_count() or 1
    return t / dt, dt, t, threads


# ----------------------------------------------------------------------------
# our arm, one GPU
# ----------------------------------------------------------------------------

def run_ours(a):
    import torch
    from moe_b200 import workloads
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        return run_ep(a)
    torch.cuda.set_device(0)
    peaks, peak_kind = load_peaks()
    t = a.tokens or 8192
    full = workloads.dsv3_shape(t, e_local=256 if not a.no_extras else a.e_local)
    # tokens of seed 0 + the weights (all 256 experts unless only the headline runs)
    weights = workloads.make_inputs(full, seed=0, device="cuda")
    shape = workloads.dsv3_shape(t, e_local=a.e_local)
    if a.zipf is None:
        inp = {k: (v[:shape.e_local] if k in WEIGHT_KEYS else v) for k, v in weights.items()}
        if not a.router_bias:   # config 2: uniform random routing, logits N(0,1) and no bias
            inp["routing_bias"] = torch.zeros_like(weights["routing_bias"])
    else:
        inp = layer_inputs(weights, shape, seed=0, zipf=a.zipf)
    if a.concentrate:
        inp["routing_bias"] = inp["routing_bias"].clone()
        inp["routing_bias"][:shape.e_local] += 10.0
    prepared = None
    if a.prepared_w2:
        from moe_b200 import prepare_gemm2_weights
        prepared = prepare_gemm2_weights(inp["gemm2_weights"], inp["gemm2_weights_scale"])
    runner = Runner(torch, shape, inp, gemm2_weights_bf16=prepared)
    clocks = ClockSampler(torch.cuda.current_device())
    # timed region: K plain forwards
    for _ in range(a.warmup):
        runner.forward()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clocks:
        start.record()
        for _ in range(a.steps):
            runner.forward()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / a.steps
    # per-kernel times: K more forwards with the library's stage events
    stages = time_stages(torch, runner, a.steps)
    active = runner.active_experts()
    n_assign = runner.assignments()
    flops = n_assign * workloads.flops_per_assignment(shape)
    value = t / (ms * 1e-3)
    fp8_peak = fp8_cublas_peak_tflops(torch)
    g1_flops = n_assign * 4 * shape.hidden * shape.inter
    g1_ms = stages["gemm1"]
    g1_bytes = active * 2 * shape.inter * shape.hidden
    roofline = {
        "kernel": "moe_gemm_kernel<GEMM1> (gate/up + SwiGLU + requant)",
        "bound": "tensor", "achieved": round(g1_flops / (g1_ms * 1e-3) / 1e12, 1),
        "peak": round(fp8_peak, 1), "unit": "TFLOP/s",
        "frac": round(g1_flops / (g1_ms * 1e-3) / 1e12 / fp8_peak, 3),
        "peak_kind": "measured on this GPU: cuBLAS FP8 e4m3 8192^3 (torch._scaled_mm)",
        "traffic": round(GEMM1_E32_DRAM_BYTES * active / GEMM1_E32_ACTIVE),
        "traffic_unit": "bytes per launch",
        "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one GEMM1 launch "
                           f"on the same-density 32-local-expert case (T=8192, experts 0-31 "
                           f"local), scaled by active experts {active}/{GEMM1_E32_ACTIVE}"),
        "hbm_view": {"achieved_gbs": round(g1_bytes / (g1_ms * 1e-3) / 1e9, 1),
                     "peak_gbs": peaks["hbm_gbs"], "peak_kind": peak_kind,
                     "frac": round(g1_bytes / (g1_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 3)},
    }
    cfg_name = "config 3, Zipf routing" if a.zipf is not None else \
        ("config 2" if shape.e_local == 256 else "same-density subset")
    if a.zipf is None:
        cfg_name += (", router bias N(0, 0.1)" if a.router_bias
                     else ", uniform random routing (zero router bias)")
    if a.concentrate:
        cfg_name = "routing concentrated on the local experts, profiling case"
    if a.prepared_w2:
        cfg_name += ", W2 prepared as bf16"
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8-e4m3 x e4m3 -> fp32 (bf16 out)", "data": "synthetic (seeded, random-init weights)",
        "config": {"workload": f"DeepSeek-V3 MoE layer, T={t}, {shape.e_local} of 256 experts "
                               f"on 1 GPU ({cfg_name})",
                   "model": "DeepSeek-V3 MoE layer", "global_batch": t, "seq_len": 1,
                   "hidden": shape.hidden, "intermediate": shape.inter, "experts": shape.e_local,
                   "top_k": 8, "parallelism": "single GPU",
                   "l2": "weights 11.3 GB > L2 (no flush needed)"},
        "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
        "fp8_peak_frac": {"nominal_4500": round(flops / (ms * 1e-3) / 1e12 / NOMINAL_FP8_TFLOPS, 3),
                          "measured_cublas": round(flops / (ms * 1e-3) / 1e12 / fp8_peak, 3)},
        "stage_ms": {k: round(v, 4) for k, v in stages.items()},
        "active_experts": active,
        "roofline": roofline,
        "clocks": clocks.summary(),
        "gpu_launches": 5 * a.steps,
    }
    layer_roof_ms = max(flops / (fp8_peak * 1e12),
                        algorithmic_bytes(shape, active, t) / (peaks["hbm_gbs"] * 1e9)) * 1e3
    line["layer_roofline"] = {"ms": round(layer_roof_ms, 4), "frac": round(layer_roof_ms / ms, 3),
                              "basis": "max(FLOPs / measured FP8 cuBLAS, bytes / measured HBM)"}
    if not a.no_extras:
        line["e2e"] = e2e_run(torch, runner, a)
        del runner
        torch.cuda.empty_cache()
        line["prepared_gemm2_bf16"] = prepared_run(torch, shape, inp, fp8_peak, a)
        line["prefill_sweep"] = prefill_sweep(torch, weights, fp8_peak, a)
        line["router_bias_t8192"] = biased_run(torch, weights, fp8_peak, a)
        line["zipf_t8192"] = zipf_run(torch, weights, fp8_peak, a)
        line["ep_config_n1"] = ep_config_n1(torch, weights, a)
        line["decode"] = decode_sweep(torch, weights, peaks)
        line["contest_shape"] = contest_sweep(torch, weights)
        line["neighbours"] = neighbours(torch, weights, fp8_peak, peaks, line["decode"])
        tps, dt, ns, threads = cpu_baseline(full, {**weights, "routing_bias": inp["routing_bias"]},
                                            a.cpu_sample_tokens, torch)
        line["cpu_baseline"] = {"value": round(tps, 3), "unit": "tokens/s", "cores": threads,
                                "kind": "port",
                                "sample": f"first {ns} tokens of the T={t} batch through the numpy "
                                          f"oracle ({dt:.1f} s; BLAS threads on {threads} cores)"}
    print(json.dumps(line))


def e2e_run(torch, runner, a):
    """Same metric through run(): every step copies its activations from pinned
    host memory and its bf16 output back to pinned host memory.  The copies run
    on two copy streams with device buffers double-buffered by step parity, so
    step i+1's inputs arrive and step i-1's output leaves while step i computes.
    Timed from an event before the first input copy to an event after the last
    output copy."""
    from moe_b200 import run
    shape, inp = runner.shape, runner.inp
    keys = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale")
    host = {k: inp[k].cpu().pin_memory() for k in keys}
    out_host = [torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16).pin_memory()
                for _ in range(2)]
    dev_in = [{k: torch.empty_like(inp[k]) for k in keys} for _ in range(2)]
    dev_out = [torch.empty(shape.t, shape.hidden, dtype=torch.bfloat16, device="cuda")
               for _ in range(2)]
    weights = [inp[k] for k in WEIGHT_KEYS]
    kw = dict(n_group=shape.n_group, topk_group=shape.topk_group, top_k=shape.top_k)
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event(enable_timing=False)   # noqa: E731
    ready, done, freed = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    for e in freed + done:
        e.record(comp)

    def copy_in(b):
        with torch.cuda.stream(h2d):
            h2d.wait_event(done[b])             # the forward that read buffer b is over
            for k in keys:
                dev_in[b][k].copy_(host[k], non_blocking=True)
            ready[b].record(h2d)

    def steps_loop(n, t0=None):
        if t0 is not None:
            t0.record(h2d)
        copy_in(0)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                copy_in(b ^ 1)
            comp.wait_event(ready[b])
            comp.wait_event(freed[b])           # buffer b's previous output has left
            args = [dev_in[b][k] for k in keys] + weights + \
                [inp["local_expert_offset"], inp["routed_scaling_factor"]]
            run(*args, dev_out[b], **kw)
            done[b].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done[b])
                out_host[b].copy_(dev_out[b], non_blocking=True)
                freed[b].record(d2h)

    steps_loop(max(3, a.warmup))
    torch.cuda.synchronize()
    steps = max(5, a.steps // 2)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps_loop(steps, t0)
    t1.record(d2h)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    h2d_bytes = sum(v.numel() * v.element_size() for v in host.values())
    return {"value": round(shape.t / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": shape.t * shape.hidden * 2,
            "path": "moe_b200.run() on device buffers filled from pinned host memory each step; "
                    "copies on two copy streams, double-buffered, overlapping compute"}


def prepared_run(torch, shape, inp, fp8_peak, a):
    """The headline workload with the one-time bf16 relayout of W2
    (``prepare_gemm2_weights``, a one-time weight relayout): GEMM2 on bf16
    operands without block-scale promotion.  The relayout runs once per layer's
    weights, outside the timed steps; its own time is reported."""
    from moe_b200 import prepare_gemm2_weights
    w2, w2s = inp["gemm2_weights"], inp["gemm2_weights_scale"]
    prepare_gemm2_weights(w2, w2s)   # warm-up
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    wb = prepare_gemm2_weights(w2, w2s)
    e.record()
    torch.cuda.synchronize()
    prep_ms = s.elapsed_time(e)
    r = Runner(torch, shape, inp, gemm2_weights_bf16=wb)
    res = prefill_point(torch, r, a.steps, a.warmup, fp8_peak)
    res["prepare_ms_once"] = round(prep_ms, 3)
    res["prepared_bytes"] = wb.numel() * 2
    res["path"] = ("run(..., gemm2_weights_bf16=prepare_gemm2_weights(W2, W2_scale)): the same "
                   "routing, GEMM1 and FP8 requant; GEMM2 on bf16(code*scale) x bf16(W2*scale)")
    del r, wb
    torch.cuda.empty_cache()
    return res


def prefill_sweep(torch, weights, fp8_peak, a):
    """Config 2 at the other token counts (all 256 experts, uniform routing:
    logits N(0,1), zero router bias)."""
    from moe_b200 import workloads
    res = {}
    for t in (1024, 4096, 16384):
        shape = workloads.dsv3_shape(t)
        r = Runner(torch, shape, layer_inputs(weights, shape, seed=30 + t, zero_bias=True))
        res[str(t)] = prefill_point(torch, r, 10, 3, fp8_peak)
        del r
        torch.cuda.empty_cache()
    return res


def biased_run(torch, weights, fp8_peak, a):
    """The headline size with config 1's router bias N(0, 0.1) instead of
    uniform routing (the headline workload of earlier measurements): the bias
    leaves ~36 experts idle and gives the hottest ~8x the mean rows."""
    from moe_b200 import workloads
    shape = workloads.dsv3_shape(8192)
    inp = {k: (v[:256] if k in WEIGHT_KEYS else v) for k, v in weights.items()}
    r = Runner(torch, shape, inp)
    res = prefill_point(torch, r, 10, 3, fp8_peak)
    counts = r.views()["counts"].float()
    res["max_rows"] = int(counts.max().item())
    del r
    torch.cuda.empty_cache()
    return res


def zipf_run(torch, weights, fp8_peak, a, s=1.2):
    """Config 3: T=8192 with expert popularity ~ Zipf(1.2) over a random
    permutation of the experts (realised through the router bias)."""
    from moe_b200 import workloads
    shape = workloads.dsv3_shape(8192)
    r = Runner(torch, shape, layer_inputs(weights, shape, seed=3, zipf=s))
    res = prefill_point(torch, r, 10, 3, fp8_peak)
    counts = r.views()["counts"].float()
    res["zipf_s"] = s
    res["histogram"] = {"max_over_mean": round(float(counts.max() / counts.mean()), 2),
                        "zero_experts": int((counts == 0).sum().item()),
                        "max_rows": int(counts.max().item()),
                        "mean_rows": round(float(counts.mean()), 1)}
    del r
    torch.cuda.empty_cache()
    return res


def ep_config_n1(torch, weights, a):
    """Config 4 on one GPU: 4096 bf16 tokens quantised 1x128 on the GPU every
    step, then the layer with all 256 experts, uniform routing (zero bias) --
    the per-GPU work of the expert-parallel runs, for v_N / (N * this)."""
    from moe_b200 import quantize_1x128, workloads
    t = 4096
    shape = workloads.dsv3_shape(t)
    inp = layer_inputs(weights, shape, seed=1000, zero_bias=True)
    g = torch.Generator(device="cuda")
    g.manual_seed(2000)
    x = torch.randn(t, shape.hidden, generator=g, device="cuda").to(torch.bfloat16)
    r = Runner(torch, shape, inp)
    q, sc = inp["hidden_states"], inp["hidden_states_scale"]

    def step():
        quantize_1x128(x, q, sc)
        r.forward()
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.steps):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / a.steps
    res = {"tokens_per_s": round(t / (ms * 1e-3), 1), "ms": round(ms, 4), "tokens": t,
           "routing": "uniform (zero bias)", "active_experts": r.active_experts()}
    del r
    torch.cuda.empty_cache()
    return res


def decode_sweep(torch, weights, peaks):
    """Decode latency (config 1, T=1..64, all 256 experts), L2 flushed before
    every step: p50 of the eager forward, p50 of the same forward replayed as
    one CUDA graph (``moe_b200.LayerGraph``), and a per-stage breakdown from a
    separate run with stage events."""
    from moe_b200 import workloads, LayerGraph
    res = {}
    flush_buf = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")

    def flush():
        flush_buf.zero_()

    def p50_of(fn, n=30, warm=5):
        for _ in range(warm):
            fn()
        per = []
        for _ in range(n):
            flush()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            per.append(s.elapsed_time(e))
        return statistics.median(per)
    for t in (1, 8, 32, 64):
        shape = workloads.dsv3_shape(t)
        r = Runner(torch, shape, layer_inputs(weights, shape, seed=1))
        r.forward()
        stages = time_stages(torch, r, 10, flush=flush)
        eager = p50_of(lambda: r.forward())
        out_g = torch.empty_like(r.out)
        graph = LayerGraph(*workloads.run_args(r.inp), out_g)
        graphed = p50_of(graph.replay)
        active = r.active_experts()
        byts = algorithmic_bytes(shape, active, t)
        roof = byts / (peaks["hbm_gbs"] * 1e9)
        res[str(t)] = {"p50_us": round(eager * 1e3, 1), "p50_us_graph": round(graphed * 1e3, 1),
                       "active_experts": active,
                       "hbm_roofline_us": round(roof * 1e6, 1),
                       "hbm_frac": round(roof / (eager * 1e-3), 3),
                       "hbm_frac_graph": round(roof / (graphed * 1e-3), 3),
                       "stage_us": {k: round(v * 1e3, 1) for k, v in stages.items()}}
        del graph, r
        torch.cuda.empty_cache()
    return res


def with_shared_expert(torch, inp, shape, seed):
    """``inp`` with one more expert after the local ones (the workloads' weight
    recipe): DeepSeek-V3's shared expert in the layout n_shared_experts=1 takes."""
    from moe_b200 import workloads
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    h, i = shape.hidden, shape.inter
    w1 = (0.02 * torch.randn(1, 2 * i, h, generator=g, device="cuda")).to(torch.bfloat16)
    w2 = (0.02 * torch.randn(1, h, i, generator=g, device="cuda")).to(torch.bfloat16)
    (q1, s1), (q2, s2) = workloads.quantize_weight_blocks(w1), workloads.quantize_weight_blocks(w2)
    out = dict(inp)
    for k, v in (("gemm1_weights", q1), ("gemm1_weights_scale", s1), ("gemm2_weights", q2),
                 ("gemm2_weights_scale", s2)):
        out[k] = torch.cat([inp[k], v])
    return out


def neighbours(torch, weights, fp8_peak, peaks, decode):
    """The ops either side of run(): the router GEMM that produces
    routing_logits, and DeepSeek-V3's shared expert fused into the layer as one
    more dispatch bucket (n_shared_experts=1, all 256 routed experts local)."""
    from moe_b200 import workloads, LayerGraph, router_logits
    res = {}
    h, e = 7168, 256
    rl = {}
    for t in (1, 64, 8192):
        g = torch.Generator(device="cuda")
        g.manual_seed(5000 + t)
        x = torch.randn(t, h, generator=g, device="cuda").to(torch.bfloat16)
        w = (0.02 * torch.randn(e, h, generator=g, device="cuda")).to(torch.bfloat16)
        out = torch.empty(t, e, device="cuda")
        for _ in range(3):
            router_logits(x, w, out)
        torch.cuda.synchronize()
        n = 20
        s, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            router_logits(x, w, out)
        en.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(en) / n * 1e3
        byts = 2 * t * h + 2 * e * h + 4 * t * e
        rl[str(t)] = {"us": round(us, 1), "tflops": round(2 * t * h * e / (us * 1e-6) / 1e12, 2),
                      "gbs": round(byts / (us * 1e-6) / 1e9, 1),
                      "hbm_roofline_us": round(byts / (peaks["hbm_gbs"] * 1e9) * 1e6, 2),
                      "path": "CUDA cores, fixed order" if t <= 128 else "tcgen05 kind::f16"}
    res["router_logits"] = {"shape": f"x [T, {h}] bf16 . w_gate [{e}, {h}]^T -> fp32",
                            "timing": "mean of 20 back-to-back calls (w_gate 3.7 MB stays in L2)",
                            "by_tokens": rl}
    # shared expert at the headline size
    shape = workloads.dsv3_shape(8192)
    inp = with_shared_expert(torch, layer_inputs(weights, shape, seed=0, zero_bias=True), shape,
                             seed=77)
    r = Runner(torch, shape, inp, n_shared=1)
    pt = prefill_point(torch, r, 10, 3, fp8_peak)
    pt["note"] = ("the headline's tokens and routing plus the shared expert: 257 dispatch "
                  "buckets; flops count the shared expert's T rows with the 8T routed ones")
    res["shared_expert_t8192"] = pt
    del r, inp
    torch.cuda.empty_cache()
    # shared expert at decode sizes: graph replay p50, L2 flushed
    flush_buf = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    dec = {}
    for t in (1, 8):
        shape = workloads.dsv3_shape(t)
        inp = with_shared_expert(torch, layer_inputs(weights, shape, seed=1), shape, seed=78)
        out_g = torch.empty(t, shape.hidden, dtype=torch.bfloat16, device="cuda")
        graph = LayerGraph(*workloads.run_args(inp), out_g, n_shared_experts=1)
        per = []
        for i in range(35):
            flush_buf.zero_()
            s, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            graph.replay()
            en.record()
            en.synchronize()
            if i >= 5:
                per.append(s.elapsed_time(en))
        dec[str(t)] = {"p50_us_graph": round(statistics.median(per) * 1e3, 1),
                       "routed_only_p50_us_graph": decode.get(str(t), {}).get("p50_us_graph")}
        del graph, inp
        torch.cuda.empty_cache()
    res["shared_expert_decode"] = dec
    del flush_buf
    torch.cuda.empty_cache()
    return res


def flashinfer_forward(inp, shape):
    """FlashInfer's trtllm_fp8_block_scale_moe (closed kernels, run as a black
    box) on the reference's inputs: DeepSeek-V3 routing, DeepSeekFp8 block
    scales, K-major weights."""
    from flashinfer.fused_moe import trtllm_fp8_block_scale_moe
    return trtllm_fp8_block_scale_moe(
        inp["routing_logits"], inp["routing_bias"], inp["hidden_states"],
        inp["hidden_states_scale"], inp["gemm1_weights"], inp["gemm1_weights_scale"],
        inp["gemm2_weights"], inp["gemm2_weights_scale"], shape.e_global, shape.top_k,
        shape.n_group, shape.topk_group, shape.inter, shape.local_expert_offset, shape.e_local,
        shape.routed_scaling_factor, routing_method_type=2)


CONTEST_TOKENS = (1, 7, 80, 901, 11984, 14107)


def contest_inputs(torch, n, weights):
    from moe_b200 import workloads
    shape = workloads.dsv3_shape(n, e_local=32, local_expert_offset=0)
    return shape, layer_inputs(weights, shape, seed=2)


def contest_weights():
    """The first 32 experts of the N=1 run's layer (the same generator draws)."""
    from moe_b200 import workloads
    return workloads.make_inputs(workloads.dsv3_shape(8192, e_local=32), seed=0, device="cuda")


# FlashInfer JIT-compiles the launcher of its MoE kernels on first use (minutes
# of nvcc).  The build is made once in this directory (git-ignored) and carried
# to the GPU box with the repository; the closed kernels themselves come from
# the installed flashinfer-cubin package.
FLASHINFER_JIT = os.path.join(REPO, "baseline", "_flashinfer_jit")


def flashinfer_env():
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", FLASHINFER_JIT)
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")


def flashinfer_jit_ready():
    import glob
    return bool(glob.glob(os.path.join(FLASHINFER_JIT, ".cache", "flashinfer", "*", "100a",
                                       "cached_ops", "fused_moe_trtllm_sm100", "*.so")))


def build_flashinfer():
    """Compile FlashInfer's MoE launcher into FLASHINFER_JIT (no GPU needed)."""
    flashinfer_env()
    from flashinfer.fused_moe.core import gen_trtllm_gen_fused_moe_sm100_module
    gen_trtllm_gen_fused_moe_sm100_module().build(verbose=False)


def run_flashinfer_contest():
    """Child process of the contest sweep: FlashInfer's kernel on the contest
    inputs, timed like ours, plus the cosine of its output against ours.
    Prints one JSON dict {n: {...}}; an exception is reported as a string."""
    flashinfer_env()
    if flashinfer_jit_ready():
        # the launcher is already compiled: skip FlashInfer's ninja up-to-date
        # check, which file times changed by copying the tree can fail
        import flashinfer.jit.core as jit_core
        jit_core.JitSpec.build = lambda self, *args, **kwargs: None
    import torch
    torch.cuda.set_device(0)
    weights = contest_weights()
    res = {}
    for n in CONTEST_TOKENS:
        shape, inp = contest_inputs(torch, n, weights)
        try:
            fo = flashinfer_forward(inp, shape)
            for _ in range(5):
                flashinfer_forward(inp, shape)
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(20):
                flashinfer_forward(inp, shape)
            e.record()
            torch.cuda.synchronize()
            fms = s.elapsed_time(e) / 20
            r = Runner(torch, shape, inp)
            r.forward()
            torch.cuda.synchronize()
            a_, b_ = r.out.float().flatten(), fo.float().flatten()
            if a_.norm() == 0 and b_.norm() == 0:
                cos = 1.0   # no token routed to a local expert: both outputs are zero
            else:
                cos = float(torch.dot(a_, b_) / (a_.norm() * b_.norm() + 1e-30))
            res[str(n)] = {"ms": round(fms, 4), "cos_vs_ours": round(cos, 6),
                           "max_abs_diff_vs_ours": round(float((a_ - b_).abs().max()), 5)}
            del r
        except Exception as exc:  # noqa: BLE001 - reported to the parent
            res[str(n)] = f"{type(exc).__name__}: {str(exc)[:300]}"
            break
    print("FLASHINFER_JSON " + json.dumps(res))


def flashinfer_contest_child():
    import subprocess
    if not flashinfer_jit_ready():
        return None, ("FlashInfer's MoE launcher is not built in baseline/_flashinfer_jit "
                      "(python bench.py --build-flashinfer, no GPU needed)")
    try:
        p = subprocess.run([sys.executable, os.path.abspath(__file__), "--flashinfer-contest"],
                           capture_output=True, text=True, timeout=300)
    except subprocess.TimeoutExpired:
        return None, "timed out after 300 s"
    for line in p.stdout.splitlines():
        if line.startswith("FLASHINFER_JSON "):
            return json.loads(line[len("FLASHINFER_JSON "):]), None
    tail = (p.stderr or p.stdout or "").strip().splitlines()[-1:] or ["no output"]
    return None, f"exit {p.returncode}: {tail[0][:300]}"


def contest_sweep(torch, weights):
    """The reference's published shape (32 local experts of 256): our layer,
    the reference's published latency, and FlashInfer's kernel timed on the same
    GPU and inputs in a child process (black box; its output is compared with
    ours there)."""
    res = {}
    for n in CONTEST_TOKENS:
        shape, inp = contest_inputs(torch, n, weights)
        r = Runner(torch, shape, inp)
        ms = time_plain(torch, r, 20, 5)
        res[str(n)] = {"ms": round(ms, 4), "reference_published_ms": REF_PUBLISHED_MS[n],
                       "speedup_vs_published": round(REF_PUBLISHED_MS[n] / ms, 2),
                       "flashinfer_implied_published_ms": FLASHINFER_IMPLIED_MS[n]}
        del r
        torch.cuda.empty_cache()
    fi, err = flashinfer_contest_child()
    for n in CONTEST_TOKENS:
        row = res[str(n)]
        got = fi.get(str(n)) if fi else None
        if isinstance(got, dict):
            row["flashinfer_ms"] = got["ms"]
            row["speedup_vs_flashinfer"] = round(got["ms"] / row["ms"], 2)
            row["cos_vs_flashinfer"] = got["cos_vs_ours"]
        else:
            row["flashinfer"] = f"unavailable: {got or err}"
    return res


# ----------------------------------------------------------------------------
# expert parallel (N > 1)
# ----------------------------------------------------------------------------

def ep_parity(torch, dist, layer, inp, bias, x_bf16, wts, world, rank, lo, shape, sample=8):
    """Each rank's EP output for its first ``sample`` tokens against the layer
    computed shard by shard with ``run()`` (the reference's own API for an
    expert shard: local_expert_offset + the rank's weight slice): every rank runs
    its shard on all ranks' sample tokens, the fp32 partials are summed over the
    ranks, and each rank compares its own rows.  Same tolerance as the tests."""
    from moe_b200 import quantize_1x128, run
    out = torch.empty(x_bf16.shape[0], shape.hidden, dtype=torch.bfloat16, device="cuda")
    layer.forward_bf16(inp["routing_logits"], bias, x_bf16, *wts, shape.routed_scaling_factor,
                       out)
    q, s = quantize_1x128(x_bf16[:sample].contiguous())
    lg = inp["routing_logits"][:sample].contiguous()
    all_q = torch.empty(world * sample, shape.hidden, dtype=torch.uint8, device="cuda")
    all_l = torch.empty(world * sample, shape.e_global, dtype=torch.float32, device="cuda")
    all_s = torch.empty(world * sample, shape.hidden // 128, dtype=torch.float32, device="cuda")
    dist.all_gather_into_tensor(all_q, q.view(torch.uint8))
    dist.all_gather_into_tensor(all_l, lg)
    dist.all_gather_into_tensor(all_s, s.t().contiguous())
    part = torch.empty(world * sample, shape.hidden, dtype=torch.bfloat16, device="cuda")
    run(all_l, bias, all_q.view(torch.float8_e4m3fn), all_s.t().contiguous(), *wts, lo,
        shape.routed_scaling_factor, part)
    ref = part.float()
    dist.all_reduce(ref)
    mine = ref[rank * sample:(rank + 1) * sample]
    got = out[:sample].float()
    err = (got - mine).abs().max()
    tol_ok = bool(((got - mine).abs() <= 1e-2 + 2e-2 * mine.abs()).all().item())
    cos = torch.dot(got.flatten(), mine.flatten()) / (got.norm() * mine.norm() + 1e-30)
    stats = torch.tensor([err.item(), -cos.item(), 0.0 if tol_ok else 1.0], device="cuda")
    dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ok = stats[2].item() == 0.0 and -stats[1].item() >= 0.9999
    return {"ok": ok, "max_abs_err": round(stats[0].item(), 5), "min_cos": round(-stats[1].item(), 7),
            "sample_tokens_per_rank": sample,
            "reference": "sum over ranks of run() on the rank's expert slice (fp32 sum of the "
                         "bf16 shard outputs), same tolerance as the tests"}


def run_ep(a):
    """Expert-parallel layer over all ranks (config 4): 256 experts sharded
    contiguously, ``a.tokens`` (default 4096) bf16 tokens per rank quantised on
    the GPU every step, uniform routing (zero router bias).  value = all ranks'
    tokens / max over ranks of the device-timed step."""
    import datetime
    import torch
    import torch.distributed as dist
    from moe_b200 import ep, workloads
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=120))
    t = a.tokens or 4096
    lo, per = ep.expert_range(rank, world, 256)
    shape = workloads.dsv3_shape(t, e_local=per, local_expert_offset=lo)
    inp = workloads.make_inputs(shape, seed=1000 + rank, device="cuda")
    shared = workloads.make_inputs(workloads.dsv3_shape(1), seed=7, device="cuda", weights=False)
    uniform_bias = torch.zeros_like(shared["routing_bias"])   # config 4: uniform routing
    skewed_bias = shared["routing_bias"]                      # N(0, 0.1), shared by the ranks
    out = torch.empty(t, shape.hidden, dtype=torch.bfloat16, device="cuda")
    wts = [inp[k] for k in WEIGHT_KEYS]

    # Config 4 starts from bf16 N(0,1) activations: every step quantises them to
    # e4m3 1x128 on the GPU before the FP8 dispatch.
    g = torch.Generator(device="cuda")
    g.manual_seed(2000 + rank)
    x_bf16 = torch.randn(t, shape.hidden, generator=g, device="cuda").to(torch.bfloat16)

    # Dispatch and combine are the library's own NVLink kernels (moe_b200.ep.FusedEP);
    # NCCL only all-gathers row counts and orders the phases.
    layer = ep.FusedEP(t, shape.hidden, shape.inter, 256)
    parity = ep_parity(torch, dist, layer, inp, uniform_bias, x_bf16, wts, world, rank, lo, shape)

    stage_names = ["send_plan", "count_allgather", "dispatch", "barrier1", "experts_combine",
                   "barrier2", "finalize"]

    def step(bias, logits, x, o, tim=None):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(8)] if tim is not None else None
        layer.forward_bf16(logits, bias, x, *wts, shape.routed_scaling_factor, o, events=evs)
        if tim is not None:
            tim.setdefault("events", []).append(evs)

    def timed(bias, steps, warmup, tim=None, clocks=None):
        for _ in range(warmup):
            step(bias, inp["routing_logits"], x_bf16, out)
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        import contextlib
        with (clocks or contextlib.nullcontext()):
            s.record()
            for _ in range(steps):
                step(bias, inp["routing_logits"], x_bf16, out, tim)
            e.record()
            torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e) / steps], device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    clocks = ClockSampler(local)
    ms_v = timed(uniform_bias, a.steps, a.warmup, clocks=clocks)
    rows_recv = layer.cnt_all.view(world, world).sum(0).tolist()
    tim = {}
    timed(uniform_bias, max(3, a.steps // 2), 1, tim=tim)
    stage_ms = {n: round(statistics.mean(ev[j].elapsed_time(ev[j + 1]) for ev in tim["events"]), 4)
                for j, n in enumerate(stage_names)}
    rows_sent = int(layer.send_cnt.sum().item())
    ms_skew = timed(skewed_bias, max(3, a.steps // 2), 2)
    rows_recv_skew = layer.cnt_all.view(world, world).sum(0).tolist()
    ms2 = ep_e2e(torch, dist, layer, inp, uniform_bias, x_bf16, wts, shape, t, a)
    dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(world * t / (ms_v * 1e-3), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_v, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8-e4m3 x e4m3 -> fp32 (bf16 out)",
            "data": "synthetic (seeded, random-init weights)",
            "config": {"workload": f"DeepSeek-V3 MoE layer, expert parallel over {world} GPUs, "
                                   f"{t} tokens per GPU of bf16 activations quantised 1x128 "
                                   f"on the GPU each step, uniform routing (config 4)",
                       "model": "DeepSeek-V3 MoE layer", "global_batch": world * t, "seq_len": 1,
                       "experts_per_gpu": per,
                       "parallelism": f"ep{world} (dispatch and combine by NVLink peer stores "
                                      f"from the library's kernels; NCCL for counts and barriers)",
                       "l2": "weights > L2 (no flush needed)"},
            "parity": parity,
            "rows_sent_rank0": rows_sent,
            # rows each rank receives (sum over sources of cnt_all[source][rank]): the
            # slowest rank sets the step time
            "rows_received_per_rank": rows_recv,
            "stage_ms_rank0": stage_ms,
            "ep_skewed": {"value": round(world * t / (ms_skew * 1e-3), 1),
                          "ms_per_step": round(ms_skew, 4),
                          "routing": "router bias N(0, 0.1) shared by all ranks",
                          "rows_received_per_rank": rows_recv_skew},
            "clocks": clocks.summary(),
            "e2e": {"value": round(world * t / (ms2 * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(ms2, 4),
                    "h2d_bytes_per_step": t * (shape.hidden * 2 + shape.e_global * 4),
                    "d2h_bytes_per_step": t * shape.hidden * 2,
                    "path": "moe_b200.ep.FusedEP.forward_bf16 on device buffers filled from pinned "
                            "host memory each step; copies on two copy streams, double-buffered"},
            "gpu_launches": 11 * a.steps,
        }
        print(json.dumps(line))
    layer.close()
    dist.destroy_process_group()


def ep_e2e(torch, dist, layer, inp, bias, x_bf16, wts, shape, t, a):
    """EP step time with every step's activations (bf16) and logits copied from
    pinned host memory and its output copied back, copies double-buffered on
    their own streams; max over ranks."""
    keys = ("routing_logits", "x")
    host = {"routing_logits": inp["routing_logits"].cpu().pin_memory(),
            "x": x_bf16.cpu().pin_memory()}
    dev_in = [{k: torch.empty_like(host[k], device="cuda") for k in keys} for _ in range(2)]
    dev_out = [torch.empty(t, shape.hidden, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    out_host = [torch.empty(t, shape.hidden, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    for e in done + freed:
        e.record(comp)

    def copy_in(b):
        with torch.cuda.stream(h2d):
            h2d.wait_event(done[b])
            for k in keys:
                dev_in[b][k].copy_(host[k], non_blocking=True)
            ready[b].record(h2d)

    def loop(n, t0=None):
        if t0 is not None:
            t0.record(h2d)
        copy_in(0)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                copy_in(b ^ 1)
            comp.wait_event(ready[b])
            comp.wait_event(freed[b])
            layer.forward_bf16(dev_in[b]["routing_logits"], bias, dev_in[b]["x"], *wts,
                               shape.routed_scaling_factor, dev_out[b])
            done[b].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done[b])
                out_host[b].copy_(dev_out[b], non_blocking=True)
                freed[b].record(d2h)

    loop(2)
    torch.cuda.synchronize()
    dist.barrier()
    steps = max(3, a.steps // 2)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    loop(steps, t0)
    t1.record(d2h)
    torch.cuda.synchronize()
    ms = torch.tensor([t0.elapsed_time(t1) / steps], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


# ----------------------------------------------------------------------------
# reference arm
# ----------------------------------------------------------------------------

def run_reference(a):
    """CPU arm: the oracle restatement of the reference algorithm on host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from moe_b200 import workloads
    t = a.tokens or 8192
    torch.set_num_threads(os.cpu_count() or 1)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    sample = min(a.cpu_sample_tokens, t)
    # only the sample's routing rows are needed; weights are generated on the
    # GPU when there is one (fast) and copied per expert
    sshape = workloads.dsv3_shape(sample)
    inp = workloads.make_inputs(sshape, seed=0, device=dev)
    inp["routing_bias"] = torch.zeros_like(inp["routing_bias"])   # config 2: uniform routing
    times = []
    threads = os.cpu_count() or 1
    for i in range(a.warmup + a.steps):
        tps, dt, ns, threads = cpu_baseline(sshape, inp, sample, torch)
        if i >= a.warmup:
            times.append(dt)
    ms = statistics.mean(times) * 1e3
    value = sample / (ms * 1e-3)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(ms, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (dequantised FP8)", "data": "synthetic (seeded)",
        "config": {"workload": f"DeepSeek-V3 MoE layer, T={t}, 256 experts (config 2); "
                               f"each step a {sample}-token sample",
                   "model": "DeepSeek-V3 MoE layer", "parallelism": "CPU host cores"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{sample} tokens per step through the numpy oracle"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def main():
    a = parse()
    if a.build_flashinfer:
        build_flashinfer()
    elif a.flashinfer_contest:
        run_flashinfer_contest()
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
