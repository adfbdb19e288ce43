"""Benchmark of the gated-delta hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extras] [--no-cpu-baseline]
    python bench.py --profile prefill|varlen|decode|verify|verify_layer|attention|in_proj   (one untimed run of a case, for ncu)

Workloads (synthetic inputs with the benchmark configs' shapes and distributions; no
dataset or checkpoint is involved):

* ``prefill`` (headline, config 1): one gated-delta layer of the 9B shape, B=1, T=4096,
  16 key / 32 value heads, bf16 with an fp32 state: causal conv1d (k=4) + SiLU over the
  8192 qkv channels, chunked gated delta rule with the final state, output-gated RMSNorm.
  A step is one such layer pass; the metric unit is tokens/s.
* ``varlen`` (config 2): 32 packed sequences (lengths U{128..2048}, seed 2) with random
  fp32 initial states and final states.
* ``decode`` (config 3): 24 stacked layers (no projections between them), 256 sequences
  with fp32 state [32, 128, 128] and conv state [8192, 3]; a step is one new token
  through the fused decode layer of all 24 layers.
* ``verify`` (config 4): 128 sequences score 5 tokens through 24 layers writing the 5
  per-token fp32 states, then roll back to an accepted length U{1..5}.
* ``attention`` (the drafter side of a delta layer, not a BASELINE config): the mask-row
  attention of one decode cycle, 32 sequences x 12 mask rows x 32 heads over 4,108 cached keys.
* ``fp8`` (not a BASELINE config): the qkv projection with the reference's fp8 weights, at a decode
  batch and at prefill with the conv, beside bf16 weights (library and cuBLAS).
* ``in_proj`` (the GEMM in front of the path, not a BASELINE config): the merged input projection
  of one 9B-shaped layer, 4096 tokens x 4096 -> 12,352, with the causal conv + SiLU fused into the
  tcgen05 GEMM's epilogue; timed beside cuBLAS's matmul followed by the conv kernel.

Multi-GPU (torchrun, one process per GPU): every rank runs its own shard with no
collective on the data path (prefill: an independent replica per GPU; decode/verify:
sequences split across ranks); the step time is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
L2_BYTES = 126 * 2 ** 20
MiB = 2 ** 20
D = 128
H, HV = 16, 32
C_QKV = 2 * H * D + HV * D  # 8192 conv channels
METRIC = "gated-delta prefill tok/s & decode tok/s per GPU, 1–8 B200, % of roofline"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the dominant kernels from the committed ncu summaries."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as fh:
            return json.load(fh)
    except Exception:
        return {}


# ------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every 10 ms (read-only queries)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, device_index: int):
        self.idx = device_index
        self.sm: list[float] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self.running = False
        self.error = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[self.idx]) if visible else self.idx
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.nvml = pynvml
            self.running = True
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        except Exception as e:  # no NVML: report the clocks as unsampled
            self.error = str(e)
        return self

    def _poll(self):
        nv = self.nvml
        while self.running:
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for name, bit in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception as e:
                self.error = str(e)
                return
            time.sleep(0.01)

    def __exit__(self, *exc):
        self.running = False
        if hasattr(self, "thread"):
            self.thread.join(timeout=2)

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"],
                    **({"error": self.error} if self.error else {})}
        busy = [x for x in self.sm if x > 0.5 * max(self.sm)] or self.sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.sm)}


# ------------------------------------------------------------------------------------------
# workloads
# ------------------------------------------------------------------------------------------
def make_prefill_inputs(seed=1, T=4096, device="cpu", pin=False):
    gen = torch.Generator().manual_seed(seed)
    qkv = torch.randn(1, T, C_QKV, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C_QKV, 4, generator=gen) * 0.5).to(torch.bfloat16)
    g = -torch.exp(torch.randn(1, T, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(1, T, HV, generator=gen)).to(torch.bfloat16)
    z = torch.randn(1, T, HV, D, generator=gen).to(torch.bfloat16)
    nw = (torch.rand(D, generator=gen) + 0.5).to(torch.bfloat16)
    out = dict(qkv=qkv, w=w, g=g, beta=beta, z=z, nw=nw)
    if pin:
        out = {k: v.pin_memory() for k, v in out.items()}
    if device != "cpu":
        out = {k: v.to(device) for k, v in out.items()}
    return out


def prefill_layer(gdn, x):
    """conv1d + SiLU -> chunked gated delta rule (final state) with the gated RMSNorm fused in."""
    return gdn.prefill_layer(x["qkv"], x["w"], x["g"], x["beta"], x["z"], x["nw"], H)


def prefill_core_bytes(T, n_seq=1, with_h0=False):
    """Algorithmic bytes of the chunk kernel: q, k at H key heads, v, o, g, beta once; states."""
    per_token = 2 * H * D * 2 + HV * D * 2 + HV * D * 2 + HV * (4 + 2)
    state = HV * D * D * 4
    return T * per_token + n_seq * state * (2 if with_h0 else 1)


def prefill_flops(T):
    return T * HV * 180_224


def chunk_plan(n_seq, packed, device, norm=False):
    """Kernels one gdn_chunk_prefill (norm: gdn_chunk_prefill_gated_norm) call launches, as the
    library chooses them: one cooperative chunk_fused_kernel when the scan CTAs (two per value
    head and sequence) plus 16 factor CTAs fit on the SMs at once; otherwise chunk_factor_kernel
    and chunk_scan_kernel, with seq_order_kernel between them for a packed batch of 2 to 1024
    sequences; then gated_rmsnorm_kernel for the norm."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    norm_k = ["gated_rmsnorm_kernel"] if norm else []
    if 2 * HV * n_seq + 16 <= sms:
        return ["chunk_fused_kernel"] + norm_k
    names = ["chunk_factor_kernel"]
    if packed and 1 < n_seq <= 1024:
        names.append("seq_order_kernel")
    return names + ["chunk_scan_kernel"] + norm_k


def varlen_lengths(seed=2, n=32):
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(128, 2049, (n,), generator=gen).tolist()


# ------------------------------------------------------------------------------------------
def timed(fn, steps, warmup, rank_sync, stream=None, inner_events=None):
    for _ in range(warmup):
        fn(0)
    torch.cuda.synchronize()
    rank_sync()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for i in range(steps):
        fn(i)
    stop.record()
    torch.cuda.synchronize()
    rank_sync()
    return start.elapsed_time(stop)


def capture(fn):
    """One CUDA graph of fn(0), after a warm-up call on a side stream (library state and the
    caching allocator are set up before the capture), as the engine captures its steps
    (inference/engine.py:337-345)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn(0)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn(0)
    torch.cuda.synchronize()
    return graph


def run_ours(args, rank, world, device, rank_sync, reduce_max):
    import jeeves_b200 as gdn

    gdn.load_library()
    hbm_peak, tc_peak, peak_kind = peaks()
    traffic = profiled_traffic()
    result = {}

    # ---------------- prefill (config 1), the headline ----------------
    T = 4096
    host = make_prefill_inputs(seed=1, T=T, pin=True)
    set_bytes = sum(v.numel() * v.element_size() for v in host.values()) + T * HV * D * 2 * 3
    n_sets = max(2, -(-2 * L2_BYTES // set_bytes))
    sets = [make_prefill_inputs(seed=1 + i, T=T, device=device) for i in range(n_sets)]
    kernel_ms = []
    ev_pairs = []

    def prefill_step(i):
        x = sets[i % n_sets]
        y = gdn.causal_conv1d(x["qkv"], x["w"])
        q = y[..., :H * D].view(1, T, H, D)
        k = y[..., H * D:2 * H * D].view(1, T, H, D)
        v = y[..., 2 * H * D:].view(1, T, HV, D)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        o, final = gdn.gated_delta_rule_chunk(q, k, v, x["g"], x["beta"], output_final_state=True)
        b.record()
        ev_pairs.append((a, b))
        gdn.gated_rms_norm(o.view(-1, D), x["z"].view(-1, D), x["nw"])

    clocks = ClockSampler(device.index).__enter__()  # sampled across every timed region below
    eager_ms = timed(prefill_step, args.steps, args.warmup, rank_sync)
    torch.cuda.synchronize()
    kernel_ms = [a.elapsed_time(b) for a, b in ev_pairs[args.warmup:]]
    eager_ms = reduce_max(eager_ms)
    # The headline: the layer as the engine runs a prefill (inference/engine.py:309-360, its extend
    # graphs): conv, then the chunk call with the gated norm, one CUDA graph per input set, replayed.
    graphs = [capture(lambda i, x=x: prefill_layer(gdn, x)) for x in sets]
    ms = reduce_max(timed(lambda i: graphs[i % n_sets].replay(), args.steps, args.warmup, rank_sync))
    ms_step = ms / args.steps
    value = world * T * args.steps / (ms / 1e3)
    k_ms = statistics.mean(kernel_ms)
    core_bytes = prefill_core_bytes(T)
    achieved = core_bytes / (k_ms / 1e3) / 1e9
    plan = chunk_plan(1, False, device)
    launches_per_step = 2 + len(plan)  # conv, the chunk kernels, gated norm

    # e2e: host buffers in, result out, through the public API. Every step uploads its inputs from
    # pinned host memory and downloads its output and final state; uploads, compute and downloads
    # run on three streams with two device input sets, so that step i+1's upload and step i-1's
    # download overlap step i's compute, as a serving pipeline would run them.
    dev_sets = [make_prefill_inputs(seed=1, T=T, device=device) for _ in range(2)]
    out_host = torch.empty(T * HV, D, dtype=torch.bfloat16).pin_memory()
    state_host = torch.empty(1, HV, D, D, dtype=torch.float32).pin_memory()
    compute = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(up):
            up.wait_event(computed[b])  # the set's previous step is done with it
            for key in ("qkv", "g", "beta", "z"):
                dev_sets[b][key].copy_(host[key], non_blocking=True)
            uploaded[b].record(up)
        compute.wait_event(uploaded[b])
        out, final = prefill_layer(gdn, dev_sets[b])
        computed[b].record(compute)
        with torch.cuda.stream(down):
            down.wait_event(computed[b])
            out_host.copy_(out.view(-1, D), non_blocking=True)
            state_host.copy_(final, non_blocking=True)
        out.record_stream(down)
        final.record_stream(down)

    def e2e_timed(steps, warmup):
        for i in range(warmup):
            e2e_step(i)
        torch.cuda.synchronize()
        rank_sync()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(compute)
        up.wait_stream(compute)
        down.wait_stream(compute)
        for i in range(steps):
            e2e_step(i)
        compute.wait_stream(up)
        compute.wait_stream(down)
        stop.record(compute)
        torch.cuda.synchronize()
        rank_sync()
        return start.elapsed_time(stop)

    e2e_ms = reduce_max(e2e_timed(args.steps, args.warmup))
    h2d = sum(host[k].numel() * host[k].element_size() for k in ("qkv", "g", "beta", "z"))
    d2h = out_host.numel() * 2 + state_host.numel() * 4

    # The bound of the e2e number: the same copies with no compute, in the same three-stream
    # pipeline (every rank at once, as they share the host's PCIe and memory), and each direction
    # alone. e2e can at best reach max(copy pipeline, device step) per step.
    out_dev = torch.empty(T * HV, D, dtype=torch.bfloat16, device=device)
    state_dev = torch.empty(1, HV, D, D, dtype=torch.float32, device=device)

    def copy_step(i, up_dir=True, down_dir=True):
        b = i % 2
        if up_dir:
            with torch.cuda.stream(up):
                up.wait_event(computed[b])
                for key in ("qkv", "g", "beta", "z"):
                    dev_sets[b][key].copy_(host[key], non_blocking=True)
                uploaded[b].record(up)
            compute.wait_event(uploaded[b])
        computed[b].record(compute)
        if down_dir:
            with torch.cuda.stream(down):
                down.wait_event(computed[b])
                out_host.copy_(out_dev, non_blocking=True)
                state_host.copy_(state_dev, non_blocking=True)

    def copies_timed(steps, warmup, **dirs):
        for i in range(warmup):
            copy_step(i, **dirs)
        torch.cuda.synchronize()
        rank_sync()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(compute)
        up.wait_stream(compute)
        down.wait_stream(compute)
        for i in range(steps):
            copy_step(i, **dirs)
        compute.wait_stream(up)
        compute.wait_stream(down)
        stop.record(compute)
        torch.cuda.synchronize()
        rank_sync()
        return start.elapsed_time(stop) / steps

    copy_ms = reduce_max(copies_timed(args.steps, args.warmup))
    h2d_ms = reduce_max(copies_timed(args.steps, args.warmup, down_dir=False))
    d2h_ms = reduce_max(copies_timed(args.steps, args.warmup, up_dir=False))
    bound_ms = max(copy_ms, ms_step)
    e2e_value = world * T * args.steps / (e2e_ms / 1e3)
    e2e_peak = world * T / (bound_ms / 1e3)

    result.update({
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "eager_ms_per_step": round(eager_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) qkv/z, g=-exp(N(-3,0.5)), beta=sigmoid(N(0,1)); no dataset)",
        "config": {"workload": "config 1: 9B-shaped prefill layer, B=1, T=4096, 16/32 heads, d=128, conv1d k=4 + SiLU, "
                               "chunked gated delta rule (final state), gated RMSNorm; replayed as one CUDA graph per "
                               "input set (eager_ms_per_step: the same step launched from Python)",
                   "tokens_per_gpu_step": T, "parallelism": f"replicas x{world} (no collective)",
                   "l2": f"inputs rotate over {n_sets} sets of {set_bytes / MiB:.0f} MiB (> L2)"},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "roofline": {"bound": "pcie (pinned host copies)", "achieved": round(e2e_value, 1),
                             "peak": round(e2e_peak, 1), "unit": "tokens/s", "frac": round(e2e_value / e2e_peak, 4),
                             "copy_pipeline_ms_per_step": round(copy_ms, 4),
                             "h2d_gbs_per_gpu": round(h2d / (h2d_ms / 1e3) / 1e9, 1),
                             "d2h_gbs_per_gpu": round(d2h / (d2h_ms / 1e3) / 1e9, 1),
                             "note": "peak = tokens per step / max(the step's copies alone in the same pipeline, the "
                                     "device step); all ranks copy at once"}},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                     "kernel": "gated_delta_rule_chunk (" + " + ".join(plan) + ")",
                     "kernel_ms": round(k_ms, 4),
                     "algorithmic_bytes": core_bytes,
                     "traffic": traffic.get("prefill", {}).get("dram_bytes_per_launch"),
                     "tensor_frac": round(prefill_flops(T) / (k_ms / 1e3) / 1e12 / tc_peak, 4)},
    })

    # ---------------- extras: varlen, decode, verify ----------------
    if args.extras:
        extra = {}
        extra["varlen"] = bench_varlen(gdn, args, device, rank_sync, reduce_max, world, hbm_peak, rank)
        # ncu traffic was captured on one GPU running the whole case; with N ranks each runs a shard
        extra["varlen"]["roofline"]["traffic"] = traffic.get("varlen", {}).get("dram_bytes_per_launch") if world == 1 else None
        extra["decode"] = bench_decode(gdn, args, device, rank, world, rank_sync, reduce_max, hbm_peak)
        extra["verify"] = bench_verify(gdn, args, device, rank, world, rank_sync, reduce_max, hbm_peak)
        extra["attention"] = bench_attention(gdn, args, device, rank, world, rank_sync, reduce_max, hbm_peak)
        extra["attention"]["roofline"]["traffic"] = (traffic.get("attention", {}).get("dram_bytes_per_launch")
                                                     if world == 1 else None)
        extra["in_proj"] = bench_in_proj(gdn, args, device, rank_sync, reduce_max, world, tc_peak)
        extra["fp8"] = bench_fp8(gdn, args, device, rank_sync, reduce_max, world, hbm_peak, tc_peak)
        result["extra"] = extra
        result["gpu_launches"] += sum(e.get("gpu_launches", 0) for e in extra.values())
    clocks.__exit__(None, None, None)
    result["clocks"] = clocks.summary()
    return result


def bench_varlen(gdn, args, device, rank_sync, reduce_max, world, hbm_peak, rank=0):
    from jeeves_b200 import sharding

    lens_all = varlen_lengths()
    Ttot_all = sum(lens_all)
    idx, lens, cu_local = sharding.local_varlen(lens_all, rank, world)  # longest-first balance
    N = len(lens)
    Ttot = sum(lens)
    gen = torch.Generator().manual_seed(2 + 1000 * rank)
    q = torch.randn(1, Ttot, H, D, generator=gen)
    q = (q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6)).to(torch.bfloat16).to(device)
    k = torch.randn(1, Ttot, H, D, generator=gen)
    k = (k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)).to(torch.bfloat16).to(device)
    v = torch.randn(1, Ttot, HV, D, generator=gen).to(torch.bfloat16).to(device)
    g = (-torch.exp(torch.randn(1, Ttot, HV, generator=gen) * 0.5 - 3.0)).to(device)
    beta = torch.sigmoid(torch.randn(1, Ttot, HV, generator=gen)).to(torch.bfloat16).to(device)
    h0 = (torch.randn(N, HV, D, D, generator=gen) * 0.02).to(device)
    cu = cu_local.to(device)

    def step(i):
        gdn.gated_delta_rule_chunk(q, k, v, g, beta, initial_state=h0, output_final_state=True, cu_seqlens=cu)

    steps = max(3, args.steps // 2)
    ms = reduce_max(timed(step, steps, args.warmup, rank_sync)) / steps
    bytes_ = prefill_core_bytes(Ttot, n_seq=N, with_h0=True)
    ach = bytes_ / (ms / 1e3) / 1e9
    return {"workload": f"config 2: 32 packed sequences U{{128..2048}} (seed 2), cu_seqlens, initial+final state; "
                        f"sequences balanced longest-first over {world} GPU(s), {N} here",
            "tokens": Ttot_all, "value": round(Ttot_all / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 4),
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(ach / hbm_peak, 4), "algorithmic_bytes": bytes_},
            "gpu_launches": len(chunk_plan(N, True, device)) * steps}


def shard(n, rank, world):
    from jeeves_b200 import sharding

    start, count = sharding.row_shard(n, rank, world)
    return count, start


def bench_decode(gdn, args, device, rank, world, rank_sync, reduce_max, hbm_peak, layers=24, B_total=256, taps=3):
    """Config 3: the 24-layer decode step (conv step, L2 norms, gated delta rule step in place, gated
    RMSNorm per layer) captured once as a CUDA graph and replayed, as the engine replays its cycle
    graphs (inference/engine.py:486); the eager (uncaptured) time is reported beside it."""
    B, _ = shard(B_total, rank, world)
    gen = torch.Generator().manual_seed(3)
    states = [torch.zeros(B, HV, D, D, device=device) for _ in range(layers)]
    for s in states:
        s.normal_(0, 0.02)
    conv_states = [torch.randn(B, C_QKV, taps, device=device).to(torch.bfloat16) for _ in range(layers)]
    w = [(torch.randn(C_QKV, 4, generator=gen) * 0.5).to(torch.bfloat16).to(device) for _ in range(layers)]
    nw = (torch.rand(D, generator=gen) + 0.5).to(torch.bfloat16).to(device)
    qkv = [torch.randn(B, C_QKV, device=device).to(torch.bfloat16) for _ in range(layers)]
    g = [(-torch.exp(torch.randn(B, HV, device=device) * 0.5 - 3.0)) for _ in range(layers)]
    beta = [torch.sigmoid(torch.randn(B, HV, device=device)).to(torch.bfloat16) for _ in range(layers)]
    z = [torch.randn(B, HV, D, device=device).to(torch.bfloat16) for _ in range(layers)]
    workspace = torch.empty(B, C_QKV, dtype=torch.bfloat16, device=device)

    def step(i):
        for l in range(layers):
            gdn.decode_layer_step(qkv[l], conv_states[l], w[l], g[l], beta[l], states[l], z[l], nw, H,
                                  workspace=workspace)

    eager_ms = reduce_max(timed(step, args.steps, args.warmup, rank_sync)) / args.steps
    graph = capture(step)
    ms = reduce_max(timed(lambda i: graph.replay(), args.steps, args.warmup, rank_sync)) / args.steps
    del graph
    unit_bytes = 2 * HV * D * D * 4 + 2 * C_QKV * taps * 2 + C_QKV * 2 + HV * 6 + 2 * HV * D * 2
    total = unit_bytes * B * layers
    ach = total / (ms / 1e3) / 1e9
    return {"workload": f"config 3: 24 layers, {B_total} sequences (state [32,128,128] fp32, conv state [8192,3]), "
                        f"one token per step, conv step + L2 + GDN step + gated norm per layer, the 24-layer step "
                        f"replayed as one CUDA graph; {B} sequences per GPU",
            "value": round(world * B / (ms / 1e3), 1), "unit": "tokens/s (sequences x steps)", "ms_per_step": round(ms, 4),
            "eager_ms_per_step": round(eager_ms, 4),
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(ach / hbm_peak, 4), "algorithmic_bytes_per_unit": unit_bytes},
            "gpu_launches": 3 * layers * args.steps * 2}  # conv step, recurrent step, norm per layer: graph and eager arms


def attention_case(B, device, K=4, Hq=HV, Hkv=HV, Dh=D, Lw=4096, seed=5):
    """The drafter's mask-row attention of one decode cycle over a delta layer's key cache
    (inference/engine.py:436-437): B sequences, M = K (K - 1) mask rows, Lw cached keys plus the
    M tail keys; every row sees the cache up to its own limit and its block's tail keys."""
    gen = torch.Generator().manual_seed(seed)
    M = K * (K - 1)
    L = Lw + M
    q = torch.randn(B, M, Hq, Dh, generator=gen).to(torch.bfloat16).to(device)
    k_cache = torch.randn(B, L, Hkv, Dh, generator=gen).to(torch.bfloat16).to(device)
    v_cache = torch.randn(B, L, Hkv, Dh, generator=gen).to(torch.bfloat16).to(device)
    block = torch.arange(K).repeat_interleave(K - 1)
    n = torch.randint(Lw // 2, Lw - K, (B,), generator=gen)
    allow_cache = torch.arange(Lw)[None, None] <= (n[:, None] + block[None])[..., None]
    allow_tail = (block[:, None] == block[None, :])[None].expand(B, -1, -1)
    allowed = torch.cat((allow_cache, allow_tail), dim=2)[:, None]
    padded = torch.full((B, 1, M, L + 16 - L % 16), float("-inf"), dtype=torch.bfloat16)
    padded[..., :L].masked_fill_(allowed, 0.0)
    mask = padded.to(device)[..., :L]
    return q, k_cache, v_cache, mask


def bench_attention(gdn, args, device, rank, world, rank_sync, reduce_max, hbm_peak, B_total=32):
    B, _ = shard(B_total, rank, world)
    q, k_cache, v_cache, mask = attention_case(B, device)
    M, L = q.shape[1], mask.shape[-1]
    scale = D ** -0.5

    def step(i):
        gdn.decode_attention(q, k_cache, v_cache, mask, scale)

    ms = reduce_max(timed(step, args.steps, args.warmup, rank_sync)) / args.steps
    bytes_ = B * L * HV * D * 2 * 2 + q.numel() * 2 * 2 + B * M * L * 2  # K, V; q and o; mask
    ach = bytes_ / (ms / 1e3) / 1e9
    splits = -(-L // 128)
    return {"workload": f"drafter mask-row attention over a delta layer's key cache: {B_total} sequences x {M} mask rows x "
                        f"{HV} heads, d=128, {L} cached keys, bf16, additive mask; {B} sequences per GPU",
            "value": round(world * B * M / (ms / 1e3), 1), "unit": "query rows/s", "ms_per_step": round(ms, 4),
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(ach / hbm_peak, 4), "algorithmic_bytes": bytes_},
            "gpu_launches": (2 if splits > 1 else 1) * args.steps}


IN_PROJ_N = C_QKV + HV * D + 2 * HV  # merged projection rows: qkv, z, b, a (12,352 at the 9B shape)


def in_proj_case(device, T=4096, K=4096, seed=6):
    """The merged input projection of one 9B-shaped gated-delta layer (hidden 4096 -> qkv 8192,
    z 4096, b 32, a 32) over T tokens, with the depthwise conv weights of the qkv channels."""
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(T, K, generator=gen).to(torch.bfloat16).to(device)
    w = (torch.randn(IN_PROJ_N, K, generator=gen) * K ** -0.5).to(torch.bfloat16).to(device)
    cw = (torch.randn(C_QKV, 4, generator=gen) * 0.5).to(torch.bfloat16).to(device)
    return x, w, cw


def bench_in_proj(gdn, args, device, rank_sync, reduce_max, world, tc_peak, T=4096, K=4096):
    """Fused projection + conv (one tcgen05 kernel) against cuBLAS's matmul followed by the
    library's conv kernel, the unfused form of the same two steps; every rank runs its own replica."""
    x, w, cw = in_proj_case(device, T, K)
    fused_ms = reduce_max(timed(lambda i: gdn.in_proj_conv(x, w, cw, C_QKV), args.steps, args.warmup, rank_sync)) / args.steps

    def unfused(i):
        y = x @ w.T
        gdn.causal_conv1d(y[None, :, :C_QKV], cw)

    unfused_ms = reduce_max(timed(unfused, args.steps, args.warmup, rank_sync)) / args.steps
    flops = 2 * T * K * IN_PROJ_N
    ach = flops / (fused_ms / 1e3) / 1e12
    return {"workload": f"merged input projection of a 9B-shaped delta layer, T={T}, hidden {K} -> {IN_PROJ_N} "
                        f"(qkv {C_QKV} with causal conv k=4 + SiLU fused in the GEMM epilogue, z, b, a), bf16; "
                        f"one replica per GPU; x and w ({(T + IN_PROJ_N) * K * 2 / 2 ** 20:.0f} MiB) exceed L2",
            "value": round(world * T / (fused_ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(fused_ms, 4),
            "unfused_ms": round(unfused_ms, 4), "unfused": "torch matmul (cuBLAS) then gdn.causal_conv1d",
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": round(ach / tc_peak, 4), "algorithmic_flops": flops},
            "gpu_launches": 2 * args.steps}  # the fused kernel, and the conv kernel of the unfused arm


def bench_fp8(gdn, args, device, rank_sync, reduce_max, world, hbm_peak, tc_peak, K=4096, N=C_QKV):
    """The qkv projection with fp8 weights (the reference's FP8Linear: e4m3 codes, fp32 row
    scales; in fp8 the engine runs in_proj_qkv on its own, inference/engine.py:155-166): at a
    decode batch (256 rows, and 32 rows, a GPU's share of 256 on 8 GPUs; bound by the weights'
    bytes) and at prefill (4096 tokens with the conv in the epilogue, bound by the tensor pipe);
    beside them the same shapes with bf16 weights through the library and through cuBLAS. Every
    arm rotates over three weight sets (201 MB of bf16 weights, more than L2), as a decode step
    reads each layer's weights once: no call finds its weights in L2."""
    gen = torch.Generator().manual_seed(8)
    ws, scales, codes = [], [], []
    for _ in range(3):
        w = (torch.randn(N, K, generator=gen) * K ** -0.5).to(torch.bfloat16).to(device)
        scale = (w.float().abs().amax(1).clamp(min=1e-12) / torch.finfo(torch.float8_e4m3fn).max).contiguous()
        ws.append(w)
        scales.append(scale)
        codes.append((w.float() / scale[:, None]).to(torch.float8_e4m3fn).contiguous())
    cw = (torch.randn(N, 4, generator=gen) * 0.5).to(torch.bfloat16).to(device)
    res = {}
    for name, M, conv in (("decode", 256, 0), ("decode_32", 32, 0), ("prefill", 4096, N)):
        x = torch.randn(M, K, generator=gen).to(torch.bfloat16).to(device)
        arms = {"fp8": lambda i: gdn.in_proj_conv(x, codes[i % 3], cw, conv, weight_scale=scales[i % 3]),
                "bf16": lambda i: gdn.in_proj_conv(x, ws[i % 3], cw, conv),
                "cublas_bf16": lambda i: x @ ws[i % 3].T}
        if conv == 0:
            # a decode-sized call takes less device time than its host-side dispatch: each arm is
            # timed as a CUDA graph of three calls (one per weight set), as the engine replays its
            # decode steps, so that the time is the device's
            ms = {}
            for k, f in arms.items():
                graph = capture(lambda i, f=f: [f(j) for j in range(3)])
                ms[k] = reduce_max(timed(lambda i: graph.replay(), args.steps, args.warmup, rank_sync)) / (3 * args.steps)
                del graph
        else:
            ms = {k: reduce_max(timed(f, args.steps, args.warmup, rank_sync)) / args.steps for k, f in arms.items()}
        entry = {k + "_ms": round(v, 4) for k, v in ms.items()}
        if conv == 0:
            bytes_ = N * K + N * 4 + M * K * 2 + M * N * 2  # codes, scales, x, out
            ach = bytes_ / (ms["fp8"] / 1e3) / 1e9
            entry["roofline"] = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                                 "frac": round(ach / hbm_peak, 4), "algorithmic_bytes": bytes_}
        else:
            ach = 2 * M * K * N / (ms["fp8"] / 1e3) / 1e12
            entry["roofline"] = {"bound": "tensor", "achieved": round(ach, 1), "peak": tc_peak, "unit": "TFLOP/s",
                                 "frac": round(ach / tc_peak, 4)}
        entry["rows"] = M
        entry["conv"] = bool(conv)
        res[name] = entry
    return {"workload": f"qkv projection {K} -> {N} with fp8 (e4m3, per-row scale) weights; decode: 256 and 32 rows, "
                        f"no conv (K split over clusters of CTAs); prefill: 4096 tokens with the causal conv + SiLU in "
                        f"the epilogue; three weight sets rotated (> L2), the decode shapes as CUDA graphs of three calls; one "
                        f"replica per GPU",
            "value": round(world * 256 / (res["decode"]["fp8_ms"] / 1e3), 1), "unit": "rows/s (decode)",
            # per step: the decode shapes 3 calls each of fp8 (row kernel, GEMM) and bf16 (GEMM); prefill fp8
            # 3 (row kernel, code conversion, GEMM on CTA pairs) and bf16 1
            **res, "gpu_launches": (2 * 3 * 3 + 4) * args.steps}


def verify_unit_bytes(design, T=5, taps=3):
    """Algorithmic bytes per (sequence, layer, step) of the verify layer, for the design built:
    conv state read and rolled forward, the ext window written and its kept columns read back, the
    pre-conv qkv of the T tokens, g / beta, z in and y out; then the recurrent state:
    * "recompute" (the reference's design, inference/engine.py:250-258): the verify reads the state,
      the commit reads and writes it once more; k and v of the T tokens are kept for the commit;
    * "snapshots": the verify reads the state and writes T per-token states; the rollback copy that
      makes snapshot j-1 live is this library's choice and is not counted;
    * "deltas": as "recompute", but the verify keeps each token's update vector (fp32) and the
      commit reads those and k instead of k and v."""
    state = HV * D * D * 4
    conv = C_QKV * taps * 2 * 3 + C_QKV * (taps + T) * 2
    io = T * C_QKV * 2 + T * HV * 6 + 2 * T * HV * D * 2
    if design == "recompute":
        return 3 * state + conv + io + 2 * T * (H * D + HV * D) * 2
    if design == "deltas":
        return 3 * state + conv + io + 2 * T * H * D * 2 + 2 * T * HV * D * 4
    return state * (1 + T) + conv + io


def verify_launches(design, B, layers):
    """Kernel launches of one config-4 step: per layer the conv step, the verify and the gated norm
    (for the kept-update-vector design below 2,048 states the norm runs inside the block verify),
    then the commits (one launch for all layers' kept update vectors, else one a layer) and the
    conv states' commit."""
    if design == "deltas":
        per_layer = 2 if B * HV < 2048 else 3
        return per_layer * layers + 1 + 1
    return 3 * layers + layers + 1


def bench_verify(gdn, args, device, rank, world, rank_sync, reduce_max, hbm_peak, layers=24, B_total=128, T=5,
                 taps=3):
    """Config 4: the verify branch of every delta layer (conv step over the conv-state window and
    the 5 new tokens, the gated delta rule outputs, gated RMSNorm), then the commit of the accepted
    tokens (recurrent state of every layer, and the conv states from the ext windows in one launch,
    inference/engine.py:471-474), the whole step replayed as one CUDA graph. Three designs: the
    reference's recompute (the commit advances each state by the accepted tokens again), kept
    update vectors (the verify runs as one tensor-core block per (row, head) state and keeps each
    token's delta; the commit applies the accepted ones in one streaming pass; states agree with
    the recompute to fp32 rounding) and per-token snapshots (the commit copies the accepted
    snapshot). The headline is the faster of the first two."""
    B, _ = shard(B_total, rank, world)
    gen = torch.Generator().manual_seed(4)
    states = [torch.zeros(B, HV, D, D, device=device).normal_(0, 0.02) for _ in range(layers)]
    conv_states = torch.randn(layers, B, C_QKV, taps, device=device).to(torch.bfloat16)
    ext = torch.empty(layers, B, C_QKV, taps + T, dtype=torch.bfloat16, device=device)
    w = [(torch.randn(C_QKV, 4, generator=gen) * 0.5).to(torch.bfloat16).to(device) for _ in range(layers)]
    nw = (torch.rand(D, generator=gen) + 0.5).to(torch.bfloat16).to(device)
    qkv = [torch.randn(B, T, C_QKV, device=device).to(torch.bfloat16) for _ in range(layers)]
    g = [(-torch.exp(torch.randn(B, T, HV, device=device) * 0.5 - 3.0)) for _ in range(layers)]
    beta = [torch.sigmoid(torch.randn(B, T, HV, device=device)).to(torch.bfloat16) for _ in range(layers)]
    z = [torch.randn(B, T, HV, D, device=device).to(torch.bfloat16) for _ in range(layers)]
    accepted = torch.randint(1, T + 1, (B,), generator=gen).to(device)
    out = {}
    for design in ("recompute", "deltas", "snapshots"):
        snaps = ([torch.empty(B, T, HV, D, D, device=device) for _ in range(layers)] if design == "snapshots"
                 else [None] * layers)
        deltas = ([torch.empty(B, T, HV, D, device=device) for _ in range(layers)] if design == "deltas"
                  else [None] * layers)

        def step(i):
            pending = [gdn.verify_layer_step(qkv[l], conv_states[l], w[l], g[l], beta[l], states[l], z[l], nw, H,
                                             ext_out=ext[l], snapshots=snaps[l], deltas=deltas[l])[1]
                       for l in range(layers)]
            gdn.verify_layers_commit(pending, states, accepted, ext=ext, conv_states=conv_states)

        graph = capture(step)
        ms = reduce_max(timed(lambda i: graph.replay(), args.steps, args.warmup, rank_sync)) / args.steps
        del graph, snaps, deltas
        unit = verify_unit_bytes(design, T, taps)
        ach = unit * B * layers / (ms / 1e3) / 1e9
        out[design] = {"ms_per_step": round(ms, 4), "value": round(world * B * T / (ms / 1e3), 1),
                       "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                                    "frac": round(ach / hbm_peak, 4), "algorithmic_bytes_per_unit": unit}}
    names = {"recompute": "recompute (the reference's: the commit advances the state by the accepted tokens)",
             "deltas": "kept update vectors (per layer one library call: the conv step, then the verify as one "
                       "tensor-core block per state as its programmatic dependent - one product of the state with the "
                       "10 k/q rows and their Gram, the 5-token recurrence unrolled per column, each token's delta "
                       "kept - and the gated norm; the commit applies the accepted ones to all 24 layers' states in "
                       "one streaming launch)"}
    head = min(("recompute", "deltas"), key=lambda d: out[d]["ms_per_step"])
    other = "deltas" if head == "recompute" else "recompute"
    best = out[head]
    return {"workload": f"config 4: 24 layers, {B_total} sequences x 5 tokens: per layer conv step over the conv-state "
                        f"window (ext kept), gated delta rule outputs, gated RMSNorm; then the commit of U{{1..5}} "
                        f"accepted tokens (recurrent states, and the conv states of all layers in one launch); the "
                        f"step replayed as one CUDA graph; {B} sequences per GPU",
            "design": names[head],
            "value": best["value"], "unit": "scored tokens/s", "ms_per_step": best["ms_per_step"],
            "roofline": best["roofline"], other: out[other], "snapshots": out["snapshots"],
            "gpu_launches": (verify_launches("recompute", B, layers) + verify_launches("deltas", B, layers) +
                             verify_launches("snapshots", B, layers)) * args.steps}


# ------------------------------------------------------------------------------------------
# CPU baseline: the reference's own eager functions (model/model.py) on the host cores when the
# reference is installed next to the repository (baseline/_ref, or JEEVES_REFERENCE); otherwise
# the oracle, a restatement of the same eager path
# ------------------------------------------------------------------------------------------
def reference_path():
    for cand in (os.environ.get("JEEVES_REFERENCE"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isfile(os.path.join(cand, "model", "model.py")):
            return cand
    return None


class CpuPath:
    """The CPU implementation timed as the baseline: the reference's eager functions
    (torch_chunk_gated_delta_rule, torch_recurrent_gated_delta_rule, causal_conv1d /
    causal_conv1d_step / eager_conv_step, GatedRMSNorm, gated_delta_rule_advance_inplace) when
    importable, else the oracle's restatement of them ("port")."""

    def __init__(self):
        path = reference_path()
        self.kind, self.where = "port", "oracle/ (fp32 PyTorch restatement of the reference's eager path)"
        self.mm = None
        if path is not None:
            try:
                if path not in sys.path:
                    sys.path.append(path)
                import model.model as mm  # the reference's own module

                self.mm, self.kind = mm, "reference"
                self.where = f"the reference's eager functions (model/model.py, imported from {os.path.relpath(path, ROOT)})"
            except Exception as e:  # fall back to the port, saying why
                self.where += f"; reference import failed: {type(e).__name__}: {e}"
        if self.mm is None:
            import oracle

            self.oracle = oracle

    def conv(self, x, w):
        return self.mm.causal_conv1d(x, w) if self.mm else self.oracle.causal_conv1d(x, w)

    def chunk(self, q, k, v, g, beta, h0=None, final=False):
        if self.mm:
            rep = v.shape[2] // q.shape[2]
            q, k = q.repeat_interleave(rep, dim=2), k.repeat_interleave(rep, dim=2)
            return self.mm.torch_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=final)
        return self.oracle.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=final)

    def recurrent(self, q, k, v, g, beta, h0=None, final=False):
        if self.mm:
            rep = v.shape[2] // q.shape[2]
            q, k = q.repeat_interleave(rep, dim=2), k.repeat_interleave(rep, dim=2)
            return self.mm.torch_recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=h0,
                                                            output_final_state=final)
        return self.oracle.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=final)

    def norm(self, x, z, w):
        if self.mm:
            mod = self.mm.GatedRMSNorm(D)
            with torch.no_grad():
                mod.weight.copy_(w.float())
            mod = mod.to(x.dtype)
            with torch.no_grad():
                return mod(x, z)
        return self.oracle.gated_rms_norm(x, z, w)

    def conv_step(self, x, state, w):
        return self.mm.causal_conv1d_step(x, state, w) if self.mm else self.oracle.causal_conv1d_step(x, state, w)

    def verify_conv(self, state, qkv, w):
        if self.mm:
            return self.mm.eager_conv_step(state, qkv, w.reshape(C_QKV, 1, -1), H * D, HV * D, D, D)
        return self.oracle.conv_step(state, qkv, w, H * D, HV * D, D, D)

    def advance(self, k, v, g, beta, state, steps):
        if self.mm:
            return self.mm.gated_delta_rule_advance_inplace(k, v, g, beta, state, steps)
        state.copy_(self.oracle.advance_gated_delta_rule(k, v, g, beta, state, steps))


def cpu_prefill_once(cpu, x, T):
    y = cpu.conv(x["qkv"], x["w"])
    q = y[..., :H * D].reshape(1, T, H, D)
    k = y[..., H * D:2 * H * D].reshape(1, T, H, D)
    v = y[..., 2 * H * D:].reshape(1, T, HV, D)
    o, S = cpu.chunk(q, k, v, x["g"], x["beta"], final=True)
    return cpu.norm(o.reshape(-1, D), x["z"].reshape(-1, D), x["nw"])


def cpu_threads():
    torch.set_num_threads(os.cpu_count() or 1)
    return torch.get_num_threads()


def cpu_baseline(cpu, T=4096, reps=2):
    cores = cpu_threads()
    x = make_prefill_inputs(seed=1, T=T)
    cpu_prefill_once(cpu, x, T)
    t0 = time.perf_counter()
    for _ in range(reps):
        cpu_prefill_once(cpu, x, T)
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(T / dt, 1), "unit": "tokens/s", "cores": cores, "kind": cpu.kind,
            "sample": f"config 1 prefill layer (conv + chunk GDN + gated norm), full T={T}, 1 warm-up + {reps} timed, "
                      f"{cpu.where} on {platform.processor() or platform.machine()}"}


def cpu_varlen(cpu):
    """Config 2 on the CPU: the reference has no packed path, so one chunk call per sequence with its
    initial and final state (the oracle's definition of the packed call), all 32 sequences once."""
    cores = cpu_threads()
    lens = varlen_lengths()
    gen = torch.Generator().manual_seed(2)
    t = 0.0
    for n, L in enumerate(lens):
        q = torch.randn(1, L, H, D, generator=gen).to(torch.bfloat16)
        k = torch.randn(1, L, H, D, generator=gen).to(torch.bfloat16)
        v = torch.randn(1, L, HV, D, generator=gen).to(torch.bfloat16)
        g = -torch.exp(torch.randn(1, L, HV, generator=gen) * 0.5 - 3.0)
        beta = torch.sigmoid(torch.randn(1, L, HV, generator=gen)).to(torch.bfloat16)
        h0 = torch.randn(1, HV, D, D, generator=gen) * 0.02
        t0 = time.perf_counter()
        cpu.chunk(q, k, v, g, beta, h0=h0, final=True)
        t += time.perf_counter() - t0
    return {"value": round(sum(lens) / t, 1), "unit": "tokens/s", "cores": cores, "kind": cpu.kind,
            "sample": f"all 32 sequences ({sum(lens)} tokens) once, one chunk call per sequence with initial and "
                      f"final state: {cpu.where}"}


def cpu_decode(cpu, B=256, layers_timed=2, layers=24, taps=4):
    """Config 3 on the CPU: the decode branch of one layer (conv step, recurrent step of one token,
    gated norm) at B=256, timed over `layers_timed` layers after one warm-up layer and extrapolated
    to the 24-layer step (a full step takes about half a minute per layer set here)."""
    cores = cpu_threads()
    gen = torch.Generator().manual_seed(3)
    w = (torch.randn(C_QKV, 4, generator=gen) * 0.5).to(torch.bfloat16)
    nw = (torch.rand(D, generator=gen) + 0.5).to(torch.bfloat16)
    conv_state = torch.randn(B, C_QKV, taps, generator=gen).to(torch.bfloat16)
    state = torch.randn(B, HV, D, D, generator=gen) * 0.02
    x = torch.randn(B, C_QKV, generator=gen).to(torch.bfloat16)
    g = -torch.exp(torch.randn(B, 1, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(B, 1, HV, generator=gen)).to(torch.bfloat16)
    z = torch.randn(B * HV, D, generator=gen).to(torch.bfloat16)

    def layer():
        nonlocal state
        y = cpu.conv_step(x, conv_state, w)
        q = y[:, None, :H * D].reshape(B, 1, H, D)
        k = y[:, None, H * D:2 * H * D].reshape(B, 1, H, D)
        v = y[:, None, 2 * H * D:].reshape(B, 1, HV, D)
        o, state = cpu.recurrent(q, k, v, g, beta, h0=state, final=True)
        cpu.norm(o.reshape(-1, D), z, nw)

    layer()
    t0 = time.perf_counter()
    for _ in range(layers_timed):
        layer()
    per_layer = (time.perf_counter() - t0) / layers_timed
    return {"value": round(B / (per_layer * layers), 1), "unit": "tokens/s (sequences x steps)", "cores": cores,
            "kind": cpu.kind, "extrapolated": True,
            "sample": f"{layers_timed} layers of the decode branch (conv step, one-token recurrent step, gated norm) "
                      f"at B={B} after 1 warm-up layer, extrapolated to the {layers}-layer step: {cpu.where}"}


def cpu_verify(cpu, B=128, T=5, layers_timed=1, layers=24, taps=4):
    """Config 4 on the CPU, the reference's recompute design: per layer the verify conv over the
    window, the recurrent outputs of the 5 tokens from the state, the gated norm, then the commit
    advance by the accepted tokens (gated_delta_rule_advance_inplace); timed over `layers_timed`
    layers after one warm-up layer and extrapolated to 24 layers."""
    cores = cpu_threads()
    gen = torch.Generator().manual_seed(4)
    w = (torch.randn(C_QKV, 4, generator=gen) * 0.5).to(torch.bfloat16)
    nw = (torch.rand(D, generator=gen) + 0.5).to(torch.bfloat16)
    conv_state = torch.randn(B, C_QKV, taps, generator=gen).to(torch.bfloat16)
    state = torch.randn(B, HV, D, D, generator=gen) * 0.02
    qkv = torch.randn(B, T, C_QKV, generator=gen).to(torch.bfloat16)
    g = -torch.exp(torch.randn(B, T, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen)).to(torch.bfloat16)
    z = torch.randn(B * T * HV, D, generator=gen).to(torch.bfloat16)
    accepted = torch.randint(1, T + 1, (B,), generator=gen)

    def layer():
        _, q, k, v = cpu.verify_conv(conv_state, qkv, w)
        o, _ = cpu.recurrent(q, k, v, g, beta, h0=state, final=False)
        cpu.norm(o.reshape(-1, D), z, nw)
        cpu.advance(k, v, g, beta, state, accepted)

    layer()
    t0 = time.perf_counter()
    for _ in range(layers_timed):
        layer()
    per_layer = (time.perf_counter() - t0) / layers_timed
    return {"value": round(B * T / (per_layer * layers), 1), "unit": "scored tokens/s", "cores": cores,
            "kind": cpu.kind, "extrapolated": True,
            "sample": f"{layers_timed} layer(s) of verify (conv over the window, 5-token recurrent outputs, gated "
                      f"norm) + commit advance at B={B} after 1 warm-up layer, extrapolated to {layers} layers: "
                      f"{cpu.where}"}


def run_reference(args, rank, world):
    """The reference's CPU implementation of the path on this box's host cores (its own eager
    functions when installed, else the oracle port), config 1."""
    if rank != 0:
        return None
    cpu = CpuPath()
    cores = cpu_threads()
    T = 4096
    x = make_prefill_inputs(seed=1, T=T)
    for _ in range(args.warmup):
        cpu_prefill_once(cpu, x, T)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_prefill_once(cpu, x, T)
    dt = time.perf_counter() - t0
    value = T * args.steps / dt
    return {"impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (same generator as the GPU arm)",
            "config": {"workload": "config 1: 9B-shaped prefill layer, B=1, T=4096, 16/32 heads (CPU, rank 0 only)"},
            "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": cores, "kind": cpu.kind,
                             "sample": f"full config-1 layer per step (conv + chunk GDN + gated norm, T={T}): "
                                       f"{cpu.where}"},
            "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def profile_case(name, device):
    """Runs one workload twice without timing, for `ncu -k ... -s 1 -c 1 python bench.py --profile NAME`."""
    import jeeves_b200 as gdn

    if name == "prefill":
        x = make_prefill_inputs(seed=1, device=device)
        for _ in range(2):
            prefill_layer(gdn, x)
    elif name == "varlen":
        lens = varlen_lengths()
        Tt, N = sum(lens), len(lens)
        q = torch.randn(1, Tt, H, D, device=device).to(torch.bfloat16)
        k = torch.randn(1, Tt, H, D, device=device).to(torch.bfloat16)
        v = torch.randn(1, Tt, HV, D, device=device).to(torch.bfloat16)
        g = -torch.rand(1, Tt, HV, device=device) * 0.1
        beta = torch.rand(1, Tt, HV, device=device).to(torch.bfloat16)
        h0 = torch.randn(N, HV, D, D, device=device) * 0.02
        cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=device)
        for _ in range(2):
            gdn.gated_delta_rule_chunk(q, k, v, g, beta, initial_state=h0, output_final_state=True, cu_seqlens=cu)
    elif name == "decode":
        B = 256
        state = torch.randn(B, HV, D, D, device=device) * 0.02
        cs = torch.randn(B, C_QKV, 3, device=device).to(torch.bfloat16)
        w = (torch.randn(C_QKV, 4, device=device) * 0.5).to(torch.bfloat16)
        qkv = torch.randn(B, C_QKV, device=device).to(torch.bfloat16)
        g = -torch.rand(B, HV, device=device) * 0.1
        beta = torch.rand(B, HV, device=device).to(torch.bfloat16)
        z = torch.randn(B, HV, D, device=device).to(torch.bfloat16)
        nw = torch.ones(D, device=device, dtype=torch.bfloat16)
        for _ in range(2):
            gdn.decode_layer_step(qkv, cs, w, g, beta, state, z, nw, H)
    elif name == "attention":
        q, k_cache, v_cache, mask = attention_case(32, device)
        for _ in range(2):
            gdn.decode_attention(q, k_cache, v_cache, mask, D ** -0.5)
    elif name == "in_proj":
        x, w, cw = in_proj_case(device)
        for _ in range(2):
            gdn.in_proj_conv(x, w, cw, C_QKV)
    elif name == "in_proj_decode":  # extra.fp8's decode shape: 256 rows, qkv 4096 -> 8192, bf16 then fp8 weights
        gen = torch.Generator().manual_seed(8)
        w = (torch.randn(C_QKV, 4096, generator=gen) * 4096 ** -0.5).to(torch.bfloat16).to(device)
        scale = (w.float().abs().amax(1).clamp(min=1e-12) / torch.finfo(torch.float8_e4m3fn).max).contiguous()
        codes = (w.float() / scale[:, None]).to(torch.float8_e4m3fn).contiguous()
        cw = (torch.randn(C_QKV, 4, generator=gen) * 0.5).to(torch.bfloat16).to(device)
        x = torch.randn(256, 4096, generator=gen).to(torch.bfloat16).to(device)
        for _ in range(2):
            gdn.in_proj_conv(x, w, cw, 0)
            gdn.in_proj_conv(x, codes, cw, 0, weight_scale=scale)
    elif name in ("verify", "verify_layer"):  # the config-4 step of bench_verify (kept update vectors):
        # 24 layers, or one layer (B = 128 rows; 268 MB of state) for captures that replay kernels
        B, T, taps = 128, 5, 3
        layers = 24 if name == "verify" else 1
        states = [torch.randn(B, HV, D, D, device=device) * 0.02 for _ in range(layers)]
        conv_states = torch.randn(layers, B, C_QKV, taps, device=device).to(torch.bfloat16)
        ext = torch.empty(layers, B, C_QKV, taps + T, dtype=torch.bfloat16, device=device)
        w = (torch.randn(C_QKV, 4, device=device) * 0.5).to(torch.bfloat16)
        nw = torch.ones(D, device=device, dtype=torch.bfloat16)
        qkv = torch.randn(B, T, C_QKV, device=device).to(torch.bfloat16)
        g = -torch.rand(B, T, HV, device=device) * 0.1
        beta = torch.rand(B, T, HV, device=device).to(torch.bfloat16)
        z = torch.randn(B, T, HV, D, device=device).to(torch.bfloat16)
        acc = torch.randint(1, T + 1, (B,), device=device)
        deltas = [torch.empty(B, T, HV, D, device=device) for _ in range(layers)]
        for _ in range(2):
            pending = [gdn.verify_layer_step(qkv, conv_states[l], w, g, beta, states[l], z, nw, H, ext_out=ext[l],
                                             deltas=deltas[l])[1] for l in range(layers)]
            gdn.verify_layers_commit(pending, states, acc, ext=ext, conv_states=conv_states)
    else:
        raise SystemExit(f"unknown profile case {name}")
    torch.cuda.synchronize()
    print(f"profile case {name}: ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-extras", dest="extras", action="store_false")
    ap.add_argument("--no-cpu-baseline", dest="cpu", action="store_false")
    ap.add_argument("--profile", choices=("prefill", "varlen", "decode", "verify", "verify_layer", "attention", "in_proj",
                                           "in_proj_decode"),
                    help="run one workload twice, untimed, for an ncu capture")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    if not torch.cuda.is_available():
        print(json.dumps({"error": "no CUDA device"}))
        sys.exit(1)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if args.profile:
        profile_case(args.profile, device)
        return
    if world > 1:
        import datetime
        import torch.distributed as dist

        # NCCL prints its version banner on file descriptor 1 when the communicator is made;
        # stdout must carry the single JSON line alone, so fd 1 points at stderr meanwhile.
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
            dist.barrier()
        finally:
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)

        def rank_sync():
            dist.barrier()

        def reduce_max(x):
            t = torch.tensor([x], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t.item()
    else:
        def rank_sync():
            pass

        def reduce_max(x):
            return x

    result = run_ours(args, rank, world, device, rank_sync, reduce_max)
    if rank == 0 and world == 1 and args.cpu:
        cpu = CpuPath()
        result["cpu_baseline"] = cpu_baseline(cpu)
        if "extra" in result:
            result["extra"]["varlen"]["cpu_baseline"] = cpu_varlen(cpu)
            result["extra"]["decode"]["cpu_baseline"] = cpu_decode(cpu)
            result["extra"]["verify"]["cpu_baseline"] = cpu_verify(cpu)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
