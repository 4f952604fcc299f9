#!/usr/bin/env python3
"""Benchmark: INT4 MoE-layer decode on B200 (Mixtral-8x7B shape).

One step = one MoE layer forward (router top-2 over 8 experts, INT4 SwiGLU
experts H=4096 F=14336 group 128, weighted combine) over one batch of T
decode tokens.  T is swept over 1/8/32/64; the headline line is T=64.

* ``value``: tokens/s with inputs resident in HBM, the layer replayed as a CUDA
  graph; 4 layers with distinct weights are rotated so no step finds its
  weights in L2 (each layer reads >= 181 MB, L2 is 126 MB).
* ``e2e``: same metric through the public API (``MoELayerInt4.forward``) with
  the activations copied host->device from pinned memory and the output
  copied back every step.
* ``roofline``: algorithmic bytes of the layer pass (touched experts' packed
  bytes + activations in/out + router weight) / measured layer time, against
  the measured HBM copy bandwidth in MEASURED_PEAKS.json.
* ``cpu_baseline``: the numpy oracle of the reference's dequant-then-matmul
  path on this host's cores, on a bounded sample.

``--impl reference`` times the reference's CPU algorithm (the oracle port;
the reference itself is Python + Triton and is not installed on the GPU box)
on the same config and prints the same JSON line with ``"impl": "reference"``.

Config 4 (``glm_c4``): one GLM-4.5-Air MoE layer (H 4096, 128 experts of
moe_ffn 1408, sigmoid top-8 with correction bias) decoding a continuous batch
of 32 sequences per GPU.  At N = 1 it is measured beside the headline; with
``--gpus N`` (under torchrun) it IS the headline: each rank owns 128/N
experts and 32 tokens of its own (weak scaling), sends each token at most once
to every rank holding one of its picks and gets the partial outputs back with
NCCL all-to-alls (``hydranet_b200/ep.py``); the whole step is one CUDA graph
per layer, the time is the max over ranks, and rank 0 checks its output
against the single-GPU layer holding all 128 experts (``parity_rel_l2``,
``index_match``).  Scaling is read from ``glm_c4`` at every N (N = 1 included).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

H, F, E, TOPK = 4096, 14336, 8, 2
SWEEP = (1, 8, 32, 64)
HEADLINE_T = 64
N_LAYERS = 4
METRIC = "INT4 MoE decode tok/s & achieved HBM GB/s vs ~8 TB/s at 1/2/4/8 B200"
WORKLOAD = "mixtral8x7b_moe_layer_decode"
# Config 4: GLM-4.5-Air MoE layer decode, 32 sequences per GPU, expert-parallel at N > 1
G_H, G_F, G_E, G_K, G_T = 4096, 1408, 128, 8, 32
G_WORKLOAD = "glm45air_moe_layer_decode_ep"
G_LAYERS = 2  # distinct layers rotated: at N = 8 one rank's 16 experts (143 MB) alone would nearly fit L2


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# Config 5: one GLM-4.5-Air MoE layer, prefill (tensor-core bound).
P_T, P_H, P_F, P_E, P_K = 8192, 4096, 1408, 128, 8


def prefill_measure(args, dev):
    """Config 5 on this GPU: GLM-4.5-Air-shape MoE layer (H 4096, moe_ffn 1408,
    128 experts, sigmoid top-8 with correction bias), 8192 bf16 tokens.  Device
    time per layer step with CUDA events (eager launches; the step's prep,
    planner and two engine launches), FLOPs 2 * T * k * 3 * H * F, against the
    measured bf16 dense peak; per-phase times with events between phases."""
    import torch
    from hydranet_b200 import synth
    from hydranet_b200.moe import MoELayerInt4
    from hydranet_b200.packing import ExpertTable
    from hydranet_b200.router import GLM4SigmoidRouter

    shape = synth.MoEShape(P_H, P_F, P_E, P_K)
    table = ExpertTable(synth.device_experts(4321, shape, dev))
    r = GLM4SigmoidRouter(hidden_dim=P_H, num_experts=P_E, experts_per_token=P_K).to(dev)
    r.set_correction_bias(torch.from_numpy(synth.host_correction_bias(3, P_E)).to(dev))
    layer = MoELayerInt4(r, table).eval()
    x = torch.randn(P_T, P_H, generator=torch.Generator(dev).manual_seed(5), device=dev).to(torch.bfloat16)
    steps = max(3, min(args.steps, 20))
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        for _ in range(args.warmup):
            layer(x)
        torch.cuda.synchronize(dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index or 0) as clk:
            ev0.record(stream)
            for _ in range(steps):
                layer(x)
            ev1.record(stream)
            torch.cuda.synchronize(dev)
        ms = ev0.elapsed_time(ev1) / steps
        evs = []

        def mark(phase):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            evs[-1].append(ev)

        for _ in range(steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            evs.append([e0])
            layer.forward_phases(x, between=mark)
            e3 = torch.cuda.Event(enable_timing=True)
            e3.record(stream)
            evs[-1].append(e3)
        torch.cuda.synchronize(dev)
    phase = {k: statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evs)
             for i, k in enumerate(("route_ms", "gateup_ms", "down_ms"))}
    flops = 2.0 * P_T * P_K * 3 * P_H * P_F
    _, tc_peak, peak_kind = peaks()
    tf = flops / (ms * 1e-3) / 1e12
    del layer, table
    torch.cuda.empty_cache()
    cpu = None
    if not args.no_cpu_baseline:
        v, n, el, nt, ne = prefill_cpu_time()
        cpu = {"value": v, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"{n} oracle steps of {nt} tokens, sigmoid top-{P_K} over {ne} experts (eight expert "
                         f"MLPs per token as in config 5), numpy float32 dequant-then-matmul, {el:.1f}s"}
    return {"workload": "glm45air_moe_layer_prefill", "tokens": P_T, "hidden": P_H, "ffn": P_F, "experts": P_E,
            "top_k": P_K, "router": "sigmoid top-8, correction bias", "steps": steps, "warmup": args.warmup,
            "ms_per_step": ms, "tok_s": P_T / (ms * 1e-3),
            "roofline": {"bound": "tensor", "achieved": tf, "peak": tc_peak, "unit": "TFLOP/s", "frac": tf / tc_peak,
                         "peak_kind": peak_kind, "flops_per_step": flops},
            "phases": phase, "clocks": clk.summary(), "cpu_baseline": cpu}


def prefill_ep(args, dev, world, rank, barrier, max_over_ranks):
    """Config 5 expert-parallel: 8192 tokens per GPU (weak scaling), the 128
    experts split over the ranks, micro-batches of 8192 / world tokens per
    rank (``ExpertParallelMoE(chunk_tokens=...)``: every grouped call sees
    8192 rows, the exchanges of one micro-batch queued beside the experts of
    the next).  Eager launches; device time per layer step with CUDA events,
    max over ranks; FLOPs per rank 2 * T * k * 3 * H * F (on average a rank
    runs T * k assignments) against the bf16 dense peak.  Parity: rank 0's
    output against one GPU holding all experts."""
    import torch
    from hydranet_b200 import synth
    from hydranet_b200.ep import ExpertParallelMoE
    from hydranet_b200.moe import MoELayerInt4
    from hydranet_b200.packing import ExpertTable
    from hydranet_b200.router import GLM4SigmoidRouter

    per = P_E // world
    chunk = P_T // world
    slots = synth.device_experts(4321, synth.MoEShape(P_H, P_F, P_E, P_K), dev)
    r = GLM4SigmoidRouter(hidden_dim=P_H, num_experts=P_E, experts_per_token=P_K).to(dev)
    r.set_correction_bias(torch.from_numpy(synth.host_correction_bias(3, P_E)).to(dev))
    layer = ExpertParallelMoE(r, ExpertTable(slots[rank * per:(rank + 1) * per]), P_E, chunk_tokens=chunk).eval()
    full = ExpertTable(slots) if rank == 0 else None
    del slots
    x = torch.randn(P_T, P_H, generator=torch.Generator(dev).manual_seed(5 + rank), device=dev).to(torch.bfloat16)
    steps = max(3, min(args.steps, 10))
    with torch.no_grad():
        y = layer(x)
        parity = None
        if rank == 0:
            ref = MoELayerInt4(r, full).eval()(x)
            parity = float((y.float() - ref.float()).norm() / ref.float().norm())
            del ref
        full = None
        del y
        for _ in range(args.warmup):
            layer(x)
        torch.cuda.synchronize(dev)
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index or 0) as clk:
            ev0.record()
            for _ in range(steps):
                layer(x)
            ev1.record()
            torch.cuda.synchronize(dev)
        ms = max_over_ranks(ev0.elapsed_time(ev1) / steps)
        barrier()
    flops = 2.0 * P_T * P_K * 3 * P_H * P_F
    _, tc_peak, peak_kind = peaks()
    tf = flops / (ms * 1e-3) / 1e12
    del layer, x
    torch.cuda.empty_cache()
    return {"workload": "glm45air_moe_layer_prefill_ep", "n_gpus": world, "tokens_per_gpu": P_T,
            "experts_per_gpu": per, "micro_batch_tokens": chunk, "hidden": P_H, "ffn": P_F, "experts": P_E,
            "top_k": P_K, "steps": steps, "ms_per_step": ms, "tok_s": world * P_T / (ms * 1e-3),
            "parity_rel_l2": parity,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": tf / tc_peak, "peak_kind": peak_kind, "flops_per_gpu_step": flops,
                         "kernel": "whole layer step per rank (route, micro-batched exchange, experts, combine)"},
            "clocks": clk.summary()}


# DRAM bytes (read + write) of one gate/up engine launch, from the ncu capture
# summarised in profiles/ (per launch, same workload); None where not captured.
GATEUP_TRAFFIC = {64: 493860096}


def blob_bytes(h, f, g=128):
    return 3 * (f * h // 2 + f * (h // g) * 2)


class ClockSampler:
    """SM clock and clock-event reasons sampled DURING the timed region.

    NVML is polled from a thread about every millisecond (read-only queries),
    so even a region of a few milliseconds gets samples; nvidia-smi at its
    shortest interval is the fallback when NVML is unavailable.
    """

    # NVML clock-event reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, gpu_index: int, period_s: float = 0.001):
        self.gpu = gpu_index
        self.period = period_s
        self.sm, self.smax, self.mask = [], 0.0, 0
        self._stop = threading.Event()
        self.t = None
        self.nvml = None

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self._physical_index())
            self.smax = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.nvml = (nv, h, reasons)
            self._poll_once()  # the timed region may be shorter than one period
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            self.nvml = None
        return self

    def _physical_index(self):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            ids = [v.strip() for v in vis.split(",") if v.strip()]
            if self.gpu < len(ids) and ids[self.gpu].isdigit():
                return int(ids[self.gpu])
        return self.gpu

    def _poll_once(self):
        nv, h, reasons = self.nvml
        self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
        self.mask |= int(reasons(h))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._poll_once()
            except Exception:
                return
            time.sleep(self.period)

    def __exit__(self, *exc):
        if self.t is not None:
            self._stop.set()
            self.t.join(timeout=2)
            try:
                self._poll_once()
            except Exception:
                pass

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = sorted(n for bit, n in self.REASONS.items() if self.mask & bit)
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.smax, "reasons": names,
                "samples": len(self.sm), "source": "nvml"}


# ---------------------------------------------------------------------------
# CPU oracle timing (the reference's dequant-then-matmul path, restated)
# ---------------------------------------------------------------------------

class OracleLayer:
    """The oracle's MoE layer at config 2 (the reference's dequant-then-matmul
    path, restated in numpy float32).  Expert weights are dequantised INT4 values
    (random nibbles times fp16 group scales), built once outside any timing,
    as the reference's dequant mode registers float weights at load time."""

    def __init__(self, T: int):
        from concurrent.futures import ThreadPoolExecutor
        from oracle import int4_ref as R
        from hydranet_b200 import synth
        self.R = R

        def make(e):
            rng = np.random.default_rng(1000 + e)
            mats = []
            for n, k in ((F, H), (F, H), (H, F)):
                packed = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
                scales = (rng.random((n, k // 128), dtype=np.float32) * np.float32(0.005)).astype(np.float16)
                mats += [packed, scales]
            return R.DequantExpert.from_packed(*mats)

        with ThreadPoolExecutor(max_workers=min(8, cpu_threads())) as ex:
            self.experts = dict(enumerate(ex.map(make, range(E))))
        self.rw = synth.host_normal(99, (E, H), 0.02)
        self.x = R.round_to_bf16(np.random.default_rng(0).standard_normal((T, H), dtype=np.float32))
        self.T = T

    def step(self):
        idx, w, _ = self.R.softmax_topk_router_ref(self.x, self.rw, TOPK, "bf16")
        return self.R.moe_combine_ref(self.x, idx, w, self.experts)


REF_INSTALL = REPO / "baseline" / "_ref"


def import_reference():
    """The reference installed unmodified in baseline/_ref, importable as the
    package ``hydranet`` (its modules use package-relative imports); None when
    it is not installed."""
    if not (REF_INSTALL / "model" / "mixtral.py").exists():
        return None
    import tempfile
    root = tempfile.mkdtemp(prefix="hn_ref_")
    os.symlink(REF_INSTALL, os.path.join(root, "hydranet"))
    sys.path.insert(0, root)
    import importlib
    return importlib.import_module("hydranet")


class ReferenceCpuLayer:
    """The reference's own ``MixtralMoELayer`` (``model/mixtral.py:259-370``) on
    the host cores in its dequant mode: float32 weights registered with its
    ``ExpertCacheManager`` on the CPU, the forward it runs without a GPU
    (router, per-expert ``F.linear`` SwiGLU, ``index_add_``).  Weights are the
    dequantised random nibbles of ``OracleLayer`` (the timing depends on the
    shapes only); built outside any timing."""

    def __init__(self, T: int):
        import torch
        import importlib
        import_reference()
        cfg = importlib.import_module("hydranet.config")
        from hydranet.cache.expert_cache import ExpertCacheManager
        from hydranet.model.mixtral import MixtralMoELayer
        torch.set_num_threads(cpu_threads())
        mc = cfg.MixtralConfig()
        mc.num_layers, mc.num_experts, mc.hidden_dim, mc.intermediate_dim = 1, E, H, F
        cc = cfg.ExpertCacheConfig(pinned_slots=0, hot_slots=E // 2, probation_slots=E - E // 2,
                                   enable_affinity_bonus=False, enable_dynamic_slots=False,
                                   max_slots_per_layer=E + 1, enable_prefetch=False)
        self.cm = ExpertCacheManager(model_config=mc, cache_config=cc, device=torch.device("cpu"),
                                     dtype=torch.float32)
        base = OracleLayer(T)
        for e, ex in base.experts.items():
            self.cm.register_expert(0, e, {"gate_proj": torch.from_numpy(ex.gate), "up_proj": torch.from_numpy(ex.up),
                                           "down_proj": torch.from_numpy(ex.down)})
        base.experts = None
        self.layer = MixtralMoELayer(mc, cc, 0, self.cm)
        with torch.no_grad():
            self.layer.router.gate.weight.copy_(torch.from_numpy(base.rw))
        self.x = torch.from_numpy(base.x).view(1, T, H)
        self.T = T

    def step(self):
        import torch
        with torch.no_grad():
            return self.layer(self.x, top_k=2)

    def close(self):
        self.cm.shutdown()


def cpu_reference_time(T: int, budget_s: float = 15.0, max_steps: int = 400):
    """tok/s of the reference's own CPU layer (``ReferenceCpuLayer``) when the
    reference is installed, else of the oracle port; returns (tok/s, steps,
    seconds, kind)."""
    try:
        layer, kind = ReferenceCpuLayer(T), "reference"
    except Exception:  # noqa: BLE001 - not installed or not importable here: the restatement
        layer, kind = OracleLayer(T), "port"
    layer.step()  # warm-up (the cache manager fills its slots)
    steps, t0 = 0, time.perf_counter()
    while True:
        layer.step()
        steps += 1
        el = time.perf_counter() - t0
        if el > budget_s or steps >= max_steps:
            break
    if hasattr(layer, "close"):
        layer.close()
    return T * steps / el, steps, el, kind


def reference_triton_bar(dev) -> dict:
    """The reference's own Triton INT4 expert MLP (``expert_mlp_int4_fused``,
    ``kernels/int4_gemm.py:211-254``) on this B200 with float16 activations,
    its native dtype: device time per call on one Mixtral expert (its models
    call it once per touched expert) at 1 and 16 tokens, and the config-2
    layer times that implies (T = 1: two calls of 1 token; T = 64: eight calls
    of 16 tokens, the mean tokens per expert)."""
    try:
        import torch
        if import_reference() is None:
            return {"unavailable": "the reference is not installed in baseline/_ref"}
        from hydranet.kernels.int4_gemm import expert_mlp_int4_fused
        from hydranet_b200 import synth
        slot = synth.device_experts(11, synth.MoEShape(H, F, 1, 1), dev)[0]
        t = slot.tensors()
        res = {"kernel": "reference expert_mlp_int4_fused (Triton 3.6), float16", "us_per_call": {}}
        for m in (1, 16):
            x = torch.randn(m, H, device=dev, dtype=torch.float16)
            for _ in range(3):
                expert_mlp_int4_fused(x, *t, group_size=128)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(20):
                expert_mlp_int4_fused(x, *t, group_size=128)
            e1.record()
            torch.cuda.synchronize(dev)
            res["us_per_call"][str(m)] = e0.elapsed_time(e1) / 20 * 1e3
        res["layer_ms_est"] = {"1": 2 * res["us_per_call"]["1"] / 1e3, "64": 8 * res["us_per_call"]["16"] / 1e3}
        return res
    except Exception as exc:  # noqa: BLE001 - the bar is context; report why it is missing
        return {"unavailable": repr(exc)[:300]}


def cpu_oracle_time(T: int, budget_s: float = 15.0, max_steps: int = 400):
    """tok/s of the oracle MoE layer on the host cores over a bounded sample."""
    layer = OracleLayer(T)
    layer.step()  # warm-up
    steps, t0 = 0, time.perf_counter()
    while True:
        layer.step()
        steps += 1
        el = time.perf_counter() - t0
        if el > budget_s or steps >= max_steps:
            break
    return T * steps / el, steps, el


def decode_engine(T: int) -> str:
    """Engine of the config-2 decode phases at batch T: the mma.sync engine runs
    segments of up to 16 tokens (8 * pick_nt), tcgen05 the larger ones."""
    return "mma.sync" if T <= 16 else "tcgen05"


def decode_launches(T: int) -> int:
    """Kernels one layer step launches at config 2, as the library itself
    reports them (``hn_moe_layer_launches``, computed from the same layout
    decisions its launch code takes): prep, gate/up and down, plus the router
    GEMM from 256 tokens, the assignment-ordered token copy from 12
    assignments per expert, and the multi-CTA planner and the combine pass
    above 4096 assignments."""
    from hydranet_b200 import _lib
    return int(_lib.load().hn_moe_layer_launches(T, H, F, E, TOPK))


def prefill_cpu_time(budget_s: float = 10.0, n_tok: int = 256, n_exp: int = 16):
    """tok/s of the oracle's prefill layer (GLM-4.5-Air shapes, sigmoid top-8,
    dequant-then-matmul in numpy float32) on the host cores, over a bounded
    sample: n_tok tokens routed over n_exp experts, so each token still runs
    eight expert MLPs (the per-token work of config 5) with fewer weights in
    host memory."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import int4_ref as R
    from hydranet_b200 import synth

    def make(e):
        rng = np.random.default_rng(2000 + e)
        mats = []
        for n, k in ((P_F, P_H), (P_F, P_H), (P_H, P_F)):
            mats += [rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8),
                     (rng.random((n, k // 128), dtype=np.float32) * np.float32(0.005)).astype(np.float16)]
        return R.DequantExpert.from_packed(*mats)

    with ThreadPoolExecutor(max_workers=min(8, cpu_threads())) as ex:
        experts = dict(enumerate(ex.map(make, range(n_exp))))
    rw = synth.host_normal(98, (n_exp, P_H), 0.02)
    x = R.round_to_bf16(np.random.default_rng(1).standard_normal((n_tok, P_H), dtype=np.float32))

    def step():
        idx, w, _ = R.sigmoid_topk_router_ref(x, rw, P_K, "f32")
        return R.moe_combine_ref(x, idx, w, experts)

    step()
    steps, t0 = 0, time.perf_counter()
    while True:
        step()
        steps += 1
        el = time.perf_counter() - t0
        if el > budget_s or steps >= 20:
            break
    return n_tok * steps / el, steps, el, n_tok, n_exp


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args):
    """The reference's CPU algorithm (the oracle port) on this host's cores, on
    the GPU arm's workload: config 2 at N = 1, config 4 under --gpus N > 1
    (rank 0 alone; its step is the whole job's layer step of N x 32 tokens,
    timed from a bounded sample)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.gpus > 1:
        v1, ms1, sample = glm_cpu_time(budget_s=max(2.0, min(args.ref_budget, 10.0)))
        line = {"impl": "reference", "metric": METRIC, "value": v1, "unit": "tok/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms1, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": G_WORKLOAD, "tokens_per_gpu": G_T, "hidden": G_H, "moe_ffn": G_F,
                           "experts": G_E, "top_k": G_K, "group_size": 128},
                "cpu_baseline": {"value": v1, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
                                 "sample": sample},
                "e2e": {"value": v1, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    T = args.tokens
    try:
        layer, kind = ReferenceCpuLayer(T), "reference"
        what = "the reference's own MixtralMoELayer.forward (dequant mode, float32 weights, torch CPU)"
    except Exception:  # noqa: BLE001 - the reference is not installed: its restatement
        layer, kind = OracleLayer(T), "port"
        what = "oracle layer steps (numpy float32 dequant-then-matmul, weights dequantised before timing)"
    for _ in range(args.warmup):
        layer.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        layer.step()
    el = time.perf_counter() - t0
    v = T * args.steps / el
    if hasattr(layer, "close"):
        layer.close()
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens": T, "hidden": H, "ffn": F, "experts": E, "top_k": TOPK,
                       "group_size": 128},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cpu_threads(), "kind": kind,
                             "sample": f"{args.steps} steps at T={T}: {what}"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


C3_LAYERS, C3_SLOTS, C3_BLOBS = 32, 126, 16


def c3_measure(args, dev) -> dict:
    """Config 3's MoE path: 32 Mixtral-shape MoE layers decoding one token at a
    time through a 126-slot cache (``SlotCache``), router logits skewed per layer by a
    Zipf(s = 1.1) expert bias (log-weights -1.1 ln(rank) over a seeded
    permutation; a harness addition, as in the config).  Experts come from 16
    distinct pinned host blobs shared round-robin by the 256 (layer, expert)
    pairs: only the bytes moved matter to the cache.  Attention and the dense
    parts of the model are out of scope, so tok/s is the MoE path alone
    (routing, one host read per layer, H2D of misses, experts)."""
    import torch
    from hydranet_b200 import ops, synth, _lib
    from hydranet_b200.router import TopKRouter
    from hydranet_b200.slot_cache import ExpertSource, SlotCache, SlotCachedMoELayer

    blobs = [s.blob.cpu().pin_memory() for s in synth.device_experts(900, synth.MoEShape(H, F, C3_BLOBS, TOPK), dev)]
    source = ExpertSource(lambda layer, expert: blobs[(layer * E + expert) % C3_BLOBS])
    cache = SlotCache(H, F, C3_LAYERS, E, C3_SLOTS, source, device=dev)
    rng = np.random.default_rng(11)

    class ZipfLayer(SlotCachedMoELayer):
        def route(self, x):
            p = ops.router_params(_lib.HN_ROUTER_SOFTMAX_TOPK, TOPK, self.router.gate.weight, logits_in_act_dtype=True,
                                  affinity_bonus=self.zipf, entropy_threshold=-1.0)  # always added to the logits
            idx, w, _ = ops.moe_route(x, p, E, keep_refs=(self.zipf,), want_logits=False)
            return idx, w

    layers = []
    for li in range(C3_LAYERS):
        r = TopKRouter(hidden_dim=H, num_experts=E, experts_per_token=TOPK).to(dev, torch.bfloat16)
        with torch.no_grad():
            r.gate.weight.copy_(torch.randn(E, H, generator=torch.Generator(dev).manual_seed(300 + li), device=dev)
                                * 0.02)
        layer = ZipfLayer(r, cache, li)
        ranks = rng.permutation(E) + 1
        layer.zipf = torch.tensor(-1.1 * np.log(ranks), dtype=torch.float32, device=dev)
        layers.append(layer)
    gen = torch.Generator(dev).manual_seed(1)

    def through(x):
        for layer in layers:
            x = layer(x)
            # keep the synthetic stream at the N(0,1) scale (attention and norms are out of scope)
            x = x / x.float().norm(dim=-1, keepdim=True).clamp_min(1e-3).to(x.dtype) * (H ** 0.5)
        return x

    n_prompt, n_tok = 512, 128
    with torch.no_grad():
        through(torch.randn(n_prompt, H, generator=gen, device=dev).to(torch.bfloat16))  # the prompt fills the cache
        x = torch.randn(1, H, generator=gen, device=dev).to(torch.bfloat16)
        torch.cuda.synchronize(dev)
        s0 = (cache.stats.hits, cache.stats.misses, cache.stats.h2d_bytes)
        t0 = time.perf_counter()
        for _ in range(n_tok):
            x = through(x)
        torch.cuda.synchronize(dev)
        el = time.perf_counter() - t0
    hits, misses, h2d = (cache.stats.hits - s0[0], cache.stats.misses - s0[1], cache.stats.h2d_bytes - s0[2])
    res = {"workload": "mixtral8x7b_moe_path_decode_126_slots", "layers": C3_LAYERS, "slots": C3_SLOTS,
           "experts_total": C3_LAYERS * E, "prompt_tokens": n_prompt, "tokens": n_tok, "batch": 1,
           "router_skew": "Zipf(s=1.1) per-expert logit bias per layer", "tok_s": n_tok / el,
           "ms_per_token": 1e3 * el / n_tok, "hit_rate": hits / max(hits + misses, 1),
           "misses_per_token": misses / n_tok, "h2d_gbs": h2d / el / 1e9,
           "timing": "host wall clock around the 128 decode tokens (each layer reads its routing back to the host)"}
    del layers, cache, blobs
    torch.cuda.empty_cache()
    return res


def glm_cpu_time(budget_s: float = 10.0, n_exp: int = 16, tok_per_exp: int = 2):
    """Host-core time of one config-4 layer step (32 tokens, sigmoid top-8 over
    128 experts) by the oracle's dequant-then-matmul path, from a bounded
    sample: n_exp expert MLPs at tok_per_exp tokens each (the mean tokens per
    expert at config 4) are timed and the layer time is that times the
    experts the step touches (115, the mean over seeded routings) / n_exp;
    the router (2 MB of fp32 weights) is timed whole.  Returns (tok/s, ms per
    layer, sample description)."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import int4_ref as R
    from hydranet_b200 import synth

    def make(e):
        rng = np.random.default_rng(3000 + e)
        mats = []
        for n, k in ((G_F, G_H), (G_F, G_H), (G_H, G_F)):
            mats += [rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8),
                     (rng.random((n, k // 128), dtype=np.float32) * np.float32(0.005)).astype(np.float16)]
        return R.DequantExpert.from_packed(*mats)

    with ThreadPoolExecutor(max_workers=min(8, cpu_threads())) as ex:
        experts = list(ex.map(make, range(n_exp)))
    rw = synth.host_normal(97, (G_E, G_H), 0.02)
    x = R.round_to_bf16(np.random.default_rng(2).standard_normal((G_T, G_H), dtype=np.float32))
    xe = x[:tok_per_exp]

    def step():
        R.sigmoid_topk_router_ref(x, rw, G_K, "f32")
        t_r = time.perf_counter()
        for e in experts:
            e(xe)
        return time.perf_counter() - t_r

    step()
    steps, t0, t_exp = 0, time.perf_counter(), 0.0
    while True:
        t_exp += step()
        steps += 1
        el = time.perf_counter() - t0
        if el > budget_s or steps >= 50:
            break
    per_step = el / steps
    t_router = per_step - t_exp / steps
    layer_s = t_router + (t_exp / steps) * 115.0 / n_exp
    return G_T / layer_s, layer_s * 1e3, (f"{steps} samples of {n_exp} expert MLPs at {tok_per_exp} tokens each "
                                          f"plus the router over {G_T} tokens (numpy float32 dequant-then-matmul); "
                                          f"layer time = router + expert time x 115/{n_exp} touched experts")


def glm_c4(args, dev, world, rank, barrier, max_over_ranks):
    """Config 4 on `world` GPUs (expert-parallel when world > 1): device time per
    layer step (CUDA graph replay, max over ranks), tok/s of the whole job
    (world * 32 / step), the parity self-check on rank 0, per-rank algorithmic
    HBM bytes (the rank's touched experts + activations) / step time, and the
    end-to-end rate through the public module with host copies."""
    import torch
    import torch.distributed as dist
    from hydranet_b200 import ops, synth
    from hydranet_b200.ep import ExpertParallelMoE
    from hydranet_b200.moe import MoELayerInt4
    from hydranet_b200.packing import ExpertTable
    from hydranet_b200.router import GLM4SigmoidRouter

    per = G_E // world
    shape = synth.MoEShape(G_H, G_F, G_E, G_K)
    layers, full_tables, routers = [], [], []
    for li in range(G_LAYERS):
        slots = synth.device_experts(7000 + li, shape, dev)  # every rank builds the same 128 experts
        r = GLM4SigmoidRouter(hidden_dim=G_H, num_experts=G_E, experts_per_token=G_K).to(dev)
        with torch.no_grad():
            r.weight.copy_(torch.randn(G_E, G_H, generator=torch.Generator(dev).manual_seed(31 + li), device=dev)
                           * 0.02)
        r.set_correction_bias(torch.from_numpy(synth.host_correction_bias(41 + li, G_E)).to(dev))
        routers.append(r)
        if world > 1:
            layers.append(ExpertParallelMoE(r, ExpertTable(slots[rank * per:(rank + 1) * per]), G_E).eval())
            full_tables.append(ExpertTable(slots) if rank == 0 and li == 0 else None)
        else:
            layers.append(MoELayerInt4(r, ExpertTable(slots)).eval())
            full_tables.append(None)
        del slots
    xs = [torch.randn(G_T, G_H, generator=torch.Generator(dev).manual_seed(500 + 10 * rank + li), device=dev)
          .to(torch.bfloat16) for li in range(G_LAYERS)]
    # touched experts of this rank (any rank's tokens) -> algorithmic bytes per step
    touched = []
    with torch.no_grad():
        for li in range(G_LAYERS):
            idx, _, _ = ops.moe_route(xs[li], routers[li].params(), G_E, want_logits=False)
            if world > 1:
                allidx = [torch.empty_like(idx) for _ in range(world)]
                dist.all_gather(allidx, idx)
                idx = torch.cat(allidx)
                idx = idx[(idx >= rank * per) & (idx < (rank + 1) * per)]
            touched.append(int(torch.unique(idx).numel()))
    algo = statistics.mean(touched) * blob_bytes(G_H, G_F) + 2 * G_T * G_H * 2 + G_E * G_H * 4
    # parity self-check on rank 0: the expert-parallel output against one GPU holding all experts
    parity, index_match = None, None
    with torch.no_grad():
        y = layers[0](xs[0])
        if rank == 0:
            if world > 1:
                ref_layer = MoELayerInt4(routers[0], full_tables[0]).eval()
                ref, ro = ref_layer(xs[0], return_routing=True)
                idx_ep, _, _ = ops.moe_route(xs[0], routers[0].params(), G_E, want_logits=False)
                index_match = bool(torch.equal(idx_ep.long(), ro.expert_indices))
                parity = float((y.float() - ref.float()).norm() / ref.float().norm())
                del ref_layer
            else:
                index_match, parity = True, 0.0
    full_tables = None
    torch.cuda.synchronize(dev)
    barrier()
    graphs, note = None, None
    with torch.no_grad():
        try:
            st = torch.cuda.Stream(dev)
            st.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(st):
                for li in range(G_LAYERS):
                    layers[li](xs[li])  # warm-up on the capture stream (workspaces, communicators)
                torch.cuda.synchronize(dev)
                graphs = []
                for li in range(G_LAYERS):
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=st):
                        layers[li](xs[li])
                    graphs.append(g)
            torch.cuda.current_stream(dev).wait_stream(st)
            torch.cuda.synchronize(dev)
        except Exception as exc:  # noqa: BLE001 - a capture failure falls back to eager steps
            graphs, note = None, repr(exc)[:200]
            torch.cuda.synchronize(dev)
        ok = torch.tensor([1 if graphs else 0], device=dev, dtype=torch.int32)
        if world > 1:
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 0:
            graphs = None

        def step(i):
            if graphs:
                graphs[i % G_LAYERS].replay()
            else:
                layers[i % G_LAYERS](xs[i % G_LAYERS])

        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index or 0) as clk:
            ev0.record()
            for i in range(args.steps):
                step(i)
            ev1.record()
            torch.cuda.synchronize(dev)
        ms_graph = max_over_ranks(ev0.elapsed_time(ev1) / args.steps) if graphs else None
        barrier()
        # the same steps launched eagerly (with NCCL all-to-alls, replaying the
        # captured graphs is not always the faster way): device time, max over ranks
        for i in range(args.warmup):
            layers[i % G_LAYERS](xs[i % G_LAYERS])
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev2.record()
        for i in range(args.steps):
            layers[i % G_LAYERS](xs[i % G_LAYERS])
        ev3.record()
        torch.cuda.synchronize(dev)
        ms_eager = max_over_ranks(ev2.elapsed_time(ev3) / args.steps)
        barrier()
        ms = min(ms_eager, ms_graph) if ms_graph is not None else ms_eager
        mode = "cuda_graph" if ms_graph is not None and ms_graph <= ms_eager else "eager"
        captured = bool(graphs)
        # graphs holding NCCL work are released before the process group goes
        for gr in graphs or []:
            gr.reset()
        graphs, g, gr = None, None, None
        torch.cuda.synchronize(dev)
        # end to end through the public module: pinned host input -> device -> layer -> host
        x_host = [xs[li].cpu().pin_memory() for li in range(G_LAYERS)]
        x_dev = torch.empty(G_T, G_H, device=dev, dtype=torch.bfloat16)
        out_host = torch.empty(G_T, G_H, dtype=torch.bfloat16).pin_memory()
        for i in range(args.warmup):
            x_dev.copy_(x_host[i % G_LAYERS], non_blocking=True)
            out_host.copy_(layers[i % G_LAYERS](x_dev), non_blocking=True)
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            x_dev.copy_(x_host[i % G_LAYERS], non_blocking=True)
            out_host.copy_(layers[i % G_LAYERS](x_dev), non_blocking=True)
        e1.record()
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        barrier()
    hbm_peak, _, peak_kind = peaks()
    gbs = algo / (ms * 1e-3) / 1e9
    res = {"workload": G_WORKLOAD, "n_gpus": world, "tokens_per_gpu": G_T, "hidden": G_H, "moe_ffn": G_F,
           "experts": G_E, "experts_per_gpu": per, "top_k": G_K, "router": "sigmoid top-8, correction bias",
           "layers_rotated": G_LAYERS, "ms_per_step": ms, "tok_s": world * G_T / (ms * 1e-3),
           "cuda_graph": mode == "cuda_graph", "launch_mode": mode, "ms_graph": ms_graph, "ms_eager": ms_eager,
           "captured": captured, "parity_rel_l2": parity, "index_match": index_match,
           "touched_experts_per_gpu": statistics.mean(touched),
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                        "peak_kind": peak_kind, "algo_bytes_per_gpu_step": algo,
                        "kernel": "whole layer step per rank (route, pack, all-to-all, experts, all-to-all, combine)"
                        if world > 1 else "whole layer step (route, experts, combine)"},
           "e2e": {"value": world * G_T / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": G_T * G_H * 2,
                   "d2h_bytes_per_step": G_T * G_H * 2, "ms_per_step": e2e_ms},
           "clocks": clk.summary()}
    if note and rank == 0:
        res["graph_note"] = note
    if world > 1:
        res["phases_ms"] = ep_phase_times(layers[0], xs[0], max(3, min(args.steps, 20)), max_over_ranks, barrier)
    del layers, routers, xs
    torch.cuda.empty_cache()
    return res


def ep_step_launches(world: int) -> int:
    """Library kernels of one expert-parallel config-4 step: the router GEMV
    and routing, pack, unpack, the local grouped call's prep, gate/up and
    down (on the mma.sync engine at these shapes), the multi-CTA planner when
    the received block holds more than 1024 slots, and the combine."""
    return 8 + (world * G_T * G_K > 1024)


def ep_phase_times(layer, x, steps, max_over_ranks, barrier) -> dict:
    """Where an expert-parallel decode step spends its time: the steps of
    ``ep_moe_forward`` launched eagerly with CUDA events between them, all
    steps queued before one synchronisation so the GPU runs ahead of the
    host (device time per phase, median over steps -- a one-off stall of
    one step does not count -- max over ranks; a phase whose launch the host
    could not issue in time also counts the wait)."""
    import torch
    import torch.distributed as dist
    from hydranet_b200.ep import CudaExchange

    ex = CudaExchange()
    world = dist.get_world_size(layer.group)
    T, H = x.shape
    names = ("route", "pack", "dispatch_all_to_all", "unpack", "local_experts", "return_all_to_all", "combine")
    times = {n: [] for n in names}
    torch.cuda.synchronize()
    barrier()
    all_ev = []
    with torch.no_grad():
        for _ in range(steps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
            all_ev.append(ev)
            ev[0].record()
            idx, w = layer.route(x)
            ev[1].record()
            send = ex.pack(x, idx, w, layer.num_experts, world)
            ev[2].record()
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=layer.group)
            ev[3].record()
            rows, ids, wts = ex.unpack(recv, H, idx.shape[1], x.dtype)
            ev[4].record()
            y = layer.local_fn(rows, ids, wts).contiguous()
            ev[5].record()
            back = torch.empty_like(y)
            dist.all_to_all_single(back, y, group=layer.group)
            ev[6].record()
            ex.combine(back.view(world, T, H), idx, layer.num_experts, world)
            ev[7].record()
    torch.cuda.synchronize()
    for ev in all_ev:
        for i, n in enumerate(names):
            times[n].append(ev[i].elapsed_time(ev[i + 1]))
    barrier()
    return {n: max_over_ranks(statistics.median(v)) for n, v in times.items()}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=HEADLINE_T)
    ap.add_argument("--ref-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", type=str, default=",".join(map(str, SWEEP)),
                    help="comma-separated token batches to time (default 1,8,32,64)")
    ap.add_argument("--layers", type=int, default=N_LAYERS, help="distinct layers rotated per step")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-5 prefill measurement")
    ap.add_argument("--no-c3", action="store_true", help="skip the config-3 MoE-path (slot cache) measurement")
    ap.add_argument("--quick", action="store_true",
                    help="headline sweep only: no CPU baseline, reference GPU bar, prefill, GLM or config-3 "
                         "(for profiler captures of the decode kernels)")
    args = ap.parse_args()
    if args.quick:
        args.no_cpu_baseline = args.no_prefill = args.no_c3 = True
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist
    from hydranet_b200 import _lib, synth
    from hydranet_b200.moe import MoELayerInt4
    from hydranet_b200.packing import ExpertTable
    from hydranet_b200.router import TopKRouter

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    _lib.load()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if world > 1:
        # expert-parallel runs measure config 4 (GLM-4.5-Air layer, 32 sequences per GPU)
        g = glm_c4(args, dev, world, rank, barrier, max_over_ranks)
        pf = None if args.no_prefill else prefill_ep(args, dev, world, rank, barrier, max_over_ranks)
        if rank == 0:
            line = {
                "metric": METRIC, "value": g["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": g["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded, weights ~N(0,0.02) INT4 g128, activations ~N(0,1))",
                "config": {"workload": G_WORKLOAD, "tokens_per_gpu": G_T, "hidden": G_H, "moe_ffn": G_F,
                           "experts": G_E, "top_k": G_K, "group_size": 128, "layers_rotated": G_LAYERS,
                           "l2": f"{G_LAYERS} distinct layers rotated (>= 2 x 130 MB of touched weights per rank)",
                           "cuda_graph": g["cuda_graph"],
                           "parallelism": f"ep{world} (experts sharded, NCCL all-to-all, one row per token and rank)"},
                "roofline": {**g["roofline"], "traffic": None},
                "e2e": g["e2e"], "gpu_launches": ep_step_launches(world) * args.steps, "clocks": g["clocks"],
                "parity_rel_l2": g["parity_rel_l2"], "index_match": g["index_match"], "glm_c4": g,
                "prefill_ep": pf, "cpu_baseline": None,
            }
            print(json.dumps(line), flush=True)
        dist.destroy_process_group()
        return

    shape = synth.MoEShape(H, F, E, TOPK)
    sweep = tuple(int(t) for t in args.sweep.split(","))
    n_layers = max(1, args.layers)
    layers = []
    for li in range(n_layers):
        table = ExpertTable(synth.device_experts(1000 * rank + li, shape, dev))
        r = TopKRouter(hidden_dim=H, num_experts=E, experts_per_token=TOPK).to(dev, torch.bfloat16)
        with torch.no_grad():
            r.gate.weight.copy_(torch.randn(E, H, generator=torch.Generator(dev).manual_seed(77 + li),
                                            device=dev) * 0.02)
        layers.append(MoELayerInt4(r, table).eval())
    torch.cuda.synchronize()
    hbm_peak, _, peak_kind = peaks()

    results = {}
    for T in sweep:
        xs = [torch.randn(T, H, generator=torch.Generator(dev).manual_seed(T * 10 + i), device=dev)
              .to(torch.bfloat16) for i in range(n_layers)]
        # routing of each layer's input (fixed per layer) -> touched experts -> algorithmic bytes
        touched = []
        with torch.no_grad():
            for li, layer in enumerate(layers):
                idx = layer.router(xs[li].view(1, T, H)).expert_indices.reshape(-1)
                touched.append(int(torch.unique(idx).numel()))
        algo_bytes = statistics.mean(touched) * blob_bytes(H, F) + 2 * T * H * 2 + E * H * 2
        # capture one graph per layer (warm up on a side stream first)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        graphs, outs = [], []
        with torch.cuda.stream(s):
            for li, layer in enumerate(layers):
                layer(xs[li])
            torch.cuda.synchronize(dev)
            for li, layer in enumerate(layers):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    outs.append(layer(xs[li]))
                graphs.append(g)
        torch.cuda.current_stream(dev).wait_stream(s)
        for i in range(args.warmup):
            graphs[i % n_layers].replay()
        torch.cuda.synchronize(dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            ev0.record()
            for i in range(args.steps):
                graphs[i % n_layers].replay()
            ev1.record()
            torch.cuda.synchronize(dev)
        ms = ev0.elapsed_time(ev1) / args.steps
        results[T] = {"ms_per_step": ms, "tok_s": T / (ms * 1e-3), "touched_experts": statistics.mean(touched),
                      "algo_bytes": algo_bytes, "gbs": algo_bytes / (ms * 1e-3) / 1e9,
                      "clocks": clk.summary()}
        results[T]["frac"] = results[T]["gbs"] / hbm_peak
        del graphs, outs
        torch.cuda.synchronize(dev)

    # per-phase device times of the headline batch, with CUDA events between
    # the layer's three launches (eager, same stream); the dominant kernel is
    # the gate/up launch
    T = args.tokens if args.tokens in results else max(results)
    xk = [torch.randn(T, H, generator=torch.Generator(dev).manual_seed(T * 10 + i), device=dev).to(torch.bfloat16)
          for i in range(n_layers)]
    stream = torch.cuda.current_stream(dev)
    evs = []

    def mark(phase):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        evs[-1].append(ev)

    with torch.no_grad():
        for i in range(args.warmup):
            layers[i % n_layers].forward_phases(xk[i % n_layers])
        torch.cuda.synchronize(dev)
        # hold the stream with a device-side sleep while the host queues every
        # timed launch, so the kernels run back to back and the events bracket
        # device time only (not host launch gaps)
        torch.cuda._sleep(int(2e8))
        for i in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            evs.append([e0])
            layers[i % n_layers].forward_phases(xk[i % n_layers], between=mark)
            e3 = torch.cuda.Event(enable_timing=True)
            e3.record(stream)
            evs[-1].append(e3)
        torch.cuda.synchronize(dev)
    prep_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    gu_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    down_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in evs)
    touched_t = results[T]["touched_experts"]
    gu_bytes = touched_t * 2 * F * (H // 2 + 2 * (H // 128)) + T * H * 2
    kernel_times = {"prep_ms": prep_ms, "gateup_ms": gu_ms, "down_ms": down_ms}
    gu_kernel = "gv_kernel gate/up (dominant)" if decode_engine(T) == "mma.sync" else \
        "tc_engine_kernel gate/up (dominant)"

    # end-to-end through the public API: pinned host input -> device -> layer -> host
    x_host = [torch.randn(T, H, generator=torch.Generator().manual_seed(5 + i)).to(torch.bfloat16).pin_memory()
              for i in range(n_layers)]
    x_dev = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
    out_host = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    with torch.no_grad():
        for i in range(args.warmup):
            x_dev.copy_(x_host[i % n_layers], non_blocking=True)
            out_host.copy_(layers[i % n_layers](x_dev), non_blocking=True)
        torch.cuda.synchronize(dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for i in range(args.steps):
            x_dev.copy_(x_host[i % n_layers], non_blocking=True)
            out_host.copy_(layers[i % n_layers](x_dev), non_blocking=True)
        ev1.record()
        torch.cuda.synchronize(dev)
    e2e_ms = ev0.elapsed_time(ev1) / args.steps
    del layers
    torch.cuda.empty_cache()

    cpu = None
    if not args.no_cpu_baseline:
        v, n, el, kind = cpu_reference_time(T, budget_s=args.ref_budget)
        what = ("the reference's own MixtralMoELayer.forward in dequant mode (float32 weights, torch CPU)"
                if kind == "reference" else "oracle layer steps (numpy float32 dequant-then-matmul)")
        cpu = {"value": v, "unit": "tok/s", "cores": cpu_threads(), "kind": kind,
               "sample": f"{n} steps at T={T} in {el:.1f}s: {what}, weights dequantised before timing"}
    triton_bar = None if args.quick else reference_triton_bar(dev)

    prefill = None if args.no_prefill else prefill_measure(args, dev)
    glm = None if args.quick else glm_c4(args, dev, 1, 0, barrier, max_over_ranks)
    c3 = None if args.no_c3 else c3_measure(args, dev)
    if glm is not None and not args.no_cpu_baseline:
        gv, gms, gsample = glm_cpu_time()
        glm["cpu_baseline"] = {"value": gv, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
                               "sample": gsample, "ms_per_step": gms}

    hr = results[T]
    line = {
        "metric": METRIC, "value": hr["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": hr["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, weights ~N(0,0.02) INT4 g128)",
        "config": {"workload": WORKLOAD, "tokens": T, "hidden": H, "ffn": F, "experts": E, "top_k": TOPK,
                   "group_size": 128, "layers_rotated": n_layers, "l2": "weights per step > L2 (126 MB), "
                   f"{n_layers} distinct layers rotated", "cuda_graph": True, "parallelism": "single"},
        "roofline": {"bound": "hbm", "achieved": gu_bytes / (gu_ms * 1e-3) / 1e9, "peak": hbm_peak,
                     "unit": "GB/s", "frac": gu_bytes / (gu_ms * 1e-3) / 1e9 / hbm_peak,
                     "traffic": GATEUP_TRAFFIC.get(T), "kernel": gu_kernel,
                     "algo_bytes_per_launch": gu_bytes, "launch_ms": gu_ms, "peak_kind": peak_kind,
                     "layer": {"achieved": hr["gbs"], "frac": hr["frac"], **kernel_times}},
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2, "ms_per_step": e2e_ms},
        "gpu_launches": decode_launches(T) * args.steps,
        "clocks": hr["clocks"],
        "cpu_baseline": cpu,
        "prefill": prefill,
        "glm_c4": glm,
        "c3_moe_path": c3,
        "reference_gpu_bar": triton_bar,
        "sweep": {str(t): {k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items() if k != "clocks"}
                  for t, r in results.items()},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
