#!/usr/bin/env python
"""Benchmark of the routed-expert MoE hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (N=1): BASELINE config 1, decode, bf16 profile -- one DeepSeek-V4
MoE layer (H=4096, I=2048, E=256, top-8, sqrtsoftplus router with a
Zipf-skewed selection bias) on T=64 tokens with every expert resident in the
HBM slot arena, synthetic seeded inputs.  A step is one layer forward.
  value : tokens/s with inputs already in HBM (device time, CUDA events);
  e2e   : tokens/s through the plugin's public forward with the tokens copied
          H2D from pinned host memory and the output read back D2H inside the
          timed region;
  roofline : the gate/up GEMM kernel (the dominant launch), algorithmic
          bytes / its event-timed duration against the measured HBM copy peak.
L2 is flushed (256 MiB write) before every timed step; steps rotate over
several token batches so routing changes.  The layer is captured once as a
CUDA graph and replayed per step (the way vLLM runs decode); the per-kernel
times behind the roofline come from an eager pass of the same steps with
CUDA events between the stages.  With N>1 (torchrun) every rank
runs the layer expert-parallel: E/N experts per rank, T=64 tokens per rank,
all-to-all dispatch and combine (weak scaling).
``--impl reference`` times the CPU restatement of the reference's
per-expert path (oracle/moe_oracle.py) on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "deepseek-v4-flash-offload_b200"))
sys.path.insert(0, ROOT)

METRIC = "MoE tok/s (bf16 & a4w4, LRU offload) at 1/2/4/8 B200; GEMM % of roofline"
UNIT = "tok/s"
L2_FLUSH_BYTES = 256 << 20


def _args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-detail", action="store_true")
    ap.add_argument("--workload", choices=["decode", "prefill", "offload"], default="decode",
                    help="decode: BASELINE config 1 (the headline); prefill: config 2 (T=2048, a4w4); "
                         "offload: config 3 (8 layers, LRU slot cache fed from pinned host memory)")
    ap.add_argument("--prefetch", action="store_true",
                    help="offload: copy the next layer's missing experts while the current layer computes")
    a = ap.parse_args(argv)
    a.warmup = max(a.warmup, 3)
    a.steps = max(a.steps, 1)
    return a


def _dist():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9 and p[1].replace(".", "").isdigit():
                    rows.append(p)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        load = [s for s in sm if s > 0.5 * mx] or sm
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# synthetic layer through the plugin's public API
# ---------------------------------------------------------------------------
def _cfg():
    from dsv4_plugin import synthetic as S
    return S.CFG1


def build_layer(device, rank: int, world: int, seed: int = 0, layer_idx: int = 3):
    """Engine + OffloadDeepseekV4MoE for one synthetic layer; the experts
    owned by this rank (all of them at world=1) are resident."""
    import types

    import torch

    from dsv4_plugin import synthetic as S
    from dsv4_plugin.core import engine as ENG
    from dsv4_plugin.models import deepseek_v4 as DV4

    cfg = _cfg()
    e_loc = cfg.n_experts // world
    lo = rank * e_loc
    eng = ENG.ExpertOffloadEngine(slot_capacity=e_loc, device=device, packed_capacity=e_loc)
    eng.bank.pin = True
    for e in range(lo, lo + e_loc):
        ex = S.make_expert(cfg, seed, e, layer_idx)
        eng.bank.register(layer_idx, e, *[torch.from_numpy(ex[k]) for k in
                                          ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")])
    ENG.reset_engine(eng)
    hf = types.SimpleNamespace(
        n_routed_experts=cfg.n_experts, n_shared_experts=None, num_experts_per_tok=cfg.topk,
        norm_topk_prob=cfg.renormalize, scoring_func=cfg.score_func, routed_scaling_factor=cfg.route_scale,
        swiglu_limit=cfg.swiglu_limit, num_hash_layers=0, vocab_size=129280, hidden_size=cfg.hidden,
        moe_intermediate_size=cfg.inter, hidden_act="silu")
    pc = types.SimpleNamespace(use_sequence_parallel_moe=False, eplb_config=None, enable_eplb=False)
    moe = DV4.OffloadDeepseekV4MoE(hf, pc, prefix=f"model.layers.{layer_idx}.mlp").to(device)
    gw, bias = S.make_gate(cfg, seed, layer_idx)
    moe.gate.weight.data.copy_(torch.from_numpy(gw))
    moe.gate.e_score_correction_bias.data.copy_(torch.from_numpy(bias))
    if world == 1:
        eng.bank.preload_all(layer_idx)
    torch.cuda.synchronize(device)
    return moe, eng


def _token_batches(n: int, tokens: int, device, rank: int):
    import torch

    from dsv4_plugin import synthetic as S
    cfg = _cfg()
    host, dev = [], []
    for r in range(n):
        x = S.make_tokens(cfg, 7 + 1000 * rank, tokens, step=r)
        h = torch.from_numpy(S.to_bf16_bits(x).astype("int16")).view(torch.bfloat16).pin_memory()
        host.append(h)
        dev.append(h.to(device))
    return host, dev


def _gemm_bytes(d: int, p: int, which: str) -> float:
    """Algorithmic HBM bytes of one launch: weights of the d active experts
    (packed E2M1 + E8M0 scales) plus the activations in and out."""
    c = _cfg()
    h, i = c.hidden, c.inter
    if which == "gate_up":
        return d * (2 * i * h // 2 + 2 * i * h // 32) + p * (h + h // 32) + p * (i + i // 32)
    return d * (h * i // 2 + h * i // 32) + p * (i + i // 32) + p * h * 2


def _layer_bytes(d: int, t: int) -> float:
    c = _cfg()
    return d * c.packed_expert_bytes() + c.n_experts * c.hidden * 4 + 2 * t * c.hidden * 2


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _traffic():
    """Per-launch DRAM bytes (read + write) of the gate/up GEMM from the
    committed ncu summary, with the algorithmic bytes of that same launch."""
    out = {}
    try:
        with open(os.path.join(ROOT, "profiles", "moe_gemm_cfg1_t64_bf16.md")) as f:
            for line in f:
                k, sep, v = line.partition(":")
                if sep and k.strip() in ("dram_bytes_per_launch", "algorithmic_bytes_per_launch"):
                    out[k.strip()] = int(v.strip())
    except (OSError, ValueError):
        return None
    return out if "dram_bytes_per_launch" in out else None


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(a):
    import torch

    rank, world, local = _dist()
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    if world > 1:
        return run_ep(a, rank, world, device)
    from dsv4_plugin.models import deepseek_v4 as DV4

    moe, eng = build_layer(device, 0, 1)
    T = a.tokens
    R = 8
    host, dev = _token_batches(R, T, device, 0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    y_host = torch.empty((T, _cfg().hidden), dtype=torch.bfloat16).pin_memory()
    plan = eng.plan_for(_cfg().n_experts, _cfg().topk, T, _cfg().swiglu_limit)
    stream = torch.cuda.current_stream(device)

    def device_steps(n, tokens_dev, record=True):
        tot, stages, ds = 0.0, [], []
        for s in range(n):
            x = tokens_dev[s % len(tokens_dev)]
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            moe.forward(x)
            e1.record(stream)
            e1.synchronize()
            if record:
                tot += e0.elapsed_time(e1)
                stages.append(plan.stage_times())
                ds.append(plan.n_active())
        return tot, stages, ds

    # the layer as a CUDA graph (how a serving engine replays decode steps):
    # the step's token batch is copied into the graph's input buffer, then the
    # whole layer (router, align, quant, two GEMMs, combine) replays.
    def capture(tokens_dev, profile_a4w4=False):
        DV4._MXFP4_GMM = profile_a4w4
        try:
            xs = torch.empty_like(tokens_dev[0])
            xs.copy_(tokens_dev[0])
            for _ in range(2):
                moe.forward(xs)
            torch.cuda.synchronize(device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                ys = moe.forward(xs)
            torch.cuda.synchronize(device)
        finally:
            DV4._MXFP4_GMM = False
        return g, xs, ys

    def graph_steps(g, xs, tokens_dev, n, record=True):
        tot = 0.0
        for s in range(n):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            xs.copy_(tokens_dev[s % len(tokens_dev)])
            g.replay()
            e1.record(stream)
            e1.synchronize()
            if record:
                tot += e0.elapsed_time(e1)
        return tot

    plan.enable_timing(False)
    g, xs, ys = capture(dev)
    graph_steps(g, xs, dev, a.warmup, record=False)
    clk = Clocks(local)
    torch.cuda.synchronize(device)
    clk.start()
    tot_ms = graph_steps(g, xs, dev, a.steps)
    torch.cuda.synchronize(device)
    clocks = clk.stop()
    ms_step = tot_ms / a.steps
    value = T * a.steps / (tot_ms / 1e3)

    # per-kernel device times of the same steps, run eagerly with CUDA events
    # between the stages (on the launching stream)
    plan.enable_timing(True)
    device_steps(2, dev, record=False)
    eager_ms, stages, ds = device_steps(a.steps, dev)
    plan.enable_timing(False)

    # roofline of the gate/up GEMM and of the whole layer
    hbm, peak_kind = _peaks()
    P = T * _cfg().topk
    g1_ms = sum(s["gate_up_gemm"] for s in stages)
    g2_ms = sum(s["down_gemm"] for s in stages)
    g1_bytes = sum(_gemm_bytes(d, P, "gate_up") for d in ds)
    g2_bytes = sum(_gemm_bytes(d, P, "down") for d in ds)
    ach1 = g1_bytes / (g1_ms / 1e3) / 1e9
    ach2 = g2_bytes / (g2_ms / 1e3) / 1e9
    lay = sum(_layer_bytes(d, T) for d in ds) / (tot_ms / 1e3) / 1e9
    traffic = _traffic()
    roofline = {"bound": "hbm", "kernel": "moe_gemm_kernel<2,false,0> (gate/up, bf16 profile)",
                "achieved": round(ach1, 1), "peak": hbm, "peak_kind": f"{peak_kind} HBM copy",
                "unit": "GB/s", "frac": round(ach1 / hbm, 4),
                "traffic": traffic["dram_bytes_per_launch"] if traffic else None,
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one gate/up launch "
                                   "(token batch 0, profiles/moe_gemm_cfg1_t64_bf16.md); algorithmic bytes of "
                                   f"that launch: {traffic.get('algorithmic_bytes_per_launch')}") if traffic else None,
                "algorithmic_bytes_per_launch": round(g1_bytes / len(ds)),
                "launch_ms": round(g1_ms / len(ds), 5)}
    detail = {"active_experts_mean": round(statistics.mean(ds), 2),
              "eager_ms_per_step": round(eager_ms / a.steps, 5),
              "stage_ms_mean": {k: round(statistics.mean(s[k] for s in stages), 5) for k in stages[0]},
              "down_gemm_roofline": {"achieved": round(ach2, 1), "frac": round(ach2 / hbm, 4)},
              "layer_roofline": {"achieved": round(lay, 1), "frac": round(lay / hbm, 4),
                                 "bytes": "D*13369344 + gate fp32 + x/y"}}

    # e2e through the public forward (graph-replayed) with host buffers
    def e2e_steps(n, record=True):
        tot = 0.0
        for s in range(n):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            xs.copy_(host[s % R], non_blocking=True)
            g.replay()
            y_host.copy_(ys, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
            if record:
                tot += e0.elapsed_time(e1)
        return tot

    e2e_steps(a.warmup, record=False)
    e2e_ms = e2e_steps(a.steps)
    e2e = {"value": round(T * a.steps / (e2e_ms / 1e3), 1), "unit": UNIT,
           "h2d_bytes_per_step": T * _cfg().hidden * 2, "d2h_bytes_per_step": T * _cfg().hidden * 2,
           "ms_per_step": round(e2e_ms / a.steps, 5),
           "api": "OffloadDeepseekV4MoE.forward replayed as a CUDA graph"}

    if not a.no_detail:
        # a4w4 profile on the same workload, and the other decode batch sizes
        g4, xs4, _ = capture(dev, profile_a4w4=True)
        graph_steps(g4, xs4, dev, 2, record=False)
        t4 = graph_steps(g4, xs4, dev, a.steps)
        detail["a4w4_value"] = round(T * a.steps / (t4 / 1e3), 1)
        del g4
        per_t = {}
        for t in (1, 8, 32):
            _, dv = _token_batches(4, t, device, 0)
            gt, xst, _ = capture(dv)
            n = max(4, a.steps // 2)
            graph_steps(gt, xst, dv, 2, record=False)
            tt = graph_steps(gt, xst, dv, n)
            plan.enable_timing(True)
            _, st, dd = device_steps(n, dv)
            plan.enable_timing(False)
            per_t[str(t)] = {"tok_s": round(t * n / (tt / 1e3), 1), "ms": round(tt / n, 5),
                             "active_experts": round(statistics.mean(dd), 1),
                             "gate_up_frac": round(sum(_gemm_bytes(d, t * 8, "gate_up") for d in dd) /
                                                   (sum(x["gate_up_gemm"] for x in st) / 1e3) / 1e9 / hbm, 4)}
            del gt
        detail["decode_T"] = per_t
    plan.status()

    cpu = None if a.no_cpu_baseline else cpu_baseline(T, budget_s=12.0)
    line = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": 1, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e2m1 x e4m3 block-scaled (bf16 profile), fp32 accumulate, bf16 out",
            "data": "synthetic (seeded; BASELINE config 1 distributions)",
            "config": {"workload": f"cfg1 decode bf16 profile: T={T} tokens, H=4096, I=2048, E=256, top-8, "
                                   "all experts resident", "tokens_per_step": T, "global_batch": T,
                       "parallelism": "single GPU",
                       "l2": "256 MiB flush before every timed step; 8 rotating token batches"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
            "gpu_launches": 7 * a.steps, "launch_mode": "CUDA graph replay per step (7 kernels)",
            "detail": detail}
    print(json.dumps(line), flush=True)


def cpu_baseline(tokens: int, budget_s: float = 12.0):
    """Oracle per-expert path (reference semantics) on the host cores, experts
    resident dequantised (the reference's hot ExpertBank), bounded sample."""
    import numpy as np

    from dsv4_plugin import synthetic as S
    from oracle import moe_oracle as O
    cfg = _cfg()
    gw, bias = S.make_gate(cfg, 0, 3)
    x = S.make_tokens(cfg, 7, tokens, step=0)
    w, idx = O.route(x, gw, bias, cfg.topk, cfg.score_func, cfg.renormalize)
    need = sorted(set(idx.reshape(-1).tolist()))
    experts = {e: S.make_expert(cfg, 0, e, 3) for e in need}
    cache = {e: O.expert_weights_f32(experts[e]) for e in need}
    n, t0 = 0, time.perf_counter()
    while True:
        O.moe_routed(x, w, idx, experts, cfg.n_experts, cfg.swiglu_limit, "bf16", deq_cache=cache)
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= 50:
            break
    dt = time.perf_counter() - t0
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"value": round(tokens * n / dt, 2), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} layer forwards of cfg1 decode T={tokens} (oracle per-expert loop, numpy fp32 BLAS, "
                      f"{len(need)} active experts resident dequantised), {dt:.1f} s"}


# ---------------------------------------------------------------------------
# config 2: prefill, a4w4 profile
# ---------------------------------------------------------------------------
FP8_DENSE_TFLOPS = 4500.0   # nominal dense B200 rate of kind::mxf8f6f4 (the bf16 profile's MMA)
FP4_DENSE_TFLOPS = 9000.0   # nominal dense B200 rate of kind::mxf4 (the a4w4 profile's MMA)


def run_prefill(a):
    """T=2048 tokens, a4w4, every expert resident; one
    step = one layer forward (router, align, MXFP4 quant, two GEMMs,
    combine), replayed as a CUDA graph."""
    import torch

    from dsv4_plugin.models import deepseek_v4 as DV4
    rank, world, local = _dist()
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    c = _cfg()
    T = 2048 if a.tokens == 64 else a.tokens
    moe, eng = build_layer(device, 0, 1)
    host, dev = _token_batches(4, T, device, 0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    plan = eng.plan_for(c.n_experts, c.topk, T, c.swiglu_limit)
    stream = torch.cuda.current_stream(device)
    DV4._MXFP4_GMM = True
    try:
        xs = torch.empty_like(dev[0])
        xs.copy_(dev[0])
        for _ in range(2):
            moe.forward(xs)
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ys = moe.forward(xs)

        def steps(n, record=True):
            tot = 0.0
            for s in range(n):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                xs.copy_(dev[s % len(dev)])
                g.replay()
                e1.record(stream)
                e1.synchronize()
                if record:
                    tot += e0.elapsed_time(e1)
            return tot

        steps(a.warmup, record=False)
        clk = Clocks(local)
        clk.start()
        tot_ms = steps(a.steps)
        clocks = clk.stop()
        # per-stage device times from an eager pass with events between the stages
        plan.enable_timing(True)
        st_list, ds = [], []
        for s in range(max(3, a.steps)):
            flush.zero_()
            moe.forward(dev[s % len(dev)])
            torch.cuda.synchronize(device)
            if s >= 1:
                st_list.append(plan.stage_times())
                ds.append(plan.n_active())
        plan.enable_timing(False)
        # end to end: host tokens in, host output back
        y_host = torch.empty((T, c.hidden), dtype=torch.bfloat16).pin_memory()
        e2e_ms = 0.0
        for s in range(a.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            xs.copy_(host[s % len(host)], non_blocking=True)
            g.replay()
            y_host.copy_(ys, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
            e2e_ms += e0.elapsed_time(e1)
        del g
    finally:
        DV4._MXFP4_GMM = False
    hbm, peak_kind = _peaks()
    P = T * c.topk
    flops = 6.0 * c.hidden * c.inter * P
    d = statistics.mean(ds)
    byts = _layer_bytes(d, T) + P * (c.hidden // 2 + c.hidden // 32) + P * (c.inter // 2 + c.inter // 32) \
        + 2 * P * c.hidden * 2
    ms = tot_ms / a.steps
    t_hbm = byts / (hbm * 1e9) * 1e3
    t_fp8 = flops / (FP8_DENSE_TFLOPS * 1e12) * 1e3
    t_fp4 = flops / (FP4_DENSE_TFLOPS * 1e12) * 1e3
    sm = {k: round(statistics.mean(x[k] for x in st_list), 5) for k in st_list[0]}
    g1_flops, g2_flops = 4.0 * c.hidden * c.inter * P, 2.0 * c.hidden * c.inter * P
    g1_bytes = _gemm_bytes(d, P, "gate_up") - P * (c.hidden + c.hidden // 32) + P * (c.hidden // 2 + c.hidden // 32)
    g1_bound = max(g1_bytes / (hbm * 1e9), g1_flops / (FP4_DENSE_TFLOPS * 1e12)) * 1e3
    line = {"metric": METRIC, "value": round(T * a.steps / (tot_ms / 1e3), 1), "unit": UNIT, "n_gpus": 1,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "e2m1 x e2m1 block-scaled (a4w4 profile), fp32 accumulate, bf16 out",
            "data": "synthetic (seeded; BASELINE config 2 shapes and distributions)",
            "config": {"workload": f"cfg2 prefill a4w4 profile: T={T} tokens, H=4096, I=2048, E=256, top-8, "
                                   "all experts resident", "tokens_per_step": T, "global_batch": T,
                       "parallelism": "single GPU", "l2": "256 MiB flush before every timed step"},
            "roofline": {"bound": "hbm" if t_hbm >= t_fp4 else "tensor",
                         "layer_bound_ms": round(max(t_hbm, t_fp4), 5), "frac": round(max(t_hbm, t_fp4) / ms, 4),
                         "hbm_ms": round(t_hbm, 5), "fp8_rate_ms": round(t_fp8, 5), "fp4_rate_ms": round(t_fp4, 5),
                         "bytes": round(byts), "flops": flops, "peak_hbm_gbs": hbm, "peak_kind": peak_kind,
                         "tensor_peak": f"{FP4_DENSE_TFLOPS:.0f} TFLOP/s nominal dense (kind::mxf4, the a4w4 MMA)",
                         "gate_up_frac": round(g1_bound / sm["gate_up_gemm"], 4)},
            "e2e": {"value": round(T * a.steps / (e2e_ms / 1e3), 1), "unit": UNIT,
                    "h2d_bytes_per_step": T * c.hidden * 2, "d2h_bytes_per_step": T * c.hidden * 2},
            "clocks": clocks, "gpu_launches": 7 * a.steps,
            "detail": {"active_experts_mean": round(d, 1), "stage_ms_mean": sm}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# config 3: offloaded multi-layer decode (LRU slot cache fed from pinned host memory)
# ---------------------------------------------------------------------------
def offload_trace(n_steps: int, n_layers: int, n_seqs: int, n_experts: int, topk: int, s: float = 1.1,
                  reuse: float = 0.7, seed: int = 1234):
    """Routing trace [steps, layers, seqs, topk]: per
    layer a Zipf(s) popularity over a random permutation of the experts; a
    sequence reuses its previous step's expert set with probability
    ``reuse``, else draws ``topk`` distinct experts by popularity."""
    import numpy as np
    rng = np.random.default_rng(seed)
    tr = np.zeros((n_steps, n_layers, n_seqs, topk), dtype=np.int32)
    for l in range(n_layers):
        rank = rng.permutation(n_experts) + 1
        p = 1.0 / rank.astype(np.float64) ** s
        p /= p.sum()
        for q in range(n_seqs):
            for st in range(n_steps):
                if st > 0 and rng.random() < reuse:
                    tr[st, l, q] = tr[st - 1, l, q]
                else:
                    tr[st, l, q] = np.sort(rng.choice(n_experts, topk, replace=False, p=p))
    return tr


def pinned_h2d_gbs(device, nbytes=1 << 30):
    import torch
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        dst.copy_(src, non_blocking=True)
    e1.record()
    e1.synchronize()
    return 3 * nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9


def run_offload(a):
    """8 MoE layers (config-1 dims), every expert of every
    layer in a pinned host pool, HBM slot budgets of 512 and 2048 packed
    slots with LRU eviction, routing from the trace above (256 decode steps
    x 8 sequences).  A step runs the 8 layers on the 8 tokens; each layer
    makes its experts resident (misses: one H2D copy per expert on the copy
    stream, which the compute stream waits for) and runs the routed-expert
    kernels.  With --prefetch the next layer's misses are issued before the
    current layer's kernels, so the copies overlap them (the experts are
    taken from the trace, i.e. a perfect predictor: an upper bound for a
    prefetch driven by the next layer's gate)."""
    import numpy as np
    import torch

    from dsv4_plugin import synthetic as S
    from dsv4_plugin.core import engine as ENG
    rank, world, local = _dist()
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    c = _cfg()
    L, T, E, K = 8, 8, c.n_experts, c.topk
    n_steps = 256
    slot = c.packed_expert_bytes()
    need = L * E * slot
    note = ""
    try:
        import psutil
        avail = psutil.virtual_memory().available
        if avail < 1.5 * need:
            L = max(1, int(avail / 1.5 / (E * slot)))
            note = f"host pool reduced to {L} layers: {avail / 2**30:.0f} GiB host memory available"
    except ImportError:
        pass
    eng = ENG.ExpertOffloadEngine(slot_capacity=0, device=device, packed_capacity=2048)
    bank = eng.bank
    bank.pin = True
    base = []
    t0 = time.perf_counter()
    for b in range(16):   # 16 distinct experts, copied into every (layer, expert) host slot
        ex = S.make_expert(c, 0, b, 0)
        bank.register(0, b, *[torch.from_numpy(ex[k]) for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")])
        base.append(bank.host_slot(0, b).clone())
    for l in range(L):
        for e in range(E):
            if l == 0 and e < 16:
                continue
            bank.register_packed(l, e, base[(e * 7 + l) % 16])
    setup_s = time.perf_counter() - t0
    tr = offload_trace(n_steps, L, T, E, K)
    x0 = torch.from_numpy(S.to_bf16_bits(S.make_tokens(c, 11, T)).astype("int16")).view(torch.bfloat16).to(device)
    g = np.random.default_rng(5)
    wts = torch.from_numpy(g.random((n_steps, L, T, K), dtype=np.float32) + 0.1)
    wts = (wts / wts.sum(-1, keepdim=True)).pin_memory()
    idx_host = torch.from_numpy(tr).pin_memory()
    stream = torch.cuda.current_stream(device)
    peak_h2d = pinned_h2d_gbs(device)
    results = []
    for budget in (512, 2048):
        eng.resize_slots(budget)
        plan = eng.plan_for(E, K, T, c.swiglu_limit)
        slot_host = torch.full((L, E), -1, dtype=torch.int32).pin_memory()
        slot_dev = torch.empty((L, E), dtype=torch.int32, device=device)
        idx_dev = torch.empty((L, T, K), dtype=torch.int32, device=device)
        w_dev = torch.empty((L, T, K), dtype=torch.float32, device=device)

        def resident(l, st):
            act = sorted(set(tr[st, l].reshape(-1).tolist()))
            return act, bank.ensure_resident(l, act, stream=stream)

        def one_step(st):
            idx_dev.copy_(idx_host[st], non_blocking=True)
            w_dev.copy_(wts[st], non_blocking=True)
            x = x0
            nxt = resident(0, st) if a.prefetch else None
            for l in range(L):
                if a.prefetch:
                    act, slots = nxt
                else:
                    # on demand, as the reference: the layer's routing reaches
                    # the host (one sync), then its misses are copied
                    stream.synchronize()
                    act, slots = resident(l, st)
                slot_host[l].fill_(-1)
                slot_host[l, torch.tensor(act, dtype=torch.long)] = torch.tensor(slots, dtype=torch.int32)
                slot_dev[l].copy_(slot_host[l], non_blocking=True)
                if a.prefetch and l + 1 < L:
                    nxt = resident(l + 1, st)   # its copies overlap this layer's kernels
                x = plan.forward(x, w_dev[l], idx_dev[l], slot_dev[l], "bf16")
                bank.mark_used(slots, stream)
            return x

        w_steps = 16
        for st in range(w_steps):
            one_step(st)
            torch.cuda.synchronize(device)   # the host slot table is reused next step
        s0 = bank.stats()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0 = time.perf_counter()
        e0.record(stream)
        for st in range(w_steps, n_steps):
            one_step(st)
            torch.cuda.synchronize(device)   # the host slot table is reused next step
        e1.record(stream)
        e1.synchronize()
        wall = time.perf_counter() - h0
        ms = e0.elapsed_time(e1)
        s1 = bank.stats()
        hits = s1["packed_hits"] - s0["packed_hits"]
        miss = s1["packed_misses"] - s0["packed_misses"]
        h2d = s1["h2d_bytes"] - s0["h2d_bytes"]
        n = n_steps - w_steps
        results.append({"slots": budget, "tok_s": round(T * n / (ms / 1e3), 1),
                        "ms_per_step": round(ms / n, 4), "hit_rate": round(hits / max(1, hits + miss), 4),
                        "misses_per_step": round(miss / n, 2), "h2d_gbs": round(h2d / (ms / 1e3) / 1e9, 2),
                        "h2d_frac_of_pinned_peak": round(h2d / (ms / 1e3) / 1e9 / peak_h2d, 4),
                        "host_wall_ms_per_step": round(wall / n * 1e3, 4)})
    best = results[0]
    line = {"metric": METRIC, "value": best["tok_s"], "unit": UNIT, "n_gpus": 1, "steps": n_steps - 16,
            "warmup": 16, "ms_per_step": best["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e2m1 x e4m3 block-scaled (bf16 profile), fp32 accumulate, bf16 out",
            "data": "synthetic routing trace (seeded; BASELINE config 3), 16 distinct expert payloads",
            "config": {"workload": f"cfg3 offloaded decode: {L} layers x {E} experts in pinned host memory, "
                                   f"T={T} tokens (8 sequences), LRU slot budgets 512 and 2048, "
                                   + ("next-layer prefetch" if a.prefetch else "on-demand copies"),
                       "tokens_per_step": T, "global_batch": T, "parallelism": "single GPU",
                       "l2": "working set (misses stream from host) larger than L2"},
            "offload": results, "pinned_h2d_peak_gbs": round(peak_h2d, 2), "setup_s": round(setup_s, 1),
            "note": note}
    print(json.dumps(line), flush=True)


def run_reference(a):
    rank, world, _ = _dist()
    if rank != 0:
        return
    import numpy as np

    from dsv4_plugin import synthetic as S
    from oracle import moe_oracle as O
    cfg = _cfg()
    T = a.tokens
    gw, bias = S.make_gate(cfg, 0, 3)
    x = S.make_tokens(cfg, 7, T, step=0)
    w, idx = O.route(x, gw, bias, cfg.topk, cfg.score_func, cfg.renormalize)
    need = sorted(set(idx.reshape(-1).tolist()))
    experts = {e: S.make_expert(cfg, 0, e, 3) for e in need}
    cache = {e: O.expert_weights_f32(experts[e]) for e in need}

    def step():
        ww, ii = O.route(x, gw, bias, cfg.topk, cfg.score_func, cfg.renormalize)
        O.moe_routed(x, ww, ii, experts, cfg.n_experts, cfg.swiglu_limit, "bf16", deq_cache=cache)

    for _ in range(a.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        step()
    dt = time.perf_counter() - t0
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    value = T * a.steps / dt
    line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(dt / a.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (bf16-rounded like the reference)",
            "data": "synthetic (seeded; BASELINE config 1 distributions)", "impl": "reference",
            "config": {"workload": f"cfg1 decode bf16 profile: T={T} tokens, H=4096, I=2048, E=256, top-8, "
                                   "all experts resident", "tokens_per_step": T, "global_batch": T,
                       "parallelism": "host cores"},
            "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"{a.steps} layer forwards (router + per-expert loop) of cfg1 T={T}; "
                                       f"{len(need)} experts resident dequantised"},
            "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ep(a, rank, world, device):
    from dsv4_plugin.parallel_ep import run_ep_bench
    line = run_ep_bench(a, rank, world, device, METRIC, UNIT, build_layer, _token_batches, Clocks,
                        L2_FLUSH_BYTES, gemm_bytes=_gemm_bytes, peaks=_peaks())
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)


def main(argv=None):
    a = _args(argv)
    if a.impl == "reference":
        run_reference(a)
    elif a.workload == "prefill":
        run_prefill(a)
    elif a.workload == "offload":
        run_offload(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
