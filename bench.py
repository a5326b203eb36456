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
    ap.add_argument("--workload", choices=["decode", "prefill", "offload", "ep1"], default="decode",
                    help="decode: BASELINE config 1 (the headline); prefill: config 2 (T=2048, a4w4); "
                         "offload: config 3 (8 layers, LRU slot cache fed from pinned host memory); "
                         "ep1: config 4 through the expert-parallel exchange on one rank (a profiling aid: "
                         "every kernel of the exchange runs, each token going to this rank)")
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
    """SM clock and clock-event reasons sampled DURING the timed region.

    NVML is polled from a thread every 2 ms (the timed regions here last tens
    of milliseconds, shorter than nvidia-smi's 200 ms loop); the device is
    found by the UUID torch reports for this process's GPU.  Without NVML,
    `nvidia-smi --query-gpu=... -lms 200` runs beside the region instead.
    The fields are those of the nvidia-smi query: clocks.sm, clocks.max.sm
    and the hw_slowdown / hw_thermal_slowdown / sw_thermal_slowdown /
    sw_power_cap reasons."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.002

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None
        self.thread = None
        self.samples = []
        self.max_mhz = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _poll(self, h):
        import pynvml
        get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), int(get_reasons(h))))
            except Exception:
                break
            time.sleep(self.PERIOD_S)

    def start(self):
        import threading
        try:
            import pynvml
            h = self._nvml_handle()
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._stop = threading.Event()
            self.thread = threading.Thread(target=self._poll, args=(h,), daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 1.0:   # the first sample precedes the region
                time.sleep(0.001)
            return
        except Exception:
            self.thread = None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def _stop_nvml(self):
        import pynvml
        self._stop.set()
        self.thread.join(timeout=5)
        rows = self.samples
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"], "source": "nvml"}
        mx = float(self.max_mhz or max(r[0] for r in rows))
        sm = [float(r[0]) for r in rows]
        load = [v for v in sm if v > 0.5 * mx] or sm
        bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
        reasons = sorted({n for _, r in rows for n, b in bits.items() if r & b})
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows),
                "source": f"nvml every {self.PERIOD_S * 1e3:.0f} ms"}

    def stop(self):
        if self.thread is not None:
            return self._stop_nvml()
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
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows),
                "source": "nvidia-smi -lms 200"}


# ---------------------------------------------------------------------------
# synthetic layer through the plugin's public API
# ---------------------------------------------------------------------------
def _cfg():
    from dsv4_plugin import synthetic as S
    return S.CFG1


def build_layer(device, rank: int, world: int, seed: int = 0, layer_idx: int = 3, owner=None):
    """Engine + OffloadDeepseekV4MoE for one synthetic layer; the experts
    owned by this rank (owner[e] == rank; default contiguous, all of them at
    world=1) are registered."""
    import types

    import torch

    from dsv4_plugin import synthetic as S
    from dsv4_plugin.core import engine as ENG
    from dsv4_plugin.models import deepseek_v4 as DV4

    cfg = _cfg()
    if owner is None:
        owner = [e // (cfg.n_experts // world) for e in range(cfg.n_experts)]
    mine = [e for e in range(cfg.n_experts) if owner[e] == rank]
    e_loc = len(mine)
    eng = ENG.ExpertOffloadEngine(slot_capacity=e_loc, device=device, packed_capacity=e_loc)
    eng.bank.pin = True
    for e in mine:
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


TRAFFIC_PROFILE = "moe_ffn_fused_cfg1_t64_bf16.md"


def _traffic():
    """Per-launch DRAM bytes (read + write) of the fused FFN launch from the
    committed ncu summary, with the algorithmic bytes of that same launch."""
    out = {}
    try:
        with open(os.path.join(ROOT, "profiles", TRAFFIC_PROFILE)) as f:
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
    # between the stages (on the launching stream): the product's fused
    # gate/up -> down launch (its time is the gate/up stage), then the two
    # GEMMs as separate launches for the per-GEMM split
    plan.enable_timing(True)
    device_steps(2, dev, record=False)
    eager_ms, stages, ds = device_steps(a.steps, dev)
    plan.set_ffn_fusion(False)
    device_steps(2, dev, record=False)
    _, stages2, ds2 = device_steps(a.steps, dev)
    plan.set_ffn_fusion(None)
    plan.enable_timing(False)

    # rooflines: the fused FFN launch (headline), each GEMM alone, the layer
    hbm, peak_kind = _peaks()
    P = T * _cfg().topk
    ffn_ms = sum(s["gate_up_gemm"] + s["down_gemm"] for s in stages)
    ffn_bytes = sum(_gemm_bytes(d, P, "gate_up") + _gemm_bytes(d, P, "down") for d in ds)
    g1_ms = sum(s["gate_up_gemm"] for s in stages2)
    g2_ms = sum(s["down_gemm"] for s in stages2)
    g1_bytes = sum(_gemm_bytes(d, P, "gate_up") for d in ds2)
    g2_bytes = sum(_gemm_bytes(d, P, "down") for d in ds2)
    ach = ffn_bytes / (ffn_ms / 1e3) / 1e9
    ach1 = g1_bytes / (g1_ms / 1e3) / 1e9
    ach2 = g2_bytes / (g2_ms / 1e3) / 1e9
    lay = sum(_layer_bytes(d, T) for d in ds) / (tot_ms / 1e3) / 1e9
    traffic = _traffic()
    roofline = {"bound": "hbm",
                "kernel": "moe_gemm_kernel<2,false,SWIGLU_FP8,64,FUSED> (gate/up + SwiGLU + FP8 requant + down in "
                          "one launch, bf16 profile)",
                "achieved": round(ach, 1), "peak": hbm, "peak_kind": f"{peak_kind} HBM copy",
                "unit": "GB/s", "frac": round(ach / hbm, 4),
                "traffic": traffic["dram_bytes_per_launch"] if traffic else None,
                "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one fused launch "
                                   f"(token batch 0, profiles/{TRAFFIC_PROFILE}); algorithmic bytes of that "
                                   f"launch: {traffic.get('algorithmic_bytes_per_launch')}") if traffic else None,
                "algorithmic_bytes_per_launch": round(ffn_bytes / len(ds)),
                "launch_ms": round(ffn_ms / len(ds), 5)}
    detail = {"active_experts_mean": round(statistics.mean(ds), 2),
              "eager_ms_per_step": round(eager_ms / a.steps, 5),
              "stage_ms_mean": {k: round(statistics.mean(s[k] for s in stages), 5) for k in stages[0]},
              "stage_ms_mean_two_gemm_launches": {k: round(statistics.mean(s[k] for s in stages2), 5)
                                                  for k in stages2[0]},
              "gate_up_gemm_roofline": {"achieved": round(ach1, 1), "frac": round(ach1 / hbm, 4),
                                        "launch_ms": round(g1_ms / len(ds2), 5)},
              "down_gemm_roofline": {"achieved": round(ach2, 1), "frac": round(ach2 / hbm, 4),
                                     "launch_ms": round(g2_ms / len(ds2), 5)},
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
            plan.set_ffn_fusion(False)
            _, st2, dd2 = device_steps(n, dv)
            plan.set_ffn_fusion(None)
            plan.enable_timing(False)
            pt = t * _cfg().topk
            per_t[str(t)] = {"tok_s": round(t * n / (tt / 1e3), 1), "ms": round(tt / n, 5),
                             "active_experts": round(statistics.mean(dd), 1),
                             "ffn_frac": round(sum(_gemm_bytes(d, pt, "gate_up") + _gemm_bytes(d, pt, "down")
                                                   for d in dd) /
                                               (sum(x["gate_up_gemm"] + x["down_gemm"] for x in st) / 1e3) / 1e9 /
                                               hbm, 4),
                             "gate_up_frac": round(sum(_gemm_bytes(d, pt, "gate_up") for d in dd2) /
                                                   (sum(x["gate_up_gemm"] for x in st2) / 1e3) / 1e9 / hbm, 4),
                             "down_frac": round(sum(_gemm_bytes(d, pt, "down") for d in dd2) /
                                                (sum(x["down_gemm"] for x in st2) / 1e3) / 1e9 / hbm, 4)}
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
            "gpu_launches": 6 * a.steps,
            "launch_mode": "CUDA graph replay per step (6 kernels: router logits, top-k, align, quantise-gather, "
                           "fused gate/up -> down, combine)",
            "detail": detail}
    if not a.no_detail:
        # the other BASELINE configurations on this GPU, after the headline's
        # resources are released: config 4 at one GPU (the strong-scaling base
        # of --gpus N) and config 3 (offloaded decode through the plugin's forward)
        from dsv4_plugin.core import engine as ENG
        del g, xs, ys, moe, eng, plan
        ENG.reset_engine(None)
        torch.cuda.synchronize(device)
        torch.cuda.empty_cache()
        for key, fn in (("config4_1gpu", lambda: ep_config4(a, 0, 1, device, steps=max(3, a.steps // 2), warmup=3)),
                        ("config3_offload", lambda: offload_bench(device))):
            try:
                detail[key] = fn()
            except Exception as exc:   # a detail must not cost the headline line
                import traceback
                traceback.print_exc()
                detail[key] = {"error": f"{type(exc).__name__}: {exc}"[:500]}
            ENG.reset_engine(None)
            torch.cuda.synchronize(device)
            torch.cuda.empty_cache()
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


def mma_peaks(device) -> dict:
    """Measured dense rate (TFLOP/s) of the two MMA kinds of the grouped GEMM
    on this GPU (dsv4_mma_peak: one CTA per SM issuing M=128, N=256
    block-scaled MMAs back to back from shared memory, CUDA events)."""
    import ctypes as C

    from dsv4_plugin._lib import check, lib
    out = {}
    for name, kind in (("mxf4", 0), ("mxf8f6f4", 1)):
        tf, ms = C.c_double(), C.c_double()
        check(lib().dsv4_mma_peak(kind, 256, 200000, device.index or 0, C.byref(tf), C.byref(ms)))
        out[name] = round(tf.value, 1)
    out["how"] = "dsv4_mma_peak: 148 CTAs x 200000 k-tiles of 128, M=128 N=256, CUDA events"
    return out


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
    peaks = mma_peaks(device)
    fp4_peak, fp8_peak = peaks["mxf4"], peaks["mxf8f6f4"]
    t_hbm = byts / (hbm * 1e9) * 1e3
    t_fp8 = flops / (fp8_peak * 1e12) * 1e3
    t_fp4 = flops / (fp4_peak * 1e12) * 1e3
    sm = {k: round(statistics.mean(x[k] for x in st_list), 5) for k in st_list[0]}
    g1_flops, g2_flops = 4.0 * c.hidden * c.inter * P, 2.0 * c.hidden * c.inter * P
    g1_bytes = _gemm_bytes(d, P, "gate_up") - P * (c.hidden + c.hidden // 32) + P * (c.hidden // 2 + c.hidden // 32)
    g1_bound = max(g1_bytes / (hbm * 1e9), g1_flops / (fp4_peak * 1e12)) * 1e3
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
                         "tensor_peak": f"{fp4_peak:.0f} TFLOP/s measured (kind::mxf4, the a4w4 MMA; "
                                        f"nominal {FP4_DENSE_TFLOPS:.0f})", "mma_peaks_tflops": peaks,
                         "gate_up_frac": round(g1_bound / sm["gate_up_gemm"], 4)},
            "e2e": {"value": round(T * a.steps / (e2e_ms / 1e3), 1), "unit": UNIT,
                    "h2d_bytes_per_step": T * c.hidden * 2, "d2h_bytes_per_step": T * c.hidden * 2},
            "clocks": clocks, "gpu_launches": 10 * a.steps,
            "launch_mode": "CUDA graph replay per step (10 kernels: gate split, tensor-core router logits, top-k, "
                           "align count / scan / place, quantise-gather, gate/up, down, combine)",
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


def _offload_layers(device, L: int, E: int, budget: int, base_payloads: int = 16):
    """Engine with every expert of L layers in the page-locked host pool
    (``base_payloads`` distinct synthetic experts copied into every host
    slot) and an HBM budget of ``budget`` slots, plus one
    OffloadDeepseekV4MoE per layer built through the plugin's constructor.
    Gate l has a one-hot row per expert on the hidden columns
    [256 l, 256 l + E), so a hidden state with value 4 on the columns of a
    set of experts routes exactly that set at layer l."""
    import types

    import torch

    from dsv4_plugin import synthetic as S
    from dsv4_plugin.core import engine as ENG
    from dsv4_plugin.models import deepseek_v4 as DV4
    c = _cfg()
    eng = ENG.ExpertOffloadEngine(slot_capacity=0, device=device, packed_capacity=budget)
    bank = eng.bank
    bank.pin = True
    base = []
    for b in range(base_payloads):
        ex = S.make_expert(c, 0, b, 0)
        bank.register(0, b, *[torch.from_numpy(ex[k]) for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")])
        base.append(bank.host_slot(0, b).clone())
    for l in range(L):
        for e in range(E):
            if l == 0 and e < base_payloads:
                continue
            bank.register_packed(l, e, base[(e * 7 + l) % base_payloads])
    ENG.reset_engine(eng)
    hf = types.SimpleNamespace(
        n_routed_experts=E, n_shared_experts=None, num_experts_per_tok=c.topk, norm_topk_prob=True,
        scoring_func="sqrtsoftplus", routed_scaling_factor=c.route_scale, swiglu_limit=c.swiglu_limit,
        num_hash_layers=0, vocab_size=129280, hidden_size=c.hidden, moe_intermediate_size=c.inter,
        hidden_act="silu")
    pc = types.SimpleNamespace(use_sequence_parallel_moe=False, eplb_config=None, enable_eplb=False)
    mods = []
    for l in range(L):
        m = DV4.OffloadDeepseekV4MoE(hf, pc, prefix=f"model.layers.{l}.mlp").to(device)
        w = torch.zeros((E, c.hidden), dtype=torch.float32)
        w[torch.arange(E), 256 * l + torch.arange(E)] = 1.0
        m.gate.weight.data.copy_(w)
        m.gate.e_score_correction_bias.data.zero_()
        mods.append(m)
    return eng, mods


def _trace_tokens(tr, E: int, hidden: int):
    """Hidden states [steps, T, H] (bf16, pinned) that route trace[step, l,
    token] at every layer l through the one-hot gates of _offload_layers."""
    import torch
    n_steps, L, T, K = tr.shape
    x = torch.zeros((n_steps, T, hidden), dtype=torch.bfloat16)
    for l in range(L):
        cols = torch.from_numpy(tr[:, l].astype("int64")) + 256 * l          # [steps, T, K]
        x.scatter_(2, cols.reshape(n_steps, T, K), 4.0)
    return x.pin_memory()


def offload_bench(device, budgets=(512, 2048), n_steps: int = 256, warm: int = 16, L: int = 8,
                  host_lru_budget: int | None = 512):
    """BASELINE config 3 through the plugin's own forward: 8 MoE layers
    (config-1 dims), every expert of every layer in a page-locked host pool,
    HBM budgets of 512 and 2048 packed slots, routing from the seeded trace
    (256 decode steps x 8 sequences; Zipf 1.1 popularity, 70 % reuse).  A
    step copies the 8 tokens' hidden states in and runs the 8 layers.

    Modes, per budget:
      device  the device-side LRU: the GPU looks the experts up and copies
              its misses from the pinned pool itself; no host synchronisation,
              so the 8-layer step is one CUDA graph;
      device+prefetch  the same, and each layer warms the next layer's
              experts on a side stream (the next layer's gate applied to this
              layer's hidden state; the synthetic hidden states encode every
              layer's trace, so the predictor is perfect here: an upper bound);
      host    the host LRU of the reference's design (one synchronisation per
              layer, cudaMemcpyAsync of each miss on a copy stream), eager.
    Reports tok/s, hit rate, H2D GB/s against the measured pinned peak, and
    for device+prefetch the share of prefetch time that overlapped the
    compute stream (CUDA-event timestamps of an eager pass)."""
    import numpy as np
    import torch

    c = _cfg()
    E, T, K = c.n_experts, 8, c.topk
    slot = c.packed_expert_bytes()
    note = ""
    try:
        import psutil
        avail = psutil.virtual_memory().available
        if avail < 1.5 * L * E * slot:
            L = max(2, int(avail / 1.5 / (E * slot)))
            note = f"host pool reduced to {L} layers: {avail / 2**30:.0f} GiB host memory available"
    except ImportError:
        pass
    t0 = time.perf_counter()
    eng, mods = _offload_layers(device, L, E, max(budgets))
    bank = eng.bank
    setup_s = time.perf_counter() - t0
    tr = offload_trace(n_steps, L, T, E, K)
    xs_host = _trace_tokens(tr, E, c.hidden)
    stream = torch.cuda.current_stream(device)
    peak_h2d = pinned_h2d_gbs(device)
    xs = torch.empty((T, c.hidden), dtype=torch.bfloat16, device=device)

    def layers():
        out = None
        for m in mods:
            out = m.forward(xs)
        return out

    def run_mode(budget, mode):
        eng.resize_slots(budget)
        bank.device_lru = mode != "host"
        eng.prefetch = mode == "device+prefetch"
        for st in range(warm):
            xs.copy_(xs_host[st], non_blocking=True)
            layers()
        torch.cuda.synchronize(device)
        g = None
        if mode != "host":
            gs = torch.cuda.Stream(device=device)
            gs.wait_stream(stream)
            with torch.cuda.stream(gs):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=gs):
                    layers()
            stream.wait_stream(gs)
            torch.cuda.synchronize(device)
        s0 = bank.stats()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for st in range(warm, n_steps):
            xs.copy_(xs_host[st], non_blocking=True)
            if g is not None:
                g.replay()
            else:
                layers()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        s1 = bank.stats()
        n = n_steps - warm
        hits = s1["packed_hits"] - s0["packed_hits"]
        miss = s1["packed_misses"] - s0["packed_misses"]
        h2d = s1["h2d_bytes"] - s0["h2d_bytes"]
        r = {"slots": budget, "mode": mode, "tok_s": round(T * n / (ms / 1e3), 1), "ms_per_step": round(ms / n, 4),
             "hit_rate": round(hits / max(1, hits + miss), 4), "misses_per_step": round(miss / n, 2),
             "h2d_gbs": round(h2d / (ms / 1e3) / 1e9, 2),
             "h2d_frac_of_pinned_peak": round(h2d / (ms / 1e3) / 1e9 / peak_h2d, 4),
             "graph": g is not None}
        if mode == "device+prefetch":
            r["prefetch_fetched_per_step"] = round((s1.get("prefetch_fetched", 0) - s0.get("prefetch_fetched", 0)) / n, 2)
            # overlap of the side stream's prefetch with the compute stream (eager pass, events)
            bank.trace = []
            spans = []
            for st in range(warm, warm + 8):
                xs.copy_(xs_host[st], non_blocking=True)
                for m in mods:
                    a0 = torch.cuda.Event(enable_timing=True)
                    a0.record(stream)
                    m.forward(xs)
                    a1 = torch.cuda.Event(enable_timing=True)
                    a1.record(stream)
                    spans.append((a0, a1))
            torch.cuda.synchronize(device)
            ref = spans[0][0]
            comp = [(ref.elapsed_time(a), ref.elapsed_time(b)) for a, b in spans]
            # prefetch i warms layer l of step i // (L - 1) and was issued by
            # layer l - 1: the part of it inside that layer's span ran under
            # its compute; the rest is time the next layer waits for
            tot = ov = 0.0
            for i, (l, a, b) in enumerate(bank.trace):
                pa, pb = ref.elapsed_time(a), ref.elapsed_time(b)
                ca, cb = comp[(i // (L - 1)) * L + l - 1]
                tot += pb - pa
                ov += max(0.0, min(pb, cb) - max(pa, ca))
            n_pf = len(bank.trace)
            bank.trace = None
            r["prefetch_overlap_frac"] = round(ov / tot, 4) if tot > 0 else None
            r["prefetch_ms_per_layer"] = round(tot / max(1, n_pf), 4)
        del g
        return r

    results = []
    for budget in budgets:
        for mode in ("device", "device+prefetch"):
            results.append(run_mode(budget, mode))
    if host_lru_budget:
        results.append(run_mode(host_lru_budget, "host"))
    plan = eng.plan_for(E, K, T, c.swiglu_limit)
    plan.status()
    if bank._dir is not None:
        bank._dir.status()
    out = {"results": results, "pinned_h2d_peak_gbs": round(peak_h2d, 2), "setup_s": round(setup_s, 1),
           "layers": L, "note": note,
           "api": "OffloadDeepseekV4MoE.forward per layer (device modes: the 8-layer step replayed as one CUDA graph)"}
    del mods, eng
    from dsv4_plugin.core import engine as ENG
    ENG.reset_engine(None)
    torch.cuda.synchronize(device)
    return out


def run_offload(a):
    """--workload offload: BASELINE config 3 as its own JSON line."""
    import torch
    rank, world, local = _dist()
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    clk = Clocks(local)
    clk.start()
    r = offload_bench(device)
    clocks = clk.stop()
    best = max((x for x in r["results"] if x["slots"] == 512), key=lambda x: x["tok_s"])
    line = {"metric": METRIC, "value": best["tok_s"], "unit": UNIT, "n_gpus": 1, "steps": 240,
            "warmup": 16, "ms_per_step": best["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e2m1 x e4m3 block-scaled (bf16 profile), fp32 accumulate, bf16 out",
            "data": "synthetic routing trace (seeded; BASELINE config 3), 16 distinct expert payloads",
            "config": {"workload": f"cfg3 offloaded decode: {r['layers']} layers x 256 experts in pinned host "
                                   "memory, T=8 tokens (8 sequences), LRU slot budgets 512 and 2048; value: "
                                   f"512 slots, {best['mode']}",
                       "tokens_per_step": 8, "global_batch": 8, "parallelism": "single GPU",
                       "l2": "working set (misses stream from host) larger than L2"},
            "offload": r, "clocks": clocks}
    print(json.dumps(line), flush=True)


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _reference_moe(cfg, layer: int = 3):
    """The reference's own per-expert MoE (model_npu.MoE over an
    offload.ExpertBank on device "cpu"), imported from the unmodified
    install in baseline/_ref.  Two shims, as the golden-fixture generator
    uses: the privateuse1 backend is named "npu" (model_npu builds
    torch.device("npu:0") at import) and model_npu.DEVICE is set to the CPU.
    The shared expert is replaced by zero: the path under test is the routed
    experts (this build's layer does not run the shared expert either)."""
    import torch
    from torch import nn

    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        torch.utils.rename_privateuse1_backend("npu")
    except RuntimeError:
        pass   # already renamed in this process
    os.environ["DSV4_PIN_HOST"] = "0"
    import model_npu as MN
    import offload as OFF
    MN.DEVICE = torch.device("cpu")
    args = MN.ModelArgs(dim=cfg.hidden, moe_inter_dim=cfg.inter, n_routed_experts=cfg.n_experts,
                        n_activated_experts=cfg.topk, score_func=cfg.score_func, route_scale=cfg.route_scale,
                        swiglu_limit=cfg.swiglu_limit, n_hash_layers=0)
    bank = OFF.ExpertBank(capacity=cfg.n_experts, device="cpu", pin=False)
    moe = MN.MoE(layer, args, bank=bank)

    class _Zero(nn.Module):
        def forward(self, x):
            return torch.zeros((), dtype=x.dtype)

    moe.shared_experts = _Zero()
    return moe, bank


def run_reference(a):
    """The reference arm: the reference's own CPU per-expert path
    (model_npu.MoE.forward with ExpertBank(device="cpu"), every used expert
    resident dequantised after the warm-up: its hot state) on the host
    cores, for the ours arm's workload: config 1 (T=64) at N=1; at N>1 a
    bounded sample (512 of the 8192 tokens per step) of config 4.  When
    baseline/_ref is absent the numpy restatement in oracle/ runs instead
    (kind "port")."""
    rank, world, _ = _dist()
    if rank != 0:
        return
    import numpy as np
    import torch

    from dsv4_plugin import synthetic as S
    cfg = _cfg()
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    if world > 1:
        T = 512
        x = S.make_tokens(cfg, 77, CFG4_TOKENS, step=0)[:T]
        workload = (f"cfg4 expert parallel on {world} ranks (8192 tokens per step, E=256, top-8); reference arm: "
                    f"{T} of the step's tokens per timed step on the host cores")
        gw, bias = S.make_gate(cfg, 0, 3)
    else:
        T = a.tokens
        x = S.make_tokens(cfg, 7, T, step=0)
        workload = f"cfg1 decode bf16 profile: T={T} tokens, H=4096, I=2048, E=256, top-8, all experts resident"
        gw, bias = S.make_gate(cfg, 0, 3)
    kind = "reference" if os.path.isfile(os.path.join(REF_DIR, "model_npu.py")) else "port"
    if kind == "reference":
        torch.set_num_threads(cores)
        moe, bank = _reference_moe(cfg)
        moe.gate.weight.data.copy_(torch.from_numpy(gw))
        moe.gate.bias.data.copy_(torch.from_numpy(bias))
        xt = torch.from_numpy(S.to_bf16_bits(x).astype(np.int16)).view(torch.bfloat16)
        ids = torch.zeros(T, dtype=torch.int64)
        with torch.no_grad():
            _, idx = moe.gate(xt, ids)
        need = sorted(set(idx.reshape(-1).tolist()))
        for e in need:
            ex = S.make_expert(cfg, 0, e, 3)
            bank.register(3, e, *[torch.from_numpy(ex[k]) for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")])

        def step():
            with torch.no_grad():
                moe(xt, ids)
        sample = (f"model_npu.MoE.forward (router + per-expert bf16 loop, baseline/_ref), T={T}, {len(need)} experts "
                  f"resident dequantised, torch {torch.get_num_threads()} threads")
        n_threads = torch.get_num_threads()
    else:
        from oracle import moe_oracle as O
        w, idx = O.route(x, gw, bias, cfg.topk, cfg.score_func, cfg.renormalize)
        need = sorted(set(idx.reshape(-1).tolist()))
        experts = {e: S.make_expert(cfg, 0, e, 3) for e in need}
        cache = {e: O.expert_weights_f32(experts[e]) for e in need}

        def step():
            ww, ii = O.route(x, gw, bias, cfg.topk, cfg.score_func, cfg.renormalize)
            O.moe_routed(x, ww, ii, experts, cfg.n_experts, cfg.swiglu_limit, "bf16", deq_cache=cache)
        sample = f"numpy restatement (oracle/), T={T}, {len(need)} experts resident dequantised"
        n_threads = cores

    for _ in range(max(1, a.warmup)):
        step()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        step()
    dt = time.perf_counter() - t0
    value = T * a.steps / dt
    line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(dt / a.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16 (the reference's CPU path)" if kind == "reference" else "fp32 (bf16-rounded like the reference)",
            "data": "synthetic (seeded; BASELINE config distributions)", "impl": "reference",
            "config": {"workload": workload, "tokens_per_step": T, "global_batch": T, "parallelism": "host cores"},
            "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": n_threads, "kind": kind,
                             "sample": f"{a.steps} timed layer forwards: {sample}"},
            "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# config 4: expert parallel on N GPUs (strong scaling of a fixed 8192-token step)
# ---------------------------------------------------------------------------
CFG4_TOKENS = 8192


def _cfg4_batches(device, rank: int, world: int, n: int = 2):
    """n seeded global batches of 8192 tokens; this rank's contiguous share
    (T/world tokens) of each, pinned on the host and on the device."""
    import torch

    from dsv4_plugin import synthetic as S
    c = _cfg()
    t = CFG4_TOKENS // world
    host, dev = [], []
    for b in range(n):
        x = S.make_tokens(c, 77, CFG4_TOKENS, step=b)[rank * t:(rank + 1) * t]
        h = torch.from_numpy(S.to_bf16_bits(x).astype("int16")).view(torch.bfloat16).pin_memory()
        host.append(h)
        dev.append(h.to(device))
    return host, dev


def _calibrated_placement(device, world: int):
    """Load-balanced expert placement from a calibration batch (a separate
    seeded 8192-token batch, not one of the timed ones): its per-expert row
    counts from the router, then ``parallel_ep.balanced_placement``.  Every
    rank computes the same placement (same inputs, deterministic kernels)."""
    import torch

    from dsv4_plugin import ops
    from dsv4_plugin import synthetic as S
    from dsv4_plugin.parallel_ep import balanced_placement
    c = _cfg()
    gw, bias = S.make_gate(c, 0, 3)
    x = S.make_tokens(c, 91, CFG4_TOKENS, step=0)
    xt = torch.from_numpy(S.to_bf16_bits(x).astype("int16")).view(torch.bfloat16).to(device)
    _, idx = ops.route_topk(xt, torch.from_numpy(gw).to(device), torch.from_numpy(bias).to(device), c.topk,
                            c.score_func, c.renormalize, c.route_scale)
    counts = torch.bincount(idx.reshape(-1).to(torch.int64), minlength=c.n_experts).cpu().tolist()
    return balanced_placement(counts, world)


def ep_config4(a, rank: int, world: int, device, profiles=("bf16", "a4w4"), steps=None, warmup=None,
               force_ep=False):
    """E=256 experts sharded e // (E/N) over N ranks, a
    fixed step of 8192 tokens split evenly (T/N per rank), Zipf-skewed
    routing, both profiles.  world == 1 runs the plain single-GPU layer (all
    256 experts resident) on all 8192 tokens: the strong-scaling base.  For
    N > 1 each rank routes its tokens, dispatches rows to the owners of their
    experts over NVLink peer memory (DSV4_EP_EXCHANGE=static: NCCL
    all-to-all), runs its experts and returns the rows; the step is one CUDA
    graph.  Per profile: tokens/s over the whole step (8192 tokens / the
    slowest rank's step time) and the per-segment times of an eager pass."""
    import torch
    import torch.distributed as dist

    from dsv4_plugin.models import deepseek_v4 as DV4
    steps = steps or a.steps
    warmup = warmup or a.warmup
    owner = None
    if world > 1 and os.environ.get("DSV4_EP_PLACEMENT", "balanced") == "balanced":
        owner = _calibrated_placement(device, world)
    moe, eng = build_layer(device, rank, world, owner=owner)
    host, dev = _cfg4_batches(device, rank, world)
    T = CFG4_TOKENS // world
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    exchange = os.environ.get("DSV4_EP_EXCHANGE", "p2p")
    epm = None
    if world > 1 or force_ep:
        from dsv4_plugin.parallel_ep import ExpertParallelMoE
        epm = ExpertParallelMoE(moe, rank, world, owner=owner)

    def fwd(x, profile):
        if epm is None:
            DV4._MXFP4_GMM = profile == "a4w4"
            try:
                return moe.forward(x)
            finally:
                DV4._MXFP4_GMM = False
        return (epm.forward_p2p if exchange == "p2p" else epm.forward_static)(x, profile)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    out = {}
    for profile in profiles:
        xs = torch.empty_like(dev[0])
        xs.copy_(dev[0])
        for _ in range(2):
            fwd(xs, profile)
        torch.cuda.synchronize(device)
        barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ys = fwd(xs, profile)
        torch.cuda.synchronize(device)
        y_host = torch.empty(tuple(ys.shape), dtype=ys.dtype).pin_memory()

        def run(n, src, e2e=False):
            ms = []
            for s in range(n):
                flush.zero_()
                barrier()
                torch.cuda.synchronize(device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                xs.copy_(src[s % len(src)], non_blocking=True)
                g.replay()
                if e2e:
                    y_host.copy_(ys, non_blocking=True)
                e1.record(stream)
                e1.synchronize()
                ms.append(e0.elapsed_time(e1))
            return ms

        run(warmup, dev)
        ms = max_over_ranks(run(steps, dev))
        run(2, host, e2e=True)
        me = max_over_ranks(run(steps, host, e2e=True))
        # eager pass: segment times (route / dispatch / experts / return / combine)
        seg = {}
        if epm is not None:
            epm.segment_times = {}
            for s in range(3):
                flush.zero_()
                barrier()
                fwd(dev[s % len(dev)], profile)
            seg = dict(epm.segment_times)
            epm.segment_times = None
            names = sorted(seg)
            seg_max = max_over_ranks([seg[k] for k in names])
            seg = {k: round(v, 5) for k, v in zip(names, seg_max)}
        # this rank's routed-expert rows and active experts (load balance)
        plan = epm.plan if epm is not None else eng.plan_for(_cfg().n_experts, _cfg().topk, T, _cfg().swiglu_limit)
        load = [float(plan.n_active())]
        if epm is not None:
            ex = epm._p2p.get(T) if exchange == "p2p" else None
            # tokens and assignments this rank received
            load.append(float(int(ex.n_recv.item())) if ex is not None else 0.0)
            n_tok = int(ex.n_recv.item()) if ex is not None else 0
            load.append(float(int((ex.recv_idx[:n_tok] >= 0).sum().item())) if ex is not None else 0.0)
        loads = [load]
        if world > 1:
            buf = torch.tensor(load, dtype=torch.float64, device=device)
            allb = [torch.empty_like(buf) for _ in range(world)]
            dist.all_gather(allb, buf)
            loads = [b.tolist() for b in allb]
        tot = sum(ms)
        out[profile] = {"tok_s": round(CFG4_TOKENS * steps / (tot / 1e3), 1), "ms_per_step": round(tot / steps, 5),
                        "e2e_tok_s": round(CFG4_TOKENS * steps / (sum(me) / 1e3), 1),
                        "step_ms_median": round(statistics.median(ms), 5),
                        "segments_ms_max_over_ranks": seg,
                        "active_experts_per_rank": [int(l[0]) for l in loads],
                        "tokens_received_per_rank": [int(l[1]) for l in loads] if world > 1 else None,
                        "assignments_received_per_rank": [int(l[2]) for l in loads] if world > 1 else None}
        del g
        torch.cuda.synchronize(device)
    if epm is not None:
        for ex in epm._p2p.values():
            ex.check_status()
    if epm is not None:
        epm.plan.status()
        epm.close()
    return out


def run_ep(a, rank, world, device):
    """--gpus N under torchrun: BASELINE config 4 at N ranks.  value = bf16
    tokens/s of the whole 8192-token step (slowest rank); rank 0 then runs
    the same 8192 tokens on its GPU alone (all 256 experts) so that the line
    carries the strong-scaling ratio of this exact workload."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if not dist.is_initialized():
        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=180))
    clk = Clocks(int(os.environ.get("LOCAL_RANK", "0")))
    clk.start()
    r = ep_config4(a, rank, world, device)
    clocks = clk.stop()
    dist.barrier()
    one = None
    if rank == 0:
        from dsv4_plugin.core import engine as ENG
        ENG.reset_engine(None)
        torch.cuda.empty_cache()
        one = ep_config4(a, 0, 1, device, steps=max(3, a.steps // 2), warmup=3)
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return
    c = _cfg()
    h = c.hidden
    T = CFG4_TOKENS // world
    bf = r["bf16"]
    scal = {p: round(r[p]["tok_s"] / one[p]["tok_s"], 3) for p in r}
    line = {"metric": METRIC, "value": bf["tok_s"], "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": bf["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "e2m1 x e4m3 block-scaled (bf16 profile), fp32 accumulate, bf16 out",
            "data": "synthetic (seeded; BASELINE config 4 distributions)",
            "config": {"workload": f"cfg4 expert parallel: 8192 tokens per step split over {world} ranks "
                                   f"({T} each), E=256 experts, {c.n_experts // world} per rank, top-8, Zipf bias; "
                                   "value: bf16 profile", "tokens_per_step": CFG4_TOKENS,
                       "global_batch": CFG4_TOKENS,
                       "parallelism": f"ep{world} (" + ("NVLink peer-memory exchange, exact counts" if
                                                        os.environ.get("DSV4_EP_EXCHANGE", "p2p") == "p2p"
                                                        else "NCCL all-to-all") +
                                           ", " + os.environ.get("DSV4_EP_PLACEMENT", "balanced") +
                                           " expert placement, one CUDA graph per step)",
                       "l2": "256 MiB flush before every timed step"},
            "e2e": {"value": bf["e2e_tok_s"], "unit": UNIT, "h2d_bytes_per_step": CFG4_TOKENS * h * 2,
                    "d2h_bytes_per_step": CFG4_TOKENS * h * 2},
            "clocks": clocks, "gpu_launches": 17 * a.steps,
            "launch_mode": "CUDA graph replay per step (17 kernels: router 3, dispatch 5 (index, count wait, rows, "
                           "rows wait, return targets), align 3, quantise-gather, gate/up, down with the return "
                           "in its epilogue, publish + wait, ordered combine)",
            "detail": {"profiles": r, "same_workload_on_1_gpu": one,
                       "strong_scaling_vs_1_gpu": scal,
                       "note": "the N=1 line of bench.py is BASELINE config 1 (decode, T=64); this line's base "
                               "for scaling is same_workload_on_1_gpu, run by rank 0 in this job"}}
    print(json.dumps(line), flush=True)


def run_ep1(a):
    """--workload ep1: BASELINE config 4's 8192-token step through the
    peer-memory exchange on a one-rank group, so that every kernel of the
    exchange (index, waits, quantised rows, return targets, the scatter-mode
    layer, publish, ordered combine) can be profiled on one GPU.  Not a
    scaling number: all tokens go to this rank and nothing crosses NVLink."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    device = torch.device("cuda:0")
    torch.cuda.set_device(device)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29611")
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=device, timeout=timedelta(seconds=120))
    try:
        r = ep_config4(a, 0, 1, device, profiles=("bf16",), force_ep=True)
    finally:
        dist.destroy_process_group()
    bf = r["bf16"]
    line = {"metric": METRIC, "value": bf["tok_s"], "unit": UNIT, "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": bf["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e2m1 x e4m3 block-scaled (bf16 profile), fp32 accumulate, bf16 out",
            "data": "synthetic (seeded; BASELINE config 4 distributions)",
            "config": {"workload": "cfg4 through the expert-parallel exchange on one rank (profiling aid)",
                       "tokens_per_step": CFG4_TOKENS, "global_batch": CFG4_TOKENS, "parallelism": "ep1",
                       "l2": "256 MiB flush before every timed step"},
            "detail": {"profiles": r}}
    print(json.dumps(line), flush=True)


def main(argv=None):
    a = _args(argv)
    if a.impl == "reference":
        run_reference(a)
    elif a.workload == "prefill":
        run_prefill(a)
    elif a.workload == "offload":
        run_offload(a)
    elif a.workload == "ep1":
        run_ep1(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
