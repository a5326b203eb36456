"""Expert parallelism: the routed-expert layer sharded over ranks by expert.

Expert e lives on rank ``e // (E / R)``.  One forward on every rank:
  1. route the rank's own tokens (the same router kernel as one GPU);
  2. dispatch: order the T*k assignments by destination rank (stable), swap
     per-destination counts with an all-to-all, then all-to-all the token
     rows (bf16) and their (expert id, route weight) pairs;
  3. local experts: the received rows run through the grouped-GEMM plan as
     tokens with exactly one expert each;
  4. return: all-to-all the output rows back to their source ranks;
  5. combine: per token, sum its k rows in ascending expert id order in
     float32 (``ops.combine_ordered``), the order of the reference's
     ``index_add_`` (deepseek_v4.py:195-197).
Each row's expert output does not depend on which other rows share its GEMM
tile, so the result equals the single-GPU layer bit for bit.  All receive
buffers are local; the exchange is NCCL (or gloo for the CPU tests).  The
reference has no expert parallelism (``ep_size = 1``, deepseek_v4.py:82).
"""

from __future__ import annotations

import statistics
import time

import torch
import torch.distributed as dist


class ExpertParallel:
    """Dispatch / combine bookkeeping of one expert-parallel layer."""

    def __init__(self, n_experts: int, rank: int, world: int, group=None):
        if n_experts % world:
            raise ValueError("n_experts must divide evenly over the ranks")
        self.n_experts, self.rank, self.world, self.group = n_experts, rank, world, group
        self.e_loc = n_experts // world
        self.expert_lo = rank * self.e_loc

    def dispatch(self, x: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor):
        """-> (x_recv [N,H], expert_recv [N] int32 global ids, w_recv [N] fp32, ctx)."""
        t, k = indices.shape
        flat_e = indices.reshape(-1).to(torch.int64)
        dest = torch.div(flat_e, self.e_loc, rounding_mode="floor")
        order = torch.sort(dest, stable=True).indices
        send = torch.bincount(dest, minlength=self.world)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        sc, rc = send.tolist(), recv.tolist()                 # host sync for the split sizes
        x_send = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
        meta_send = torch.stack([flat_e.index_select(0, order).to(torch.int32),
                                 weights.reshape(-1).float().index_select(0, order).view(torch.int32)], 1)
        n = sum(rc)
        x_recv = x.new_empty((n, x.shape[1]))
        meta_recv = meta_send.new_empty((n, 2))
        dist.all_to_all_single(x_recv, x_send, rc, sc, group=self.group)
        dist.all_to_all_single(meta_recv, meta_send, rc, sc, group=self.group)
        ctx = {"order": order, "sc": sc, "rc": rc, "indices": indices, "t": t, "k": k}
        return x_recv, meta_recv[:, 0].contiguous(), meta_recv[:, 1].contiguous().view(torch.float32), ctx

    def combine_rows(self, y_recv: torch.Tensor, ctx):
        """Send the expert outputs back; -> (rows [P,H] in send order, order [T,k])."""
        p = ctx["t"] * ctx["k"]
        back = y_recv.new_empty((p, y_recv.shape[1]))
        dist.all_to_all_single(back, y_recv.contiguous(), ctx["sc"], ctx["rc"], group=self.group)
        order = ctx["order"]
        pos = torch.empty_like(order)
        pos[order] = torch.arange(p, device=order.device)
        srt = torch.argsort(ctx["indices"].to(torch.int64), dim=1, stable=True)
        ordered = pos.view(ctx["t"], ctx["k"]).gather(1, srt)
        return back, ordered


class ExpertParallelMoE:
    """Expert-parallel forward of an ``OffloadDeepseekV4MoE`` whose bank
    holds this rank's experts."""

    def __init__(self, moe, rank: int, world: int, group=None):
        self.moe = moe
        self.ep = ExpertParallel(moe.n_routed_experts, rank, world, group)
        bank = moe.engine.bank
        lo, n = self.ep.expert_lo, self.ep.e_loc
        slots = bank.ensure_resident(moe.layer_idx, list(range(lo, lo + n)))
        table = torch.full((moe.n_routed_experts,), -1, dtype=torch.int32)
        table[lo:lo + n] = torch.tensor(slots, dtype=torch.int32)
        self.slot_of = table.to(bank.device)
        self.plan = None

    def forward(self, hs: torch.Tensor, profile: str = "bf16") -> torch.Tensor:
        from dsv4_plugin import ops
        moe = self.moe
        w, idx = moe._route(hs, None)
        x_recv, e_recv, w_recv, ctx = self.ep.dispatch(hs, w, idx)
        n = x_recv.shape[0]
        plan = moe.engine.plan_for(moe.n_routed_experts, 1, max(n, 1), moe.swiglu_limit or 0.0)
        self.plan = plan
        y_recv = plan.forward(x_recv, w_recv.view(-1, 1), e_recv.view(-1, 1), self.slot_of, profile) if n else \
            x_recv.new_empty((0, hs.shape[1]))
        moe.engine.bank.mark_used(None)
        rows, order = self.ep.combine_rows(y_recv, ctx)
        return ops.combine_ordered(rows, order)


def run_ep_bench(a, rank, world, device, metric, unit, build_layer, token_batches, Clocks, flush_bytes):
    """Weak-scaling bench: T tokens per rank, E/R experts per rank."""
    import os

    if not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))
    moe, eng = build_layer(device, rank, world)
    epm = ExpertParallelMoE(moe, rank, world)
    T = a.tokens
    host, dev = token_batches(8, T, device, rank)
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def steps(n, record=True):
        ms = []
        for s in range(n):
            flush.zero_()
            dist.barrier()
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            epm.forward(dev[s % len(dev)])
            e1.record(stream)
            e1.synchronize()
            if record:
                ms.append(e0.elapsed_time(e1))
        return ms

    steps(a.warmup, record=False)
    clk = Clocks(int(os.environ.get("LOCAL_RANK", "0")))
    dist.barrier()
    torch.cuda.synchronize(device)
    clk.start()
    ms = steps(a.steps)
    dist.barrier()
    torch.cuda.synchronize(device)
    clocks = clk.stop()
    # per-step max over ranks (device time)
    t = torch.tensor(ms, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    tot_ms = float(t.sum().item())
    value = world * T * a.steps / (tot_ms / 1e3)

    # e2e: host tokens in, host output back, same exchange
    y_host = torch.empty((T, moe.gate.weight.shape[1]), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(dev[0])

    def e2e_steps(n, record=True):
        out = []
        for s in range(n):
            flush.zero_()
            dist.barrier()
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            xd.copy_(host[s % len(host)], non_blocking=True)
            y = epm.forward(xd)
            y_host.copy_(y, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
            if record:
                out.append(e0.elapsed_time(e1))
        return out

    e2e_steps(2, record=False)
    te = torch.tensor(e2e_steps(a.steps), dtype=torch.float64, device=device)
    dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.sum().item())
    epm.plan.status()
    del epm
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return None
    h = moe.gate.weight.shape[1]
    return {"metric": metric, "value": round(value, 1), "unit": unit, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(tot_ms / a.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "e2m1 x e4m3 block-scaled (bf16 profile), fp32 accumulate, bf16 out",
            "data": "synthetic (seeded; BASELINE config 1 distributions)",
            "config": {"workload": f"cfg1 decode bf16 profile, expert parallel: T={T} tokens per rank, "
                                   f"E={moe.n_routed_experts} experts, {moe.n_routed_experts // world} per rank",
                       "tokens_per_step": T * world, "global_batch": T * world,
                       "parallelism": f"ep{world} (NCCL all-to-all dispatch/combine)",
                       "l2": "256 MiB flush before every timed step; 8 rotating token batches per rank"},
            "e2e": {"value": round(world * T * a.steps / (e2e_ms / 1e3), 1), "unit": unit,
                    "h2d_bytes_per_step": T * h * 2, "d2h_bytes_per_step": T * h * 2},
            "clocks": clocks, "gpu_launches": 8 * a.steps,
            "detail": {"step_ms_median": round(statistics.median(t.tolist()), 5)}}
