"""Expert parallelism: the routed-expert layer sharded over ranks by expert.

Expert e lives on rank ``owner[e]``: by default ``e // (E / R)``; a
load-balanced placement (``balanced_placement``, the static counterpart of
the EPLB hooks the reference's layer carries, deepseek_v4.py:74-85) puts
E / R experts on every rank so that the expected rows per rank are as even
as the expert loads allow.  One forward on every rank:
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

import torch
import torch.distributed as dist

from dsv4_plugin._lib import ROWS_BF16, ROWS_FP8, ROWS_MXFP4


def contiguous_placement(n_experts: int, world: int) -> list:
    """owner[e] = e // (E / R)."""
    if n_experts % world:
        raise ValueError("n_experts must divide evenly over the ranks")
    return [e // (n_experts // world) for e in range(n_experts)]


def balanced_placement(loads, world: int) -> list:
    """Experts to ranks, E / R per rank, evening out the expected rows per
    rank: experts in descending load, each to the least-loaded rank that has
    room (ties: lower rank; equal loads: lower expert id first).  ``loads``:
    per-expert row counts of a calibration batch."""
    loads = [float(v) for v in loads]
    n = len(loads)
    if n % world:
        raise ValueError("n_experts must divide evenly over the ranks")
    room = [n // world] * world
    tot = [0.0] * world
    owner = [0] * n
    for e in sorted(range(n), key=lambda i: (-loads[i], i)):
        r = min((r for r in range(world) if room[r] > 0), key=lambda r: (tot[r], r))
        owner[e] = r
        room[r] -= 1
        tot[r] += loads[e]
    return owner


class ExpertParallel:
    """Dispatch / combine bookkeeping of one expert-parallel layer."""

    def __init__(self, n_experts: int, rank: int, world: int, group=None, owner=None):
        self.n_experts, self.rank, self.world, self.group = n_experts, rank, world, group
        self.owner = list(owner) if owner is not None else contiguous_placement(n_experts, world)
        if len(self.owner) != n_experts or sorted(set(self.owner)) != list(range(world)):
            raise ValueError("owner must map every expert to a rank in [0, world)")
        self.local = [e for e in range(n_experts) if self.owner[e] == rank]
        self.e_loc = len(self.local)
        self._owner_dev = {}

    def owner_tensor(self, device) -> torch.Tensor:
        t = self._owner_dev.get(str(device))
        if t is None:
            t = torch.tensor(self.owner, dtype=torch.int32, device=device)
            self._owner_dev[str(device)] = t
        return t

    def dispatch(self, x: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor):
        """-> (x_recv [N,H], expert_recv [N] int32 global ids, w_recv [N] fp32, ctx)."""
        t, k = indices.shape
        flat_e = indices.reshape(-1).to(torch.int64)
        dest = self.owner_tensor(flat_e.device).to(torch.int64).index_select(0, flat_e)
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


class StaticExchange:
    """Dispatch / return with a fixed capacity of C = T*k rows per peer.

    The exact exchange above needs the per-peer row counts on the host (one
    synchronisation per step).  Here every rank sends C rows to every peer
    (the worst case: all of its assignments on one peer), padding rows carry
    expert id -1, which the routed-expert kernels skip.  Every step is a
    device operation with a shape known in advance, so the whole layer
    (router, exchange, experts, return, combine) can be captured in one CUDA
    graph, NCCL collectives included.  Bookkeeping uses only ops without
    host synchronisation (stable sort, scatter_add, cumsum, gathers)."""

    def __init__(self, n_experts: int, rank: int, world: int, tokens: int, topk: int, hidden: int, device,
                 group=None, dtype=torch.bfloat16, owner=None):
        self.n_experts, self.rank, self.world, self.group = n_experts, rank, world, group
        self.owner = torch.tensor(owner if owner is not None else contiguous_placement(n_experts, world),
                                  dtype=torch.int32, device=device)
        self.t, self.k, self.h = tokens, topk, hidden
        self.cap = tokens * topk
        n = world * self.cap
        self.send_x = torch.empty((n, hidden), dtype=dtype, device=device)
        self.recv_x = torch.empty_like(self.send_x)
        self.send_meta = torch.empty((n, 2), dtype=torch.int32, device=device)
        self.recv_meta = torch.empty_like(self.send_meta)
        self.back = torch.empty_like(self.send_x)
        self._p = torch.arange(tokens * topk, device=device)
        self._dev = None

    def pack(self, x: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor):
        """Fill the send buffers; -> pos [P] (slot of each assignment).  On
        CUDA one library call (``dsv4_ep_dispatch_pack``), which also fills
        the combine order; elsewhere the same bookkeeping in torch ops."""
        if x.is_cuda:
            from dsv4_plugin._lib import check, lib
            if self._dev is None:
                p = self.t * self.k
                self._dev = {"pos": torch.empty(p, dtype=torch.int32, device=x.device),
                             "ordered": torch.empty((self.t, self.k), dtype=torch.int32, device=x.device),
                             "status": torch.zeros(1, dtype=torch.int32, device=x.device)}
            d = self._dev
            x, w, i = x.contiguous(), weights.contiguous().float(), indices.contiguous().to(torch.int32)
            check(lib().dsv4_ep_dispatch_pack(x.data_ptr(), w.data_ptr(), i.data_ptr(), self.t, self.k, self.h,
                                              self.n_experts, self.world, self.owner.data_ptr(),
                                              self.send_x.data_ptr(),
                                              self.send_meta.data_ptr(), d["pos"].data_ptr(),
                                              d["ordered"].data_ptr(), d["status"].data_ptr(),
                                              torch.cuda.current_stream(x.device).cuda_stream))
            return d["pos"]
        flat_e = indices.reshape(-1).to(torch.int64)
        dest = self.owner.to(torch.int64).index_select(0, flat_e)
        order = torch.sort(dest, stable=True).indices
        counts = torch.zeros(self.world, dtype=torch.int64, device=dest.device)
        counts.scatter_add_(0, dest, torch.ones_like(dest))
        start = torch.cumsum(counts, 0) - counts
        rank_sorted = self._p - start.index_select(0, dest.index_select(0, order))
        rank = torch.empty_like(rank_sorted)
        rank[order] = rank_sorted
        pos = dest * self.cap + rank
        self.send_meta[:, 0].fill_(-1)   # padding: empty assignment, weight 0
        self.send_meta[:, 1].fill_(0)
        self.send_meta[pos, 0] = flat_e.to(torch.int32)
        self.send_meta[pos, 1] = weights.reshape(-1).float().view(torch.int32)
        self.send_x[pos] = x.index_select(0, torch.div(self._p, self.k, rounding_mode="floor"))
        return pos

    def exchange(self):
        dist.all_to_all_single(self.recv_x, self.send_x, group=self.group)
        dist.all_to_all_single(self.recv_meta, self.send_meta, group=self.group)
        return self.recv_x, self.recv_meta[:, 0], self.recv_meta[:, 1].view(torch.float32)

    def give_back(self, y_recv: torch.Tensor):
        dist.all_to_all_single(self.back, y_recv, group=self.group)
        return self.back

    def order(self, pos: torch.Tensor, indices: torch.Tensor):
        """Per token, its k slots in ascending expert id order [T, k]."""
        if self._dev is not None and pos.is_cuda:
            return self._dev["ordered"]
        srt = torch.argsort(indices.to(torch.int64), dim=1, stable=True)
        return pos.view(self.t, self.k).gather(1, srt)


class _DevPtr:
    """A device buffer owned by the library, seen as a torch tensor."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3}


class P2PExchange:
    """Exchange over NVLink peer memory (``dsv4_ep_*``) with exact per-peer
    counts, one row per (token, destination rank): each source first
    publishes how many of its tokens go to every owner, then writes each such
    token once, compactly, straight into the owner's receive block (mapped
    through CUDA IPC) with its k picks, the other ranks' experts set to -1.
    The owner runs the layer (top-k over its received tokens) on exactly the
    tokens it received (a device-side count, no host synchronisation) and
    writes every assignment's output straight back.  Device flags with a
    per-step epoch replace the collectives; the step can be captured in a
    CUDA graph.  Creating it is collective (the IPC handles are gathered)."""

    def __init__(self, n_experts: int, rank: int, world: int, tokens: int, topk: int, hidden: int, device,
                 group=None, owner=None):
        import ctypes as C

        from dsv4_plugin._lib import check, lib
        self.n_experts, self.rank, self.world, self.group = n_experts, rank, world, group
        self.t, self.k, self.h = tokens, topk, hidden
        self.device = torch.device(device)
        self.owner = torch.tensor(owner if owner is not None else contiguous_placement(n_experts, world),
                                  dtype=torch.int32, device=self.device)
        nb = lib().dsv4_ep_ipc_handle_bytes()
        handle = C.create_string_buffer(nb)
        self._h = C.c_void_p()
        check(lib().dsv4_ep_create(C.byref(self._h), self.device.index, rank, world, tokens, topk, hidden, handle))
        mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8).to(self.device)
        every = torch.empty(world * nb, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        allh = every.cpu().numpy().tobytes()
        check(lib().dsv4_ep_connect(self._h, C.create_string_buffer(allh, len(allh))))
        rx, ri, rw, rn, bk = (C.c_void_p() for _ in range(5))
        check(lib().dsv4_ep_buffers(self._h, C.byref(rx), C.byref(ri), C.byref(rw), C.byref(rn), C.byref(bk)))
        rows = world * tokens
        dev = self.device
        self.recv_x = torch.as_tensor(_DevPtr(rx.value, (rows, hidden), "<i2"), device=dev).view(torch.bfloat16)
        self.recv_idx = torch.as_tensor(_DevPtr(ri.value, (rows, topk), "<i4"), device=dev)
        self.recv_w = torch.as_tensor(_DevPtr(rw.value, (rows, topk), "<f4"), device=dev)
        self.n_recv = torch.as_tensor(_DevPtr(rn.value, (1,), "<i4"), device=dev)
        self.back = torch.as_tensor(_DevPtr(bk.value, (tokens * topk, hidden), "<i2"),
                                    device=dev).view(torch.bfloat16)
        self.ordered = torch.empty((tokens, topk), dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        # the receive rows seen as quantised rows (uint8 [rows, row_bytes]) per format
        self._recv_q = {}
        for fmt in (ROWS_FP8, ROWS_MXFP4):
            rb = int(lib().dsv4_ep_row_bytes(fmt, hidden))
            self._recv_q[fmt] = torch.as_tensor(_DevPtr(rx.value, (rows, rb), "|u1"), device=dev)

    def dispatch(self, x: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor, row_format: int = ROWS_BF16):
        """-> (recv_x, recv_indices, recv_weights, n_recv): the received tokens
        (the first *n_recv rows of the buffers) and their device-side count.
        With ``row_format`` ROWS_FP8 / ROWS_MXFP4 the tokens are quantised at
        the source and recv_x is uint8 [rows, row_bytes] of quantised rows."""
        from dsv4_plugin._lib import check, lib
        x, w, i = x.contiguous(), weights.contiguous().float(), indices.contiguous().to(torch.int32)
        if x.shape[0] != self.t:
            raise ValueError(f"the exchange was made for {self.t} tokens, got {x.shape[0]}")
        check(lib().dsv4_ep_dispatch_q(self._h, x.data_ptr(), w.data_ptr(), i.data_ptr(), self.t, self.n_experts,
                                       self.owner.data_ptr(), self.ordered.data_ptr(), int(row_format),
                                       self.status.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream))
        rx = self.recv_x if row_format == ROWS_BF16 else self._recv_q[row_format]
        return rx, self.recv_idx, self.recv_w, self.n_recv

    def return_targets(self) -> int:
        """Device address of the table of each received assignment's return
        destination (filled by ``dispatch``), for ``MoEPlan.forward_scatter``."""
        import ctypes as C

        from dsv4_plugin._lib import check, lib
        t = C.c_void_p()
        check(lib().dsv4_ep_return_targets(self._h, C.byref(t)))
        return t.value

    def returned(self):
        """After the scatter-mode layer wrote the rows into the sources'
        ``back``: announce it and wait for every owner; -> ``back``."""
        from dsv4_plugin._lib import check, lib
        check(lib().dsv4_ep_return_published(self._h, self.status.data_ptr(),
                                             torch.cuda.current_stream(self.device).cuda_stream))
        return self.back

    def give_back(self, rows: torch.Tensor, row_of_assignment: torch.Tensor | None = None):
        """Send the output of every received assignment (token j, pick s) --
        ``rows[row_of_assignment[j*k + s]]``, or ``rows[j*k + s]`` -- back to
        its source; -> this rank's ``back`` rows [T*k, H] (assignment order)."""
        from dsv4_plugin._lib import check, lib
        check(lib().dsv4_ep_return(self._h, rows.data_ptr(),
                                   None if row_of_assignment is None else row_of_assignment.data_ptr(),
                                   self.status.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream))
        return self.back

    def check_status(self):
        """Raise when a device-side step failed (e.g. a wait ran out)."""
        torch.cuda.current_stream(self.device).synchronize()
        code = int(self.status.item())
        if code:
            self.status.zero_()
            from dsv4_plugin._lib import Dsv4Error
            raise Dsv4Error(code, "expert-parallel exchange reported this status")

    def close(self):
        """Collective: unmap the peers' blocks and free this rank's."""
        from dsv4_plugin._lib import lib
        if self._h:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            lib().dsv4_ep_destroy(self._h)
            self._h = None


class ExpertParallelMoE:
    """Expert-parallel forward of an ``OffloadDeepseekV4MoE`` whose bank
    holds this rank's experts (``owner[e] == rank``; default contiguous)."""

    def __init__(self, moe, rank: int, world: int, group=None, owner=None):
        self.moe = moe
        self.ep = ExpertParallel(moe.n_routed_experts, rank, world, group, owner)
        bank = moe.engine.bank
        local = self.ep.local
        slots = bank.ensure_resident(moe.layer_idx, local)
        table = torch.full((moe.n_routed_experts,), -1, dtype=torch.int32)
        table[torch.tensor(local, dtype=torch.long)] = torch.tensor(slots, dtype=torch.int32)
        self.slot_of = table.to(bank.device)
        self.plan = None
        self._static = {}
        self._p2p = {}
        self.segment_times = None   # set to {} to time the segments of eager forward_static / forward_p2p calls
        # the peer-memory path returns the rows from the down GEMM's epilogue
        # (DSV4_EP_FUSED_RETURN=0: a separate return kernel after the layer)
        import os
        self.fused_return = os.environ.get("DSV4_EP_FUSED_RETURN", "1") != "0"
        # the tokens cross NVLink quantised in the profile's format (FP8 rows
        # for bf16, MXFP4 for a4w4; DSV4_EP_QUANT_DISPATCH=0: bf16 rows)
        self.quant_dispatch = os.environ.get("DSV4_EP_QUANT_DISPATCH", "1") != "0"

    def forward_static(self, hs: torch.Tensor, profile: str = "bf16") -> torch.Tensor:
        """The same layer through ``StaticExchange``: no host synchronisation,
        so the call can be captured in a CUDA graph.  Equals ``forward`` bit
        for bit."""
        from dsv4_plugin import ops
        moe = self.moe
        t = hs.shape[0]
        ex = self._static.get(t)
        if ex is None:
            ex = StaticExchange(moe.n_routed_experts, self.ep.rank, self.ep.world, t, moe.topk, hs.shape[1],
                                hs.device, self.ep.group, owner=self.ep.owner)
            self._static[t] = ex
        marks = [] if self.segment_times is not None else None

        def mark():
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append(ev)

        mark()
        w, idx = moe._route(hs, None)
        mark()
        pos = ex.pack(hs, w, idx)
        mark()
        x_recv, e_recv, w_recv = ex.exchange()
        mark()
        plan = moe.engine.plan_for(moe.n_routed_experts, 1, x_recv.shape[0], moe.swiglu_limit or 0.0)
        self.plan = plan
        y_recv = plan.forward(x_recv, w_recv.view(-1, 1), e_recv.view(-1, 1), self.slot_of, profile)
        mark()
        back = ex.give_back(y_recv)
        mark()
        y = ops.combine_ordered(back, ex.order(pos, idx))
        mark()
        if marks is not None:
            marks[-1].synchronize()
            names = ("route", "pack", "dispatch_a2a", "experts", "return_a2a", "combine")
            self.segment_times = {n: marks[i].elapsed_time(marks[i + 1]) for i, n in enumerate(names)}
        return y

    def forward_p2p(self, hs: torch.Tensor, profile: str = "bf16") -> torch.Tensor:
        """The same layer through ``P2PExchange`` (NVLink peer memory, exact
        counts, each token once per destination rank): no collectives, no host
        synchronisation; capturable in a CUDA graph.  The owner runs the
        experts (top-k, foreign picks -1) on exactly the tokens it received
        and returns each assignment's output straight from the layer's sorted
        output (no combine pass on the owner).  Equals ``forward`` bit for
        bit.  The first call with a new token count is collective (it maps
        the peers' buffers)."""
        from dsv4_plugin import ops
        moe = self.moe
        t = hs.shape[0]
        ex = self._p2p.get(t)
        if ex is None:
            ex = P2PExchange(moe.n_routed_experts, self.ep.rank, self.ep.world, t, moe.topk, hs.shape[1],
                             hs.device, self.ep.group, owner=self.ep.owner)
            self._p2p[t] = ex
        marks = [] if self.segment_times is not None else None

        def mark():
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append(ev)

        mark()
        w, idx = moe._route(hs, None)
        mark()
        fmt = ROWS_BF16
        if self.fused_return and self.quant_dispatch:
            fmt = ROWS_MXFP4 if profile == "a4w4" else ROWS_FP8
        x_recv, i_recv, w_recv, n_recv = ex.dispatch(hs, w, idx, fmt)
        mark()
        plan = moe.engine.plan_for(moe.n_routed_experts, moe.topk, x_recv.shape[0], moe.swiglu_limit or 0.0)
        self.plan = plan
        if self.fused_return:
            # the down GEMM's epilogue stores every output row straight into
            # its source's `back` over NVLink, tile by tile
            plan.forward_scatter(x_recv, w_recv, i_recv, self.slot_of, ex.return_targets(), profile,
                                 n_tokens_dev=n_recv, x_format=fmt)
            mark()
            back = ex.returned()
        else:
            rows, inv = plan.forward_rows(x_recv, w_recv, i_recv, self.slot_of, profile, n_tokens_dev=n_recv)
            mark()
            back = ex.give_back(rows, inv)
        mark()
        y = ops.combine_ordered(back, ex.ordered)
        mark()
        if marks is not None:
            marks[-1].synchronize()
            names = ("route", "dispatch", "experts", "return", "combine")
            self.segment_times = {n: marks[i].elapsed_time(marks[i + 1]) for i, n in enumerate(names)}
        return y

    def close(self):
        """Collective: release the peer-memory exchanges."""
        for ex in self._p2p.values():
            ex.close()
        self._p2p.clear()

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
