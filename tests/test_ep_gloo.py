"""Expert-parallel dispatch / combine bookkeeping on CPU with gloo, world 2.

Each rank routes its own tokens to experts owned by either rank; a stand-in
expert function (row-independent, exact) replaces the GPU GEMM.  The result
after dispatch -> local compute -> return -> ordered combine must equal the
same computation done locally on one rank, bit for bit."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _expert_fn(x, e, w):
    """Stand-in expert: exact in bf16 so any reordering bug shows."""
    return (x.float() * (e.float() + 1.0).unsqueeze(1) * w.unsqueeze(1)).to(torch.bfloat16)


def _combine_py(rows, order):
    t, k = order.shape
    y = torch.zeros(t, rows.shape[1], dtype=torch.float32)
    for i in range(t):
        for j in range(k):
            p = int(order[i, j])
            if p >= 0:
                y[i] += rows[p].float()
    return y.to(torch.bfloat16)


def _local_reference(x, w, idx):
    t, k = idx.shape
    y = torch.zeros(t, x.shape[1], dtype=torch.float32)
    srt = torch.argsort(idx, dim=1, stable=True)
    for i in range(t):
        for j in srt[i].tolist():
            y[i] += _expert_fn(x[i:i + 1], idx[i, j:j + 1], w[i, j:j + 1])[0].float()
    return y.to(torch.bfloat16)


def _owner(kind, n_experts, world):
    if kind is None:
        return None
    g = torch.Generator().manual_seed(7)
    perm = torch.randperm(n_experts, generator=g).tolist()   # a scattered placement, E / R per rank
    owner = [0] * n_experts
    for i, e in enumerate(perm):
        owner[e] = i % world
    return owner


def _worker(rank, world, port, n_experts, tokens, topk, out, placement=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dsv4_plugin.parallel_ep import ExpertParallel
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(tokens, 64, generator=g).to(torch.bfloat16)
        idx = torch.stack([torch.randperm(n_experts, generator=g)[:topk] for _ in range(tokens)]).to(torch.int32) \
            if tokens else torch.zeros((0, topk), dtype=torch.int32)
        if tokens:
            idx[: tokens // 2, 0] = n_experts - 1          # skew toward the last rank
        w = torch.rand(tokens, topk, generator=g)
        ep = ExpertParallel(n_experts, rank, world, owner=_owner(placement, n_experts, world))
        x_recv, e_recv, w_recv, ctx = ep.dispatch(x, w, idx)
        assert set(e_recv.tolist()) <= set(ep.local)
        y_recv = _expert_fn(x_recv, e_recv, w_recv)
        rows, order = ep.combine_rows(y_recv, ctx)
        y = _combine_py(rows, order)
        ref = _local_reference(x, w, idx)
        out[rank] = bool(torch.equal(y.view(torch.int16), ref.view(torch.int16)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,placement", [(0, None), (1, None), (37, None), (37, "scattered")])
def test_ep_dispatch_combine_gloo_world2(tokens, placement):
    world, n_experts, topk = 2, 16, 4
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), n_experts, tokens, topk, out, placement), nprocs=world, join=True)
    assert dict(out) == {0: True, 1: True}


def test_balanced_placement_evens_the_rows_per_rank():
    from dsv4_plugin.parallel_ep import balanced_placement, contiguous_placement
    rng = np.random.default_rng(0)
    loads = (1.0 / (1 + rng.permutation(256)) ** 1.1) * 10000     # Zipf(1.1) over a random permutation
    for world in (2, 4, 8):
        own = balanced_placement(loads, world)
        assert [own.count(r) for r in range(world)] == [256 // world] * world
        per = np.bincount(own, weights=loads, minlength=world)
        cont = np.bincount(contiguous_placement(256, world), weights=loads, minlength=world)
        assert per.max() / per.mean() <= cont.max() / cont.mean()
        # no rank above the mean by more than 5 %, except the one that must
        # hold the heaviest expert, which then carries the lightest others
        fill = np.sort(loads)[: 256 // world - 1].sum()
        assert per.max() <= max(loads.max() + fill, 1.05 * per.mean())


def _worker_static(rank, world, port, n_experts, tokens, topk, out, placement=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dsv4_plugin.parallel_ep import StaticExchange
        g = torch.Generator().manual_seed(200 + rank)
        x = torch.randn(tokens, 64, generator=g).to(torch.bfloat16)
        idx = torch.stack([torch.randperm(n_experts, generator=g)[:topk] for _ in range(tokens)]).to(torch.int32)
        idx[: tokens // 2, 0] = n_experts - 1
        w = torch.rand(tokens, topk, generator=g)
        owner = _owner(placement, n_experts, world)
        ex = StaticExchange(n_experts, rank, world, tokens, topk, 64, "cpu", owner=owner)
        own = torch.tensor(owner if owner is not None else [e // (n_experts // world) for e in range(n_experts)])
        pos = ex.pack(x, w, idx)
        x_recv, e_recv, w_recv = ex.exchange()
        valid = e_recv >= 0
        ok = bool((own[e_recv[valid].to(torch.int64)] == rank).all())
        # every assignment destined to this rank arrives exactly once
        to_rank = torch.bincount(own[idx.reshape(-1).to(torch.int64)], minlength=world)
        dist.all_reduce(to_rank)
        ok = ok and int(valid.sum()) == int(to_rank[rank])
        y_recv = torch.zeros_like(x_recv)
        y_recv[valid] = _expert_fn(x_recv[valid], e_recv[valid], w_recv[valid])
        back = ex.give_back(y_recv)
        y = _combine_py(back, ex.order(pos, idx))
        ref = _local_reference(x, w, idx)
        out[rank] = ok and bool(torch.equal(y.view(torch.int16), ref.view(torch.int16)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,placement", [(1, None), (29, None), (29, "scattered")])
def test_ep_static_exchange_gloo_world2(tokens, placement):
    """Fixed-capacity exchange (padding rows with expert -1): same result as
    the local computation, and every assignment reaches its owner once."""
    world, n_experts, topk = 2, 16, 4
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker_static, args=(world, _free_port(), n_experts, tokens, topk, out, placement), nprocs=world,
             join=True)
    assert dict(out) == {0: True, 1: True}
