"""Expert-parallel dispatch / combine bookkeeping on CPU with gloo, world 2.

Each rank routes its own tokens to experts owned by either rank; a stand-in
expert function (row-independent, exact) replaces the GPU GEMM.  The result
after dispatch -> local compute -> return -> ordered combine must equal the
same computation done locally on one rank, bit for bit."""

import os
import socket

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


def _worker(rank, world, port, n_experts, tokens, topk, out):
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
        ep = ExpertParallel(n_experts, rank, world)
        x_recv, e_recv, w_recv, ctx = ep.dispatch(x, w, idx)
        assert bool(((e_recv >= ep.expert_lo) & (e_recv < ep.expert_lo + ep.e_loc)).all())
        y_recv = _expert_fn(x_recv, e_recv, w_recv)
        rows, order = ep.combine_rows(y_recv, ctx)
        y = _combine_py(rows, order)
        ref = _local_reference(x, w, idx)
        out[rank] = bool(torch.equal(y.view(torch.int16), ref.view(torch.int16)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens", [0, 1, 37])
def test_ep_dispatch_combine_gloo_world2(tokens):
    world, n_experts, topk = 2, 16, 4
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), n_experts, tokens, topk, out), nprocs=world, join=True)
    assert dict(out) == {0: True, 1: True}


def _worker_static(rank, world, port, n_experts, tokens, topk, out):
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
        ex = StaticExchange(n_experts, rank, world, tokens, topk, 64, "cpu")
        pos = ex.pack(x, w, idx)
        x_recv, e_recv, w_recv = ex.exchange()
        valid = e_recv >= 0
        e_loc = n_experts // world
        ok = bool(((e_recv[valid] >= rank * e_loc) & (e_recv[valid] < (rank + 1) * e_loc)).all())
        # every assignment destined to this rank arrives exactly once
        to_rank = torch.bincount(idx.reshape(-1).to(torch.int64) // e_loc, minlength=world)
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


@pytest.mark.parametrize("tokens", [1, 29])
def test_ep_static_exchange_gloo_world2(tokens):
    """Fixed-capacity exchange (padding rows with expert -1): same result as
    the local computation, and every assignment reaches its owner once."""
    world, n_experts, topk = 2, 16, 4
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker_static, args=(world, _free_port(), n_experts, tokens, topk, out), nprocs=world, join=True)
    assert dict(out) == {0: True, 1: True}
