"""Expert-parallel layer on the GPU (NCCL).  The EP forward must equal the
single-GPU layer bit for bit.  World 1 runs in every GPU session; world 2
needs two GPUs and is skipped otherwise."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsv4_plugin import synthetic as S

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _scattered(n_experts, world):
    g = torch.Generator().manual_seed(11)
    perm = torch.randperm(n_experts, generator=g).tolist()
    owner = [0] * n_experts
    for i, e in enumerate(perm):
        owner[e] = i % world
    return owner


def _run(rank, world, port, tokens, out, scattered=False):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, root, os.path.join(root, "deepseek-v4-flash-offload_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from datetime import timedelta

    from helpers import make_plugin_layer

    from dsv4_plugin.parallel_ep import ExpertParallelMoE
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        cfg = S.CFG0
        allx = {e: S.make_expert(cfg, 0, e, 3) for e in range(cfg.n_experts)}
        full, _ = make_plugin_layer(cfg, allx, dev)
        x = S.make_tokens(cfg, 50 + rank, tokens)
        xt = torch.from_numpy(S.to_bf16_bits(x).astype(np.int16)).view(torch.bfloat16).to(dev)
        full.engine.bank.preload_all(3)
        ref = full.forward(xt).clone()
        owner = _scattered(cfg.n_experts, world) if scattered else \
            [e // (cfg.n_experts // world) for e in range(cfg.n_experts)]
        mine = {e: allx[e] for e in range(cfg.n_experts) if owner[e] == rank}
        part, _ = make_plugin_layer(cfg, mine, dev)
        epm = ExpertParallelMoE(part, rank, world, owner=owner if scattered else None)
        for profile in ("bf16", "a4w4"):
            from dsv4_plugin.models import deepseek_v4 as DV4
            DV4._MXFP4_GMM = profile == "a4w4"
            try:
                ref = full.forward(xt).clone()
                got = epm.forward(xt, profile)
            finally:
                DV4._MXFP4_GMM = False
            torch.cuda.synchronize(dev)
            epm.plan.status()
            out[(rank, profile)] = bool(torch.equal(got.view(torch.int16), ref.view(torch.int16)))
        # fixed-capacity exchange, eager and captured in a CUDA graph with its NCCL calls
        ref = full.forward(xt).clone()
        got = epm.forward_static(xt)
        torch.cuda.synchronize(dev)
        epm.plan.status()
        out[(rank, "static")] = bool(torch.equal(got.view(torch.int16), ref.view(torch.int16)))
        xs = xt.clone()
        epm.forward_static(xs)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ys = epm.forward_static(xs)
        g.replay()
        torch.cuda.synchronize(dev)
        out[(rank, "graph")] = bool(torch.equal(ys.view(torch.int16), ref.view(torch.int16)))
        del g
        torch.cuda.synchronize(dev)
        # exchange over NVLink peer memory, eager and captured (the return
        # fused into the down GEMM), both profiles with the tokens sent
        # quantised at their source (FP8 / MXFP4 rows) and as bf16 rows, and
        # with a separate return kernel
        from dsv4_plugin.models import deepseek_v4 as DV4
        ok = True
        for profile in ("bf16", "a4w4"):
            DV4._MXFP4_GMM = profile == "a4w4"
            try:
                refp = full.forward(xt).clone()
            finally:
                DV4._MXFP4_GMM = False
            for quant in (True, False):
                epm.quant_dispatch = quant
                got = epm.forward_p2p(xt, profile)
                epm._p2p[xt.shape[0]].check_status()
                ok = ok and bool(torch.equal(got.view(torch.int16), refp.view(torch.int16)))
        epm.quant_dispatch = True
        epm.fused_return = False
        got = epm.forward_p2p(xt)
        epm._p2p[xt.shape[0]].check_status()
        epm.fused_return = True
        out[(rank, "p2p")] = ok and bool(torch.equal(got.view(torch.int16), ref.view(torch.int16)))
        epm.forward_p2p(xs)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ys = epm.forward_p2p(xs)
        for _ in range(3):
            g.replay()
        epm._p2p[xs.shape[0]].check_status()
        out[(rank, "p2p_graph")] = bool(torch.equal(ys.view(torch.int16), ref.view(torch.int16)))
        del g
        epm.close()
        del epm
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens", [1, 24])
def test_ep_world1_equals_single_gpu(tokens):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_run, args=(1, _port(), tokens, out), nprocs=1, join=True)
    assert dict(out) == {(0, "bf16"): True, (0, "a4w4"): True, (0, "static"): True, (0, "graph"): True,
                         (0, "p2p"): True, (0, "p2p_graph"): True}


@pytest.mark.parametrize("scattered", [False, True])
def test_ep_world2_equals_single_gpu(scattered):
    """World 2, contiguous and scattered expert placement (expert_owner map)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_run, args=(2, _port(), 33, out, scattered), nprocs=2, join=True)
    assert all(out.values()) and len(out) == 12


@pytest.mark.parametrize("world,tokens,topk,scattered", [(2, 33, 8, False), (8, 64, 8, False), (4, 300, 6, False),
                                                       (4, 300, 6, True)])
def test_dispatch_pack_kernel_matches_torch_bookkeeping(world, tokens, topk, scattered):
    """dsv4_ep_dispatch_pack against the same bookkeeping in torch ops (the
    CPU path of StaticExchange.pack): slots, metadata, rows, combine order."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dsv4_plugin.parallel_ep import StaticExchange
    n_experts, h = 64, 256
    g = torch.Generator().manual_seed(tokens)
    x = torch.randn(tokens, h, generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(n_experts, generator=g)[:topk] for _ in range(tokens)]).to(torch.int32)
    w = torch.rand(tokens, topk, generator=g)
    owner = _scattered(n_experts, world) if scattered else None
    ref = StaticExchange(n_experts, 0, world, tokens, topk, h, "cpu", owner=owner)
    pos_ref = ref.pack(x, w, idx)
    ord_ref = ref.order(pos_ref, idx)
    dev = StaticExchange(n_experts, 0, world, tokens, topk, h, "cuda", owner=owner)
    pos = dev.pack(x.cuda(), w.cuda(), idx.cuda())
    torch.cuda.synchronize()
    assert torch.equal(pos.cpu().to(torch.int64), pos_ref)
    assert torch.equal(dev.send_meta.cpu(), ref.send_meta)
    valid = ref.send_meta[:, 0] >= 0
    assert torch.equal(dev.send_x.cpu()[valid].view(torch.int16), ref.send_x[valid].view(torch.int16))
    assert torch.equal(dev.order(pos, idx).cpu().to(torch.int64), ord_ref)
    assert int(dev._dev["status"].item()) == 0


@pytest.mark.parametrize("scattered", [False, True])
def test_ep_world4_equals_single_gpu(scattered):
    if torch.cuda.device_count() < 4:
        pytest.skip("needs four GPUs")
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_run, args=(4, _port(), 40, out, scattered), nprocs=4, join=True)
    assert all(out.values()) and len(out) == 24


def _run_timeout(rank, world, port, out):
    """Rank 1 leaves between steps (it makes no further exchange calls); rank
    0's next dispatch waits for flags that nothing sets, runs out after the
    bounded wait and reports DSV4_ETIMEOUT; its stream finishes and the
    context stays usable.  Both ranks then destroy their handles."""
    import sys
    import time
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, root, os.path.join(root, "deepseek-v4-flash-offload_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from datetime import timedelta

    from dsv4_plugin._lib import DSV4_ETIMEOUT, Dsv4Error
    from dsv4_plugin.parallel_ep import P2PExchange
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        n_experts, tokens, topk, hidden = 16, 8, 4, 256
        g = torch.Generator().manual_seed(rank)
        x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(dev)
        idx = torch.stack([torch.randperm(n_experts, generator=g)[:topk] for _ in range(tokens)]).to(torch.int32)
        w = torch.rand(tokens, topk, generator=g).to(dev)
        ex = P2PExchange(n_experts, rank, world, tokens, topk, hidden, dev)
        rows = torch.zeros((world * tokens * topk, hidden), dtype=torch.bfloat16, device=dev)
        ex.dispatch(x, w, idx.to(dev))
        ex.give_back(rows)               # a stand-in expert output for every received assignment
        ex.check_status()
        out[(rank, "step1")] = True
        dist.barrier()
        if rank == 0:
            t0 = time.time()
            ex.dispatch(x, w, idx.to(dev))
            ex.give_back(rows)
            try:
                ex.check_status()
                out[(rank, "timeout")] = False
            except Dsv4Error as err:
                out[(rank, "timeout")] = err.code == DSV4_ETIMEOUT
            out[(rank, "seconds")] = time.time() - t0
            torch.zeros(1, device=dev).add_(1).item()   # the context still runs work
        dist.barrier()
        ex.close()
    finally:
        dist.destroy_process_group()


def test_ep_peer_wait_times_out_when_a_rank_leaves():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_run_timeout, args=(2, _port(), out), nprocs=2, join=True)
    assert out[(0, "step1")] and out[(1, "step1")]
    assert out[(0, "timeout")]
    assert out[(0, "seconds")] < 30.0
