"""The router entry point that allocates nothing (dsv4_route_topk_noalloc).

It serves callers that cannot allocate device memory while they route a
batch, e.g. a serving engine whose cache pool already holds nearly all free
HBM.  Its logits scratch is a fixed device array inside the library, so this
test checks, through the C ABI, that two calls in a row give the same
weights and expert ids as the workspace-taking dsv4_route_topk (same
tolerance as the other router tests), and that a batch larger than the
fixed scratch is refused with a clear error.  This file is collected last.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from dsv4_plugin import synthetic as S

pytestmark = pytest.mark.gpu
MAX_LOGITS = 65536


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dsv4_plugin import _lib
    return _lib


def _inputs(T, seed):
    cfg = S.CFG1
    gw, bias = S.make_gate(cfg, seed)
    x = S.make_tokens(cfg, seed, T)
    xt = torch.from_numpy(S.to_bf16_bits(x).astype(np.int16)).view(torch.bfloat16).cuda()
    return cfg, xt, torch.from_numpy(gw).cuda(), torch.from_numpy(bias).cuda()


def _route(L, noalloc, cfg, xt, gw, bias):
    T = xt.shape[0]
    w = torch.empty((T, cfg.topk), dtype=torch.float32, device="cuda")
    i = torch.empty((T, cfg.topk), dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    args = (xt.data_ptr(), gw.data_ptr(), bias.data_ptr(), None, None, 0, T, cfg.hidden, cfg.n_experts, cfg.topk,
            2, 1, cfg.route_scale, w.data_ptr(), i.data_ptr())
    if noalloc:
        L.check(L.lib().dsv4_route_topk_noalloc(*args, s))
    else:
        nb = L.lib().dsv4_route_workspace_bytes(T, cfg.hidden, cfg.n_experts)
        ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
        L.check(L.lib().dsv4_route_topk(*args, ws.data_ptr(), nb, s))
    torch.cuda.synchronize()
    return w.cpu().numpy(), i.cpu().numpy()


def test_noalloc_router_matches_workspace_router_on_two_calls(L):
    for T, seed in ((64, 1), (200, 2)):
        cfg, xt, gw, bias = _inputs(T, seed)
        w_ref, i_ref = _route(L, False, cfg, xt, gw, bias)
        w_na, i_na = _route(L, True, cfg, xt, gw, bias)
        assert np.array_equal(np.sort(i_na, -1), np.sort(i_ref, -1))
        np.testing.assert_allclose(np.take_along_axis(w_na, np.argsort(i_na, -1), -1),
                                   np.take_along_axis(w_ref, np.argsort(i_ref, -1), -1), rtol=1e-5, atol=1e-7)


def test_noalloc_router_refuses_batches_beyond_its_scratch(L):
    cfg = S.CFG1
    T = MAX_LOGITS // cfg.n_experts + 1
    xt = torch.zeros((T, cfg.hidden), dtype=torch.bfloat16, device="cuda")
    gw = torch.zeros((cfg.n_experts, cfg.hidden), dtype=torch.float32, device="cuda")
    w = torch.empty((T, cfg.topk), dtype=torch.float32, device="cuda")
    i = torch.empty((T, cfg.topk), dtype=torch.int32, device="cuda")
    rc = L.lib().dsv4_route_topk_noalloc(xt.data_ptr(), gw.data_ptr(), None, None, None, 0, T, cfg.hidden,
                                         cfg.n_experts, cfg.topk, 2, 1, 1.5, w.data_ptr(), i.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == L.DSV4_EINVAL
    assert b"fixed scratch" in L.lib().dsv4_last_error_string()
