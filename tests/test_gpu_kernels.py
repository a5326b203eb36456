"""GPU parity of the element-wise kernels, router and align against the
oracle and the reference's golden fixtures.  Bit-exact where the reference
is integer / byte / exactly-rounded work."""

import os

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from dsv4_plugin import synthetic as S

from helpers import bf16_tensor, bf16_to_np

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dsv4_plugin import ops as _ops
    return _ops


def _gold(name):
    return np.load(os.path.join(GOLD, name))


@pytest.mark.parametrize("tag", ["a", "b"])
def test_dequant_golden(ops, tag):
    g = _gold("ops.npz")
    wp = torch.from_numpy(g[f"deq_{tag}_wp"]).cuda()
    ws = torch.from_numpy(g[f"deq_{tag}_ws"]).cuda()
    out = ops.dequant_fp4_weight(wp, ws)
    got = out.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, g[f"deq_{tag}_out"])


def test_dequant_full_size_bit_exact(ops):
    ex = S.make_expert(S.CFG1, 3, 0)
    for w in ("w1", "w2"):
        out = ops.dequant_fp4_weight(torch.from_numpy(ex[w + "p"]).cuda(), torch.from_numpy(ex[w + "s"]).cuda())
        ref = O.bf16_bits(O.dequant_fp4_weight(ex[w + "p"], ex[w + "s"]))
        assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)


def test_slot_dequant_matches_checkpoint_dequant(ops):
    cfg = S.CFG0
    ex = S.make_expert(cfg, 5, 2)
    slot = ops.pack_expert(*[torch.from_numpy(ex[k]) for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")],
                           cfg.hidden, cfg.inter).cuda()
    d = ops.slot_dequant(slot, cfg.hidden, cfg.inter)
    for w in ("w1", "w2", "w3"):
        ref = O.bf16_bits(O.dequant_fp4_weight(ex[w + "p"], ex[w + "s"]))
        assert np.array_equal(d[w].cpu().view(torch.int16).numpy().view(np.uint16), ref)


def test_act_quant_golden_and_exhaustive(ops):
    g = _gold("ops.npz")
    x = torch.from_numpy(g["aq_x"].view(np.int16)).view(torch.bfloat16).cuda()
    ops.act_quant(x, 128, "ue8m0", None, True)
    assert np.array_equal(x.cpu().view(torch.int16).numpy().view(np.uint16), g["aq_y"])
    # every finite bf16 value, shuffled into 128-blocks, against the reference
    xt = torch.from_numpy(g["aq_all_x"].view(np.int16)).view(torch.bfloat16).cuda()
    ops.act_quant(xt, 128, "ue8m0", None, True)
    assert np.array_equal(xt.cpu().view(torch.int16).numpy().view(np.uint16), g["aq_all_y"])


def test_mx_quant_bit_exact(ops):
    rng = np.random.default_rng(1)
    x = S.bf16_exact(rng.standard_normal((64, 1024)).astype(np.float32) * np.float32(3.0))
    x[3, :32] = 0.0
    x[4, 32:64] = 1e-30
    x[5, 64:96] = 6.0 * 2.0 ** np.arange(32)
    # a block scaled by 1 (max 6): the E2M1 grid, every tie between grid
    # points (to the even code), values that round to +-0, and saturation
    ties = [6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 0.1, 0.3, 4.9, 5.1, 5.9, 1.0, 1.5, 3.0]
    x[6, 96:128] = np.array(ties + [-v for v in ties], np.float32)
    x[7, 128:160] = np.array(ties + [-v for v in ties], np.float32) * np.float32(2.0 ** -20)
    x = S.bf16_exact(x)
    q, s = ops.dynamic_mx_quant(bf16_tensor(x))
    vals, k, _ = O.mx_quant_fp4(x)
    assert np.array_equal(q.cpu().numpy(), O.pack_fp4(vals))
    assert np.array_equal(s.cpu().numpy(), (k + 127).astype(np.uint8))


def _sets(a):
    return np.sort(np.asarray(a), axis=-1)


def test_route_golden_cfg0(ops):
    g = _gold("layer_cfg0.npz")
    x = bf16_tensor(O.bf16_from_bits(g["x"]))
    cfg = S.CFG0
    w, i = ops.route_topk(x, torch.from_numpy(g["gate_w"]).cuda(), torch.zeros(cfg.n_experts).cuda(), cfg.topk,
                          "softmax", False)
    assert np.array_equal(_sets(i.cpu().numpy()), _sets(g["oracle_idx"]))
    ow = np.take_along_axis(g["oracle_w"], np.argsort(g["oracle_idx"], -1), -1)
    gw = np.take_along_axis(w.cpu().numpy(), np.argsort(i.cpu().numpy(), -1), -1)
    np.testing.assert_allclose(gw, ow, rtol=1e-5, atol=1e-7)
    for func, wk, ik in (("sqrtsoftplus", "sq_w", "sq_idx"), ("sigmoid", "sig_w", "sig_idx")):
        w, i = ops.route_topk(x, torch.from_numpy(g["sq_gate_w"]).cuda(), torch.from_numpy(g["sq_bias"]).cuda(),
                              cfg.topk, func, True)
        assert np.array_equal(_sets(i.cpu().numpy()), _sets(g[ik]))
        np.testing.assert_allclose(np.take_along_axis(w.cpu().numpy(), np.argsort(i.cpu().numpy(), -1), -1),
                                   np.take_along_axis(g[wk], np.argsort(g[ik], -1), -1), rtol=1e-5, atol=1e-7)
    w, i = ops.route_topk(x, torch.from_numpy(g["sq_gate_w"]).cuda(), None, cfg.topk, "sqrtsoftplus", True,
                          tid2eid=torch.from_numpy(g["hash_tid2eid"]).cuda(),
                          input_ids=torch.from_numpy(g["hash_ids"]).cuda())
    assert np.array_equal(i.cpu().numpy(), g["hash_idx"])
    np.testing.assert_allclose(w.cpu().numpy(), g["hash_w"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("T", [64, 512])
def test_route_cfg1_matches_reference_plugin(ops, T):
    """Config 1 (E=256, H=4096, sqrtsoftplus, Zipf bias, renormalised):
    the GPU router against the reference plugin's own ``_route`` run on the
    CPU (route_cfg1.npz).  T=512 takes the tensor-core logits kernel."""
    g = _gold("route_cfg1.npz")
    cfg = S.CFG1
    gw, bias = S.make_gate(cfg, 0)
    x = S.make_tokens(cfg, 0, T)
    w, i = ops.route_topk(bf16_tensor(x), torch.from_numpy(gw).cuda(), torch.from_numpy(bias).cuda(), cfg.topk,
                          cfg.score_func, cfg.renormalize)
    i, w = i.cpu().numpy(), w.cpu().numpy()
    assert np.array_equal(_sets(i), _sets(g[f"t{T}_idx"]))
    np.testing.assert_allclose(np.take_along_axis(w, np.argsort(i, -1), -1),
                               np.take_along_axis(g[f"t{T}_w"], np.argsort(g[f"t{T}_idx"], -1), -1),
                               rtol=1e-5, atol=1e-6)


def test_route_hash_rejects_token_ids_outside_the_table(ops):
    """A token id outside [0, vocab) reads no table row: its picks come out
    as expert id E, which the layer's align rejects (the reference raises
    an IndexError on the host for the same input)."""
    cfg = S.CFG0
    vocab = 50
    rng = np.random.default_rng(3)
    tid2eid = rng.integers(0, cfg.n_experts, size=(vocab, cfg.topk)).astype(np.int32)
    ids = np.array([0, 49, 50, -1, 7, 1 << 40], dtype=np.int64)
    x = bf16_tensor(S.make_tokens(cfg, 1, len(ids)))
    gw = torch.from_numpy(S.make_gate(cfg, 0)[0]).cuda()
    w, i = ops.route_topk(x, gw, None, cfg.topk, "sqrtsoftplus", True, tid2eid=torch.from_numpy(tid2eid).cuda(),
                          input_ids=torch.from_numpy(ids).cuda())
    i = i.cpu().numpy()
    for t, tok in enumerate(ids.tolist()):
        if 0 <= tok < vocab:
            assert np.array_equal(i[t], tid2eid[tok])
        else:
            assert np.all(i[t] == cfg.n_experts)
    al = ops.moe_align(torch.from_numpy(i).cuda(), cfg.n_experts)
    assert int(al["status"].item()) == -1   # DSV4_EINVAL


@pytest.mark.parametrize("T", [1, 8, 64, 255, 300, 2048])
def test_route_cfg1_matches_oracle(ops, T):
    """Decode sizes run the 64 x 64 split-K kernel, from 256 tokens the
    128 x 128 one (300: a ragged last token tile)."""
    cfg = S.CFG1
    gw, bias = S.make_gate(cfg, 0)
    x = S.make_tokens(cfg, 0, T)
    w, i = ops.route_topk(bf16_tensor(x), torch.from_numpy(gw).cuda(), torch.from_numpy(bias).cuda(), cfg.topk,
                          cfg.score_func, cfg.renormalize)
    ow, oi = O.route(x, gw, bias, cfg.topk, cfg.score_func, cfg.renormalize)
    assert np.array_equal(_sets(i.cpu().numpy()), _sets(oi))
    np.testing.assert_allclose(np.take_along_axis(w.cpu().numpy(), np.argsort(i.cpu().numpy(), -1), -1),
                               np.take_along_axis(ow, np.argsort(oi, -1), -1), rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("T,k,E", [(0, 8, 256), (1, 8, 256), (64, 8, 256), (2048, 8, 256), (8192, 8, 256),
                                   (16, 4, 16), (33, 6, 1024)])
def test_align_bit_exact(ops, T, k, E):
    rng = np.random.default_rng(T * 31 + E)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]) if T else np.zeros((0, k), np.int64)
    if T:
        # skew: token-majority on a few experts
        idx[: T // 2, 0] = 3
    res = ops.moe_align(torch.from_numpy(idx.astype(np.int32)).cuda(), E)
    ref = O.moe_align(idx.reshape(T, k), E)
    assert int(res["status"].item()) == 0
    assert np.array_equal(res["counts"].cpu().numpy(), ref["counts"])
    assert np.array_equal(res["offsets"].cpu().numpy(), ref["offsets"])
    assert np.array_equal(res["sorted_flat"].cpu().numpy(), ref["order"])
    assert np.array_equal(res["inv"].cpu().numpy(), ref["inv"])
    na = int(res["n_active"].item())
    assert na == ref["active"].size
    assert np.array_equal(res["active"].cpu().numpy()[:na], ref["active"])


@pytest.mark.parametrize("T", [64, 2048])
def test_align_with_empty_assignments(ops, T):
    """Expert id -1 marks an empty assignment (the padding rows of the
    expert-parallel exchange): it gets inv = -1 and no sorted row, and the
    other assignments sort exactly as without it.  T=64 (512 assignments)
    takes the one-pass path, T=2048 (16384) the two-pass path."""
    E, k = 256, 8
    rng = np.random.default_rng(77 + T)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])
    idx[rng.random(idx.shape) < 0.3] = -1
    res = ops.moe_align(torch.from_numpy(idx.astype(np.int32)).cuda(), E)
    flat = idx.reshape(-1)
    valid = np.nonzero(flat >= 0)[0]
    order = valid[np.argsort(flat[valid], kind="stable")]
    counts = np.bincount(flat[valid], minlength=E)
    inv = np.full(flat.size, -1, np.int64)
    inv[order] = np.arange(order.size)
    assert int(res["status"].item()) == 0
    assert np.array_equal(res["counts"].cpu().numpy(), counts)
    assert np.array_equal(res["offsets"].cpu().numpy(), np.concatenate([[0], np.cumsum(counts)]))
    assert np.array_equal(res["sorted_flat"].cpu().numpy()[:order.size], order)
    assert np.array_equal(res["inv"].cpu().numpy(), inv)


def test_align_rejects_out_of_range_expert(ops):
    idx = torch.tensor([[0, 1], [2, 99]], dtype=torch.int32).cuda()
    res = ops.moe_align(idx, 16)
    assert int(res["status"].item()) == -1


def test_mma_peak_probe_reports_a_plausible_rate(ops):
    """The tensor-core rate probe behind the prefill roofline: positive, and
    below twice the nominal dense rate of each kind (9 PF/s mxf4, 4.5 PF/s
    mxf8f6f4) -- far above it would mean the MMAs did not run."""
    import ctypes as C

    from dsv4_plugin._lib import check, lib
    for kind, nominal in ((0, 9000.0), (1, 4500.0)):
        tf, ms = C.c_double(), C.c_double()
        check(lib().dsv4_mma_peak(kind, 256, 20000, 0, C.byref(tf), C.byref(ms)))
        assert 0.05 * nominal < tf.value < 2.0 * nominal, (kind, tf.value)
