"""Pin the CPU oracle against fixtures produced by the reference's own code
(``tests/golden/make_golden.py``).  CPU only."""

import hashlib
import os

import numpy as np
import pytest

from oracle import moe_oracle as O
from dsv4_plugin import synthetic as S

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name), allow_pickle=False)


def _bf16(bits):
    return O.bf16_from_bits(np.asarray(bits, dtype=np.uint16))


def _e4m3_decode(b):
    b = b.astype(np.int32)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    v = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1 + m / 8.0) * 2.0 ** (e - 7))
    return (s * v).astype(np.float32)


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_dequant_matches_reference(tag):
    g = _load("ops.npz")
    out = O.dequant_fp4_weight(g[f"deq_{tag}_wp"], g[f"deq_{tag}_ws"])
    ref32 = g[f"deq_{tag}_out_f32"]
    assert np.array_equal(out, ref32, equal_nan=True)
    ref16 = g[f"deq_{tag}_out"]
    got16 = O.bf16_bits(O.bf16_round(out))
    fin = np.isfinite(O.bf16_from_bits(ref16))
    assert np.array_equal(got16[fin], ref16[fin])          # bit-exact, incl. the sign of zero


def test_act_quant_roundtrip_matches_reference():
    g = _load("ops.npz")
    x = _bf16(g["aq_x"])
    y = O.act_quant_rt(x)
    assert np.array_equal(O.bf16_bits(y), g["aq_y"])


def test_act_quant_exhaustive_matches_reference():
    g = _load("ops.npz")
    y = O.act_quant_rt(_bf16(g["aq_all_x"]))
    assert np.array_equal(O.bf16_bits(y), g["aq_all_y"])     # incl. the sign of zero and overflow to inf


def test_pow2_scale_exhaustive_over_bf16_amax():
    g = _load("ops.npz")
    amax = O.bf16_from_bits(g["scale_pats"])
    assert np.array_equal(O.fp8_block_scale_exp(amax), g["scale_exp"])


def test_e4m3_cast_exhaustive_over_bf16():
    g = _load("ops.npz")
    v = O.bf16_from_bits(g["e4m3_in"])
    assert np.array_equal(O.e4m3_round(v), _e4m3_decode(g["e4m3_out"]))


def test_fp4_round_tie_rule():
    g = _load("ops.npz")
    assert np.array_equal(O.e2m1_round(g["r4_in"]), g["r4_out"])


@pytest.fixture(scope="module")
def layer0():
    g = _load("layer_cfg0.npz")
    cfg = S.CFG0
    experts = [S.make_expert(cfg, 0, e) for e in range(cfg.n_experts)]
    gate_w, _ = S.make_gate(cfg, 0)
    x = S.make_tokens(cfg, 0, 16)
    h = hashlib.sha256()
    for a in [gate_w, x] + [experts[e][k] for e in range(cfg.n_experts)
                            for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")]:
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.digest() == g["inputs_sha"].tobytes(), "synthetic generator drifted from the fixture"
    return g, cfg, experts, gate_w, x


def _sets(idx):
    return np.sort(np.asarray(idx), axis=-1)


def _aligned(w, idx):
    o = np.argsort(idx, axis=-1)
    return np.take_along_axis(w, o, axis=-1)


def test_router_softmax_matches_reference(layer0):
    g, cfg, experts, gate_w, x = layer0
    w, idx = O.route(x, gate_w, np.zeros(cfg.n_experts, np.float32), cfg.topk, "softmax", False)
    assert np.array_equal(_sets(idx), _sets(g["oracle_idx"]))
    assert np.array_equal(_sets(idx), _sets(g["plugin_softmax_idx"]))
    np.testing.assert_allclose(_aligned(w, idx), _aligned(g["oracle_w"], g["oracle_idx"]), rtol=1e-5, atol=1e-6)


def test_router_sqrtsoftplus_and_sigmoid_match_reference(layer0):
    g, cfg, experts, gate_w, x = layer0
    for func, wk, ik in (("sqrtsoftplus", "sq_w", "sq_idx"), ("sigmoid", "sig_w", "sig_idx")):
        w, idx = O.route(x, g["sq_gate_w"], g["sq_bias"], cfg.topk, func, True)
        assert np.array_equal(_sets(idx), _sets(g[ik]))
        np.testing.assert_allclose(_aligned(w, idx), _aligned(g[wk], g[ik]), rtol=1e-5, atol=1e-6)


def test_router_hash_matches_reference(layer0):
    g, cfg, experts, gate_w, x = layer0
    w, idx = O.route(x, g["sq_gate_w"], None, cfg.topk, "sqrtsoftplus", True,
                     tid2eid=g["hash_tid2eid"], input_ids=g["hash_ids"])
    assert np.array_equal(idx, g["hash_idx"])
    np.testing.assert_allclose(w, g["hash_w"], rtol=1e-5, atol=1e-6)
    assert int(g["hash_missing_ids_raises"][0]) == 1
    with pytest.raises(RuntimeError):
        O.route(x, g["sq_gate_w"], None, cfg.topk, tid2eid=g["hash_tid2eid"], input_ids=None)


@pytest.mark.parametrize("T", [64, 512])
def test_router_cfg1_matches_reference_plugin(T):
    """Config-1-sized routing (E=256, H=4096, sqrtsoftplus, Zipf bias,
    renormalised, x1.5): the oracle against the reference plugin's own
    ``_route`` run on the CPU (route_cfg1.npz)."""
    g = _load("route_cfg1.npz")
    cfg = S.CFG1
    gw, bias = S.make_gate(cfg, 0)
    x = S.make_tokens(cfg, 0, T)
    h = hashlib.sha256()
    for a in (gw, bias, x):
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.digest() == g[f"t{T}_sha"].tobytes(), "synthetic generator drifted from the fixture"
    w, idx = O.route(x, gw, bias, cfg.topk, cfg.score_func, cfg.renormalize)
    assert np.array_equal(_sets(idx), _sets(g[f"t{T}_idx"]))
    np.testing.assert_allclose(_aligned(w, idx), _aligned(g[f"t{T}_w"], g[f"t{T}_idx"]), rtol=1e-5, atol=1e-6)


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_moe_bf16_matches_reference(layer0):
    g, cfg, experts, gate_w, x = layer0
    w, idx = O.route(x, gate_w, np.zeros(cfg.n_experts, np.float32), cfg.topk, "softmax", False)
    y = O.moe_routed(x, w, idx, experts, cfg.n_experts, 10.0, "bf16")
    ref = _bf16(g["oracle_y"])
    plug = _bf16(g["plugin_bf16_y"])
    # the reference's grouped path equals its per-expert loop exactly
    assert np.array_equal(ref, plug)
    # oracle: float32 BLAS accumulation vs the reference's bf16 CPU matmul
    assert _rel(y, ref) <= 1e-2
    assert np.mean(y == ref) > 0.9


def test_moe_routes_sqrtsoftplus_and_hash_match_reference(layer0):
    g, cfg, experts, gate_w, x = layer0
    w, idx = O.route(x, g["sq_gate_w"], g["sq_bias"], cfg.topk, "sqrtsoftplus", True)
    y = O.moe_routed(x, w, idx, experts, cfg.n_experts, 10.0, "bf16")
    assert _rel(y, _bf16(g["sq_y"])) <= 1e-2
    w, idx = O.route(x, g["sq_gate_w"], None, cfg.topk, "sqrtsoftplus", True,
                     tid2eid=g["hash_tid2eid"], input_ids=g["hash_ids"])
    y = O.moe_routed(x, w, idx, experts, cfg.n_experts, 10.0, "bf16")
    assert _rel(y, _bf16(g["hash_y"])) <= 1e-2


def test_moe_a4w4_matches_reference_data_flow(layer0):
    g, cfg, experts, gate_w, x = layer0
    w, idx = O.route(x, gate_w, np.zeros(cfg.n_experts, np.float32), cfg.topk, "softmax", False)
    y = O.moe_routed(x, w, idx, experts, cfg.n_experts, 10.0, "a4w4")
    assert _rel(y, _bf16(g["plugin_a4w4_y"])) <= 1e-2


def test_lru_model_matches_reference_bank():
    g = _load("bank_lru.npz")
    m = O.LruModel(4)
    for e in range(4):
        m.get((0, e))
    m.get((0, 0))
    m.get((1, 0))
    assert [list(k) for k in m.keys()] == g["s1_keys"].tolist()
    assert [m.hits, m.misses, m.evictions] == g["s1_stats"].tolist()
    m2 = O.LruModel(7)
    for L, e in g["s2_trace"]:
        m2.get((int(L), int(e)))
    assert [list(k) for k in m2.keys()] == g["s2_keys"].tolist()
    assert [m2.hits, m2.misses, m2.evictions] == g["s2_stats"][:3].tolist()
    mp = O.LruModel(int(g["s2_stats"][5]))
    for L, e in g["s2_trace"][:150]:
        mp.get((int(L), int(e)))
    assert [list(k) for k in mp.keys()] == g["s2_pkeys"].tolist()
    assert [mp.hits, mp.misses] == g["s2_stats"][3:5].tolist()
    m0 = O.LruModel(0)
    m0.get((0, 0))
    m0.get((0, 0))
    assert [len(m0.keys()), m0.misses] == g["s0_stats"].tolist()
    # ExpertBank.get returns the dequantised bf16 expert
    assert np.array_equal(O.bf16_bits(O.dequant_fp4_weight(g["get_w1_src"], g["get_w1s_src"])), g["get_w1"])


def test_shared_expert_matches_reference():
    """The shared expert (model_npu.Expert in "fp8" mode, weights from
    npu_ops.dequant_fp8_weight) run by the reference on the CPU
    (shared_cfg0.npz): the oracle's FP8 dequant is bit-exact and its output
    equals the reference's to bf16 rounding of a float32 BLAS sum."""
    import hashlib
    g = _load("shared_cfg0.npz")
    cfg = S.CFG0
    sh = S.make_shared_expert(cfg, 0, 3)
    h = hashlib.sha256()
    for k in sorted(sh):
        h.update(np.ascontiguousarray(sh[k]).tobytes())
    assert h.digest() == g["sha"].tobytes(), "synthetic generator drifted from the fixture"
    for w in ("w1", "w2"):
        assert np.array_equal(O.bf16_bits(O.dequant_fp8_weight(sh[w], sh[w + "s"])), g[f"deq_{w}"])
    x = _bf16(g["x"])
    y = O.shared_expert(x, O.shared_weights_f32(sh), cfg.swiglu_limit)
    ref = _bf16(g["y"])
    assert _rel(y, ref) <= 1e-2
    assert np.mean(y == ref) > 0.9
