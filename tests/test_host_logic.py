"""Host-side logic of the plugin surface, on CPU: checkpoint key parsing,
the weight-load tee, patch installation, the slot LRU bookkeeping and the
layer constructor.  Fixtures come from the reference (tests/golden)."""

import os
import sys
import types

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import moe_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
os.environ.setdefault("DSV4_PIN_HOST", "0")


def test_expert_name_parsing_matches_reference():
    from dsv4_plugin.core.engine import is_expert_weight, parse_expert_name
    g = np.load(os.path.join(GOLD, "engine_names.npz"))
    for name, parsed, main, anyk in zip(g["names"], g["parsed"], g["is_main"], g["is_any"]):
        r = parse_expert_name(str(name))
        got = (-9, -9, -9, -9) if r is None else (r[0], r[1], int(r[2][1]), 0 if r[3] == "weight" else 1)
        assert tuple(parsed) == got, name
        assert is_expert_weight(str(name)) == bool(main), name
        assert is_expert_weight(str(name), include_mtp=True) == bool(anyk), name


def test_slot_lru_matches_reference_bank_traces():
    from dsv4_plugin.core.bank import SlotLRU
    g = np.load(os.path.join(GOLD, "bank_lru.npz"))
    lru = SlotLRU(4)
    for e in range(4):
        lru.lookup([(0, e)])
    lru.lookup([(0, 0)])
    lru.lookup([(1, 0)])
    assert [list(k) for k in lru.od] == g["s1_keys"].tolist()
    assert [lru.hits, lru.misses, lru.evictions] == g["s1_stats"].tolist()
    lru = SlotLRU(7)
    for L, e in g["s2_trace"]:
        lru.lookup([(int(L), int(e))])
    assert [list(k) for k in lru.od] == g["s2_keys"].tolist()
    assert [lru.hits, lru.misses, lru.evictions] == g["s2_stats"][:3].tolist()
    # slots are a bijection over the resident keys
    assert sorted(lru.od.values()) == sorted(set(lru.od.values()))


def test_slot_lru_batch_never_evicts_itself():
    from dsv4_plugin.core.bank import SlotLRU
    lru = SlotLRU(3)
    lru.lookup([(0, 1), (0, 2), (0, 3)])
    slots, misses = lru.lookup([(0, 3), (0, 4), (0, 1)])      # 4 must evict 2, not 3 or 1
    assert [k for k, _ in misses] == [(0, 4)]
    assert (0, 2) not in lru and (0, 3) in lru and (0, 1) in lru
    assert len(set(slots)) == 3
    with pytest.raises(MemoryError):
        lru.lookup([(0, 5), (0, 6), (0, 7), (0, 8)])


def test_slot_lru_random_against_oracle_model():
    from dsv4_plugin.core.bank import SlotLRU
    rng = np.random.default_rng(3)
    for cap in (1, 5, 17):
        lru, ref = SlotLRU(cap), O.LruModel(cap)
        for _ in range(500):
            k = (int(rng.integers(0, 3)), int(rng.integers(0, 30)))
            lru.lookup([k])
            ref.get(k)
        assert list(lru.od) == ref.keys()
        assert (lru.hits, lru.misses, lru.evictions) == (ref.hits, ref.misses, ref.evictions)


def test_slot_lru_batches_against_oracle_model():
    """Whole-layer batches (sorted, distinct keys, as a layer's active
    experts): slots, misses and counts equal the batch model's."""
    from dsv4_plugin.core.bank import SlotLRU
    rng = np.random.default_rng(11)
    for cap in (8, 24, 40):
        lru, ref = SlotLRU(cap), O.SlotLruModel(cap)
        for _ in range(300):
            layer = int(rng.integers(0, 3))
            n = int(rng.integers(1, min(cap, 24) + 1))
            keys = [(layer, int(e)) for e in sorted(rng.choice(64, n, replace=False).tolist())]
            s1, m1 = lru.lookup(keys)
            s2, m2 = ref.lookup(keys)
            assert s1 == s2 and [k for k, _ in m1] == m2
        assert (lru.hits, lru.misses, lru.evictions) == (ref.hits, ref.misses, ref.evictions)
        assert list(lru.od.items()) == list(ref.od.items())


def _six(seed, h=256, i=128):
    g = torch.Generator().manual_seed(seed)
    pk = lambda n, k: torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=g)  # noqa: E731
    sc = lambda n, k: torch.randint(118, 131, (n, k // 32), dtype=torch.uint8, generator=g)  # noqa: E731
    return pk(i, h), sc(i, h), pk(h, i), sc(h, i), pk(i, h), sc(i, h)


def test_engine_capture_and_bank_registration_on_cpu():
    from dsv4_plugin.core.engine import ExpertOffloadEngine
    eng = ExpertOffloadEngine(slot_capacity=8, device="cpu")
    t = _six(1)
    names = [f"layers.3.ffn.experts.5.{w}.{k}" for w in ("w1", "w2", "w3") for k in ("weight", "scale")]
    parts = dict(zip(("w1p", "w1s", "w2p", "w2s", "w3p", "w3s"), t))
    key = {"weight": "p", "scale": "s"}
    for j, n in enumerate(names):
        w, k = n.split(".")[-2:]
        assert eng.capture(n, parts[w + key[k]])
        assert eng.stats()["parked"] == (1 if j < 5 else 0)
    assert eng.captured == 1 and eng.bank.has(3, 5) and eng.bank.num_experts() == 1
    assert not eng.capture("layers.3.ffn.gate.weight", torch.zeros(1))
    s = eng.stats()
    assert s["packed_capacity"] == 32 and s["capacity"] == 8 and s["captured"] == 1
    # the host pool holds the kernel-native slot; unpacking returns the inputs
    from dsv4_plugin import ops
    back = ops.unpack_expert(eng.bank.host_slot(3, 5), 256, 128)
    for k, v in parts.items():
        assert torch.equal(back[k], v)
    with pytest.raises(RuntimeError, match="CUDA"):
        eng.bank.ensure_resident(3, [5])


def _fake_target(name="dsv4_fake_vllm_v4"):
    mod = types.ModuleType(name)

    class DeepseekV4MoE(nn.Module):
        pass

    class DeepseekV4ForCausalLM:
        def load_weights(self, weights):
            return set(n for n, _ in weights)

    mod.DeepseekV4MoE = DeepseekV4MoE
    mod.DeepseekV4ForCausalLM = DeepseekV4ForCausalLM
    mod.get_tensor_model_parallel_world_size = lambda: 1
    mod.get_tensor_model_parallel_rank = lambda: 0
    sys.modules[name] = mod
    return mod


def test_install_patches_and_load_weights_tee(monkeypatch):
    import dsv4_plugin
    from dsv4_plugin.core import engine as ENG
    from dsv4_plugin.models import deepseek_v4 as DV4
    mod = _fake_target()
    monkeypatch.setenv("DSV4_PATCH_MODULE", mod.__name__)
    monkeypatch.setattr(DV4, "_PATCHED", False)
    eng = ENG.ExpertOffloadEngine(slot_capacity=64, device="cpu")
    ENG.reset_engine(eng)
    orig_moe = mod.DeepseekV4MoE
    dsv4_plugin.register_model()
    dsv4_plugin.register_model()                     # idempotent
    assert issubclass(mod.DeepseekV4MoE, DV4.OffloadDeepseekV4MoE)
    assert issubclass(mod.DeepseekV4MoE, orig_moe)
    assert mod.DeepseekV4ForCausalLM.load_weights is DV4._offload_load_weights
    assert mod._DSV4_OFFLOAD_PATCHED

    # tee: 2 layers x 3 experts x 6 blocks (+ MTP and dense keys) through the patched load_weights
    six = _six(7)
    stream, expect_pass = [], []
    for L in (0, 4):
        for e in (0, 1, 9):
            for w, (p, s) in zip(("w1", "w2", "w3"), ((six[0], six[1]), (six[2], six[3]), (six[4], six[5]))):
                stream.append((f"model.layers.{L}.ffn.experts.{e}.{w}.weight", p))
                stream.append((f"model.layers.{L}.ffn.experts.{e}.{w}.scale", s))
    for n in ("mtp.0.ffn.experts.3.w1.weight", "model.layers.0.ffn.gate.weight", "model.embed.weight"):
        stream.append((n, torch.zeros(1)))
        expect_pass.append(n)
    # the shared expert of layer 4 (FP8): teed into the engine and passed on
    from dsv4_plugin import synthetic as S
    sh = S.make_shared_expert(S.MoEConfig("t", 256, 128, 8, 2, "softmax", False), 2, 4)
    for w in ("w1", "w2", "w3"):
        for kind, key in (("weight", w), ("scale", w + "s")):
            n = f"model.layers.4.ffn.shared_experts.{w}.{kind}"
            stream.append((n, torch.from_numpy(sh[key])))
            expect_pass.append(n)
    got = mod.DeepseekV4ForCausalLM().load_weights(iter(stream))
    assert got == set(expect_pass)
    assert eng.captured == 6 and eng.stats()["parked"] == 0
    assert eng.shared_slot(4) is not None and eng.shared_slot(0) is None
    ENG.reset_engine(None)


def test_layer_constructor_fields(monkeypatch):
    from dsv4_plugin.core import engine as ENG
    from dsv4_plugin.models import deepseek_v4 as DV4
    mod = _fake_target("dsv4_fake_vllm_v4b")
    monkeypatch.setenv("DSV4_PATCH_MODULE", mod.__name__)
    ENG.reset_engine(ENG.ExpertOffloadEngine(slot_capacity=4, device="cpu"))
    cfg = types.SimpleNamespace(n_routed_experts=16, n_shared_experts=None, num_experts_per_tok=4,
                                norm_topk_prob=True, scoring_func="sqrtsoftplus", routed_scaling_factor=1.5,
                                swiglu_limit=10.0, num_hash_layers=3, vocab_size=100, hidden_size=256,
                                moe_intermediate_size=128, hidden_act="silu")
    pc = types.SimpleNamespace(use_sequence_parallel_moe=False, eplb_config=None, enable_eplb=False)
    m = DV4.OffloadDeepseekV4MoE(cfg, pc, prefix="model.layers.2.mlp")
    assert m.layer_idx == 2 and m.hash and m.gate.tid2eid.shape == (100, 4)
    assert m.gate.e_score_correction_bias is None
    m5 = DV4.OffloadDeepseekV4MoE(cfg, pc, prefix="model.layers.5.mlp")
    assert not m5.hash and m5.gate.e_score_correction_bias.shape == (16,)
    assert dict(m5.named_parameters()).keys() == {"gate.weight", "gate.e_score_correction_bias"}
    mdraft = DV4.OffloadDeepseekV4MoE(cfg, pc, prefix="model.layers.1.mlp", is_draft_layer=True)
    assert not mdraft.hash
    with pytest.raises(RuntimeError, match="input_ids"):
        m._route(torch.zeros(2, 256), None)
    ENG.reset_engine(None)


def test_gate_split_terms_sum_to_the_gate_exactly():
    """The tensor-core router splits the fp32 gate into hi = bf16(w),
    mid = bf16(w - hi), lo = bf16(w - hi - mid) (gate_split_kernel in
    csrc/route.cu, round to nearest even).  Every residual is exact in fp32,
    the last one is already a bf16 value, and the three terms add up to w
    exactly, so the bf16 products x * term lose nothing.  This holds for
    |w| below bf16's largest finite value (3.39e38); larger fp32 values round
    to infinity in the first term."""
    rng = np.random.default_rng(5)
    n = 200000
    w = (rng.standard_normal(n) * 10.0 ** rng.integers(-30, 30, n)).astype(np.float32)
    w = np.concatenate([w, np.float32([0.0, -0.0, 1.0, -1.0, 3.3e38, -3.3e38, 1.1754944e-38,
                                       np.nextafter(np.float32(1), np.float32(2))])])

    def bf16(v):
        b = v.view(np.uint32).astype(np.uint64)
        return ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)

    hi = bf16(w)
    r1 = (w - hi).astype(np.float32)
    mid = bf16(r1)
    r2 = (r1 - mid).astype(np.float32)
    lo = bf16(r2)
    assert np.array_equal(lo, r2)
    assert np.array_equal(hi.astype(np.float64) + mid.astype(np.float64) + lo.astype(np.float64),
                          w.astype(np.float64))


def test_engine_captures_the_shared_expert_from_the_weight_stream():
    """Shared-expert tensors in the checkpoint's names are parsed, parked and
    packed into the FP8 slot once all six arrived (on the CPU here)."""
    from dsv4_plugin import ops
    from dsv4_plugin.core.engine import ExpertOffloadEngine, is_shared_expert_weight, parse_shared_name
    from dsv4_plugin import synthetic as S
    assert parse_shared_name("model.layers.7.ffn.shared_experts.w2.scale") == (7, "w2", "scale")
    assert not is_shared_expert_weight("layers.7.ffn.experts.3.w2.scale")
    assert not is_shared_expert_weight("layers.7.ffn.shared_experts.w2.bias")
    cfg = S.CFG0
    sh = S.make_shared_expert(cfg, 1, 7)
    eng = ExpertOffloadEngine(slot_capacity=1, device="cpu")
    names = [(f"layers.7.ffn.shared_experts.{w}.{kind}", sh[w + ("" if kind == "weight" else "s")])
             for w in ("w1", "w2", "w3") for kind in ("weight", "scale")]
    for j, (n, t) in enumerate(names):
        assert eng.capture_shared(n, torch.from_numpy(t))
        assert (eng.shared_slot(7) is None) == (j < 5)
    ref = ops.pack_shared_expert(*[torch.from_numpy(sh[k]) for k in ("w1", "w1s", "w2", "w2s", "w3", "w3s")],
                                 cfg.hidden, cfg.inter)
    assert torch.equal(eng.shared_slot(7), ref)
    assert ref.numel() == ops.shared_slot_bytes(cfg.hidden, cfg.inter) == 3 * cfg.hidden * cfg.inter * 33 // 32
