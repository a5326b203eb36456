"""Generate golden fixtures by running the REFERENCE's own Python code on CPU.

Run in the development container, where the reference checkout exists:

    python tests/golden/make_golden.py --ref <path-to-reference-checkout>

It imports the reference modules (``npu_ops``, ``offload``, ``model_npu``,
``dsv4_plugin.models.deepseek_v4``, ``dsv4_plugin.core.engine``) with two
shims, and writes small ``.npz`` fixtures beside this script:

  * ``torch.utils.rename_privateuse1_backend("npu")`` before ``model_npu``
    (its module-level ``torch.device("npu:0")``), then ``DEVICE = cpu``;
  * stub ``torch_npu`` and ``vllm_ascend.models.deepseek_v4`` modules: the
    grouped matmul stub is a per-group ``x @ w`` (the reference states the
    vendor GMM is bit-exact against the per-expert ``F.linear``), the MX
    quant stub is this build's MXFP4 rule (so the a4w4 fixture pins the
    plugin's data flow, not the closed NPU op's rounding).

``--only route_cfg1`` writes just the config-1 routing fixture
(``route_cfg1.npz``), ``--only shared_cfg0`` just the shared-expert fixture
(``shared_cfg0.npz``), and leave the others as they are.

Large inputs (expert weights) are not stored: they come from the seeded
generator in ``dsv4_plugin/synthetic.py`` and the fixture stores their
SHA-256 so a test can detect generator drift.  The fixtures are consumed by
``tests/test_oracle_golden.py`` (CPU) and the GPU parity tests.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys
import types

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _load_synthetic():
    path = os.path.join(REPO, "deepseek-v4-flash-offload_b200", "dsv4_plugin", "synthetic.py")
    spec = importlib.util.spec_from_file_location("_dsv4_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["_dsv4_synthetic"] = mod
    spec.loader.exec_module(mod)
    return mod


def _sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _mx_quant_rule(x: torch.Tensor):
    """Build's MXFP4 rule: scale exponent floor(log2(amax/6)) computed exactly,
    E2M1 round-to-nearest-even, saturating at 6.  Returns (values, scale) as
    float tensors so the stub GMM can multiply them directly."""
    xf = x.float().reshape(-1, x.shape[-1] // 32, 32)
    amax = xf.abs().amax(-1, keepdim=True)
    m, e = torch.frexp(torch.where(amax > 0, amax, torch.ones_like(amax)))
    k = (e - 1) - 3 + ((m * 2) >= 1.5).to(e.dtype)
    k = torch.where(amax > 0, k.clamp(-127, 127), torch.full_like(k, -127))
    v = torch.ldexp(xf, -k.float())
    a = v.abs().clamp(max=6.0)
    q = torch.where(a < 2, torch.full_like(a, 0.5), torch.where(a < 4, torch.ones_like(a), torch.full_like(a, 2.0)))
    r = torch.minimum(torch.round(a / q) * q, torch.full_like(a, 6.0))
    r = torch.where(v < 0, -r, r)
    return r.reshape(x.shape), torch.ldexp(torch.ones_like(k.float()), k.float()).reshape(*x.shape[:-1], x.shape[-1] // 32)


def install_stubs():
    tnpu = types.ModuleType("torch_npu")
    tnpu.float4_e2m1fn_x2 = "float4_e2m1fn_x2"
    tnpu.float8_e8m0fnu = torch.float8_e8m0fnu

    def npu_grouped_matmul(x, weight, split_item=2, group_list_type=1, group_type=0,
                           group_list=None, bias=None, scale=None, per_token_scale=None,
                           output_dtype=None, x_dtype=None, weight_dtype=None,
                           scale_dtype=None, per_token_scale_dtype=None):
        xs = x[0]
        counts = [int(c) for c in group_list]
        outs = []
        o = 0
        if scale is None:
            for g, c in enumerate(counts):
                outs.append((xs[o:o + c] @ weight[g]).to(xs.dtype))
                o += c
            return [torch.cat(outs, 0)]
        # a4w4 stub: x holds dequantised activations (see the quant stub);
        # weight / scale are the plugin's stacked transposed views
        # [g, K/2, N] and [g, K/64, N, 2] of the packed expert tensors.
        from npu_ops import dequant_fp4_weight
        wstack, sstack = weight[0], scale[0]
        for g, c in enumerate(counts):
            wp = wstack[g].transpose(0, 1).contiguous()
            n = wp.shape[0]
            ws = sstack[g].permute(1, 0, 2).reshape(n, -1).contiguous()
            wd = dequant_fp4_weight(wp, ws, torch.float32)
            outs.append((xs[o:o + c].float() @ wd.T).to(torch.bfloat16))
            o += c
        return [torch.cat(outs, 0)]

    def npu_dynamic_mx_quant(x, dst_type=None):
        v, s = _mx_quant_rule(x)
        deq = (v.reshape(-1, x.shape[-1] // 32, 32) * s.reshape(-1, x.shape[-1] // 32, 1)).reshape(x.shape)
        # the a4w4 stub carries dequantised activations; scale of one keeps
        # the plugin's reshape of the per-token scale valid.
        return deq, torch.ones(*x.shape[:-1], x.shape[-1] // 32)

    tnpu.npu_grouped_matmul = npu_grouped_matmul
    tnpu.npu_dynamic_mx_quant = npu_dynamic_mx_quant
    sys.modules["torch_npu"] = tnpu

    va = types.ModuleType("vllm_ascend")
    vam = types.ModuleType("vllm_ascend.models")
    v4 = types.ModuleType("vllm_ascend.models.deepseek_v4")

    class DeepseekV4MoE(nn.Module):
        pass

    class AscendDeepseekV4ForCausalLM:
        def load_weights(self, weights):
            return set(n for n, _ in weights)

    v4.DeepseekV4MoE = DeepseekV4MoE
    v4.AscendDeepseekV4ForCausalLM = AscendDeepseekV4ForCausalLM
    v4.get_tensor_model_parallel_world_size = lambda: 1
    v4.get_tensor_model_parallel_rank = lambda: 0
    va.models = vam
    vam.deepseek_v4 = v4
    sys.modules["vllm_ascend"] = va
    sys.modules["vllm_ascend.models"] = vam
    sys.modules["vllm_ascend.models.deepseek_v4"] = v4


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def from_f32_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def make_route_cfg1(DV4, S):
    """Config-1-sized routing through the reference plugin's own ``_route``
    (deepseek_v4.py:118-148): sqrtsoftplus scores, the Zipf-shaped bias,
    renormalisation and route_scale 1.5, at T = 64 and 512.  The inputs come
    from the seeded generator; the fixture stores their SHA-256 and the
    outputs only (``route_cfg1.npz``)."""
    cfg = S.CFG1
    gw, bias = S.make_gate(cfg, 0)
    out = {}
    for T in (64, 512):
        x = S.make_tokens(cfg, 0, T)
        m = DV4.OffloadDeepseekV4MoE.__new__(DV4.OffloadDeepseekV4MoE)
        nn.Module.__init__(m)
        m.hash = False
        m.topk = cfg.topk
        m.renormalize = cfg.renormalize
        m.scoring_func = cfg.score_func
        m.routed_scaling_factor = 1.5
        m.n_routed_experts = cfg.n_experts
        m.layer_idx = 0
        m.gate = types.SimpleNamespace(weight=torch.from_numpy(gw), e_score_correction_bias=torch.from_numpy(bias),
                                       tid2eid=None)
        w, i = m._route(from_f32_bf16(x), None)
        out[f"t{T}_sha"] = np.frombuffer(bytes.fromhex(_sha(gw, bias, x)), dtype=np.uint8)
        out[f"t{T}_w"] = w.numpy().copy()
        out[f"t{T}_idx"] = i.numpy().astype(np.int64)
    np.savez_compressed(os.path.join(HERE, "route_cfg1.npz"), **out)


def make_shared_cfg0(O, MN, S):
    """shared_cfg0.npz: the reference's shared expert (model_npu.Expert in
    "fp8" mode: weights from npu_ops.dequant_fp8_weight, as its loader sets
    them) on config-0 dims, and the dequant of the FP8 weights themselves.
    The FP8 bytes come from synthetic.make_shared_expert (SHA-256 stored)."""
    cfg = S.CFG0
    sh = S.make_shared_expert(cfg, 0, 3)
    x = S.make_tokens(cfg, 5, 16)
    ex = MN.Expert(cfg.hidden, cfg.inter, mode="fp8", swiglu_limit=cfg.swiglu_limit)
    for w in ("w1", "w2", "w3"):
        deq = O.dequant_fp8_weight(torch.from_numpy(sh[w]).view(torch.float8_e4m3fn),
                                   torch.from_numpy(sh[w + "s"]).view(torch.float8_e8m0fnu), 128, torch.bfloat16)
        getattr(ex, w).weight.data.copy_(deq)
    with torch.no_grad():
        y = ex(from_f32_bf16(x))
    out = {"x": bf16_bits(from_f32_bf16(x)), "y": bf16_bits(y),
           "sha": np.frombuffer(bytes.fromhex(_sha(*[sh[k] for k in sorted(sh)])), dtype=np.uint8)}
    for w in ("w1", "w2"):
        deq = O.dequant_fp8_weight(torch.from_numpy(sh[w]).view(torch.float8_e4m3fn),
                                   torch.from_numpy(sh[w + "s"]).view(torch.float8_e8m0fnu), 128, torch.bfloat16)
        out[f"deq_{w}"] = bf16_bits(deq)
    np.savez_compressed(os.path.join(HERE, "shared_cfg0.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    ap.add_argument("--only", choices=["route_cfg1", "shared_cfg0"], default=None,
                    help="write only this fixture (the others stay as they are)")
    args = ap.parse_args()
    os.environ["DSV4_PIN_HOST"] = "0"
    sys.path.insert(0, args.ref)
    install_stubs()
    torch.utils.rename_privateuse1_backend("npu")
    import npu_ops as O  # noqa: E402
    import offload  # noqa: E402
    import model_npu as MN  # noqa: E402
    MN.DEVICE = torch.device("cpu")
    import dsv4_plugin.models.deepseek_v4 as DV4  # noqa: E402
    import dsv4_plugin.core.engine as ENG  # noqa: E402
    S = _load_synthetic()
    torch.set_num_threads(8)
    if args.only == "route_cfg1":
        make_route_cfg1(DV4, S)
        print("wrote route_cfg1.npz to", HERE)
        return
    if args.only == "shared_cfg0":
        make_shared_cfg0(O, MN, S)
        print("wrote shared_cfg0.npz to", HERE)
        return

    # ---------------------------------------------------------------- ops
    rng = np.random.default_rng(20240601)
    ops = {}
    for tag, (n, kh, lo, hi) in {"a": (8, 64, 118, 131), "b": (16, 256, 100, 150),
                                  "c": (4, 512, 0, 255)}.items():
        wp = rng.integers(0, 256, (n, kh), dtype=np.uint8)
        ws = rng.integers(lo, hi, (n, kh * 2 // 32), dtype=np.uint8)
        out = O.dequant_fp4_weight(torch.from_numpy(wp).view(torch.int8),
                                   torch.from_numpy(ws).view(torch.float8_e8m0fnu), torch.bfloat16)
        ops[f"deq_{tag}_wp"], ops[f"deq_{tag}_ws"], ops[f"deq_{tag}_out"] = wp, ws, bf16_bits(out)
        outf = O.dequant_fp4_weight(torch.from_numpy(wp).view(torch.int8),
                                    torch.from_numpy(ws).view(torch.float8_e8m0fnu), torch.float32)
        ops[f"deq_{tag}_out_f32"] = outf.numpy().copy()

    # act_quant in place (the plugin's call form, deepseek_v4.py:170)
    g = torch.Generator().manual_seed(7)
    rows = []
    base = torch.randn(64, 512, generator=g)
    for mul in (1.0, 3.0, 1e-3, 1e3, 1e-6, 200.0):
        rows.append(base[:8] * mul)
    special = torch.zeros(8, 512)
    special[1] = 448.0
    special[2, ::3] = -448.0 * 4
    special[3] = torch.arange(512) * 1e-3
    special[4] = 2.0 ** torch.arange(-20, 20).repeat(13)[:512].float()
    special[5, 7] = 1e-5
    special[6] = -special[4]
    special[7] = torch.linspace(-1000, 1000, 512)
    rows.append(special)
    xa = torch.cat(rows, 0).to(torch.bfloat16)
    ya = O.act_quant(xa.clone(), 128, "ue8m0", None, True)
    ops["aq_x"], ops["aq_y"] = bf16_bits(xa), bf16_bits(ya)

    # every finite bf16 value, shuffled into 128-blocks, through act_quant
    allv = (np.arange(0, 0x10000, dtype=np.uint32) << 16).view(np.float32)
    allv = allv[np.isfinite(allv)]
    allv = np.random.default_rng(0).permutation(allv)
    allv = allv[: (allv.size // 128) * 128].reshape(-1, 128)
    xall = torch.from_numpy(allv.copy()).to(torch.bfloat16)
    ops["aq_all_x"] = bf16_bits(xall)
    ops["aq_all_y"] = bf16_bits(O.act_quant(xall.clone(), 128, "ue8m0", None, True))

    # exhaustive: pow2 scale exponent for every positive finite bf16 amax
    pats = np.arange(1, 0x7F80, dtype=np.uint16)
    amax = torch.from_numpy((pats.astype(np.uint32) << 16).view(np.float32))
    s = O._fast_pow2_scale(amax.clamp(min=1e-4), 1.0 / O.FP8_MAX)
    ops["scale_pats"] = pats
    ops["scale_exp"] = torch.log2(s).round().to(torch.int32).numpy()

    # exhaustive e4m3 cast of every bf16 value in [-448, 448]
    allb = np.arange(0, 0x10000, dtype=np.uint32).astype(np.uint16)
    vals = (allb.astype(np.uint32) << 16).view(np.float32)
    keep = np.isfinite(vals) & (np.abs(vals) <= 448.0)
    v = torch.from_numpy(vals[keep].copy())
    ops["e4m3_in"] = allb[keep]
    ops["e4m3_out"] = v.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()

    # _round_fp4 on the reference test's grid plus every half point
    grid = torch.cat([torch.arange(-6.0, 6.001, 0.01), torch.arange(-6.0, 6.01, 0.25),
                      torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -2.5, -5.0])])
    ops["r4_in"] = grid.numpy().astype(np.float32)
    ops["r4_out"] = O._round_fp4(grid).numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **ops)

    # ------------------------------------------------------------- layer
    layer = {}
    cfg = S.CFG0
    seed = 0
    experts = [S.make_expert(cfg, seed, e) for e in range(cfg.n_experts)]
    gate_w, _ = S.make_gate(cfg, seed)
    x = S.make_tokens(cfg, seed, 16)
    layer["inputs_sha"] = np.frombuffer(
        bytes.fromhex(_sha(gate_w, x, *[experts[e][k] for e in range(cfg.n_experts)
                                         for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")])),
        dtype=np.uint8)
    layer["x"] = S.to_bf16_bits(x)
    layer["gate_w"] = gate_w

    margs = MN.ModelArgs(dim=cfg.hidden, moe_inter_dim=cfg.inter, n_routed_experts=cfg.n_experts,
                         n_activated_experts=cfg.topk, score_func="softmax", route_scale=1.5,
                         swiglu_limit=10.0, n_hash_layers=0, vocab_size=1000)
    bank = offload.ExpertBank(capacity=cfg.n_experts, device="cpu", pin=False)
    for e, ex in enumerate(experts):
        bank.register(0, e, *[torch.from_numpy(ex[k]) for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")])
    moe = MN.MoE(0, margs, bank=bank)

    class _Zero(nn.Module):
        def forward(self, x, weights=None):
            return torch.zeros_like(x)

    moe.shared_experts = _Zero()
    moe.gate.weight.data.copy_(torch.from_numpy(gate_w))
    moe.gate.bias.data.zero_()
    xt = from_f32_bf16(x)
    ids = torch.zeros(16, dtype=torch.long)
    wb, ib = moe.gate(xt, ids)
    yb = moe(xt, ids)
    layer["oracle_w"] = wb.numpy().copy()
    layer["oracle_idx"] = ib.numpy().astype(np.int64)
    layer["oracle_y"] = bf16_bits(yb)

    def make_plugin(gw, bias, score, renorm, topk, n_exp, tid2eid=None):
        m = DV4.OffloadDeepseekV4MoE.__new__(DV4.OffloadDeepseekV4MoE)
        nn.Module.__init__(m)
        m.hash = tid2eid is not None
        m.topk = topk
        m.renormalize = renorm
        m.scoring_func = score
        m.routed_scaling_factor = 1.5
        m.swiglu_limit = 10.0
        m.n_routed_experts = n_exp
        m.is_sequence_parallel = False
        m.shared_experts = None
        m.layer_idx = 0
        m.engine = types.SimpleNamespace(get=bank.get, get_packed=bank.get_packed)
        m.gate = types.SimpleNamespace(weight=torch.from_numpy(gw),
                                       e_score_correction_bias=None if bias is None else torch.from_numpy(bias),
                                       tid2eid=None if tid2eid is None else torch.from_numpy(tid2eid))
        return m

    # plugin, softmax without renormalisation == oracle semantics
    p = make_plugin(gate_w, np.zeros(cfg.n_experts, np.float32), "softmax", False, cfg.topk, cfg.n_experts)
    wp_, ip_ = p._route(xt, None)
    layer["plugin_softmax_w"] = wp_.numpy().copy()
    layer["plugin_softmax_idx"] = ip_.numpy().astype(np.int64)
    layer["plugin_bf16_y"] = bf16_bits(p._routed(xt, None))
    DV4._MXFP4_GMM = True
    try:
        layer["plugin_a4w4_y"] = bf16_bits(p._routed(xt, None))
    finally:
        DV4._MXFP4_GMM = False

    # plugin, sqrtsoftplus + bias + renormalise (the DeepSeek-V4 router)
    brng = np.random.default_rng(11)
    bias = (brng.standard_normal(cfg.n_experts) * 0.1).astype(np.float32)
    gw2 = S.bf16_exact(brng.standard_normal((cfg.n_experts, cfg.hidden)).astype(np.float32) / np.float32(32.0))
    p2 = make_plugin(gw2, bias, "sqrtsoftplus", True, cfg.topk, cfg.n_experts)
    w2_, i2_ = p2._route(xt, None)
    layer["sq_gate_w"], layer["sq_bias"] = gw2, bias
    layer["sq_w"], layer["sq_idx"] = w2_.numpy().copy(), i2_.numpy().astype(np.int64)
    layer["sq_y"] = bf16_bits(p2._routed(xt, None))
    # sigmoid scoring
    p3 = make_plugin(gw2, bias, "sigmoid", True, cfg.topk, cfg.n_experts)
    w3_, i3_ = p3._route(xt, None)
    layer["sig_w"], layer["sig_idx"] = w3_.numpy().copy(), i3_.numpy().astype(np.int64)

    # hash routing (deepseek_v4.py:133-138)
    tid = brng.integers(0, cfg.n_experts, (1000, cfg.topk)).astype(np.int32)
    in_ids = brng.integers(0, 1000, (16,)).astype(np.int64)
    p4 = make_plugin(gw2, None, "sqrtsoftplus", True, cfg.topk, cfg.n_experts, tid2eid=tid)
    w4_, i4_ = p4._route(xt, torch.from_numpy(in_ids))
    layer["hash_tid2eid"], layer["hash_ids"] = tid, in_ids
    layer["hash_w"], layer["hash_idx"] = w4_.numpy().copy(), i4_.numpy().astype(np.int64)
    layer["hash_y"] = bf16_bits(p4._routed(xt, torch.from_numpy(in_ids)))
    try:
        p4._route(xt, None)
        layer["hash_missing_ids_raises"] = np.array([0])
    except RuntimeError:
        layer["hash_missing_ids_raises"] = np.array([1])
    np.savez_compressed(os.path.join(HERE, "layer_cfg0.npz"), **layer)

    # ------------------------------------------------------------- bank LRU
    lru = {}

    def small(seed_):
        gg = torch.Generator().manual_seed(seed_)
        return tuple(torch.randint(lo, hi, shp, dtype=torch.uint8, generator=gg)
                     for (lo, hi, shp) in ((0, 256, (64, 32)), (100, 150, (64, 2)), (0, 256, (64, 32)),
                                           (100, 150, (64, 2)), (0, 256, (64, 32)), (100, 150, (64, 2))))

    # the reference's own LRU scenario (test_offload.py:67-79)
    b = offload.ExpertBank(capacity=4, device="cpu", pin=False)
    for e in range(5):
        b.register(0, e, *small(100 + e))
    for e in range(3):
        b.register(1, e, *small(200 + e))
    for e in range(4):
        b.get(0, e)
    b.get(0, 0)
    b.get(1, 0)
    st = b.stats()
    lru["s1_keys"] = np.array(list(b._cache.keys()), dtype=np.int64)
    lru["s1_stats"] = np.array([st["hits"], st["misses"], st["evictions"]], dtype=np.int64)
    # a long random trace, bf16 and packed caches
    b2 = offload.ExpertBank(capacity=7, device="cpu", pin=False)
    os.environ.pop("DSV4_PACKED_SLOTS", None)
    for L in range(2):
        for e in range(10):
            b2.register(L, e, *small(300 + 10 * L + e))
    tr = np.random.default_rng(5)
    trace = np.stack([tr.integers(0, 2, 300), np.minimum(tr.zipf(1.3, 300) - 1, 9)], axis=1)
    for L, e in trace:
        b2.get(int(L), int(e))
    for L, e in trace[:150]:
        b2.get_packed(int(L), int(e))
    st2 = b2.stats()
    lru["s2_trace"] = trace.astype(np.int64)
    lru["s2_keys"] = np.array(list(b2._cache.keys()), dtype=np.int64)
    lru["s2_pkeys"] = np.array(list(b2._packed_cache.keys()), dtype=np.int64)
    lru["s2_stats"] = np.array([st2["hits"], st2["misses"], st2["evictions"], st2["packed_hits"],
                                st2["packed_misses"], st2["packed_capacity"]], dtype=np.int64)
    b0 = offload.ExpertBank(capacity=0, device="cpu", pin=False)
    b0.register(0, 0, *small(7))
    b0.get(0, 0)
    b0.get(0, 0)
    lru["s0_stats"] = np.array([len(b0._cache), b0.stats()["misses"]], dtype=np.int64)
    d = b.get(1, 0)
    lru["get_w1"] = bf16_bits(d["w1"])
    lru["get_w1_src"] = small(200)[0].numpy()
    lru["get_w1s_src"] = small(200)[1].numpy()
    np.savez_compressed(os.path.join(HERE, "bank_lru.npz"), **lru)

    # ------------------------------------------------------------- engine
    names = []
    for L in (0, 3, 42):
        for e in (0, 7, 255):
            for w in ("w1", "w2", "w3"):
                for kind in ("weight", "scale"):
                    names.append(f"layers.{L}.ffn.experts.{e}.{w}.{kind}")
                    names.append(f"model.layers.{L}.ffn.experts.{e}.{w}.{kind}")
    names += ["mtp.0.ffn.experts.7.w1.weight", "mtp.0.ffn.experts.7.w2.scale",
              "layers.3.ffn.gate.weight", "layers.3.ffn.gate.bias", "layers.3.ffn.shared_experts.w1.weight",
              "layers.3.attn.wq_a.weight", "layers.3.ffn.experts.5.w4.weight", "embed.weight",
              "layers.10.ffn.experts.12.w3.scale_inv", "xlayers.1.ffn.experts.2.w1.weight"]
    parsed = []
    for n in names:
        r = ENG.parse_expert_name(n)
        parsed.append((-9, -9, -9, -9) if r is None else (r[0], r[1], int(r[2][1]), 0 if r[3] == "weight" else 1))
    eng = {"names": np.array(names), "parsed": np.array(parsed, dtype=np.int64),
           "is_main": np.array([ENG.is_expert_weight(n) for n in names]),
           "is_any": np.array([ENG.is_expert_weight(n, include_mtp=True) for n in names])}
    np.savez_compressed(os.path.join(HERE, "engine_names.npz"), **eng)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
