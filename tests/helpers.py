"""Shared helpers of the parity tests: synthetic layers on the GPU, oracle runs."""

from __future__ import annotations

import numpy as np
import torch

from dsv4_plugin import synthetic as S
from oracle import moe_oracle as O


def bf16_tensor(a: np.ndarray, device="cuda") -> torch.Tensor:
    bits = S.to_bf16_bits(a).astype(np.int16)
    return torch.from_numpy(bits).view(torch.bfloat16).to(device)


def bf16_to_np(t: torch.Tensor) -> np.ndarray:
    bits = t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
    return O.bf16_from_bits(bits)


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


class SyntheticLayer:
    """Experts of one synthetic layer packed into a device slot arena
    (slot e holds expert e)."""

    def __init__(self, cfg: S.MoEConfig, seed: int = 0, layer: int = 0, n_experts: int | None = None,
                 device="cuda"):
        from dsv4_plugin import ops
        self.cfg = cfg
        self.n = n_experts or cfg.n_experts
        self.experts = [S.make_expert(cfg, seed, e, layer) for e in range(self.n)]
        self.gate_w, self.bias = S.make_gate(cfg, seed, layer)
        nb = ops.expert_slot_bytes(cfg.hidden, cfg.inter)
        host = torch.empty((self.n, nb), dtype=torch.uint8)
        for e, ex in enumerate(self.experts):
            ops.pack_expert(*[torch.from_numpy(ex[k]) for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")],
                            cfg.hidden, cfg.inter, out=host[e])
        self.arena = host.to(device)
        self.slot_of = torch.arange(self.n, dtype=torch.int32, device=device)
        # dequantised experts are cached only for the small configuration
        self.deq_cache = {} if cfg.hidden * cfg.inter <= 1024 * 512 else None

    def oracle(self, x: np.ndarray, weights: np.ndarray, idx: np.ndarray, profile="bf16") -> np.ndarray:
        return O.moe_routed(x, weights, idx, self.experts, self.n, self.cfg.swiglu_limit, profile,
                            deq_cache=self.deq_cache)


def make_plugin_layer(cfg: S.MoEConfig, experts: dict, device, layer_idx: int = 3, seed: int = 0,
                      slots: int | None = None, shared: dict | None = None):
    """OffloadDeepseekV4MoE for a synthetic layer built through the plugin's
    public API, with ``experts`` {eid: six tensors} registered in a fresh
    engine (which becomes the process-wide one), and with ``shared`` (the
    FP8 shared expert of synthetic.make_shared_expert) fused in."""
    import types

    from dsv4_plugin.core import engine as ENG
    from dsv4_plugin.models import deepseek_v4 as DV4

    n = slots or len(experts)
    eng = ENG.ExpertOffloadEngine(slot_capacity=n, device=device, packed_capacity=n)
    for e, ex in experts.items():
        eng.bank.register(layer_idx, e, *[torch.from_numpy(ex[k]) for k in
                                          ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")])
    if shared is not None:
        eng.register_shared(layer_idx, *[torch.from_numpy(shared[k]) for k in ("w1", "w1s", "w2", "w2s", "w3", "w3s")])
    ENG.reset_engine(eng)
    hf = types.SimpleNamespace(
        n_routed_experts=cfg.n_experts, n_shared_experts=1 if shared is not None else None,
        num_experts_per_tok=cfg.topk,
        norm_topk_prob=cfg.renormalize, scoring_func=cfg.score_func, routed_scaling_factor=cfg.route_scale,
        swiglu_limit=cfg.swiglu_limit, num_hash_layers=0, vocab_size=1000, hidden_size=cfg.hidden,
        moe_intermediate_size=cfg.inter, hidden_act="silu")
    pc = types.SimpleNamespace(use_sequence_parallel_moe=False, eplb_config=None, enable_eplb=False)
    moe = DV4.OffloadDeepseekV4MoE(hf, pc, prefix=f"model.layers.{layer_idx}.mlp").to(device)
    gw, bias = S.make_gate(cfg, seed, layer_idx)
    moe.gate.weight.data.copy_(torch.from_numpy(gw))
    if bias is not None:
        moe.gate.e_score_correction_bias.data.copy_(torch.from_numpy(bias))
    else:
        moe.gate.e_score_correction_bias.data.zero_()
    return moe, eng
