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
