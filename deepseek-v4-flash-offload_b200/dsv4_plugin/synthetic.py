"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (there is no checkpoint or dataset on the box).

Everything is numpy and deterministic in (seed, expert id), so a test, the
oracle and the bench can regenerate any subset of experts independently.

Configurations (H hidden, I expert intermediate, E experts, k top-k):
  * ``cfg0``: H=1024, I=512,  E=16,  k=4, softmax router, gate ~N(0,0.02)
  * ``cfg1``: H=4096, I=2048, E=256, k=8, sqrtsoftplus router with
    renormalisation, logits ~N(0,1) and a Zipf(s=1.1)-shaped per-expert
    selection bias (the ``e_score_correction_bias`` of the real model) so the
    load is skewed.
Expert weights: E2M1 codes uniform over the 16 nibble values (bytes uniform
0..255), E8M0 scale bytes uniform in [118, 130].
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int
    inter: int
    n_experts: int
    topk: int
    score_func: str
    renormalize: bool
    route_scale: float = 1.5
    swiglu_limit: float = 10.0
    gate_std: float | None = None      # None: 1/sqrt(hidden) (logits ~N(0,1))
    zipf_s: float | None = None         # None: no selection bias
    zipf_bias_scale: float = 0.3

    def packed_expert_bytes(self) -> int:
        h, i = self.hidden, self.inter
        return 3 * i * h // 2 + 3 * i * h // 32


CFG0 = MoEConfig("cfg0", 1024, 512, 16, 4, "softmax", False, gate_std=0.02)
CFG1 = MoEConfig("cfg1", 4096, 2048, 256, 8, "sqrtsoftplus", True, zipf_s=1.1, zipf_bias_scale=0.3)
CONFIGS = {"cfg0": CFG0, "cfg1": CFG1}


def _rng(*key: int) -> np.random.Generator:
    return np.random.default_rng(list(key))


def make_expert(cfg: MoEConfig, seed: int, eid: int, layer: int = 0) -> dict:
    """Six packed tensors of one expert in the checkpoint layout
    (``layers.N.ffn.experts.M.w{1,2,3}.{weight,scale}``):
    w1/w3 [I, H/2] + [I, H/32], w2 [H, I/2] + [H, I/32], all uint8."""
    h, i = cfg.hidden, cfg.inter
    g = _rng(seed, 1000 + layer, eid)
    out = {}
    for w, (n, k) in (("w1", (i, h)), ("w2", (h, i)), ("w3", (i, h))):
        out[w + "p"] = g.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
        out[w + "s"] = g.integers(118, 131, size=(n, k // 32), dtype=np.uint8)
    return out


def make_shared_expert(cfg: MoEConfig, seed: int, layer: int = 0) -> dict:
    """The shared expert of a layer in the checkpoint's FP8 form: w1 / w3
    [I, H] and w2 [H, I] E4M3 bytes (sign random, exponent field 0..8 and
    any mantissa: |v| <= 3.75, no NaN codes) with one E8M0 scale byte per
    128 x 128 block, uniform in [118, 126] (``w1s`` [ceil(I/128),
    ceil(H/128)] ...).  The shared intermediate size is ``inter`` (one
    shared expert)."""
    h, i = cfg.hidden, cfg.inter
    g = _rng(seed, 4000 + layer)
    out = {}
    for w, (n, k) in (("w1", (i, h)), ("w2", (h, i)), ("w3", (i, h))):
        sign = g.integers(0, 2, size=(n, k), dtype=np.uint8) << 7
        expo = g.integers(0, 9, size=(n, k), dtype=np.uint8) << 3
        mant = g.integers(0, 8, size=(n, k), dtype=np.uint8)
        out[w] = (sign | expo | mant).astype(np.uint8)
        out[w + "s"] = g.integers(118, 127, size=((n + 127) // 128, (k + 127) // 128), dtype=np.uint8)
    return out


def bf16_exact(a: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (RNE) and return float32 holding the bf16 value."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def make_gate(cfg: MoEConfig, seed: int, layer: int = 0):
    """Gate weight [E, H] float32 (bf16-exact values, as the fp32 upcast of a
    bf16 checkpoint tensor) and the selection bias [E] float32 or None."""
    g = _rng(seed, 2000 + layer)
    std = cfg.gate_std if cfg.gate_std is not None else 1.0 / np.sqrt(cfg.hidden)
    w = bf16_exact(g.standard_normal((cfg.n_experts, cfg.hidden), dtype=np.float32) * np.float32(std))
    bias = None
    if cfg.zipf_s is not None:
        rank = g.permutation(cfg.n_experts) + 1
        bias = (-cfg.zipf_bias_scale * cfg.zipf_s * np.log(rank)).astype(np.float32)
    return w, bias


def make_tokens(cfg: MoEConfig, seed: int, n_tokens: int, step: int = 0,
                std: float = 1.0) -> np.ndarray:
    """Hidden states [T, H] as bf16-exact float32, ~N(0, std)."""
    g = _rng(seed, 3000 + step, n_tokens)
    return bf16_exact(g.standard_normal((n_tokens, cfg.hidden), dtype=np.float32) * np.float32(std))


def to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """bf16-exact float32 -> uint16 bit patterns (for torch.bfloat16 views)."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
