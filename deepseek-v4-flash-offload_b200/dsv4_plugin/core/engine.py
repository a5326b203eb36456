"""Expert offload engine: weight-stream capture + the shared expert bank.

Same surface as the reference's ``dsv4_plugin.core.engine``
(engine.py:22-116): ``parse_expert_name``, ``is_expert_weight``,
``ExpertOffloadEngine(slot_capacity, device)`` with ``capture / get /
get_packed / stats`` and the process-wide ``get_engine()``.  The checkpoint
key format is the model's own and therefore identical:
``[model.]layers.N.ffn.experts.M.w{1,2,3}.{weight,scale}`` (main layers) and
``mtp.N.ffn.experts.M...`` (speculative-decoding draft layers, mapped to
layer ``-1 - N`` and not consumed by default).

In addition the engine owns the per-device routed-expert plans
(``plan_for``) so every decoder layer shares one slot arena and workspace.
"""

from __future__ import annotations

import os
import re
import weakref

import torch

from dsv4_plugin.core.bank import ExpertBank

_NAME = re.compile(r"(?:^|\.)(?:layers\.(?P<layer>\d+)|mtp\.(?P<mtp>\d+))\.ffn\.experts\.(?P<eid>\d+)"
                   r"\.(?P<w>w[123])\.(?P<kind>weight|scale)$")
_KIND = {"weight": "p", "scale": "s"}
_SHARED = re.compile(r"(?:^|\.)layers\.(?P<layer>\d+)\.ffn\.shared_experts\.(?P<w>w[123])\.(?P<kind>weight|scale)$")


def parse_expert_name(name: str):
    """-> (layer, eid, "w1"|"w2"|"w3", "weight"|"scale") or None."""
    m = _NAME.search(name)
    if m is None:
        return None
    layer = int(m["layer"]) if m["layer"] is not None else -1 - int(m["mtp"])
    return layer, int(m["eid"]), m["w"], m["kind"]


def parse_shared_name(name: str):
    """``[model.]layers.N.ffn.shared_experts.w{1,2,3}.{weight,scale}`` ->
    (layer, "w1"|"w2"|"w3", "weight"|"scale") or None."""
    m = _SHARED.search(name)
    return None if m is None else (int(m["layer"]), m["w"], m["kind"])


def is_shared_expert_weight(name: str) -> bool:
    return parse_shared_name(name) is not None


def is_expert_weight(name: str, include_mtp: bool = False) -> bool:
    """True for routed-expert tensors of the main layers (and of the MTP draft
    layers when ``include_mtp``)."""
    p = parse_expert_name(name)
    return p is not None and (include_mtp or p[0] >= 0)


class ExpertOffloadEngine:
    """Host pool of packed experts + device slot cache, per (layer, eid)."""

    def __init__(self, slot_capacity: int, device="cuda", dtype=torch.bfloat16, packed_capacity=None):
        self.bank = ExpertBank(capacity=slot_capacity, device=device, dtype=dtype, packed_capacity=packed_capacity)
        self._pending = {}
        self.captured = 0
        self._plans = {}
        self._layers = {}
        # DSV4_PREFETCH=0: no next-layer prefetch on the side stream
        self.prefetch = os.environ.get("DSV4_PREFETCH", "1") != "0"
        # the shared experts, fused into the routed launches: layer -> device FP8 slot
        self.shared = {}
        self._shared_pending = {}

    def capture(self, name: str, tensor: torch.Tensor) -> bool:
        """Park one expert tensor; register the expert once all six arrived."""
        parsed = parse_expert_name(name)
        if parsed is None:
            return False
        layer, eid, w, kind = parsed
        slots = self._pending.setdefault((layer, eid), {})
        slots[w + _KIND[kind]] = tensor.detach().to("cpu")
        if len(slots) >= 6:
            self.bank.register(layer, eid, *[slots[k] for k in ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")])
            del self._pending[(layer, eid)]
            self.captured += 1
        return True

    def register_layer(self, layer: int, module) -> None:
        """MoE layers register here so that a layer can warm the next one."""
        self._layers[int(layer)] = weakref.ref(module)

    def layer(self, layer: int):
        r = self._layers.get(int(layer))
        return r() if r is not None else None

    def capture_shared(self, name: str, tensor: torch.Tensor) -> bool:
        """Park one shared-expert tensor (E4M3 weight or E8M0 block scale);
        once all six of a layer arrived, pack them into the layer's FP8 slot
        on the device."""
        parsed = parse_shared_name(name)
        if parsed is None:
            return False
        layer, w, kind = parsed
        parts = self._shared_pending.setdefault(layer, {})
        parts[w + ("" if kind == "weight" else "s")] = tensor.detach().to("cpu")
        if len(parts) >= 6:
            self.register_shared(layer, *[parts[k] for k in ("w1", "w1s", "w2", "w2s", "w3", "w3s")])
            del self._shared_pending[layer]
        return True

    def register_shared(self, layer: int, w1, s1, w2, s2, w3, s3) -> torch.Tensor:
        """Pack a layer's shared expert (w1 / w3 [I, H], w2 [H, I] E4M3; block
        scales E8M0) into its FP8 slot and keep it on the device."""
        from dsv4_plugin import ops
        inter, hidden = w1.shape
        slot = ops.pack_shared_expert(w1, s1, w2, s2, w3, s3, hidden, inter)
        dev = self.bank.device
        self.shared[int(layer)] = slot.to(dev) if dev.type == "cuda" else slot
        return self.shared[int(layer)]

    def shared_slot(self, layer: int):
        return self.shared.get(int(layer))

    def get(self, layer: int, eid: int):
        return self.bank.get(layer, eid)

    def get_packed(self, layer: int, eid: int):
        return self.bank.get_packed(layer, eid)

    def plan_for(self, n_experts: int, topk: int, n_tokens: int, swiglu_limit: float, with_shared: bool = False):
        """Routed-expert plan able to take ``n_tokens`` tokens, shared by the
        layers (with the shared expert fused in when ``with_shared``)."""
        from dsv4_plugin.ops import MoEPlan
        key = (n_experts, topk, float(swiglu_limit), bool(with_shared))
        plan = self._plans.get(key)
        if plan is None or plan.max_tokens < n_tokens:
            cap = 1 << max(6, (max(n_tokens, 1) - 1).bit_length())
            plan = MoEPlan(self.bank.hidden, self.bank.inter, n_experts, topk, cap, swiglu_limit, self.bank.arena,
                           with_shared=with_shared)
            self._plans[key] = plan
        return plan

    def resize_slots(self, packed_capacity: int):
        """New HBM budget of packed slots; plans bound to the old arena are dropped."""
        self.bank.resize_slots(packed_capacity)
        self._plans.clear()

    def stats(self):
        s = self.bank.stats()
        s["captured"] = self.captured
        s["parked"] = len(self._pending)
        return s

    def __repr__(self):
        return f"ExpertOffloadEngine({self.bank!r}, captured={self.captured})"


_ENGINE: ExpertOffloadEngine | None = None


def get_engine(slot_capacity: int | None = None, device=None) -> ExpertOffloadEngine:
    """Process-wide engine; ``slot_capacity`` only applies on first call
    (env ``DSV4_EXPERT_SLOTS``, default 512 bf16-equivalent slots)."""
    global _ENGINE
    if _ENGINE is None:
        if slot_capacity is None:
            slot_capacity = int(os.environ.get("DSV4_EXPERT_SLOTS", "512"))
        if device is None:
            device = f"cuda:{torch.cuda.current_device()}" if torch.cuda.is_available() else "cpu"
        _ENGINE = ExpertOffloadEngine(slot_capacity=slot_capacity, device=device)
    return _ENGINE


def reset_engine(engine: ExpertOffloadEngine | None = None):
    """Replace (or drop) the process-wide engine; used by tests and benches."""
    global _ENGINE
    _ENGINE = engine
