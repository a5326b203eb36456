"""Takeover of DeepSeek-V4's MoE layer: routed experts on the B200 kernels.

Same surface as the reference plugin (dsv4_plugin/models/deepseek_v4.py):
  * ``OffloadDeepseekV4MoE(config, parallel_config, quant_config=None,
    prefix="", is_draft_layer=False)`` with ``_route``, ``_routed`` and
    ``forward(hidden_states, input_ids=None)``;
  * ``_offload_load_weights(self, weights)``: tee of the weight stream,
    routed experts into the host pool, everything else to the original;
  * ``install_patches()``: idempotent swap of ``DeepseekV4MoE`` and
    ``load_weights`` in the target vLLM module;
  * module flag ``_MXFP4_GMM`` (env ``DSV4_MXFP4_GMM=1``) selects the a4w4
    profile, else bf16;
  * the shared expert: its FP8 weights are teed into the engine at load and
    ``forward`` runs it inside the routed launches (``DSV4_FUSED_SHARED=0``
    keeps the vLLM dense MLP added afterwards, as the reference does).
The patch target is the first importable module of ``DSV4_PATCH_MODULE``
(comma separated; default: vLLM's CUDA DeepSeek-V4 model module, then the
vllm-ascend one the reference patches).

Routing runs ``ops.route_topk``; the experts run ``ops.MoEPlan.forward``
over the engine's slot arena.  There is no CPU path: a CPU tensor raises.
"""

from __future__ import annotations

import importlib
import os

import torch
from torch import nn

from dsv4_plugin import ops
from dsv4_plugin.core.engine import get_engine, is_expert_weight, is_shared_expert_weight

_PATCHED = False
_MXFP4_GMM = os.environ.get("DSV4_MXFP4_GMM", "0") == "1"
# DSV4_FUSED_SHARED=0: the shared expert stays the vLLM dense MLP added after
# the routed output (the reference's structure); by default its FP8 weights
# are captured at load and it runs inside the routed launches
_FUSED_SHARED = os.environ.get("DSV4_FUSED_SHARED", "1") != "0"
# decode batches route in one launch in the layer plan's workspace
# (DSV4_PLAN_ROUTE=0: the two-kernel router with its own workspace)
_PLAN_ROUTE = os.environ.get("DSV4_PLAN_ROUTE", "0") != "0"
DEFAULT_TARGETS = ("vllm.model_executor.models.deepseek_v4", "vllm_ascend.models.deepseek_v4")


def _targets():
    env = os.environ.get("DSV4_PATCH_MODULE")
    return tuple(t.strip() for t in env.split(",") if t.strip()) if env else DEFAULT_TARGETS


def target_module():
    """The vLLM module whose ``DeepseekV4MoE`` this plugin replaces, or None."""
    for name in _targets():
        try:
            return importlib.import_module(name)
        except ImportError:
            continue
    return None


class _ExpertsFacade:
    """Stand-in for FusedMoE: satisfies code that reads ``moe.experts``."""

    is_internal_router = False

    def __init__(self, moe):
        self._moe = moe

    def update_expert_map(self):
        pass


class _Gate(nn.Module):
    """Router parameters under the checkpoint names ``gate.weight`` (fp32
    [E, H]), ``gate.e_score_correction_bias`` / ``gate.tid2eid``."""

    def __init__(self, hidden: int, n_experts: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(n_experts, hidden, dtype=torch.float32), requires_grad=False)
        self.e_score_correction_bias = None
        self.tid2eid = None


class OffloadDeepseekV4MoE(nn.Module):
    """DeepSeek-V4 MoE layer whose routed experts live in the expert bank."""

    def __init__(self, config, parallel_config, quant_config=None, prefix="", is_draft_layer=False):
        nn.Module.__init__(self)  # the vLLM parent would build FusedMoE with every expert on the device
        v4 = target_module()
        ws = getattr(v4, "get_tensor_model_parallel_world_size", None)
        rk = getattr(v4, "get_tensor_model_parallel_rank", None)
        self.tp_size = ws() if ws else 1
        self.tp_rank = rk() if rk else 0
        self.layer_idx = int(prefix.split(sep=".")[-2])
        self.routed_scaling_factor = getattr(config, "routed_scaling_factor", 1.5)
        self.swiglu_limit = getattr(config, "swiglu_limit", None)
        self.n_routed_experts = config.n_routed_experts
        self.n_shared_experts = config.n_shared_experts
        self.topk = config.num_experts_per_tok
        self.renormalize = config.norm_topk_prob
        self.num_expert_group = getattr(config, "n_group", 1)
        self.topk_group = getattr(config, "topk_group", 1)
        self.scoring_func = getattr(config, "scoring_func", "softmax")
        self.is_sequence_parallel = bool(getattr(parallel_config, "use_sequence_parallel_moe", False))

        self.gate = _Gate(config.hidden_size, config.n_routed_experts)

        eplb = getattr(parallel_config, "eplb_config", None)
        self.enable_eplb = bool(getattr(parallel_config, "enable_eplb", False))
        self.n_redundant_experts = getattr(eplb, "num_redundant_experts", 0) if eplb is not None else 0
        self.n_logical_experts = self.n_routed_experts
        self.n_physical_experts = self.n_logical_experts + self.n_redundant_experts
        self.ep_size = 1
        self.n_local_physical_experts = self.n_physical_experts
        self.physical_expert_start = 0
        self.physical_expert_end = self.n_local_physical_experts

        mlp = getattr(v4, "DeepseekV2MLP", None)
        if config.n_shared_experts is None or mlp is None:
            self.shared_experts = None
        else:
            self.shared_experts = mlp(
                hidden_size=config.hidden_size,
                intermediate_size=config.moe_intermediate_size * config.n_shared_experts,
                hidden_act=config.hidden_act, swiglu_limit=self.swiglu_limit, quant_config=quant_config,
                is_sequence_parallel=self.is_sequence_parallel, reduce_results=False,
                prefix=f"{prefix}.shared_experts")

        self.hash = self.layer_idx < getattr(config, "num_hash_layers", 0) and not is_draft_layer
        if self.hash:
            self.gate.tid2eid = nn.Parameter(
                torch.zeros(config.vocab_size, config.num_experts_per_tok, dtype=torch.int32), requires_grad=False)
        else:
            self.gate.e_score_correction_bias = nn.Parameter(
                torch.zeros(config.n_routed_experts, dtype=torch.float32), requires_grad=False)
        self.engine = get_engine()
        self.engine.register_layer(self.layer_idx, self)
        self.experts = _ExpertsFacade(self)

    # -- routing ------------------------------------------------------------
    def _route(self, hs: torch.Tensor, input_ids: torch.Tensor | None, out=None, workspace=None, plan=None):
        """(weights fp32 [T, k], indices int32 [T, k]); deepseek_v4.py:118-148.
        A decode batch (< 256 tokens) with the layer's plan routes in one
        launch in the plan's workspace (``MoEPlan.route``)."""
        tid2eid = getattr(self.gate, "tid2eid", None) if self.hash else None
        if self.hash and input_ids is None:
            raise RuntimeError("hash-layer routing needs input_ids (forward_context.input_ids is missing)")
        bias = None if self.hash else getattr(self.gate, "e_score_correction_bias", None)
        if plan is not None and out is None and hs.shape[0] < 256 and _PLAN_ROUTE:
            return plan.route(hs, self.gate.weight, bias, self.topk, self.scoring_func, self.renormalize,
                              self.routed_scaling_factor, tid2eid=tid2eid,
                              input_ids=input_ids if self.hash else None)
        return ops.route_topk(hs, self.gate.weight, bias, self.topk, self.scoring_func, self.renormalize,
                              self.routed_scaling_factor, tid2eid=tid2eid,
                              input_ids=input_ids if self.hash else None, out=out, workspace=workspace)

    # -- routed experts -------------------------------------------------------
    def _slot_table(self, indices: torch.Tensor):
        """(device expert -> slot table, slots to mark as read or None).

        Every expert of the layer resident (``preload_all``): the bank's static
        table.  Otherwise, with a page-locked pool: the device-side LRU
        (``ExpertBank.acquire``), no host synchronisation; once created it
        owns the arena.  Otherwise the host LRU, which needs the active
        experts on the host (one synchronisation per layer)."""
        bank = self.engine.bank
        if bank._dir is None:
            table = bank.resident_table(self.layer_idx, self.n_routed_experts)
            if table is not None:
                return table, None
        if bank.device_directory(self.n_routed_experts) is not None:
            return bank.acquire(self.layer_idx, indices), None
        active = torch.unique(indices).tolist()            # one host sync per layer
        slots = bank.ensure_resident(self.layer_idx, active)
        host = torch.full((self.n_routed_experts,), -1, dtype=torch.int32)
        host[torch.tensor(active, dtype=torch.long)] = torch.tensor(slots, dtype=torch.int32)
        return host.to(indices.device, non_blocking=True), slots

    def _prefetch_next(self, hs: torch.Tensor, input_ids):
        """Warm the next layer's predicted experts while this layer computes
        (the prefetch the reference's design notes plan, line 82, but do not
        implement): the next layer's gate applied to this layer's hidden
        states, or its hash table on the same token ids, on the bank's side
        stream."""
        bank = self.engine.bank
        nxt = self.engine.layer(self.layer_idx + 1) if self.engine.prefetch else None
        if nxt is None or bank._dir is None or (nxt.hash and input_ids is None):
            return
        t, k = hs.shape[0], nxt.topk
        # buffers allocated on this stream (graph-capture safe), used on the side stream
        pw = torch.empty((t, k), dtype=torch.float32, device=hs.device)
        pi = torch.empty((t, k), dtype=torch.int32, device=hs.device)
        ws = torch.empty(max(ops.route_workspace_bytes(t, hs.shape[1], nxt.n_routed_experts), 4),
                         dtype=torch.uint8, device=hs.device)
        side = bank.prefetch_stream()
        for x in (hs, pw, pi, ws):
            x.record_stream(side)
        bank.prefetch(self.layer_idx + 1, lambda: nxt._route(hs, input_ids, out=(pw, pi), workspace=ws)[1])

    def _routed_experts(self, hs, weights, indices, profile, input_ids=None, shared_slot=None):
        slot_of, slots = self._slot_table(indices)
        if slots is None and self.engine.bank._dir is not None:
            self._prefetch_next(hs, input_ids)
        plan = self.engine.plan_for(self.n_routed_experts, self.topk, hs.shape[0], self.swiglu_limit or 0.0,
                                    with_shared=shared_slot is not None)
        y = plan.forward(hs, weights, indices, slot_of, profile, shared_slot=shared_slot)
        if slots is not None and not torch.cuda.is_current_stream_capturing():
            self.engine.bank.mark_used(slots)
        return y

    def _plan(self, n_tokens: int, with_shared: bool = False):
        return self.engine.plan_for(self.n_routed_experts, self.topk, n_tokens, self.swiglu_limit or 0.0,
                                    with_shared=with_shared)

    def _routed(self, hs: torch.Tensor, input_ids: torch.Tensor | None = None) -> torch.Tensor:
        """Routed-expert output [T, H] bf16; profile from ``_MXFP4_GMM``."""
        weights, indices = self._route(hs, input_ids, plan=self._plan(hs.shape[0]))
        return self._routed_experts(hs, weights, indices, "a4w4" if _MXFP4_GMM else "bf16", input_ids)

    def _routed_mxfp4(self, hs: torch.Tensor, input_ids: torch.Tensor | None = None) -> torch.Tensor:
        weights, indices = self._route(hs, input_ids, plan=self._plan(hs.shape[0]))
        return self._routed_experts(hs, weights, indices, "a4w4", input_ids)

    def _shared_slot(self):
        """The layer's shared expert as an FP8 slot for the fused launches, or
        None (no shared expert, not captured, or DSV4_FUSED_SHARED=0)."""
        if not _FUSED_SHARED or self.n_shared_experts in (None, 0):
            return None
        return self.engine.shared_slot(self.layer_idx)

    def forward(self, hidden_states: torch.Tensor, input_ids=None) -> torch.Tensor:
        num_tokens, hidden_dim = hidden_states.shape
        hs = hidden_states.view(-1, hidden_dim)
        if self.hash and input_ids is None:
            from vllm.forward_context import get_forward_context
            input_ids = getattr(get_forward_context(), "input_ids", None)
        v4 = target_module() if self.is_sequence_parallel else None
        if self.is_sequence_parallel:
            hs = v4.sequence_parallel_chunk(hs)
            if input_ids is not None:
                input_ids = v4.sequence_parallel_chunk(input_ids)
        sh = self._shared_slot()
        if sh is not None:
            # routed experts + shared expert in one pass: the shared expert is
            # every token's last assignment, added in fp32 before the one bf16
            # rounding (model_npu.py:531-533)
            weights, indices = self._route(hs, input_ids, plan=self._plan(hs.shape[0], with_shared=True))
            out = self._routed_experts(hs, weights, indices, "a4w4" if _MXFP4_GMM else "bf16", input_ids,
                                       shared_slot=sh)
        else:
            out = self._routed(hs, input_ids)
            if self.shared_experts is not None:
                out = out + self.shared_experts(hs)
        if self.is_sequence_parallel:
            out = v4.tensor_model_parallel_all_gather(out, 0)[:num_tokens]
        return out.view(num_tokens, hidden_dim)


def _offload_load_weights(self, weights):
    """Weight-stream tee (deepseek_v4.py:272-288): main-layer routed experts
    go to the engine's host pool, everything else (MTP experts included) to
    the original ``load_weights``.  Shared-expert tensors are also copied into
    the engine (for the fused launches) and still passed on."""
    engine = get_engine()
    it = iter(weights)

    def filtered():
        for name, w in it:
            if is_expert_weight(name):
                engine.capture(name, w)
            else:
                if _FUSED_SHARED and is_shared_expert_weight(name):
                    engine.capture_shared(name, w)
                yield name, w

    return _ORIG_LOAD_WEIGHTS(self, filtered())


def _missing_load_weights(self, weights):
    raise RuntimeError("no original load_weights: the vLLM DeepSeek-V4 model module is not importable")


_ORIG_LOAD_WEIGHTS = _missing_load_weights


def install_patches():
    """Idempotently install the MoE class and the load_weights tee."""
    global _PATCHED, _ORIG_LOAD_WEIGHTS
    if _PATCHED:
        return
    v4 = target_module()
    if v4 is None:
        raise ImportError(f"none of the patch targets {_targets()} is importable")
    if not getattr(v4, "_DSV4_OFFLOAD_PATCHED", False):
        base = getattr(v4, "DeepseekV4MoE", None)
        if base is not None and base is not OffloadDeepseekV4MoE and not issubclass(OffloadDeepseekV4MoE, base):
            cls = type("OffloadDeepseekV4MoE", (OffloadDeepseekV4MoE, base), {})
        else:
            cls = OffloadDeepseekV4MoE
        v4.DeepseekV4MoE = cls
        model_cls = None
        for name in ("DeepseekV4ForCausalLM", "AscendDeepseekV4ForCausalLM"):
            model_cls = getattr(v4, name, None)
            if model_cls is not None:
                break
        if model_cls is not None:
            _ORIG_LOAD_WEIGHTS = model_cls.load_weights
            model_cls.load_weights = _offload_load_weights
        v4._DSV4_OFFLOAD_PATCHED = True
    _PATCHED = True
