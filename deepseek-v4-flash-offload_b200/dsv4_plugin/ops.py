"""torch-facing wrappers of the CUDA library, named after the reference ops.

| here                    | reference                                           |
|-------------------------|-----------------------------------------------------|
| ``dequant_fp4_weight``  | npu_ops.dequant_fp4_weight (npu_ops.py:142-158)     |
| ``act_quant``           | npu_ops.act_quant, inplace form (npu_ops.py:73-98)  |
| ``dynamic_mx_quant``    | torch_npu.npu_dynamic_mx_quant (deepseek_v4.py:212) |
| ``route_topk``          | OffloadDeepseekV4MoE._route (deepseek_v4.py:118-148)|
| ``moe_align``           | the align block of _routed (deepseek_v4.py:154-164) |
| ``MoEPlan.forward``     | _routed / _routed_mxfp4 (deepseek_v4.py:150-245)    |

All tensors must live on a CUDA device; work runs on the current torch
stream.  There is no CPU path.
"""

from __future__ import annotations

import ctypes as C

import torch

from ._lib import PROFILES, ROWS_BF16, ROWS_FP8, ROWS_MXFP4, SCORE_FUNCS, check, lib  # noqa: F401

_E8M0 = getattr(torch, "float8_e8m0fnu", None)


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("dsv4 ops need CUDA tensors (there is no CPU path)")


def _u8(t: torch.Tensor) -> torch.Tensor:
    if t.dtype in (torch.uint8, torch.int8) or (_E8M0 is not None and t.dtype == _E8M0):
        return t.contiguous().view(torch.uint8)
    raise TypeError(f"expected a uint8/int8/e8m0 tensor, got {t.dtype}")


def dequant_fp4_weight(w_packed: torch.Tensor, scale: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """[N, K//2] packed E2M1 + [N, K//32] E8M0 -> [N, K] bf16 (bit-exact)."""
    if out_dtype != torch.bfloat16:
        raise NotImplementedError("the CUDA dequant produces bf16")
    _need_cuda(w_packed, scale)
    w, s = _u8(w_packed), _u8(scale)
    n, kh = w.shape
    out = torch.empty((n, kh * 2), dtype=torch.bfloat16, device=w.device)
    check(lib().dsv4_dequant_mxfp4(w.data_ptr(), s.data_ptr(), out.data_ptr(), n, kh * 2, _stream(w.device)))
    return out


def act_quant(x: torch.Tensor, block_size: int = 128, scale_fmt: str = "ue8m0", scale_dtype=None,
              inplace: bool = False):
    """FP8-E4M3 round trip per 128 with a power-of-two scale, in place.

    Only the in-place form used by the routed-expert path is provided."""
    if not inplace or block_size != 128 or scale_fmt != "ue8m0":
        raise NotImplementedError("only act_quant(x, 128, 'ue8m0', _, inplace=True) is provided")
    _need_cuda(x)
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise TypeError("act_quant expects a contiguous bf16 tensor")
    check(lib().dsv4_act_quant_fp8_rt(x.data_ptr(), x.numel() // x.shape[-1], x.shape[-1], _stream(x.device)))
    return x


def dynamic_mx_quant(x: torch.Tensor):
    """bf16 [.., C] -> (packed E2M1 uint8 [.., C//2], E8M0 uint8 [.., C//32])."""
    _need_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError("dynamic_mx_quant expects bf16")
    x = x.contiguous()
    cols = x.shape[-1]
    rows = x.numel() // cols
    q = torch.empty((*x.shape[:-1], cols // 2), dtype=torch.uint8, device=x.device)
    s = torch.empty((*x.shape[:-1], cols // 32), dtype=torch.uint8, device=x.device)
    check(lib().dsv4_act_quant_mxfp4(x.data_ptr(), rows, cols, q.data_ptr(), s.data_ptr(), _stream(x.device)))
    return q, s


def route_topk(x: torch.Tensor, gate_weight: torch.Tensor, bias: torch.Tensor | None, topk: int,
               score_func: str = "sqrtsoftplus", renormalize: bool = True, route_scale: float = 1.5,
               tid2eid: torch.Tensor | None = None, input_ids: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None, out=None):
    """Router of the MoE layer.  Returns (weights fp32 [T,k], indices int32 [T,k]),
    written into ``out`` = (weights, indices) when given."""
    _need_cuda(x, gate_weight, bias, tid2eid, input_ids)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    x = x.contiguous()
    w = gate_weight.contiguous().float()
    t, h = x.shape
    e = w.shape[0]
    if tid2eid is not None:
        if input_ids is None:
            raise RuntimeError("hash routing needs input_ids (forward_context.input_ids is missing)")
        tid2eid = tid2eid.to(torch.int32).contiguous()
        input_ids = input_ids.to(torch.int64).reshape(-1).contiguous()
        if input_ids.numel() != t:
            raise ValueError("input_ids must have one id per token")
    b = None if bias is None else bias.float().contiguous()
    need = lib().dsv4_route_workspace_bytes(t, h, e)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 4), dtype=torch.uint8, device=x.device)
    if out is not None:
        wo, io = out
        if (wo.shape != (t, topk) or io.shape != (t, topk) or wo.dtype != torch.float32 or io.dtype != torch.int32
                or not (wo.is_contiguous() and io.is_contiguous())):
            raise ValueError("out must be contiguous (float32 [T, k], int32 [T, k]) tensors")
    else:
        wo = torch.empty((t, topk), dtype=torch.float32, device=x.device)
        io = torch.empty((t, topk), dtype=torch.int32, device=x.device)
    check(lib().dsv4_route_topk(
        x.data_ptr(), w.data_ptr(), None if b is None else b.data_ptr(),
        None if tid2eid is None else tid2eid.data_ptr(), None if input_ids is None else input_ids.data_ptr(),
        0 if tid2eid is None else tid2eid.shape[0], t, h, e, topk, SCORE_FUNCS[score_func], int(bool(renormalize)), float(route_scale),
        wo.data_ptr(), io.data_ptr(), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
        _stream(x.device)))
    return wo, io


def route_workspace_bytes(n_tokens: int, hidden: int, n_experts: int) -> int:
    n = lib().dsv4_route_workspace_bytes(n_tokens, hidden, n_experts)
    if n < 0:
        check(int(n))
    return int(n)


def moe_align(indices: torch.Tensor, n_experts: int) -> dict:
    """Stable counting sort of the [T,k] expert indices (int32) on the GPU."""
    _need_cuda(indices)
    idx = indices.to(torch.int32).contiguous()
    t, k = idx.shape
    p = t * k
    dev = idx.device
    out = {
        "counts": torch.empty(n_experts, dtype=torch.int32, device=dev),
        "offsets": torch.empty(n_experts + 1, dtype=torch.int32, device=dev),
        "sorted_flat": torch.empty(max(p, 1), dtype=torch.int32, device=dev),
        "inv": torch.empty(max(p, 1), dtype=torch.int32, device=dev),
        "active": torch.full((n_experts,), -1, dtype=torch.int32, device=dev),
        "n_active": torch.zeros(1, dtype=torch.int32, device=dev),
        "status": torch.zeros(1, dtype=torch.int32, device=dev),
    }
    o = out
    check(lib().dsv4_moe_align(idx.data_ptr(), t, k, n_experts, o["counts"].data_ptr(), o["offsets"].data_ptr(),
                               o["sorted_flat"].data_ptr(), o["inv"].data_ptr(), o["active"].data_ptr(),
                               o["n_active"].data_ptr(), o["status"].data_ptr(), _stream(dev)))
    out["sorted_flat"] = out["sorted_flat"][:p]
    out["inv"] = out["inv"][:p]
    return out


def combine_ordered(rows: torch.Tensor, order: torch.Tensor) -> torch.Tensor:
    """y[t] = bf16(sum_j rows[order[t, j]]) in float32, j ascending; -1 skips."""
    _need_cuda(rows, order)
    rows = rows.contiguous()
    o = order.to(torch.int32).contiguous()
    t, k = o.shape
    y = torch.empty((t, rows.shape[1]), dtype=torch.bfloat16, device=rows.device)
    check(lib().dsv4_moe_combine_ordered(rows.data_ptr(), o.data_ptr(), t, k, rows.shape[1], y.data_ptr(),
                                         _stream(rows.device)))
    return y


def expert_slot_bytes(hidden: int, inter: int) -> int:
    n = lib().dsv4_expert_slot_bytes(hidden, inter)
    if n < 0:
        check(int(n))
    return int(n)


def pack_expert(w1p, w1s, w2p, w2s, w3p, w3s, hidden: int, inter: int, out=None) -> torch.Tensor:
    """Pack the six checkpoint tensors of one expert (CPU) into one slot
    (CPU uint8 tensor, optionally written into ``out``)."""
    ts = [t.detach().contiguous().view(torch.uint8) if t.dtype != torch.uint8 else t.detach().contiguous()
          for t in (w1p, w1s, w2p, w2s, w3p, w3s)]
    for t in ts:
        if t.is_cuda:
            raise ValueError("pack_expert packs host tensors")
    nb = expert_slot_bytes(hidden, inter)
    if out is None:
        out = torch.empty(nb, dtype=torch.uint8)
    if out.is_cuda or out.numel() < nb or not out.is_contiguous():
        raise ValueError("out must be a contiguous host uint8 buffer of at least the slot size")
    check(lib().dsv4_pack_expert_host(*[t.data_ptr() for t in ts], hidden, inter, out.data_ptr()))
    return out


def shared_slot_bytes(hidden: int, inter: int) -> int:
    n = lib().dsv4_shared_slot_bytes(hidden, inter)
    if n < 0:
        check(int(n))
    return int(n)


def pack_shared_expert(w1, s1, w2, s2, w3, s3, hidden: int, inter: int, out=None) -> torch.Tensor:
    """Pack the shared expert's FP8 checkpoint tensors (w1 / w3 [I, H], w2
    [H, I] E4M3 bytes; s* [ceil(N/128), ceil(K/128)] E8M0 bytes; host) into
    its FP8 slot (host uint8 tensor)."""
    ts = [t.detach().contiguous().view(torch.uint8) if t.dtype != torch.uint8 else t.detach().contiguous()
          for t in (w1, s1, w2, s2, w3, s3)]
    for t in ts:
        if t.is_cuda:
            raise ValueError("pack_shared_expert packs host tensors")
    nb = shared_slot_bytes(hidden, inter)
    if out is None:
        out = torch.empty(nb, dtype=torch.uint8)
    if out.is_cuda or out.numel() < nb or not out.is_contiguous():
        raise ValueError("out must be a contiguous host uint8 buffer of at least the slot size")
    check(lib().dsv4_pack_shared_host(*[t.data_ptr() for t in ts], hidden, inter, out.data_ptr()))
    return out


def unpack_expert(slot: torch.Tensor, hidden: int, inter: int) -> dict:
    """Inverse of ``pack_expert`` (host tensors) -> six checkpoint tensors."""
    s = slot.detach().cpu().contiguous()
    h, i = hidden, inter
    out = {"w1p": torch.empty((i, h // 2), dtype=torch.uint8), "w1s": torch.empty((i, h // 32), dtype=torch.uint8),
           "w2p": torch.empty((h, i // 2), dtype=torch.uint8), "w2s": torch.empty((h, i // 32), dtype=torch.uint8),
           "w3p": torch.empty((i, h // 2), dtype=torch.uint8), "w3s": torch.empty((i, h // 32), dtype=torch.uint8)}
    check(lib().dsv4_unpack_expert_host(s.data_ptr(), h, i, *[out[k].data_ptr() for k in
                                                            ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")]))
    return out


def slot_dequant(slot: torch.Tensor, hidden: int, inter: int) -> dict:
    """bf16 w1/w2/w3 of one device-resident slot (ExpertBank.get semantics)."""
    _need_cuda(slot)
    dev = slot.device
    w1 = torch.empty((inter, hidden), dtype=torch.bfloat16, device=dev)
    w3 = torch.empty((inter, hidden), dtype=torch.bfloat16, device=dev)
    w2 = torch.empty((hidden, inter), dtype=torch.bfloat16, device=dev)
    check(lib().dsv4_slot_dequant(slot.data_ptr(), hidden, inter, w1.data_ptr(), w2.data_ptr(), w3.data_ptr(),
                                  _stream(dev)))
    return {"w1": w1, "w2": w2, "w3": w3}


class MoEPlan:
    """Binds a slot arena (uint8 CUDA tensor [n_slots, slot_bytes]) and a
    workspace to the layer dims; ``forward`` runs the fused routed-expert
    layer on the current stream."""

    def __init__(self, hidden: int, inter: int, n_experts: int, topk: int, max_tokens: int,
                 swiglu_limit: float, arena: torch.Tensor, with_shared: bool = False):
        _need_cuda(arena)
        if arena.dtype != torch.uint8 or not arena.is_contiguous() or arena.dim() != 2:
            raise TypeError("arena must be a contiguous uint8 CUDA tensor [n_slots, slot_bytes]")
        if arena.shape[1] != expert_slot_bytes(hidden, inter):
            raise ValueError("arena row size must equal the expert slot size")
        self.hidden, self.inter, self.n_experts, self.topk = hidden, inter, n_experts, topk
        self.with_shared = bool(with_shared)
        self.max_tokens = int(max_tokens)
        self.arena = arena
        self.device = arena.device
        sh = int(self.with_shared)
        nb = lib().dsv4_moe_workspace_bytes_ex(hidden, inter, n_experts, topk, self.max_tokens, sh)
        if nb < 0:
            check(int(nb))
        self.workspace = torch.empty(int(nb), dtype=torch.uint8, device=self.device)
        h = C.c_void_p()
        check(lib().dsv4_moe_plan_create_ex(C.byref(h), hidden, inter, n_experts, topk, self.max_tokens,
                                            float(swiglu_limit), arena.data_ptr(), arena.shape[0],
                                            self.workspace.data_ptr(), int(nb), sh))
        self._h = h

    def forward(self, x: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor, slot_of: torch.Tensor,
                profile: str = "bf16", out: torch.Tensor | None = None,
                shared_slot: torch.Tensor | None = None) -> torch.Tensor:
        """Routed experts (plus the shared expert, whose FP8 slot a plan made
        ``with_shared`` takes) of the [T, H] bf16 tokens -> [T, H] bf16."""
        _need_cuda(x, weights, indices, slot_of)
        x = x.contiguous()
        if x.dtype != torch.bfloat16:
            raise TypeError("x must be bf16")
        t = x.shape[0]
        if t > self.max_tokens:
            raise ValueError(f"{t} tokens exceed the plan's max_tokens={self.max_tokens}")
        w = weights.contiguous().float()
        idx = indices.contiguous().to(torch.int32)
        so = slot_of.contiguous().to(torch.int32)
        if so.numel() < self.n_experts:
            raise ValueError("slot_of needs one entry per expert")
        if out is None:
            out = torch.empty((t, self.hidden), dtype=torch.bfloat16, device=x.device)
        if self.with_shared:
            if shared_slot is None or not shared_slot.is_cuda or shared_slot.dtype != torch.uint8:
                raise ValueError("this plan runs the shared expert: pass its FP8 slot (uint8 CUDA tensor)")
            check(lib().dsv4_moe_forward_shared(self._h, PROFILES[profile], x.data_ptr(), t, w.data_ptr(),
                                                idx.data_ptr(), so.data_ptr(), shared_slot.data_ptr(), out.data_ptr(),
                                                _stream(x.device)))
            return out
        check(lib().dsv4_moe_forward(self._h, PROFILES[profile], x.data_ptr(), t, w.data_ptr(), idx.data_ptr(),
                                     so.data_ptr(), out.data_ptr(), _stream(x.device)))
        return out

    def route(self, x: torch.Tensor, gate_weight: torch.Tensor, bias: torch.Tensor | None, topk: int,
              score_func: str = "sqrtsoftplus", renormalize: bool = True, route_scale: float = 1.5,
              tid2eid: torch.Tensor | None = None, input_ids: torch.Tensor | None = None):
        """``route_topk`` for a decode batch (< 256 tokens) in this plan's
        workspace: one launch (partial logits, grid barrier, top-k) when the
        grid fits on the GPU.  Returns (weights fp32 [T,k], indices int32 [T,k])."""
        _need_cuda(x, gate_weight, bias, tid2eid, input_ids)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        x = x.contiguous()
        w = gate_weight.contiguous().float()
        t = x.shape[0]
        if tid2eid is not None:
            if input_ids is None:
                raise RuntimeError("hash routing needs input_ids (forward_context.input_ids is missing)")
            tid2eid = tid2eid.to(torch.int32).contiguous()
            input_ids = input_ids.to(torch.int64).reshape(-1).contiguous()
            if input_ids.numel() != t:
                raise ValueError("input_ids must have one id per token")
        b = None if bias is None else bias.float().contiguous()
        wo = torch.empty((t, topk), dtype=torch.float32, device=x.device)
        io = torch.empty((t, topk), dtype=torch.int32, device=x.device)
        check(lib().dsv4_moe_route(
            self._h, x.data_ptr(), w.data_ptr(), None if b is None else b.data_ptr(),
            None if tid2eid is None else tid2eid.data_ptr(), None if input_ids is None else input_ids.data_ptr(),
            0 if tid2eid is None else tid2eid.shape[0], t, topk, SCORE_FUNCS[score_func], int(bool(renormalize)),
            float(route_scale), wo.data_ptr(), io.data_ptr(), _stream(x.device)))
        return wo, io

    def forward_rows(self, x: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor, slot_of: torch.Tensor,
                     profile: str = "bf16", n_tokens_dev: torch.Tensor | None = None):
        """The layer without its combine, for a token count that may be known
        only on the device (``n_tokens_dev``: int32 [1]; the first n rows of
        ``x`` / ``weights`` / ``indices`` are used, at most ``x.shape[0]``).
        Returns (rows bf16 [row capacity, H], inv int32 [T * k]): the output of
        assignment a is ``rows[inv[a]]``; both live in the plan's workspace
        until its next forward."""
        _need_cuda(x, weights, indices, slot_of)
        if x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise TypeError("x must be contiguous bf16")
        t = x.shape[0]
        if t > self.max_tokens:
            raise ValueError(f"{t} tokens exceed the plan's max_tokens={self.max_tokens}")
        w = weights if weights.dtype == torch.float32 and weights.is_contiguous() else weights.contiguous().float()
        idx = indices if indices.dtype == torch.int32 and indices.is_contiguous() else \
            indices.contiguous().to(torch.int32)
        so = slot_of.contiguous().to(torch.int32)
        check(lib().dsv4_moe_forward_rows(self._h, PROFILES[profile], x.data_ptr(), t,
                                          None if n_tokens_dev is None else n_tokens_dev.data_ptr(), w.data_ptr(),
                                          idx.data_ptr(), so.data_ptr(), None, _stream(x.device)))
        return self.output_rows(t * self.topk)

    def forward_scatter(self, x: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor, slot_of: torch.Tensor,
                        assign_dst_ptr: int, profile: str = "bf16", n_tokens_dev: torch.Tensor | None = None,
                        x_format: int = ROWS_BF16) -> None:
        """The layer whose down GEMM stores the output row of assignment a
        straight to the device address table ``assign_dst_ptr`` [T * k]
        (another GPU's memory included; null entries are dropped).  With
        ``x_format`` ROWS_FP8 (bf16 profile) or ROWS_MXFP4 (a4w4), x is uint8
        [T, row_bytes] rows quantised at their source."""
        _need_cuda(x, weights, indices, slot_of)
        if x_format == ROWS_BF16 and (x.dtype != torch.bfloat16 or not x.is_contiguous()):
            raise TypeError("x must be contiguous bf16")
        if x_format != ROWS_BF16 and (x.dtype != torch.uint8 or not x.is_contiguous()):
            raise TypeError("quantised rows must be a contiguous uint8 tensor")
        t = x.shape[0]
        if t > self.max_tokens:
            raise ValueError(f"{t} tokens exceed the plan's max_tokens={self.max_tokens}")
        w = weights if weights.dtype == torch.float32 and weights.is_contiguous() else weights.contiguous().float()
        idx = indices if indices.dtype == torch.int32 and indices.is_contiguous() else \
            indices.contiguous().to(torch.int32)
        so = slot_of.contiguous().to(torch.int32)
        check(lib().dsv4_moe_forward_scatter_q(self._h, PROFILES[profile], x.data_ptr(), int(x_format), t,
                                               None if n_tokens_dev is None else n_tokens_dev.data_ptr(),
                                               w.data_ptr(), idx.data_ptr(), so.data_ptr(), assign_dst_ptr,
                                               _stream(x.device)))

    def output_rows(self, n_assign: int):
        rp, ip = C.c_void_p(), C.c_void_p()
        check(lib().dsv4_moe_output_rows(self._h, C.byref(rp), C.byref(ip)))
        rows = torch.as_tensor(_DevArray(rp.value, (self._rows_cap(), self.hidden), "<i2"), device=self.device)
        inv = torch.as_tensor(_DevArray(ip.value, (max(n_assign, 1),), "<i4"), device=self.device)
        return rows.view(torch.bfloat16), inv[:n_assign]

    def _rows_cap(self) -> int:
        # padded row capacity of the plan (same rule as the library's workspace layout)
        p = self.max_tokens * self.topk
        bn = 128
        return (p + (bn - 1) * min(self.n_experts, p) + bn - 1) // bn * bn + bn

    STAGES = ("align", "quant_gather", "gate_up_gemm", "down_gemm", "combine")

    def set_gemm_tile(self, tokens_per_tile: int = 0) -> None:
        """Tokens per GEMM tile: 64, 112, or 0 for the library default."""
        check(lib().dsv4_moe_set_gemm_tile(self._h, int(tokens_per_tile)))

    def set_ffn_fusion(self, enable=None) -> None:
        """Gate/up and down GEMMs in one launch (True), two (False), or the
        library's choice (None: one launch with the decode tile)."""
        check(lib().dsv4_moe_set_ffn_fusion(self._h, -1 if enable is None else int(bool(enable))))

    def enable_timing(self, enable: bool = True) -> None:
        check(lib().dsv4_moe_enable_timing(self._h, int(bool(enable))))

    def stage_times(self) -> dict:
        """ms per stage of the last forward (waits for it)."""
        buf = (C.c_float * 5)()
        check(lib().dsv4_moe_stage_times(self._h, buf, 5))
        return dict(zip(self.STAGES, [float(v) for v in buf]))

    def n_active(self) -> int:
        """Active experts of the last forward (synchronises)."""
        ptrs = [C.c_void_p() for _ in range(6)]
        check(lib().dsv4_moe_debug_align(self._h, *[C.byref(p) for p in ptrs]))
        buf = (C.c_int32 * 1)()
        torch.cuda.synchronize(self.device)
        _memcpy_d2h(buf, ptrs[5].value, 4)
        return int(buf[0])

    def status(self) -> None:
        """Synchronise and raise if a kernel recorded an error."""
        check(lib().dsv4_moe_status(self._h, _stream(self.device)))

    def debug_align(self, n_tokens: int) -> dict:
        ptrs = [C.c_void_p() for _ in range(6)]
        check(lib().dsv4_moe_debug_align(self._h, *[C.byref(p) for p in ptrs]))
        p = n_tokens * self.topk
        e = self.n_experts
        names = ("counts", "offsets", "sorted_flat", "inv", "active", "n_active")
        sizes = (e, e + 1, p, p, e, 1)
        out = {}
        for name, ptr, n in zip(names, ptrs, sizes):
            if n == 0:
                out[name] = torch.zeros(0, dtype=torch.int32)
                continue
            buf = (C.c_int32 * n)()
            torch.cuda.synchronize(self.device)
            _memcpy_d2h(buf, ptr.value, 4 * n)
            out[name] = torch.tensor(list(buf), dtype=torch.int32)
        return out

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib().dsv4_moe_plan_destroy(h)
            except Exception:
                pass
            self._h = None


class _DevArray:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3}


def _memcpy_d2h(dst, src_ptr: int, nbytes: int):
    """Copy device memory at a raw address into a ctypes buffer via torch."""
    import numpy as np
    arr = np.frombuffer(dst, dtype=np.uint8)
    # wrap the device address as a torch tensor through __cuda_array_interface__
    class _View:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (src_ptr, False), "version": 3}
    t = torch.as_tensor(_View(), device="cuda")
    arr[:] = t.cpu().numpy()
