"""CPU oracle for the routed-expert MoE hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The shipped path is the CUDA library
under ``deepseek-v4-flash-offload_b200/csrc`` and fails loudly when that
library is missing.

It restates, in numpy, the algorithm of the reference plugin
``ErnestW2019/deepseek-v4-flash-offload`` for the routed-expert path.  Each
function names the reference lines it follows.  Parity is pinned by
``tests/test_oracle_golden.py`` against fixtures that
``tests/golden/make_golden.py`` produced by running the reference's own
Python code on the CPU.

Number formats used throughout:
  * packed MXFP4 weights: uint8 ``[N, K//2]``, low nibble = even k
    (npu_ops.py:146), E2M1 code table npu_ops.py:20-23;
  * E8M0 scales: uint8, value ``2**(byte-127)`` (npu_ops.py:35-44);
  * bf16 values are carried as float32 arrays holding exactly-representable
    bf16 numbers (``bf16_round`` does the rounding, RNE like torch).
"""

from __future__ import annotations

import numpy as np

# E2M1 nibble -> value (npu_ops.py:20-23).  Nibble 8 decodes to +0.0 there,
# so the dequantised bf16 bit pattern of code 8 is 0x0000.
FP4_TABLE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                      0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)
FP8_MAX = 448.0
FP4_MAX = 6.0
_F32_1_OVER_448 = np.float32(1.0 / 448.0)
_F32_1E_4 = np.float32(1e-4)


# ---------------------------------------------------------------------------
# scalar format helpers
# ---------------------------------------------------------------------------
def e8m0_to_f32(s: np.ndarray) -> np.ndarray:
    """UE8M0 byte -> float32 ``2**(s-127)`` (npu_ops.py:35-44)."""
    return np.ldexp(np.float32(1.0), s.astype(np.int32) - 127).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even), returned as float32.

    Same rounding as torch's ``.to(torch.bfloat16)``; NaN stays NaN.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Upper 16 bits of float32 values that are already bf16-exact."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _exponent(a: np.ndarray):
    """For finite a > 0: (E, m) with a = m * 2**E, m in [1, 2) (exact)."""
    m, e = np.frexp(a.astype(np.float32))  # a = m * 2**e, m in [0.5, 1)
    return (e - 1).astype(np.int32), (m * 2).astype(np.float32)


def ceil_log2_exact(v: np.ndarray) -> np.ndarray:
    """Exact ceil(log2(v)) for float32 v > 0."""
    e, m = _exponent(v)
    return np.where(m == 1.0, e, e + 1).astype(np.int32)


def e4m3_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values in [-448, 448] to the nearest float8 e4m3fn value
    (ties to even), as torch's ``.to(torch.float8_e4m3fn)`` does for
    in-range inputs (npu_ops.py:95)."""
    x = x.astype(np.float32)
    a = np.abs(x)
    e, _ = _exponent(np.where(a > 0, a, np.float32(1.0)))
    e = np.maximum(e, -6)                      # subnormal quantum is 2**-9
    q = np.ldexp(np.float32(1.0), e - 3)       # 3 mantissa bits
    r = np.rint(a / q) * q                     # np.rint = ties to even
    r = np.minimum(r, np.float32(FP8_MAX))
    # the cast keeps the sign of zero (and of values that round to zero)
    return np.copysign(r, x).astype(np.float32)


def e2m1_round(x: np.ndarray) -> np.ndarray:
    """Round to the nearest E2M1 value, ties to the even code, saturating at
    +-6.  Tie rule of ``_round_fp4`` (npu_ops.py:53-67)."""
    x = x.astype(np.float32)
    a = np.minimum(np.abs(x), np.float32(FP4_MAX))
    # binades: [0,2) step 0.5, [2,4) step 1, [4,6] step 2
    q = np.where(a < 2.0, 0.5, np.where(a < 4.0, 1.0, 2.0)).astype(np.float32)
    r = np.rint(a / q) * q
    r = np.minimum(r, np.float32(FP4_MAX))
    return np.where(x < 0, -r, r).astype(np.float32)


def e2m1_code(v: np.ndarray) -> np.ndarray:
    """E2M1-representable float32 value -> 4-bit code (sign bit 3)."""
    a = np.abs(v)
    mag = np.searchsorted(FP4_TABLE[:8], a).astype(np.uint8)
    sign = (np.signbit(v) & (a > 0)).astype(np.uint8) << 3
    return (mag | sign).astype(np.uint8)


# ---------------------------------------------------------------------------
# weight dequant (npu_ops.py:132-158)
# ---------------------------------------------------------------------------
# byte -> (value of the low nibble, value of the high nibble), as one 8-byte word
_BYTE_PAIRS = np.ascontiguousarray(np.stack([FP4_TABLE[np.arange(256) & 0xF], FP4_TABLE[np.arange(256) >> 4]],
                                            axis=-1)).view(np.uint64).reshape(256)


def dequant_fp4_weight(w_packed: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """[N, K//2] packed E2M1 + [N, K//32] E8M0 -> float32 [N, K].

    Low nibble is element 2j, high nibble 2j+1 (npu_ops.py:146); the per-32
    scale multiplies 32 consecutive k (npu_ops.py:155-157).  Every result is
    exact in bf16 for the scale range used here, so the float32 result equals
    the reference's bf16 output.
    """
    u = w_packed.view(np.uint8)
    n, kh = u.shape
    # one gather per byte through a 256-entry table of value pairs (low nibble first)
    vals = np.take(_BYTE_PAIRS, u).view(np.float32).reshape(n, kh * 2 // 32, 32)
    s = e8m0_to_f32(scale.view(np.uint8))
    vals *= s[:, :, None]
    return vals.reshape(n, kh * 2)


# ---------------------------------------------------------------------------
# activation quantisation
# ---------------------------------------------------------------------------
def fp8_block_scale_exp(amax: np.ndarray) -> np.ndarray:
    """Exponent k of the per-128 power-of-two scale 2**k of ``act_quant``:
    amax clamped to >= 1e-4, v = amax * (1/448) in float32, clamped to
    >= 2**-126, k = ceil(log2(v)) (npu_ops.py:47-50, 89-92)."""
    a = np.maximum(amax.astype(np.float32), _F32_1E_4)
    v = (a * _F32_1_OVER_448).astype(np.float32)
    v = np.maximum(v, np.float32(2.0 ** -126))
    return ceil_log2_exact(v)


def act_quant_rt(x: np.ndarray, block: int = 128) -> np.ndarray:
    """FP8-E4M3 round trip with a per-``block`` power-of-two scale, applied
    to bf16 values: ``act_quant(x, 128, "ue8m0", None, inplace=True)``
    (npu_ops.py:73-98).  Returns bf16-exact float32 values."""
    xf = x.astype(np.float32)
    shp = xf.shape
    xb = xf.reshape(-1, shp[-1] // block, block)
    k = fp8_block_scale_exp(np.abs(xb).max(axis=-1, keepdims=True))
    y = e4m3_round(np.clip(np.ldexp(xb, -k), -FP8_MAX, FP8_MAX))
    with np.errstate(over="ignore"):      # y * 2**k may overflow to inf, as in float32 torch
        return bf16_round(np.ldexp(y, k)).reshape(shp)


def act_quant_fp8(x: np.ndarray, block: int = 128):
    """Same quantisation as ``act_quant_rt`` but returns the parts:
    (e4m3 values as float32 [.., C], scale exponents int32 [.., C//block])."""
    xf = x.astype(np.float32)
    shp = xf.shape
    xb = xf.reshape(-1, shp[-1] // block, block)
    k = fp8_block_scale_exp(np.abs(xb).max(axis=-1, keepdims=True))
    y = e4m3_round(np.clip(np.ldexp(xb, -k), -FP8_MAX, FP8_MAX))
    return y.reshape(shp), k[..., 0].reshape(*shp[:-1], shp[-1] // block)


def mx_scale_exp(amax: np.ndarray) -> np.ndarray:
    """E8M0 exponent of the a4w4 activation scale: floor(log2(amax / 6)),
    computed exactly, clamped to [-127, 127]; amax == 0 gives -127.

    This is the scale rule the build specifies for ``npu_dynamic_mx_quant``
    (deepseek_v4.py:212, 240), a closed CANN op whose exact rule the
    reference does not pin."""
    a = amax.astype(np.float32)
    pos = a > 0
    e, m = _exponent(np.where(pos, a, np.float32(1.0)))
    k = e - 3 + (m >= 1.5).astype(np.int32)
    k = np.clip(k, -127, 127)
    return np.where(pos, k, -127).astype(np.int32)


def mx_quant_fp4(x: np.ndarray, block: int = 32):
    """MXFP4 quantisation per ``block`` along the last dim.

    Returns (values: E2M1 values float32 [.., C], scale_exp int32 [.., C//32],
    dequantised float32 [.., C]).  Element rounding: RNE with saturation at
    +-6, the tie rule of npu_ops.py:53-67."""
    xf = x.astype(np.float32)
    shp = xf.shape
    xb = xf.reshape(-1, shp[-1] // block, block)
    k = mx_scale_exp(np.abs(xb).max(axis=-1, keepdims=True))
    q = e2m1_round(np.ldexp(xb, -k))
    deq = np.ldexp(q, k)
    return (q.reshape(shp), k[..., 0].reshape(*shp[:-1], shp[-1] // block),
            deq.reshape(shp).astype(np.float32))


def pack_fp4(values: np.ndarray) -> np.ndarray:
    """E2M1 values [.., C] -> packed uint8 [.., C//2], low nibble = even."""
    c = e2m1_code(values)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


# ---------------------------------------------------------------------------
# router (deepseek_v4.py:118-148; model_npu.py:447-466)
# ---------------------------------------------------------------------------
def _softplus(x):
    # torch.nn.functional.softplus (beta=1, threshold=20)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def route(x: np.ndarray, gate_w: np.ndarray, bias: np.ndarray | None, topk: int,
          score_func: str = "sqrtsoftplus", renormalize: bool = True,
          route_scale: float = 1.5, tid2eid: np.ndarray | None = None,
          input_ids: np.ndarray | None = None):
    """Returns (weights float32 [T,k], indices int64 [T,k]).

    logits = x.float() @ W.T; scores by ``score_func``; selection by
    top-k of scores + bias (or the hash table ``tid2eid[input_ids]``);
    weights are the *unbiased* scores of the chosen experts, optionally
    renormalised, times ``route_scale``.  Indices come out in descending
    order of the biased score; the reference uses ``sorted=False`` so only
    the per-row set is specified (test_moe_align.py:156-158).
    """
    logits = x.astype(np.float32) @ gate_w.astype(np.float32).T
    if score_func == "softmax":
        z = logits - logits.max(axis=-1, keepdims=True)
        ez = np.exp(z)
        scores = (ez / ez.sum(axis=-1, keepdims=True)).astype(np.float32)
    elif score_func == "sigmoid":
        scores = (1.0 / (1.0 + np.exp(-logits))).astype(np.float32)
    else:
        scores = np.sqrt(_softplus(logits)).astype(np.float32)
    if tid2eid is not None:
        if input_ids is None:
            raise RuntimeError("hash routing needs input_ids")
        idx = tid2eid[np.asarray(input_ids).reshape(-1)].astype(np.int64)
    else:
        choice = scores if bias is None else (scores + bias.astype(np.float32)).astype(np.float32)
        # stable descending sort: equal scores keep ascending expert id
        idx = np.argsort(-choice, axis=-1, kind="stable")[:, :topk].astype(np.int64)
    w = np.take_along_axis(scores, idx, axis=1).astype(np.float32)
    if renormalize:
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    w = (w * np.float32(route_scale)).astype(np.float32)
    return w, idx


# ---------------------------------------------------------------------------
# moe_align (deepseek_v4.py:154-164)
# ---------------------------------------------------------------------------
def moe_align(indices: np.ndarray, n_experts: int):
    """Stable counting sort of the flattened (token, slot) assignments by
    expert id.

    Returns dict(order [P] flat index in sorted order, row [P] = order//k,
    counts [E], offsets [E+1], active [D] ascending expert ids,
    group_list [D] = counts[active], inv [P] sorted position of each flat
    index).  ``torch.argsort`` in the reference is not stable; every output
    of the layer is invariant to the order inside a group, and this build
    fixes it to token-major (stable)."""
    t, k = indices.shape
    flat = indices.reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=n_experts).astype(np.int64)
    offsets = np.zeros(n_experts + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(counts)
    active = np.nonzero(counts > 0)[0].astype(np.int64)
    inv = np.empty_like(order)
    inv[order] = np.arange(order.size)
    return dict(order=order, row=order // k, counts=counts, offsets=offsets,
                active=active, group_list=counts[active], inv=inv)


# ---------------------------------------------------------------------------
# routed experts
# ---------------------------------------------------------------------------
def silu(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def _swiglu(gate, up, w, limit):
    """deepseek_v4.py:184-187 / model_npu.py:512-515."""
    if limit and limit > 0:
        up = np.clip(up, -limit, limit)
        gate = np.minimum(gate, np.float32(limit))
    return (silu(gate) * up * w).astype(np.float32)


def e4m3_value(b: np.ndarray) -> np.ndarray:
    """E4M3 (fn) byte -> float32, exact: sign, 4-bit exponent (bias 7), 3-bit
    mantissa, subnormals at exponent 0; 0x7F / 0xFF are NaN."""
    b = b.astype(np.uint32)
    e = ((b >> 3) & 15).astype(np.int32)
    m = (b & 7).astype(np.float32)
    v = np.where(e == 0, np.ldexp(m / np.float32(8.0), -6),
                 np.ldexp(np.float32(1.0) + m / np.float32(8.0), e - 7)).astype(np.float32)
    v = np.where((b & 0x7F) == 0x7F, np.float32(np.nan), v)
    return np.where(b & 0x80, -v, v).astype(np.float32)


def dequant_fp8_weight(w: np.ndarray, scale: np.ndarray, block: int = 128) -> np.ndarray:
    """[N, K] E4M3 bytes * E8M0 scale per 128 x 128 block -> float32
    (npu_ops.py:161-167); exact in bf16 for the scales used here."""
    n, k = w.shape
    s = e8m0_to_f32(scale.view(np.uint8))
    s = np.repeat(np.repeat(s, block, axis=0)[:n], block, axis=1)[:, :k]
    return (e4m3_value(w) * s).astype(np.float32)


def shared_weights_f32(sh: dict) -> dict:
    """Dequantised shared expert {"w1", "w2", "w3"} (model_npu.Linear in "fp8"
    mode holds dequant_fp8_weight(...) as bf16, model_npu.py:94-117)."""
    return {w: dequant_fp8_weight(sh[w], sh[w + "s"]) for w in ("w1", "w2", "w3")}


def shared_expert(x: np.ndarray, wd: dict, swiglu_limit: float = 10.0) -> np.ndarray:
    """model_npu.Expert.forward in "fp8" mode (model_npu.py:469-491): every
    Linear FP8-round-trips its input (act_quant per 128), the bf16 GEMM
    outputs are rounded to bf16, SwiGLU with the clamp and no route weight,
    bf16(h) round-tripped again, bf16 output [T, H]."""
    xq = act_quant_rt(x)
    gate = bf16_round(xq @ wd["w1"].T)
    up = bf16_round(xq @ wd["w3"].T)
    h = bf16_round(_swiglu(gate, up, np.float32(1.0), swiglu_limit))
    return bf16_round(act_quant_rt(h) @ wd["w2"].T)


def expert_weights_f32(expert: dict) -> dict:
    """Dequantise one expert's six packed tensors (offload.py:77-84)."""
    return {w: dequant_fp4_weight(expert[w + "p"], expert[w + "s"]) for w in ("w1", "w2", "w3")}


def moe_routed(x: np.ndarray, weights: np.ndarray, indices: np.ndarray,
               experts, n_experts: int, swiglu_limit: float = 10.0,
               profile: str = "bf16", deq_cache: dict | None = None,
               shared: dict | None = None) -> np.ndarray:
    """Routed-expert output [T, H] (bf16-exact float32) for one layer.

    ``experts[e]`` is a dict of the six packed tensors
    (w1p,w1s,w2p,w2s,w3p,w3s).  Profile ``bf16`` follows the per-expert loop
    of model_npu.py:507-533 and the grouped path of deepseek_v4.py:169-197:
    FP8 round trip of x, gate/up GEMMs rounded to bf16, SwiGLU with clamp,
    times the route weight, FP8 round trip of bf16(h), down GEMM rounded to
    bf16, float32 ``index_add_`` in ascending expert order, cast to bf16.
    Profile ``a4w4`` follows deepseek_v4.py:199-245 with the MXFP4
    activation quantisation of ``mx_quant_fp4``.  With ``shared`` (the
    dequantised shared expert) its output is added in fp32 after the routed
    rows, as model_npu.MoE.forward does.
    """
    t, h = x.shape
    al = moe_align(indices, n_experts)
    sw = weights.reshape(-1)[al["order"]]
    if profile == "bf16":
        xq = act_quant_rt(x)
    else:
        xq = mx_quant_fp4(x)[2]
    y = np.zeros((t, h), dtype=np.float32)
    for e in al["active"]:
        lo, hi = al["offsets"][e], al["offsets"][e + 1]
        rows = al["row"][lo:hi]
        if deq_cache is not None and int(e) in deq_cache:
            wd = deq_cache[int(e)]
        else:
            wd = expert_weights_f32(experts[int(e)])
            if deq_cache is not None:
                deq_cache[int(e)] = wd
        xe = xq[rows]
        gate = bf16_round(xe @ wd["w1"].T)
        up = bf16_round(xe @ wd["w3"].T)
        hh = bf16_round(_swiglu(gate, up, sw[lo:hi, None], swiglu_limit))
        if profile == "bf16":
            hq = act_quant_rt(hh)
        else:
            hq = mx_quant_fp4(hh)[2]
        out = bf16_round(hq @ wd["w2"].T)
        # index_add_ in sorted order: per token, experts ascend
        np.add.at(y, rows, out)
    if shared is not None:
        # MoE.forward: y = y + self.shared_experts(x) in fp32, then one
        # rounding to bf16 (model_npu.py:532-533); ``shared`` holds the
        # dequantised weights (shared_weights_f32)
        y = y + shared_expert(x, shared, swiglu_limit)
    return bf16_round(y)


# ---------------------------------------------------------------------------
# ExpertBank LRU bookkeeping (offload.py:86-129)
# ---------------------------------------------------------------------------
class LruModel:
    """Hit / miss / eviction bookkeeping of ``ExpertBank.get``
    (offload.py:86-100): an OrderedDict keyed by (layer, eid); a hit moves
    the key to the MRU end; a miss inserts it when capacity > 0 and pops
    from the LRU end while over capacity."""

    def __init__(self, capacity: int):
        from collections import OrderedDict
        self.capacity = int(capacity)
        self.od = OrderedDict()
        self.hits = self.misses = self.evictions = 0

    def get(self, key) -> bool:
        if key in self.od:
            self.hits += 1
            self.od.move_to_end(key)
            return True
        self.misses += 1
        if self.capacity > 0:
            self.od[key] = True
            while len(self.od) > self.capacity:
                self.od.popitem(last=False)
                self.evictions += 1
        return False

    def keys(self):
        return list(self.od.keys())


class SlotLruModel:
    """Packed-slot LRU of ``ExpertBank.get_packed`` (offload.py:103-129) as a
    batch: the reference calls ``get_packed`` once per active expert of a
    layer (deepseek_v4.py:216) and keeps the tensors of that layer alive in
    Python, so its OrderedDict may evict a key of the same layer.  A slot
    arena cannot: every expert of a layer must sit in its own slot while the
    layer's kernels run.  So a lookup walks the layer's keys in the given
    order, a hit moves its key to the most-recently-used end, and a miss
    takes a free slot (lowest index first) or evicts the least recently used
    key that is NOT part of the batch.  ``lookup`` returns (slots, missed
    keys).  When no batch is at risk of evicting itself the hit / miss /
    eviction counts equal ``LruModel``'s on the same key sequence
    (``self_evictions_avoided`` counts the cases where they differ)."""

    def __init__(self, capacity: int):
        from collections import OrderedDict
        self.capacity = int(capacity)
        self.od = OrderedDict()          # key -> slot, least recently used first
        self.free = list(range(self.capacity))
        self.hits = self.misses = self.evictions = 0
        self.self_evictions_avoided = 0

    def lookup(self, keys):
        batch = set(keys)
        if len(batch) > self.capacity:
            raise MemoryError(f"{len(batch)} experts needed at once but only {self.capacity} slots")
        slots, missed = [], []
        for k in keys:
            if k in self.od:
                self.hits += 1
                self.od.move_to_end(k)
                slots.append(self.od[k])
                continue
            self.misses += 1
            if self.free:
                s = self.free.pop(0)
            else:
                lru = next(iter(self.od))
                if lru in batch:
                    self.self_evictions_avoided += 1
                victim = next(v for v in self.od if v not in batch)
                s = self.od.pop(victim)
                self.evictions += 1
            self.od[k] = s
            slots.append(s)
            missed.append(k)
        return slots, missed
