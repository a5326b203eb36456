"""C-ABI library checks that need no GPU: it builds, loads, exports every
entry point of include/dsv4moe.h, and its host-only functions (slot packing)
match a Python restatement of the slot layout."""

import ctypes as C
import importlib.util
import os

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "deepseek-v4-flash-offload_b200")


@pytest.fixture(scope="module")
def lib():
    spec = importlib.util.spec_from_file_location("dsv4_build_ext", os.path.join(PKG, "build_ext.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    from dsv4_plugin import _lib
    return _lib


def test_exports_every_header_symbol(lib):
    names = lib.header_symbols(os.path.join(ROOT, "include", "dsv4moe.h"))
    assert len(names) >= 20
    raw = C.CDLL(lib.LIB_PATH)
    missing = [n for n in names if not hasattr(raw, n)]
    assert not missing, missing
    # the ctypes table covers the header exactly
    assert sorted(lib.SIGNATURES) == names
    assert lib.lib().dsv4_abi_version() == 2


def test_slot_bytes(lib):
    L = lib.lib()
    assert L.dsv4_expert_slot_bytes(4096, 2048) == 13369344
    assert L.dsv4_expert_slot_bytes(1024, 512) == 835584
    assert L.dsv4_expert_slot_bytes(1000, 512) == lib.DSV4_EINVAL
    assert L.dsv4_expert_slot_bytes(1152, 512) == lib.DSV4_EINVAL   # hidden must pair 128-row tiles


def test_dispatch_row_bytes(lib):
    """Bytes of one dispatched token row per format: bf16 2H; FP8 H codes
    + H/128 exponents; MXFP4 H/2 codes + H/32 scales; padded to 16."""
    L = lib.lib()
    assert L.dsv4_ep_row_bytes(lib.ROWS_BF16, 4096) == 8192
    assert L.dsv4_ep_row_bytes(lib.ROWS_FP8, 4096) == 4128
    assert L.dsv4_ep_row_bytes(lib.ROWS_MXFP4, 4096) == 2176
    assert L.dsv4_ep_row_bytes(lib.ROWS_FP8, 1024) == 1040        # 1024 + 8, padded to 16
    assert L.dsv4_ep_row_bytes(lib.ROWS_MXFP4, 1024) == 544
    assert L.dsv4_ep_row_bytes(3, 4096) == lib.DSV4_EINVAL
    assert L.dsv4_ep_row_bytes(lib.ROWS_FP8, 1000) == lib.DSV4_EINVAL


def _pack_py(w, sc, k, row_of, wout, sout):
    """Python restatement of the paired slot layout (256-row pairs x 128 K)."""
    rows = w.shape[0]
    for r in range(rows):
        R = row_of(r)
        for kt in range(k // 128):
            off = ((R // 256) * (k // 128) + kt) * 16384 + (R % 256) * 64
            wout[off: off + 64] = w[r, kt * 64: kt * 64 + 64]
        rr = R % 128
        for kb in range(k // 32):
            off = ((R // 256) * (k // 128) + kb // 4) * 1024 + ((R % 256) // 128) * 512 + (rr % 32) * 16 + \
                (rr // 32) * 4 + kb % 4
            sout[off] = sc[r, kb]


def test_pack_unpack_round_trip(lib):
    from dsv4_plugin import ops
    from dsv4_plugin import synthetic as S
    cfg = S.CFG0
    ex = S.make_expert(cfg, 11, 3)
    t = {k: torch.from_numpy(v) for k, v in ex.items()}
    slot = ops.pack_expert(t["w1p"], t["w1s"], t["w2p"], t["w2s"], t["w3p"], t["w3s"], cfg.hidden, cfg.inter)
    h, i = cfg.hidden, cfg.inter
    sb = slot.numpy()
    assert sb.size == 835584
    w13, s13 = np.zeros(i * h, np.uint8), np.zeros(2 * i * h // 32, np.uint8)
    _pack_py(ex["w1p"], ex["w1s"], h, lambda r: (r // 128) * 256 + r % 128, w13, s13)
    _pack_py(ex["w3p"], ex["w3s"], h, lambda r: (r // 128) * 256 + 128 + r % 128, w13, s13)
    w2, s2 = np.zeros(h * i // 2, np.uint8), np.zeros(h * i // 32, np.uint8)
    _pack_py(ex["w2p"], ex["w2s"], i, lambda r: r, w2, s2)
    o = i * h + h * i // 2
    assert np.array_equal(sb[: i * h], w13)
    assert np.array_equal(sb[i * h: o], w2)
    assert np.array_equal(sb[o: o + s13.size], s13)
    assert np.array_equal(sb[o + s13.size:], s2)
    back = ops.unpack_expert(slot, h, i)
    for k in ex:
        assert np.array_equal(back[k].numpy(), ex[k]), k


def test_errors_are_codes_not_crashes(lib):
    L = lib.lib()
    rc = L.dsv4_pack_expert_host(None, None, None, None, None, None, 1024, 512, None)
    assert rc == lib.DSV4_EINVAL
    assert b"null pointer" in L.dsv4_last_error_string()
    with pytest.raises(lib.Dsv4Error):
        lib.check(rc)


def test_ops_refuse_cpu_tensors(lib):
    from dsv4_plugin import ops
    with pytest.raises(ValueError, match="no CPU path"):
        ops.dequant_fp4_weight(torch.zeros(4, 16, dtype=torch.uint8), torch.zeros(4, 1, dtype=torch.uint8))
    with pytest.raises(ValueError, match="no CPU path"):
        ops.route_topk(torch.zeros(2, 256, dtype=torch.bfloat16), torch.zeros(16, 256), None, 4)


def test_slotcache_c_abi_on_cpu():
    """The LRU slot cache is host code: batch semantics, refusal of an
    oversized batch, snapshot order and statistics through the C ABI."""
    import ctypes

    import numpy as np

    from dsv4_plugin._lib import DSV4_ENOMEM, check, lib
    L = lib()
    h = ctypes.c_void_p()
    check(L.dsv4_slotcache_create(ctypes.byref(h), 3))

    def lookup(keys):
        lay = np.array([k[0] for k in keys], np.int64)
        exp = np.array([k[1] for k in keys], np.int64)
        slots = np.empty(len(keys), np.int32)
        miss = np.empty(len(keys), np.uint8)
        rc = L.dsv4_slotcache_lookup(h, lay.ctypes.data, exp.ctypes.data, len(keys), slots.ctypes.data,
                                     miss.ctypes.data)
        return rc, slots.tolist(), miss.tolist()

    def snapshot():
        lay, exp, sl, n = np.empty(8, np.int64), np.empty(8, np.int64), np.empty(8, np.int32), np.zeros(1, np.int64)
        check(L.dsv4_slotcache_snapshot(h, lay.ctypes.data, exp.ctypes.data, sl.ctypes.data, 8, n.ctypes.data))
        return [((int(lay[i]), int(exp[i])), int(sl[i])) for i in range(int(n[0]))]

    def stats():
        out = np.zeros(4, np.int64)
        check(L.dsv4_slotcache_stats(h, out.ctypes.data))
        return out.tolist()

    try:
        assert lookup([(0, 1), (0, 2), (0, 1)]) == (0, [0, 1, 0], [1, 1, 0])   # free slots 0, 1, ... first
        assert snapshot() == [((0, 2), 1), ((0, 1), 0)]                       # LRU first
        assert lookup([(5, 7)]) == (0, [2], [1])
        rc, slots, miss = lookup([(5, 7), (0, 9), (0, 2)])                    # (0, 9) evicts (0, 1), not (0, 2)
        assert rc == 0 and miss == [0, 1, 0] and slots == [2, 0, 1]
        assert L.dsv4_slotcache_slot_of(h, 0, 1) == -1 and L.dsv4_slotcache_slot_of(h, 0, 9) == 0
        assert stats() == [3, 4, 1, 3]                                         # hits, misses, evictions, resident
        before = snapshot()
        assert lookup([(1, 1), (1, 2), (1, 3), (1, 4)])[0] == DSV4_ENOMEM      # 4 keys, 3 slots
        assert snapshot() == before and stats() == [3, 4, 1, 3]                # nothing changed
        check(L.dsv4_slotcache_clear(h))
        assert snapshot() == [] and stats() == [3, 4, 1, 0]
        assert lookup([(2, 2)]) == (0, [0], [1])
    finally:
        L.dsv4_slotcache_destroy(h)
