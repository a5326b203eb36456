"""Expert bank: packed MXFP4 experts in pinned host memory + an HBM slot cache.

Mirrors ``offload.ExpertBank`` of the reference (offload.py:22-151): same
constructor arguments, ``register / has / num_experts / get / get_packed /
invalidate / stats`` and the same LRU semantics (a hit moves the key to the
MRU end, a miss inserts it and evicts from the LRU end while over capacity,
capacity 0 never caches).

The B200 design differs underneath:
  * an expert is packed once, at ``register``, into ONE contiguous slot in
    the layout the tensor cores read (``ops.pack_expert``), carved out of
    large pinned host blocks;
  * the device side is one arena of ``packed_capacity`` slots; a miss is a
    single ``cudaMemcpyAsync`` of the slot on a dedicated copy stream, and
    the compute stream waits on an event instead of the host;
  * a slot is only overwritten after the kernels that last read it are done
    (per-slot events recorded by ``mark_used``).
``get`` (bf16 dequantised experts, reference semantics) is kept for API and
test parity; the routed-expert kernels never use it.
"""

from __future__ import annotations

import collections
import ctypes
import os

import numpy as np
import torch

KEYS6 = ("w1p", "w1s", "w2p", "w2s", "w3p", "w3s")


class SlotLRU:
    """LRU bookkeeping of (layer, eid) -> slot index, host only, in the
    library (``dsv4_slotcache_*``, csrc/slotcache.cpp).

    ``lookup(keys)`` returns (slots, misses) for a batch of keys that must
    all be resident at the same time: keys of the batch are never evicted by
    other keys of the same batch.  ``od`` is a snapshot of the resident keys
    in LRU order (least recently used first) with their slots."""

    def __init__(self, capacity: int):
        from dsv4_plugin._lib import check, lib
        self.capacity = int(capacity)
        h = ctypes.c_void_p()
        check(lib().dsv4_slotcache_create(ctypes.byref(h), self.capacity))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                from dsv4_plugin._lib import lib
                lib().dsv4_slotcache_destroy(h)
            except Exception:   # interpreter shutdown: the process frees it
                pass
            self._h = None

    def lookup(self, keys):
        from dsv4_plugin._lib import DSV4_ENOMEM, check, lib
        n = len(keys)
        lay = np.fromiter((k[0] for k in keys), dtype=np.int64, count=n)
        exp = np.fromiter((k[1] for k in keys), dtype=np.int64, count=n)
        slots = np.empty(n, dtype=np.int32)
        miss = np.empty(n, dtype=np.uint8)
        rc = lib().dsv4_slotcache_lookup(self._h, lay.ctypes.data, exp.ctypes.data, n, slots.ctypes.data,
                                         miss.ctypes.data)
        if rc == DSV4_ENOMEM:
            raise MemoryError(f"{len(set(keys))} experts needed at once but only {self.capacity} slots")
        check(rc)
        sl = slots.tolist()
        return sl, [(keys[i], sl[i]) for i in np.flatnonzero(miss).tolist()]

    def slot_of(self, k) -> int:
        from dsv4_plugin._lib import lib
        return int(lib().dsv4_slotcache_slot_of(self._h, int(k[0]), int(k[1])))

    def _stats(self):
        from dsv4_plugin._lib import check, lib
        out = np.zeros(4, dtype=np.int64)
        check(lib().dsv4_slotcache_stats(self._h, out.ctypes.data))
        return out

    @property
    def hits(self) -> int:
        return int(self._stats()[0])

    @property
    def misses(self) -> int:
        return int(self._stats()[1])

    @property
    def evictions(self) -> int:
        return int(self._stats()[2])

    @property
    def od(self) -> collections.OrderedDict:
        from dsv4_plugin._lib import check, lib
        n = max(len(self), 1)
        lay = np.empty(n, dtype=np.int64)
        exp = np.empty(n, dtype=np.int64)
        slots = np.empty(n, dtype=np.int32)
        got = np.zeros(1, dtype=np.int64)
        check(lib().dsv4_slotcache_snapshot(self._h, lay.ctypes.data, exp.ctypes.data, slots.ctypes.data, n,
                                            got.ctypes.data))
        m = int(got[0])
        return collections.OrderedDict(((int(lay[i]), int(exp[i])), int(slots[i])) for i in range(m))

    def clear(self):
        from dsv4_plugin._lib import check, lib
        check(lib().dsv4_slotcache_clear(self._h))

    def __contains__(self, k):
        return self.slot_of(k) >= 0

    def __len__(self):
        return int(self._stats()[3])


class ExpertBank:
    """Host-resident packed experts + device LRU slot cache.

    ``capacity``: experts kept dequantised (bf16) by ``get`` (reference
    semantics).  ``packed_capacity`` (env ``DSV4_PACKED_SLOTS``, default
    ``4 * capacity``, the same HBM budget): packed slots of the arena the
    routed-expert kernels read.  ``pin`` (env ``DSV4_PIN_HOST``, default on):
    page-locked host pool; a failed pin degrades once to pageable memory.
    """

    def __init__(self, capacity: int, device, dtype=torch.bfloat16, verbose=False, pin=None,
                 hidden: int | None = None, inter: int | None = None, packed_capacity: int | None = None,
                 block_slots: int = 16):
        self.capacity = int(capacity)
        self.device = torch.device(device)
        self.dtype = dtype
        self.verbose = verbose
        if pin is None:
            pin = os.environ.get("DSV4_PIN_HOST", "1") == "1"
        self.pin = bool(pin)
        if packed_capacity is None:
            packed_capacity = int(os.environ.get("DSV4_PACKED_SLOTS", str(4 * self.capacity)))
        self.packed_capacity = int(packed_capacity)
        self.hidden, self.inter = hidden, inter
        self.block_slots = int(block_slots)
        self._host = {}                 # (layer, eid) -> host uint8 slot view
        self._blocks = []               # pinned (or pageable) host blocks
        self._block_used = 0
        self._cache = collections.OrderedDict()   # (layer, eid) -> bf16 dict (get)
        self.hits = self.misses = self.evictions = 0
        self._lru = SlotLRU(self.packed_capacity)
        self._arena = None
        self._slot_events = {}
        self._copy_stream = None
        self.h2d_bytes = 0
        self.h2d_copies = 0
        self._tables = {}               # layer -> (epoch, device slot table)
        self._epoch = 0
        self._all_event = None

    # -- host pool ----------------------------------------------------------
    @property
    def slot_bytes(self) -> int:
        from dsv4_plugin import ops
        return ops.expert_slot_bytes(self.hidden, self.inter)

    def _new_host_slot(self) -> torch.Tensor:
        nb = self.slot_bytes
        if not self._blocks or self._block_used == self.block_slots:
            blk = None
            if self.pin:
                try:
                    blk = torch.empty((self.block_slots, nb), dtype=torch.uint8, pin_memory=True)
                except RuntimeError as exc:   # pinned memory unavailable: degrade once
                    print(f"[ExpertBank] pin_memory failed, using pageable memory: {exc}", flush=True)
                    self.pin = False
            if blk is None:
                blk = torch.empty((self.block_slots, nb), dtype=torch.uint8)
            self._blocks.append(blk)
            self._block_used = 0
        s = self._blocks[-1][self._block_used]
        self._block_used += 1
        return s

    def register(self, layer, eid, w1p, w1s, w2p, w2s, w3p, w3s):
        """Pack and store one expert's six checkpoint tensors (offload.py:59-68)."""
        from dsv4_plugin import ops
        if self.hidden is None:
            self.inter, kh = w1p.shape
            self.hidden = kh * 2
        key = (int(layer), int(eid))
        dst = self._host.get(key)
        if dst is None:
            dst = self._new_host_slot()
        ops.pack_expert(w1p, w1s, w2p, w2s, w3p, w3s, self.hidden, self.inter, out=dst)
        self._host[key] = dst
        if key in self._lru:        # stale device copy
            self.invalidate()

    def register_packed(self, layer, eid, slot: torch.Tensor):
        """Store an expert that is already in the packed slot layout (for
        example a slot written earlier by ``host_slot``), without repacking."""
        if self.hidden is None:
            raise RuntimeError("register_packed needs hidden/inter (pass them to the constructor)")
        if slot.dtype != torch.uint8 or slot.numel() != self.slot_bytes:
            raise ValueError(f"a packed slot is {self.slot_bytes} uint8 bytes")
        key = (int(layer), int(eid))
        dst = self._host.get(key)
        if dst is None:
            dst = self._new_host_slot()
        dst.copy_(slot.reshape(-1))
        self._host[key] = dst
        if key in self._lru:
            self.invalidate()

    def has(self, layer, eid):
        return (int(layer), int(eid)) in self._host

    def num_experts(self):
        return len(self._host)

    def host_slot(self, layer, eid) -> torch.Tensor:
        return self._host[(int(layer), int(eid))]

    # -- device arena -------------------------------------------------------
    def _need_cuda(self):
        if self.device.type != "cuda":
            raise RuntimeError("the expert slot cache needs a CUDA device (there is no CPU path)")

    @property
    def arena(self) -> torch.Tensor:
        self._need_cuda()
        if self._arena is None:
            self._arena = torch.empty((self.packed_capacity, self.slot_bytes), dtype=torch.uint8,
                                      device=self.device)
        return self._arena

    def _stream(self):
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)
        return self._copy_stream

    def ensure_resident(self, layer, eids, stream=None):
        """Make experts (layer, e) for e in ``eids`` resident in the arena.

        Returns their slot indices.  Misses are copied H2D on the bank's copy
        stream; ``stream`` (default: current) waits for those copies on the
        device.  Replaces the per-expert ``get_packed`` loop of
        deepseek_v4.py:216."""
        self._need_cuda()
        keys = [(int(layer), int(e)) for e in eids]
        for k in keys:
            if k not in self._host:
                raise KeyError(f"expert {k} was never registered")
        arena = self.arena
        slots, misses = self._lru.lookup(keys)
        if misses:
            cs = self._stream()
            if self._all_event is not None:
                cs.wait_event(self._all_event)   # kernels that read every slot
            for k, s in misses:
                ev = self._slot_events.get(s)
                if ev is not None:
                    cs.wait_event(ev)        # last kernels reading slot s are done
                with torch.cuda.stream(cs):
                    arena[s].copy_(self._host[k], non_blocking=True)
                self.h2d_bytes += self.slot_bytes
                self.h2d_copies += 1
            done = torch.cuda.Event()
            done.record(cs)
            (stream or torch.cuda.current_stream(self.device)).wait_event(done)
        return slots

    def resident_table(self, layer, n_experts):
        """Device int32 [n_experts] expert -> slot table of ``layer`` when
        every expert of the layer is resident, else None.  Built once per
        residency epoch; using it does not touch the LRU order."""
        layer = int(layer)
        epoch = self._epoch + self._lru.evictions
        hit = self._tables.get(layer)
        if hit is not None and hit[0] == epoch:
            return hit[1]
        keys = [(layer, e) for e in range(n_experts)]
        if not all(k in self._lru for k in keys):
            return None
        t = torch.tensor([self._lru.slot_of(k) for k in keys], dtype=torch.int32).to(self.device)
        self._tables[layer] = (epoch, t)
        return t

    def resize_slots(self, packed_capacity: int):
        """Change the HBM budget to ``packed_capacity`` slots.  Drops every
        resident expert (the host pool stays) and waits for the kernels
        that read the old arena."""
        self._need_cuda()
        torch.cuda.synchronize(self.device)
        self._arena = None
        self.packed_capacity = int(packed_capacity)
        self._lru = SlotLRU(self.packed_capacity)
        self._slot_events.clear()
        self._all_event = None
        self._tables.clear()
        self._epoch += 1
        self.h2d_bytes = self.h2d_copies = 0

    def mark_used(self, slots, stream=None):
        """Record that kernels enqueued so far on ``stream`` read ``slots``
        (``None``: possibly any slot)."""
        ev = torch.cuda.Event()
        ev.record(stream or torch.cuda.current_stream(self.device))
        if slots is None:
            self._all_event = ev
            return
        for s in slots:
            self._slot_events[int(s)] = ev

    def preload_all(self, layer=None):
        """Copy every registered expert (of ``layer``) into the arena."""
        keys = [k for k in self._host if layer is None or k[0] == layer]
        by_layer = collections.defaultdict(list)
        for L, e in keys:
            by_layer[L].append(e)
        out = {}
        for L, es in by_layer.items():
            for e, s in zip(es, self.ensure_resident(L, es)):
                out[(L, e)] = s
        return out

    # -- reference API ------------------------------------------------------
    def get(self, layer, eid):
        """bf16 {"w1","w2","w3"} on the device (offload.py:86-100 semantics)."""
        from dsv4_plugin import ops
        key = (int(layer), int(eid))
        cached = self._cache.get(key)
        if cached is not None:
            self.hits += 1
            self._cache.move_to_end(key)
            return cached
        self.misses += 1
        self._need_cuda()
        slot = self._host[key].to(self.device, non_blocking=True)
        vals = ops.slot_dequant(slot, self.hidden, self.inter)
        if self.capacity > 0:
            self._cache[key] = vals
            while len(self._cache) > self.capacity:
                self._cache.popitem(last=False)
                self.evictions += 1
        return vals

    def get_packed(self, layer, eid):
        """Packed expert on the device (offload.py:103-129 semantics):
        ``w{1,2,3}p`` ([N, K//2] uint8) and ``w{1,2,3}s`` ([N, K//32] E8M0)
        in checkpoint order, plus ``slot`` (the resident slot, kernel layout)
        and ``slot_index``.  The checkpoint-order tensors are copies made
        from the host pool; the kernels read the slot."""
        from dsv4_plugin import ops
        s = self.ensure_resident(layer, [eid])[0]
        parts = ops.unpack_expert(self._host[(int(layer), int(eid))], self.hidden, self.inter)
        out = {k: v.to(self.device) for k, v in parts.items()}
        out["slot"] = self.arena[s]
        out["slot_index"] = s
        return out

    def invalidate(self):
        self._cache.clear()
        self._lru.clear()
        self._slot_events.clear()
        self._all_event = None
        self._tables.clear()
        self._epoch += 1

    def stats(self):
        tot = self.hits + self.misses
        lru = self._lru
        ptot = lru.hits + lru.misses
        return {"hits": self.hits, "misses": self.misses, "evictions": self.evictions,
                "hit_rate": (self.hits / tot) if tot else 0.0,
                "cached": len(self._cache), "capacity": self.capacity,
                "packed_hits": lru.hits, "packed_misses": lru.misses,
                "packed_hit_rate": (lru.hits / ptot) if ptot else 0.0,
                "packed_cached": len(lru), "packed_capacity": self.packed_capacity,
                "packed_evictions": lru.evictions,
                "pinned": self.pin, "h2d_bytes": self.h2d_bytes, "h2d_copies": self.h2d_copies}

    def __repr__(self):
        s = self.stats()
        return (f"ExpertBank(experts={self.num_experts()}, packed={s['packed_cached']}/"
                f"{s['packed_capacity']}, packed_hit_rate={s['packed_hit_rate']:.3f})")
