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


class _DevView:
    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


class SlotDirectory:
    """The bank's LRU kept on the device (``dsv4_slotdir_*``,
    csrc/slotdir.cu): same semantics as ``SlotLRU``, but the router's expert
    ids never leave the GPU.  ``acquire`` enqueues, on a stream, the lookup of
    a layer's batch and the GPU's own copies of the missed experts from the
    page-locked host pool, so an offloaded layer has no host synchronisation
    and can be captured in a CUDA graph.  ``table(layer)`` is the device
    expert -> slot table the grouped GEMM reads."""

    DEMAND, PREFETCH = 0, 1
    MAX_SLOTS = 32768

    def __init__(self, arena: torch.Tensor, n_layers: int, n_experts: int):
        from dsv4_plugin._lib import check, lib
        self.n_layers, self.n_experts = int(n_layers), int(n_experts)
        self.n_slots, self.slot_bytes = int(arena.shape[0]), int(arena.shape[1])
        self.device = arena.device
        nb = lib().dsv4_slotdir_workspace_bytes(self.n_layers, self.n_experts, self.n_slots)
        if nb < 0:
            check(int(nb))
        self.workspace = torch.empty(int(nb), dtype=torch.uint8, device=self.device)
        h = ctypes.c_void_p()
        check(lib().dsv4_slotdir_create(ctypes.byref(h), self.n_layers, self.n_experts, arena.data_ptr(),
                                        self.n_slots, self.slot_bytes, self.workspace.data_ptr(), int(nb)))
        self._h = h
        self._arena = arena
        self._tables = {}

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                from dsv4_plugin._lib import lib
                lib().dsv4_slotdir_destroy(h)
            except Exception:
                pass
            self._h = None

    def set_sources(self, items):
        """items: iterable of (layer, expert, page-locked host slot tensor)."""
        from dsv4_plugin._lib import check, lib
        items = [(int(L), int(e), t) for L, e, t in items if 0 <= int(L) < self.n_layers]
        if not items:
            return
        lay = np.array([i[0] for i in items], dtype=np.int32)
        exp = np.array([i[1] for i in items], dtype=np.int32)
        ptrs = (ctypes.c_void_p * len(items))(*[i[2].data_ptr() for i in items])
        check(lib().dsv4_slotdir_set_sources(self._h, len(items), lay.ctypes.data, exp.ctypes.data, ptrs))

    def acquire(self, layer: int, indices: torch.Tensor, mode: int = 0, stream=None):
        from dsv4_plugin._lib import check, lib
        idx = indices if indices.dtype == torch.int32 and indices.is_contiguous() else \
            indices.contiguous().to(torch.int32)
        st = stream or torch.cuda.current_stream(self.device)
        check(lib().dsv4_slotdir_acquire(self._h, int(layer), idx.data_ptr(), idx.numel(), int(mode),
                                         st.cuda_stream))
        return idx

    def table(self, layer: int) -> torch.Tensor:
        t = self._tables.get(int(layer))
        if t is None:
            from dsv4_plugin._lib import check, lib
            p = ctypes.c_void_p()
            check(lib().dsv4_slotdir_table(self._h, int(layer), ctypes.byref(p)))
            t = torch.as_tensor(_DevView(p.value, self.n_experts, "<i4"), device=self.device)
            self._tables[int(layer)] = t
        return t

    def counters(self, stream=None) -> dict:
        from dsv4_plugin._lib import check, lib
        out = np.zeros(8, dtype=np.int64)
        st = stream or torch.cuda.current_stream(self.device)
        check(lib().dsv4_slotdir_stats(self._h, out.ctypes.data, st.cuda_stream))
        names = ("hits", "misses", "evictions", "prefetch_hits", "prefetch_fetched", "prefetch_evictions",
                 "prefetch_skipped", "acquires")
        return dict(zip(names, (int(v) for v in out)))

    def status(self, stream=None) -> None:
        from dsv4_plugin._lib import check, lib
        st = stream or torch.cuda.current_stream(self.device)
        check(lib().dsv4_slotdir_status(self._h, st.cuda_stream))

    def snapshot(self, stream=None):
        """(keys [S] int32 = layer * n_experts + expert or -1, stamps [S] int64)."""
        from dsv4_plugin._lib import check, lib
        keys = np.empty(self.n_slots, dtype=np.int32)
        stamps = np.empty(self.n_slots, dtype=np.int64)
        st = stream or torch.cuda.current_stream(self.device)
        check(lib().dsv4_slotdir_snapshot(self._h, keys.ctypes.data, stamps.ctypes.data, st.cuda_stream))
        return keys, stamps

    def clear(self, stream=None):
        from dsv4_plugin._lib import check, lib
        st = stream or torch.cuda.current_stream(self.device)
        check(lib().dsv4_slotdir_clear(self._h, st.cuda_stream))


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
        self._dir = None                # SlotDirectory when the bank offloads with device-side lookups
        self._prefetch_stream = None
        self._prefetch_done = None      # event: the last prefetch enqueued on the side stream
        self.trace = None               # list: (layer, start, end) timing events of each prefetch
        # DSV4_DEVICE_LRU=0 keeps the host LRU (one synchronisation per layer)
        self.device_lru = os.environ.get("DSV4_DEVICE_LRU", "1") != "0"

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
        self._new_source(key, dst)
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
        self._new_source(key, dst)
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

    # -- device-side LRU ------------------------------------------------------
    def _new_source(self, key, host_slot):
        if self._dir is not None:
            if key[0] >= self._dir.n_layers:
                self._dir = None            # rebuilt, larger, at the next acquire
                self.invalidate()
            else:
                self._dir.set_sources([(key[0], key[1], host_slot)])
                if key[0] in self._dir_touched:   # an older copy of the expert may be resident
                    self.invalidate()

    def device_directory(self, n_experts: int):
        """The device-side LRU (created on first use), or None when the pool
        is not page-locked (the GPU can only read pinned host memory) or
        ``DSV4_DEVICE_LRU=0``."""
        if not (self.device_lru and self.pin and self.device.type == "cuda"):
            return None
        if self.packed_capacity > SlotDirectory.MAX_SLOTS:
            return None
        if self._dir is None:
            if not all(t.is_pinned() for t in self._host.values()):
                return None
            n_layers = max([k[0] for k in self._host if k[0] >= 0] + [0]) + 1
            self._lru.clear()               # the directory starts empty: one owner of the arena
            self._tables.clear()
            torch.cuda.synchronize(self.device)
            self._dir = SlotDirectory(self.arena, n_layers, n_experts)
            self._dir.set_sources((L, e, t) for (L, e), t in self._host.items() if L >= 0)
            self._dir_touched = set()
        return self._dir

    def acquire(self, layer: int, indices: torch.Tensor, stream=None) -> torch.Tensor:
        """Device path of ``ensure_resident``: make the experts named by the
        router's ``indices`` (device [T, k]) resident, on ``stream``, without
        reading them on the host.  Waits (on the device) for the last
        prefetch first.  Returns the layer's device expert -> slot table."""
        d = self._dir
        st = stream or torch.cuda.current_stream(self.device)
        if self._prefetch_done is not None:
            st.wait_event(self._prefetch_done)
            self._prefetch_done = None
        d.acquire(layer, indices, SlotDirectory.DEMAND, st)
        self._dir_touched.add(int(layer))
        return d.table(layer)

    def prefetch_stream(self):
        if self._prefetch_stream is None:
            self._prefetch_stream = torch.cuda.Stream(device=self.device)
        return self._prefetch_stream

    def prefetch(self, layer: int, predict, stream=None) -> None:
        """Copy the experts that ``predict()`` (called on the side stream,
        returns device [T, k] expert ids) names for ``layer`` while the
        current stream keeps computing.  The next ``acquire`` waits for it on
        the device.  The prefetch never evicts the experts of the demand batch
        in flight."""
        d = self._dir
        if d is None or not 0 <= int(layer) < d.n_layers:
            return
        cur = stream or torch.cuda.current_stream(self.device)
        side = self.prefetch_stream()
        fork = torch.cuda.Event()
        fork.record(cur)
        side.wait_event(fork)
        with torch.cuda.stream(side):
            t0 = None
            if self.trace is not None:   # timing events: eager runs only
                t0 = torch.cuda.Event(enable_timing=True)
                t0.record(side)
            idx = predict()
            d.acquire(layer, idx, SlotDirectory.PREFETCH, side)
            done = torch.cuda.Event(enable_timing=t0 is not None)
            done.record(side)
            if t0 is not None:
                self.trace.append((int(layer), t0, done))
        self._dir_touched.add(int(layer))
        self._prefetch_done = done

    def join_prefetch(self, stream=None) -> None:
        if self._prefetch_done is not None:
            (stream or torch.cuda.current_stream(self.device)).wait_event(self._prefetch_done)
            self._prefetch_done = None

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
        self._dir = None
        self._prefetch_done = None
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
        if self._dir is not None:
            self.join_prefetch()
            self._dir.clear()
            self._dir_touched = set()
        self._slot_events.clear()
        self._all_event = None
        self._tables.clear()
        self._epoch += 1

    def stats(self):
        """offload.py:135-146 keys; the packed_* counters come from the
        device directory when the bank offloads through it (synchronises)."""
        tot = self.hits + self.misses
        lru = self._lru
        ph, pm, pe, pc = lru.hits, lru.misses, lru.evictions, len(lru)
        h2d_b, h2d_n = self.h2d_bytes, self.h2d_copies
        extra = {}
        if self._dir is not None:
            c = self._dir.counters()
            keys, _ = self._dir.snapshot()
            ph, pm, pe, pc = ph + c["hits"], pm + c["misses"], pe + c["evictions"], int((keys >= 0).sum())
            fetched = c["misses"] + c["prefetch_fetched"]
            h2d_b, h2d_n = h2d_b + fetched * self.slot_bytes, h2d_n + fetched
            extra = {"device_lru": True, **{k: v for k, v in c.items() if k.startswith("prefetch")}}
        ptot = ph + pm
        return {"hits": self.hits, "misses": self.misses, "evictions": self.evictions,
                "hit_rate": (self.hits / tot) if tot else 0.0,
                "cached": len(self._cache), "capacity": self.capacity,
                "packed_hits": ph, "packed_misses": pm,
                "packed_hit_rate": (ph / ptot) if ptot else 0.0,
                "packed_cached": pc, "packed_capacity": self.packed_capacity,
                "packed_evictions": pe,
                "pinned": self.pin, "h2d_bytes": h2d_b, "h2d_copies": h2d_n, **extra}

    def __repr__(self):
        s = self.stats()
        return (f"ExpertBank(experts={self.num_experts()}, packed={s['packed_cached']}/"
                f"{s['packed_capacity']}, packed_hit_rate={s['packed_hit_rate']:.3f})")
