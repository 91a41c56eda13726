"""Host-tier expert cache: the reference's ExpertCache (tinygiant/cache.py:11-160)
moved one tier up.  There it maps the relayout file and mlock-pins hot experts in
RAM; here the relayout bytes sit in pinned host memory (the layer files read with
pread, or any ggml expert blobs), hot experts are pinned in HBM, and every other
expert is copied into an HBM slot on demand on a side stream, least recently used
slot first, so the next layer's misses can be fetched while the current layer
computes.

    cache = HostTierCache(model, host_layers, cache_slots=24)
    cache.pin(layer, ids)                    # resident for the cache's lifetime
    cache.prefetch(layer + 1, next_ids)      # start the copies of the misses
    cache.forward(layer, ids, weights, x)    # x += sum_j w_j expert_j(RMSNorm(x) * norm)

Device memory of the slots comes from torch; the copies and repacks are ordered
with CUDA events (a slot is overwritten only after the last kernel reading it)."""
from __future__ import annotations

import ctypes
from collections import OrderedDict

import numpy as np

from ._lib import check


class HostTierCache:
    def __init__(self, model, host_layers, cache_slots: int = 24, staging: int = 2, layout: str = "ggml"):
        """model: an engine.MoEModel (its shape, norms and kernels); host_layers[l]: a
        pinned uint8 torch tensor holding layer l's E expert blobs (Q4_0,
        expert-contiguous relayout order) in `layout`: "ggml" blobs are repacked on the
        device after each copy, "rows" blobs (a version-4 relayout) are copied into their
        slot as they are."""
        assert layout in ("ggml", "rows")
        self.rows = layout == "rows"
        import torch
        self.torch = torch
        self.model = model
        self.lib = model.lib
        self.eb = model.expert_bytes
        self.host = host_layers
        for h in host_layers:
            assert h.is_pinned() and h.dtype == torch.uint8 and h.numel() == model.n_experts * self.eb
        dev = torch.device("cuda", model.device)
        self.slots = torch.empty((cache_slots, self.eb), dtype=torch.uint8, device=dev)
        self.stage = torch.empty((staging, self.eb), dtype=torch.uint8, device=dev)
        self.n_stage, self.next_stage = staging, 0
        self.copy_stream = torch.cuda.Stream(device=dev)
        self.ready = [torch.cuda.Event() for _ in range(cache_slots)]   # slot contents landed
        self.used = [torch.cuda.Event() for _ in range(cache_slots)]    # last kernel reading it done
        self.free = list(range(cache_slots))
        self.lru: OrderedDict = OrderedDict()   # (layer, expert) -> slot, oldest first
        self.pinned = {}                        # (layer, expert) -> device tensor (row-split)
        self.hits = self.misses = self.pinned_hits = 0
        self.bytes_h2d = 0
        self.prefetched = set()   # loaded by prefetch, not yet requested: a miss when requested

    # ------------------------------------------------------------ pinning
    def pin(self, layer: int, ids):
        """Copy experts `ids` of `layer` into HBM for the cache's lifetime (synchronous)."""
        torch = self.torch
        for e in ids:
            key = (layer, int(e))
            if key in self.pinned:
                continue
            dst = torch.empty(self.eb, dtype=torch.uint8, device=self.slots.device)
            raw = self.host[layer][int(e) * self.eb:(int(e) + 1) * self.eb]
            if self.rows:
                dst.copy_(raw)
            else:
                self.stage[0].copy_(raw)
                check(self.lib.tgx_repack_experts(self.model.handle, ctypes.c_void_p(self.stage[0].data_ptr()),
                                                  ctypes.c_void_p(dst.data_ptr()), 1,
                                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), self.lib)
            self.pinned[key] = dst
        torch.cuda.synchronize()

    def pin_from_profile(self, reader, n_per_layer: int) -> int:
        """Pin each layer's n most active experts by the relayout's activation profile
        (the reference's ExpertCache.pin_hot_experts, tinygiant/cache.py:84-100);
        returns how many were pinned."""
        count = 0
        for layer in range(len(self.host)):
            ids = reader.hot_experts(layer, n_per_layer)
            if ids:
                self.pin(layer, ids)
                count += len(ids)
        return count

    # ------------------------------------------------------------ the HBM slot tier
    def _load(self, key, protect):
        """Start loading expert key into a slot (evicting the least recently used slot not
        in `protect`); returns the slot."""
        if self.free:
            slot = self.free.pop()
        else:
            victim = next((k for k in self.lru if k not in protect), None)
            if victim is None:
                raise RuntimeError("HostTierCache: every slot is needed by the current request; add cache_slots")
            slot = self.lru.pop(victim)
            self.prefetched.discard(victim)
        layer, e = key
        cs = self.copy_stream
        cs.wait_event(self.used[slot])          # no kernel still reads the old contents
        st = self.stage[self.next_stage]
        self.next_stage = (self.next_stage + 1) % self.n_stage
        with self.torch.cuda.stream(cs):
            src = self.host[layer][e * self.eb:(e + 1) * self.eb]
            if self.rows:   # already in the kernels' layout: straight into the slot
                self.slots[slot].copy_(src, non_blocking=True)
            else:
                st.copy_(src, non_blocking=True)
                check(self.lib.tgx_repack_experts(self.model.handle, ctypes.c_void_p(st.data_ptr()),
                                                  ctypes.c_void_p(self.slots[slot].data_ptr()), 1,
                                                  ctypes.c_void_p(cs.cuda_stream)), self.lib)
            self.ready[slot].record(cs)
        self.bytes_h2d += self.eb
        self.lru[key] = slot
        return slot

    def prefetch(self, layer: int, ids):
        """Start copying the experts of `layer` that are neither pinned nor cached."""
        keys = [(layer, int(e)) for e in ids]
        protect = set(keys)
        for key in keys:
            if key not in self.pinned and key not in self.lru:
                self._load(key, protect)
                self.prefetched.add(key)

    def resident(self, layer: int, ids, count: bool = True):
        """Device pointers of experts `ids` (loading misses); hits/misses are counted."""
        keys = [(layer, int(e)) for e in ids]
        protect = set(keys)
        ptrs, slots = [], []
        for key in keys:
            if key in self.pinned:
                self.pinned_hits += count
                self.hits += count
                ptrs.append(self.pinned[key].data_ptr())
                continue
            if key in self.lru:
                if key in self.prefetched:    # a miss whose copy the prefetch already started
                    self.prefetched.discard(key)
                    self.misses += count
                else:
                    self.hits += count
                self.lru.move_to_end(key)
                slot = self.lru[key]
            else:
                self.misses += count
                slot = self._load(key, protect)
            slots.append(slot)
            ptrs.append(self.slots[slot].data_ptr())
        return ptrs, slots

    def forward(self, layer: int, ids, weights, x, stream=None):
        """x (cuda f32[embed]) += sum_j weights[j] * expert_{ids[j]}(RMSNorm(x) * norm_layer)."""
        torch = self.torch
        stream = stream or torch.cuda.current_stream()
        ptrs, slots = self.resident(layer, ids)
        for s in slots:
            stream.wait_event(self.ready[s])
        arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
        w = np.ascontiguousarray(weights, dtype=np.float32)
        check(self.lib.tgx_experts_forward(self.model.handle, layer, arr, w.ctypes.data, len(ptrs),
                                           ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(stream.cuda_stream)),
              self.lib)
        for s in slots:
            self.used[s].record(stream)

    @property
    def hit_rate(self) -> float:
        n = self.hits + self.misses
        return self.hits / n if n else 0.0
