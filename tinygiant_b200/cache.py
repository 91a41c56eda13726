"""Host-tier expert cache: the reference's ExpertCache (tinygiant/cache.py:11-160)
moved one tier up.  There it maps the relayout file and mlock-pins hot experts in
RAM; here the relayout bytes sit in pinned host memory (the layer files read with
pread, or any ggml expert blobs), hot experts are pinned in HBM, and every other
expert is copied into an HBM slot on demand on a side stream, least recently used
slot first, so the next layer's misses can be fetched while the current layer
computes.

    cache = HostTierCache(model, host_layers, cache_slots=24, index=reader.index)
    cache.pin(layer, ids)                    # resident for the cache's lifetime
    cache.prefetch(layer + 1, next_ids)      # start the copies of the misses
    cache.forward(layer, ids, weights, x)    # x += sum_j w_j expert_j(RMSNorm(x) * norm)

The reference's ExpertCache surface is kept: get(layer, eid) counts the access and
returns the resident expert; pin_hot_experts (the relayout's static activation
profile), pin_from_usage (calibration counts, then the profile) and pin_nonuniform
(a per-layer pin count) choose experts exactly as tinygiant/cache.py:72-152 does and
pin them in HBM.

Device memory of the slots comes from torch; the copies and repacks are ordered
with CUDA events (a slot is overwritten only after the last kernel reading it)."""
from __future__ import annotations

import ctypes
from collections import OrderedDict

import numpy as np

from ._lib import check


def select_pins(access_counts: dict, profile: dict, pins_per_layer: dict, n_layers: int):
    """The experts the reference's pin_from_usage / pin_nonuniform pin
    (tinygiant/cache.py:84-152), as (layer, expert) pairs in pinning order: per layer,
    the pins_per_layer[layer] most accessed experts of the calibration counts (ties: the
    smaller id first), then, while fewer are chosen, the relayout profile's
    expert_ranking[layer] in its order, skipping experts already chosen."""
    per_layer = {}
    for (layer, expert), cnt in access_counts.items():
        per_layer.setdefault(layer, []).append((-cnt, expert))
    out = []
    for layer in range(n_layers):
        n_pin = pins_per_layer.get(layer, 0)
        if n_pin <= 0:
            continue
        chosen = []
        for _, e in sorted(per_layer.get(layer, []))[:n_pin]:
            chosen.append(int(e))
        if len(chosen) < n_pin and str(layer) in profile:
            for e in profile[str(layer)]["expert_ranking"]:
                if len(chosen) >= n_pin:
                    break
                if int(e) not in chosen:
                    chosen.append(int(e))
        out.extend((layer, e) for e in chosen)
    return out


def select_hot(profile: dict, n_per_layer: int):
    """The experts the reference's pin_hot_experts pins (tinygiant/cache.py:72-82): the
    first n of every profiled layer's expert_ranking, layers in numeric order."""
    out = []
    for key in sorted(profile.keys(), key=int):
        out.extend((int(key), int(e)) for e in profile[key]["expert_ranking"][:n_per_layer])
    return out


class HostTierCache:
    def __init__(self, model, host_layers, cache_slots: int = 24, staging: int = 2, layout: str = "ggml",
                 index: dict | None = None):
        """model: an engine.MoEModel (its shape, norms and kernels); host_layers[l]: a
        pinned uint8 torch tensor holding layer l's E expert blobs (Q4_0,
        expert-contiguous relayout order) in `layout`: "ggml" blobs are repacked on the
        device after each copy, "rows" blobs (a version-4 relayout) are copied into their
        slot as they are.  index: the relayout's index.json (its activation_profile feeds
        pin_hot_experts and the backfill of pin_from_usage / pin_nonuniform)."""
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
        self.access_counts = {}                 # (layer, expert) -> requests, as the reference counts them
        self.index = index or {}
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
                # the staging ring belongs to the copy stream (_load): wait until it is done
                # with every slot before this stream reuses one
                torch.cuda.current_stream().wait_stream(self.copy_stream)
                self.stage[0].copy_(raw)
                check(self.lib.tgx_repack_experts(self.model.handle, ctypes.c_void_p(self.stage[0].data_ptr()),
                                                  ctypes.c_void_p(dst.data_ptr()), 1,
                                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), self.lib)
            self.pinned[key] = dst
        torch.cuda.synchronize()

    def _pin_pairs(self, pairs) -> int:
        by_layer = {}
        for layer, e in pairs:
            if layer < len(self.host):
                by_layer.setdefault(layer, []).append(e)
        for layer, ids in by_layer.items():
            self.pin(layer, ids)
        return sum(len(v) for v in by_layer.values())

    def pin_hot_experts(self, n_per_layer: int) -> int:
        """tinygiant/cache.py:72-82: pin the top n_per_layer experts of every layer by the
        relayout's static activation profile; resets the hit counters; returns the count."""
        profile = self.index.get("activation_profile")
        if not profile:
            return 0
        count = self._pin_pairs(select_hot(profile, n_per_layer))
        self.hits = self.misses = self.pinned_hits = 0
        return count

    def pin_from_usage(self, n_per_layer: int, n_layers: int) -> int:
        """tinygiant/cache.py:84-113: pin each layer's n_per_layer most requested experts
        since the last reset (calibration), backfilled from the static profile; resets
        the hit counters and the request counts; returns the count."""
        return self.pin_nonuniform({layer: n_per_layer for layer in range(n_layers)}, n_layers)

    def pin_nonuniform(self, pins_per_layer: dict, n_layers: int) -> int:
        """tinygiant/cache.py:115-152: pin pins_per_layer[layer] experts per layer, from
        the request counts first and the static profile after; resets the counters."""
        pairs = select_pins(self.access_counts, self.index.get("activation_profile", {}), pins_per_layer, n_layers)
        count = self._pin_pairs(pairs)
        self.hits = self.misses = self.pinned_hits = 0
        self.access_counts = {}
        return count

    def record(self, layer: int, ids):
        """Count requests of experts `ids` of `layer` without loading them (calibration
        from routing decided elsewhere)."""
        for e in ids:
            key = (layer, int(e))
            self.access_counts[key] = self.access_counts.get(key, 0) + 1

    def get(self, layer: int, expert_id: int):
        """The reference's ExpertCache.get (tinygiant/cache.py:154-160): count the request
        and return the expert, resident in HBM (a uint8 cuda tensor in the kernels'
        row-split layout).  The current stream is made to wait for its copy.  A slot's
        expert stays valid until a later request evicts it; a pinned one for the cache's
        lifetime."""
        ptrs, slots = self.resident(layer, [expert_id])
        key = (layer, int(expert_id))
        if key in self.pinned:
            return self.pinned[key]
        self.torch.cuda.current_stream().wait_event(self.ready[slots[0]])
        return self.slots[slots[0]]

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
            if count:
                self.access_counts[key] = self.access_counts.get(key, 0) + 1
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
