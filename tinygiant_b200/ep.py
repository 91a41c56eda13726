"""Experts sharded over GPUs (expert parallelism), one process per GPU.

Rank r of G holds experts [r*E/G, (r+1)*E/G) of every layer; the routers, FFN norms
and the optional shared expert (n_shared=1: slot k of every token, weight 1) are
replicated, so every rank routes every token the same way.  A token's shared-expert
output is computed by the rank holding the fewest of its routed experts.  One MoE layer
(tinygiant/engine.py:229-258 for each of T tokens) is

    tgx_ep_moe_partial   y[(t, j)] for the (token, slot) pairs whose expert is local, else 0
    all_reduce(y, SUM)   over the expert-parallel group (NCCL on GPUs)
    tgx_ep_combine       x[t] += sum_j w[t][j] * y[(t, j)] in slot order

Each element of y has one nonzero contribution, so the sum is exact and the result is
bit-identical to the single-GPU batched path (and, through it, to the CPU oracle).
The all-reduce moves T * top_k * embed floats per layer.  After enable_p2p() the
exchange is direct instead: the down kernels store each (token, slot) sum into every
rank's exchange buffer over NVLink and the combine waits on per-rank epoch flags.
moe_layer_dispatch / decode_dispatch instead shard the tokens: each rank routes its own,
sends each (token, slot) pair's Q8_0 row to its expert's holder and gets the pair's y
back (NCCL all-to-alls), so bytes per rank fall as 1/G (tgx_ep_dispatch*).
After enable_fused(), decode_step(x) runs all layers of one token in one persistent
kernel per rank (the one-GPU fused step over the local experts), the per-slot down
values crossing NVLink as tagged words inside the kernel.

    ep = EPMoEModel(rank=r, size=G, device=local_rank)
    ep.fill_synthetic(seed)            # or load_experts(layer, first, blob) for the local range
    ep.decode(X)                       # X: cuda f32[T][embed], all layers, in place
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _constants as C
from ._lib import TgxShape, check, get_lib
from .engine import _dev_ptr, _stream_handle


def expert_range(n_experts: int, rank: int, size: int):
    """(first, count) of the experts rank `rank` of `size` holds."""
    if size < 1 or not 0 <= rank < size or n_experts % size:
        raise ValueError("need 0 <= rank < size and n_experts divisible by size")
    n = n_experts // size
    return rank * n, n


def shared_owner(routed_ids, t: int, n_experts: int, size: int) -> int:
    """The rank that computes token t's shared-expert output: the one holding the fewest
    of the token's routed experts, ties to rank (t + i) mod size with the smallest i
    (the rule the partial step's kernels apply)."""
    e_n = n_experts // size
    counts = [0] * size
    for e in routed_ids:
        counts[int(e) // e_n] += 1
    best, best_n = 0, 1 << 30
    for i in range(size):
        r = (t + i) % size
        if counts[r] < best_n:
            best, best_n = r, counts[r]
    return best


class EPMoEModel:
    def __init__(self, embed=C.EMBED_DIM, inter=C.EXPERT_INTERMEDIATE, n_experts=C.N_EXPERTS,
                 top_k=C.N_EXPERTS_USED, n_layers=C.N_LAYERS, rank=0, size=1, device=0, group=None, n_shared=0):
        self.lib = get_lib()
        self.shape = TgxShape(embed, inter, n_experts, top_k, n_layers, C.RMS_EPS)
        self.embed, self.inter, self.n_experts, self.top_k, self.n_layers = embed, inter, n_experts, top_k, n_layers
        self.rank, self.size, self.device, self.group, self.n_shared = rank, size, device, group, n_shared
        h = ctypes.c_void_p()
        check(self.lib.tgx_ep_create(device, ctypes.byref(self.shape), n_shared, rank, size, ctypes.byref(h)),
              self.lib)
        self._ep = h
        first, n = ctypes.c_int(), ctypes.c_int()
        check(self.lib.tgx_ep_expert_range(h, ctypes.byref(first), ctypes.byref(n)), self.lib)
        self.first, self.n_local = first.value, n.value
        assert (self.first, self.n_local) == expert_range(n_experts, rank, size)
        self.expert_bytes = C.expert_bytes(embed, inter)
        self._y = {}

    def close(self, barrier: bool = True):
        """Free the context.  With the NVLink exchange every rank first drops its
        mappings of the others' regions, then a barrier, then the regions are freed."""
        if self._ep:
            if getattr(self, "p2p", False):
                self.lib.tgx_ep_p2p_disconnect(self._ep)
                if self.size > 1 and barrier:
                    import torch.distributed as dist
                    if dist.is_initialized():
                        dist.barrier(group=self.group)
                self.p2p = False
            self.lib.tgx_ep_destroy(self._ep)
            self._ep = None

    def __del__(self):
        try:
            self.close(barrier=False)   # never a collective from the garbage collector
        except Exception:
            pass

    # ---------------------------------------------------------------- weights
    def fill_synthetic(self, seed: int, w_sigma: float = 0.02, r_sigma: float = 0.02):
        """The weights MoEModel.fill_synthetic(seed) gives the same experts."""
        check(self.lib.tgx_ep_fill_synthetic(self._ep, seed, w_sigma, r_sigma), self.lib)

    def load_experts(self, layer: int, first: int, blob: np.ndarray):
        """ggml Q4_0 experts [first, first + n) of a layer (inside the local range)."""
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        n = blob.size // self.expert_bytes
        assert n * self.expert_bytes == blob.size
        check(self.lib.tgx_ep_load_experts(self._ep, layer, first, n, blob.ctypes.data, 0), self.lib)

    def load_shared(self, layer: int, blob: np.ndarray):
        """The layer's shared expert (n_shared = 1): one ggml Q4_0 blob gate | up | down."""
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        assert blob.size == self.expert_bytes
        check(self.lib.tgx_ep_load_shared(self._ep, layer, blob.ctypes.data, 0), self.lib)

    def read_expert(self, layer: int, e: int) -> np.ndarray:
        """Expert e (local routed id, or n_experts for the shared expert) as a ggml blob."""
        out = np.empty(self.expert_bytes, np.uint8)
        check(self.lib.tgx_ep_read_expert(self._ep, layer, e, out.ctypes.data), self.lib)
        return out

    def set_router(self, layer: int, R: np.ndarray):
        R = np.ascontiguousarray(R, dtype=np.float32)
        assert R.shape == (self.n_experts, self.embed)
        check(self.lib.tgx_ep_set_router(self._ep, layer, R.ctypes.data, 0), self.lib)

    def set_ffn_norm(self, layer: int, w: np.ndarray):
        w = np.ascontiguousarray(w, dtype=np.float32)
        assert w.shape == (self.embed,)
        check(self.lib.tgx_ep_set_ffn_norm(self._ep, layer, w.ctypes.data, 0), self.lib)

    def set_kernels(self, kernels: int):
        """0 auto, 1 dp4a, 2 tensor cores (tcgen05) for the expert matmuls (same bits);
        3 tensor cores with the fast epilogue (within the accumulation-order tolerance)."""
        check(self.lib.tgx_ep_set_kernels(self._ep, kernels), self.lib)

    def status(self, stream=None):
        check(self.lib.tgx_ep_status(self._ep, _stream_handle(stream)), self.lib)

    # ---------------------------------------------------------------- compute
    def y_buffer(self, T: int):
        """The per-step exchange buffer for T tokens (reused, one per T)."""
        import torch
        if T not in self._y:
            n = int(self.lib.tgx_ep_y_floats(self._ep, T))
            self._y[T] = torch.empty(n, dtype=torch.float32, device=torch.device("cuda", self.device))
        return self._y[T]

    def partial(self, layer: int, X, Y, stream=None):
        check(self.lib.tgx_ep_moe_partial(self._ep, layer, _dev_ptr(X), X.shape[0], _dev_ptr(Y),
                                          _stream_handle(stream)), self.lib)

    def combine(self, X, Y, stream=None):
        check(self.lib.tgx_ep_combine(self._ep, _dev_ptr(X), X.shape[0], _dev_ptr(Y), _stream_handle(stream)),
              self.lib)

    def enable_p2p(self, t_max: int, exchange=None):
        """Switch the exchange from the all-reduce to direct NVLink stores between the
        ranks' down kernels (tgx_ep_p2p_*).  exchange(bytes) -> list of every rank's bytes
        in rank order; default: torch.distributed.all_gather_object on self.group."""
        n = int(self.lib.tgx_ep_p2p_handle_bytes())
        h = (ctypes.c_uint8 * n)()
        check(self.lib.tgx_ep_p2p_init(self._ep, t_max, h), self.lib)
        mine = bytes(h)
        if exchange is None:
            if self.size == 1:
                handles = [mine]
            else:
                import torch.distributed as dist
                handles = [None] * self.size
                dist.all_gather_object(handles, mine, group=self.group)
        else:
            handles = exchange(mine)
        assert len(handles) == self.size and handles[self.rank] == mine
        buf = (ctypes.c_uint8 * (n * self.size)).from_buffer_copy(b"".join(handles))
        check(self.lib.tgx_ep_p2p_connect(self._ep, buf), self.lib)
        self.p2p = True

    def _gather_handles(self, mine: bytes, exchange):
        if exchange is not None:
            return exchange(mine)
        if self.size == 1:
            return [mine]
        import torch.distributed as dist
        handles = [None] * self.size
        dist.all_gather_object(handles, mine, group=self.group)
        return handles

    def enable_fused(self, exchange=None):
        """Set up the one-kernel decode step over the local experts (tgx_ep_fused_*):
        every rank must call it, after its weights, routers and norms are set (later
        router changes are picked up too).  exchange as for enable_p2p."""
        n = int(self.lib.tgx_ep_p2p_handle_bytes())
        h = (ctypes.c_uint8 * n)()
        check(self.lib.tgx_ep_fused_init(self._ep, h), self.lib)
        mine = bytes(h)
        handles = self._gather_handles(mine, exchange)
        assert len(handles) == self.size and handles[self.rank] == mine
        buf = (ctypes.c_uint8 * (n * self.size)).from_buffer_copy(b"".join(handles))
        check(self.lib.tgx_ep_fused_connect(self._ep, buf), self.lib)
        self.p2p = True   # close() disconnects the mappings before the barrier
        self.fused = True

    def decode_step(self, x, stream=None):
        """All layers of one token (cuda f32[embed], the same on every rank) in place,
        in one kernel per rank; every rank ends with the same x."""
        assert x.dim() == 1 and x.shape[0] == self.embed and x.is_contiguous()
        check(self.lib.tgx_ep_decode_step(self._ep, _dev_ptr(x), _stream_handle(stream)), self.lib)

    def fused_trace(self, x, stream=None) -> np.ndarray:
        """decode_step with phase stamps: u64 [layers][CTAs][32] (globaltimer ns at
        0..15, clock64 at 16..31)."""
        ctas = ctypes.c_int()
        check(self.lib.tgx_ep_fused_info(self._ep, ctypes.byref(ctas), None), self.lib)
        out = np.zeros((self.n_layers, ctas.value, 32), np.uint64)
        check(self.lib.tgx_ep_fused_trace(self._ep, _dev_ptr(x), out.ctypes.data, _stream_handle(stream)), self.lib)
        return out

    def fused_routing(self, layer: int):
        """(expert ids, weights) of the last fused step at `layer`."""
        idx = np.zeros(self.top_k, np.int32)
        w = np.zeros(self.top_k, np.float32)
        check(self.lib.tgx_ep_fused_last_routing(self._ep, layer, idx.ctypes.data, w.ctypes.data), self.lib)
        return idx, w

    def set_wait_limit(self, cycles: int):
        check(self.lib.tgx_ep_set_wait_limit(self._ep, int(cycles)), self.lib)

    def fused_status(self, stream=None):
        check(self.lib.tgx_ep_fused_status(self._ep, _stream_handle(stream)), self.lib)

    def fused_epoch(self) -> int:
        e = ctypes.c_uint()
        check(self.lib.tgx_ep_fused_epoch(self._ep, ctypes.byref(e)), self.lib)
        return e.value

    def fused_recover(self, max_over_ranks=None):
        """After a failed step on any rank: every rank calls this; it restarts all ranks'
        launch count at one above the largest (max_over_ranks(int) -> int; default: a
        MAX all-reduce over self.group)."""
        e = self.fused_epoch()
        if max_over_ranks is not None:
            top = int(max_over_ranks(e))
        elif self.size == 1:
            top = e
        else:
            import torch
            import torch.distributed as dist
            dev = "cpu" if dist.get_backend(self.group) == "gloo" else torch.device("cuda", self.device)
            t = torch.tensor([e], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            top = int(t.item())
        check(self.lib.tgx_ep_fused_reset(self._ep, top + 1), self.lib)

    # ---------------------------------------------------------------- token dispatch
    def record_bytes(self) -> int:
        return int(self.lib.tgx_ep_record_bytes(self._ep))

    def _cuda(self, name: str, n: int, dtype):
        """A reused device buffer of at least n elements (grown by doubling)."""
        import torch
        b = self._y.get(name)
        if b is None or b.numel() < n:
            b = torch.empty(max(n, 2 * (b.numel() if b is not None else 0)), dtype=dtype,
                            device=torch.device("cuda", self.device))
            self._y[name] = b
        return b[:n]

    def dispatch(self, layer: int, X, stream=None):
        """Route this rank's tokens X (cuda f32[T][embed]); returns (send, counts): the
        records grouped by destination rank (uint8 [T * slots * record_bytes]) and the
        records per rank (cuda int32 [size])."""
        import torch
        T = X.shape[0]
        ks = self.top_k + self.n_shared
        send = self._cuda("d_send", T * ks * self.record_bytes(), torch.uint8)
        counts = self._cuda("d_counts", self.size, torch.int32)
        check(self.lib.tgx_ep_dispatch(self._ep, layer, _dev_ptr(X), T, send.data_ptr(), counts.data_ptr(),
                                       _stream_handle(stream)), self.lib)
        return send, counts

    def dispatch_experts(self, layer: int, recv, n_recv: int, stream=None):
        """The expert FFNs of n_recv received records: cuda f32 [n_recv][embed]."""
        import torch
        y = self._cuda("d_yr", max(1, n_recv) * self.embed, torch.float32)[: n_recv * self.embed]
        check(self.lib.tgx_ep_dispatch_experts(self._ep, layer, recv.data_ptr() if n_recv else None, n_recv,
                                               y.data_ptr() if n_recv else None, _stream_handle(stream)), self.lib)
        return y.view(n_recv, self.embed)

    def dispatch_combine(self, X, y_back, stream=None):
        check(self.lib.tgx_ep_dispatch_combine(self._ep, _dev_ptr(X), X.shape[0], y_back.data_ptr(),
                                               _stream_handle(stream)), self.lib)

    def moe_layer_dispatch(self, layer: int, X, stream=None, stats=None):
        """MoE block `layer` for this rank's tokens X (cuda f32[T][embed]) in place, the
        pairs dispatched to their experts' holders and back with NCCL all-to-alls over
        self.group.  stats (dict), when given, accumulates the bytes this rank received."""
        import torch
        import torch.distributed as dist
        rb = self.record_bytes()
        if X.shape[0] > 0:
            send, counts = self.dispatch(layer, X, stream)
        else:   # no tokens here: still take part in every exchange
            send = self._cuda("d_send", 1, torch.uint8)
            counts = self._cuda("d_counts", self.size, torch.int32)
            counts.zero_()
        rcounts = self._cuda("d_rcounts", self.size, torch.int32)
        if self.size > 1:
            dist.all_to_all_single(rcounts, counts, group=self.group)
        else:
            rcounts.copy_(counts)
        both = torch.cat([counts, rcounts]).cpu().tolist()
        sc, rc = both[: self.size], both[self.size:]
        n_send, n_recv = sum(sc), sum(rc)
        recv = self._cuda("d_recv", max(1, n_recv) * rb, torch.uint8)[: n_recv * rb]
        if self.size > 1:
            dist.all_to_all_single(recv, send[: n_send * rb], [c * rb for c in rc], [c * rb for c in sc],
                                   group=self.group)
        else:
            recv.copy_(send[: n_send * rb])
        y = self.dispatch_experts(layer, recv, n_recv, stream)
        y_back = self._cuda("d_yback", max(1, n_send) * self.embed, torch.float32)[: n_send * self.embed]
        if self.size > 1:
            dist.all_to_all_single(y_back, y.reshape(-1), [c * self.embed for c in sc],
                                   [c * self.embed for c in rc], group=self.group)
        else:
            y_back.copy_(y.reshape(-1))
        if X.shape[0] > 0:
            self.dispatch_combine(X, y_back, stream)
        if stats is not None:
            stats["recv_bytes"] = stats.get("recv_bytes", 0) + n_recv * rb + n_send * self.embed * 4
            stats["layers"] = stats.get("layers", 0) + 1

    def decode_dispatch(self, X, stream=None, stats=None):
        """All layers chained on this rank's tokens X in place (token dispatch)."""
        for layer in range(self.n_layers):
            self.moe_layer_dispatch(layer, X, stream, stats)

    def enable_dispatch_p2p(self, t_max: int, exchange=None):
        """Token dispatch without host syncs (tgx_ep_dispatch_p2p_*): records and y rows
        travel through the ranks' IPC regions over NVLink.  t_max: the most tokens a rank
        passes to one call.  exchange as for enable_p2p."""
        n = int(self.lib.tgx_ep_p2p_handle_bytes())
        h = (ctypes.c_uint8 * n)()
        check(self.lib.tgx_ep_dispatch_p2p_init(self._ep, t_max, h), self.lib)
        mine = bytes(h)
        handles = self._gather_handles(mine, exchange)
        assert len(handles) == self.size and handles[self.rank] == mine
        buf = (ctypes.c_uint8 * (n * self.size)).from_buffer_copy(b"".join(handles))
        check(self.lib.tgx_ep_dispatch_p2p_connect(self._ep, buf), self.lib)
        self.p2p = True   # close() disconnects the mappings before the barrier

    def moe_layer_dispatch_p2p(self, layer: int, X, stream=None):
        """MoE block `layer` for this rank's tokens X (cuda f32[T][embed], 1 <= T <= t_max) in
        place; every rank calls it for the same layers in the same order."""
        assert X.dim() == 2 and X.shape[1] == self.embed and X.shape[0] >= 1
        check(self.lib.tgx_ep_moe_layer_dispatch_p2p(self._ep, layer, _dev_ptr(X), X.shape[0],
                                                     _stream_handle(stream)), self.lib)

    def decode_dispatch_p2p(self, X, stream=None):
        for layer in range(self.n_layers):
            self.moe_layer_dispatch_p2p(layer, X, stream)

    def dispatch_p2p_counts(self):
        """(records received, records sent) by the last call."""
        r, s = ctypes.c_int(), ctypes.c_int()
        check(self.lib.tgx_ep_dispatch_p2p_counts(self._ep, ctypes.byref(r), ctypes.byref(s)), self.lib)
        return r.value, s.value

    def dispatch_p2p_status(self, stream=None):
        check(self.lib.tgx_ep_dispatch_p2p_status(self._ep, _stream_handle(stream)), self.lib)

    def p2p_status(self, stream=None):
        check(self.lib.tgx_ep_p2p_status(self._ep, _stream_handle(stream)), self.lib)

    def moe_layer(self, layer: int, X, stream=None):
        """MoE block `layer` for the T tokens of X (cuda f32[T][embed]) in place."""
        assert X.dim() == 2 and X.shape[1] == self.embed
        if getattr(self, "p2p", False):
            check(self.lib.tgx_ep_moe_layer_p2p(self._ep, layer, _dev_ptr(X), X.shape[0], _stream_handle(stream)),
                  self.lib)
            return
        import torch.distributed as dist
        Y = self.y_buffer(X.shape[0])
        self.partial(layer, X, Y, stream)
        if self.size > 1:
            dist.all_reduce(Y, op=dist.ReduceOp.SUM, group=self.group)
        self.combine(X, Y, stream)

    def decode(self, X, stream=None):
        """All layers chained on X in place."""
        for layer in range(self.n_layers):
            self.moe_layer(layer, X, stream)
