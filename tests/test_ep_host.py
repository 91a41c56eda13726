"""The expert-parallel exchange schemes on CPU: world_size 2 and 4 `gloo` ranks, the
oracle as the per-rank compute: the all-reduce of y over replicated tokens, and token
dispatch (EPMoEModel.moe_layer_dispatch's host logic).  Each rank computes y for the (token, slot) pairs whose
expert it holds (zeros elsewhere), the ranks all-reduce y, and every rank combines in
slot order; the result must equal the oracle's unsharded MoE block bit for bit
(tinygiant/engine.py:229-258).  Also the expert partition itself."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

H, I, E, K, T, L = 256, 256, 8, 4, 5, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(seed=7):
    from oracle import oracle as O
    blobs = [O.quantize_q4_0(O.fill_normal(E * 3 * H * I, seed + 2 * l, 0.05)) for l in range(L)]
    routers = [O.fill_normal(E * H, seed + 2 * l + 1, 0.05).reshape(E, H) for l in range(L)]
    norms = [np.linspace(0.5, 1.5, H).astype(np.float32) for _ in range(L)]
    shared = [O.quantize_q4_0(O.fill_normal(3 * H * I, seed + 50 + l, 0.05)) for l in range(L)]
    X = np.stack([O.fill_normal(H, 100 + t, 1.0) for t in range(T)])
    return blobs, routers, norms, shared, X


def _worker(rank, world, port, out_path, with_shared):
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from tinygiant_b200.ep import expert_range
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tinygiant_b200.ep import shared_owner
        blobs, routers, norms, shared, X = _model()
        first, n = expert_range(E, rank, world)
        eb = O.expert_bytes(H, I)
        KS = K + (1 if with_shared else 0)
        X = X.copy()
        for l in range(L):
            Y = np.zeros((T, KS, H), np.float32)
            W = np.ones((T, KS), np.float32)          # the shared slot has weight 1
            for t in range(T):
                _, idx, w, _ = O.moe_block(blobs[l], routers[l], X[t], K, H, I, normw=norms[l])
                W[t, :K] = w
                scale = np.float32(O.rms_scale(X[t]))
                normed = (X[t] * scale).astype(np.float32) * norms[l]
                for j, e in enumerate(idx):
                    if first <= e < first + n:
                        Y[t, j] = O.expert_stages(blobs[l][e * eb:(e + 1) * eb], normed, H, I)["y"]
                if with_shared and shared_owner(idx, t, E, world) == rank:
                    Y[t, K] = O.expert_stages(shared[l], normed, H, I)["y"]
            Yt = torch.from_numpy(Y)
            dist.all_reduce(Yt, op=dist.ReduceOp.SUM)
            Y = Yt.numpy()
            for t in range(T):
                acc = np.zeros(H, np.float32)
                for j in range(KS):
                    acc = (acc + (W[t, j] * Y[t, j]).astype(np.float32)).astype(np.float32)
                X[t] = (X[t] + acc).astype(np.float32)
        if rank == 0:
            np.save(out_path, X)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,with_shared", [(2, False), (4, False), (2, True), (4, True)])
def test_ep_exchange_matches_unsharded_oracle(tmp_path, world, with_shared):
    import torch.multiprocessing as mp
    from oracle import oracle as O
    out = str(tmp_path / "x.npy")
    mp.start_processes(_worker, args=(world, _free_port(), out, with_shared), nprocs=world, start_method="spawn",
                       join=True)
    got = np.load(out)
    blobs, routers, norms, shared, X = _model()
    ref = X.copy()
    for l in range(L):
        ref = O.moe_block_batched(blobs[l], routers[l], ref, K, H, I, normw=norms[l],
                                  shared=shared[l] if with_shared else None)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


class _OracleDispatch:
    """EPMoEModel's token-dispatch host logic (moe_layer_dispatch: the count and record
    all-to-alls, the reverse all-to-all of y, the sizes) on CPU tensors, with the three
    device steps done by the oracle: routing of this rank's tokens, one record per
    (token, slot) pair in destination-rank order (the shared slot stays here), the
    experts of received records, the combine in slot order.  A record carries the expert
    id, the pair index and the normed input row as floats."""

    def __init__(self, rank, world, model, with_shared):
        from oracle import oracle as O
        from tinygiant_b200.ep import EPMoEModel, expert_range
        self.O, self.rank, self.size, self.group = O, rank, world, None
        self.blobs, self.routers, self.norms, self.shared, _ = model
        self.first, self.n_local = expert_range(E, rank, world)
        self.top_k, self.n_shared, self.embed, self.n_layers = K, 1 if with_shared else 0, H, L
        self.eb = O.expert_bytes(H, I)
        self._y = {}
        self.moe_layer_dispatch = EPMoEModel.moe_layer_dispatch.__get__(self)
        self.decode_dispatch = EPMoEModel.decode_dispatch.__get__(self)

    def record_bytes(self):
        return 16 + 4 * H

    def _cuda(self, name, n, dtype):
        import torch
        b = self._y.get(name)
        if b is None or b.numel() < n:
            b = torch.zeros(max(n, 1), dtype=dtype)
            self._y[name] = b
        return b[:n]

    def dispatch(self, layer, X, stream=None):
        import torch
        O, ks = self.O, self.top_k + self.n_shared
        x = X.numpy()
        recs, dest, self.w = [], [], np.ones((len(x), ks), np.float32)
        for t in range(len(x)):
            _, idx, w, _ = O.moe_block(self.blobs[layer], self.routers[layer], x[t], K, H, I, normw=self.norms[layer])
            self.w[t, :K] = w
            normed = (x[t] * np.float32(O.rms_scale(x[t]))).astype(np.float32) * self.norms[layer]
            for j in range(ks):
                e = int(idx[j]) if j < K else E
                hdr = np.array([e, t * ks + j, 0, 0], np.int32).tobytes()
                recs.append(hdr + normed.astype(np.float32).tobytes())
                dest.append(e // self.n_local if j < K else self.rank)
        order = sorted(range(len(recs)), key=lambda i: dest[i])          # destination-major
        self.slot = np.empty(len(recs), np.int64)
        self.slot[order] = np.arange(len(recs))
        send = torch.frombuffer(bytearray(b"".join(recs[i] for i in order)), dtype=torch.uint8)
        counts = torch.tensor(np.bincount(dest, minlength=self.size), dtype=torch.int32)
        return send, counts

    def dispatch_experts(self, layer, recv, n_recv, stream=None):
        import torch
        rb, out = self.record_bytes(), np.zeros((n_recv, H), np.float32)
        raw = recv.numpy().tobytes()
        for i in range(n_recv):
            r = raw[i * rb:(i + 1) * rb]
            e = int(np.frombuffer(r[:4], np.int32)[0])
            normed = np.frombuffer(r[16:], np.float32)
            blob = self.shared[layer] if e == E else self.blobs[layer][e * self.eb:(e + 1) * self.eb]
            assert e == E or self.first <= e < self.first + self.n_local
            out[i] = self.O.expert_stages(blob, normed, H, I)["y"]
        return torch.from_numpy(out)

    def dispatch_combine(self, X, y_back, stream=None):
        ks = self.top_k + self.n_shared
        y = y_back.numpy().reshape(-1, H)
        x = X.numpy()
        for t in range(len(x)):
            acc = np.zeros(H, np.float32)
            for j in range(ks):
                acc = (acc + (self.w[t, j] * y[self.slot[t * ks + j]]).astype(np.float32)).astype(np.float32)
            x[t] = (x[t] + acc).astype(np.float32)


def _dispatch_worker(rank, world, port, out_path, with_shared):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = _model()
        ep = _OracleDispatch(rank, world, model, with_shared)
        X = torch.from_numpy(np.array_split(model[4], world)[rank].copy())
        stats = {}
        ep.decode_dispatch(X, stats=stats)
        parts = [None] * world
        dist.all_gather_object(parts, (X.numpy(), stats["recv_bytes"]))
        if rank == 0:
            np.save(out_path, np.concatenate([p[0] for p in parts]))
            np.save(out_path + ".bytes.npy", np.array([p[1] for p in parts]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,with_shared", [(2, False), (4, False), (2, True)])
def test_token_dispatch_matches_unsharded_oracle(tmp_path, world, with_shared):
    # each rank holds its own share of the tokens; pairs travel to their experts' holders
    # and back through gloo all-to-alls driven by EPMoEModel.moe_layer_dispatch
    import torch.multiprocessing as mp
    from oracle import oracle as O
    out = str(tmp_path / "x.npy")
    mp.start_processes(_dispatch_worker, args=(world, _free_port(), out, with_shared), nprocs=world,
                       start_method="spawn", join=True)
    got = np.load(out)
    blobs, routers, norms, shared, X = _model()
    ref = X.copy()
    for l in range(L):
        ref = O.moe_block_batched(blobs[l], routers[l], ref, K, H, I, normw=norms[l],
                                  shared=shared[l] if with_shared else None)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # every rank received records and y rows, and no rank all T tokens' pairs
    recv = np.load(out + ".bytes.npy")
    ks = K + (1 if with_shared else 0)
    assert (recv > 0).all() and recv.max() < L * T * ks * (16 + 4 * H + 4 * H)


def test_shared_owner_rule():
    from tinygiant_b200.ep import shared_owner
    # 8 experts over 4 ranks (2 each): the rank with the fewest routed slots, rotation for ties
    assert shared_owner([0, 1, 2, 3], 0, 8, 4) == 2          # ranks 2, 3 hold none; 2 first from t=0
    assert shared_owner([0, 1, 2, 3], 3, 8, 4) == 3          # from t=3 the rotation starts at rank 3
    assert shared_owner([0, 2, 4, 6], 1, 8, 4) == 1          # all hold one: rank (t mod 4)
    assert shared_owner([5], 0, 8, 1) == 0
    # balance at batch 1: over many tokens each rank takes a share
    rng = np.random.default_rng(0)
    owners = [shared_owner(rng.choice(256, 8, replace=False), t, 256, 8) for t in range(4000)]
    counts = np.bincount(owners, minlength=8)
    assert counts.min() > 0.08 * 4000


def test_expert_range_partitions():
    from tinygiant_b200.ep import expert_range
    for E_, G in ((128, 1), (128, 2), (128, 8), (256, 8), (8, 4)):
        spans = [expert_range(E_, r, G) for r in range(G)]
        assert [f for f, _ in spans] == [r * (E_ // G) for r in range(G)]
        assert sum(n for _, n in spans) == E_
    for bad in ((128, 3, 3), (128, 0, 3), (10, 0, 4), (8, 2, 2)):
        with pytest.raises(ValueError):
            expert_range(*bad)
