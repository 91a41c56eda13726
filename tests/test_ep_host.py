"""The expert-parallel exchange scheme on CPU: world_size 2 and 4 `gloo` ranks, the
oracle as the per-rank compute.  Each rank computes y for the (token, slot) pairs whose
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
