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

H, I, E, K, T, L = 256, 256, 8, 4, 3, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(seed=7):
    from oracle import oracle as O
    blobs = [O.quantize_q4_0(O.fill_normal(E * 3 * H * I, seed + 2 * l, 0.05)) for l in range(L)]
    routers = [O.fill_normal(E * H, seed + 2 * l + 1, 0.05).reshape(E, H) for l in range(L)]
    norms = [np.linspace(0.5, 1.5, H).astype(np.float32) for _ in range(L)]
    X = np.stack([O.fill_normal(H, 100 + t, 1.0) for t in range(T)])
    return blobs, routers, norms, X


def _worker(rank, world, port, out_path):
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from tinygiant_b200.ep import expert_range
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blobs, routers, norms, X = _model()
        first, n = expert_range(E, rank, world)
        eb = O.expert_bytes(H, I)
        X = X.copy()
        for l in range(L):
            Y = np.zeros((T, K, H), np.float32)
            W = np.zeros((T, K), np.float32)
            for t in range(T):
                _, idx, w, _ = O.moe_block(blobs[l], routers[l], X[t], K, H, I, normw=norms[l])
                W[t] = w
                scale = np.float32(O.rms_scale(X[t]))
                normed = (X[t] * scale).astype(np.float32) * norms[l]
                for j, e in enumerate(idx):
                    if first <= e < first + n:
                        Y[t, j] = O.expert_stages(blobs[l][e * eb:(e + 1) * eb], normed, H, I)["y"]
            Yt = torch.from_numpy(Y)
            dist.all_reduce(Yt, op=dist.ReduceOp.SUM)
            Y = Yt.numpy()
            for t in range(T):
                acc = np.zeros(H, np.float32)
                for j in range(K):
                    acc = (acc + (W[t, j] * Y[t, j]).astype(np.float32)).astype(np.float32)
                X[t] = (X[t] + acc).astype(np.float32)
        if rank == 0:
            np.save(out_path, X)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_exchange_matches_unsharded_oracle(tmp_path, world):
    import torch.multiprocessing as mp
    from oracle import oracle as O
    out = str(tmp_path / "x.npy")
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    got = np.load(out)
    blobs, routers, norms, X = _model()
    ref = X.copy()
    for l in range(L):
        ref = O.moe_block_batched(blobs[l], routers[l], ref, K, H, I, normw=norms[l])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_expert_range_partitions():
    from tinygiant_b200.ep import expert_range
    for E_, G in ((128, 1), (128, 2), (128, 8), (256, 8), (8, 4)):
        spans = [expert_range(E_, r, G) for r in range(G)]
        assert [f for f, _ in spans] == [r * (E_ // G) for r in range(G)]
        assert sum(n for _, n in spans) == E_
    for bad in ((128, 3, 3), (128, 0, 3), (10, 0, 4), (8, 2, 2)):
        with pytest.raises(ValueError):
            expert_range(*bad)
