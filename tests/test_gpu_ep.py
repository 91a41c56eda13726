"""GPU parity of expert parallelism (tgx_ep_*): the sharded path must equal the
single-GPU batched path with all experts (itself bit-exact to the CPU oracle) bit for
bit.  On one GPU, G ranks are emulated by G contexts on the same device whose y
buffers are summed with torch (each element has one nonzero term, so the sum is
exact); no kernel waits on another.  With two or more GPUs, a torchrun job runs the
real NCCL exchange (tests/ep_worker.py)."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8


@pytest.mark.parametrize("G", [2, 4, 8])
@pytest.mark.parametrize("T", [1, 5, 64, 300])
def test_ep_emulated_matches_single_gpu(G, T):
    import torch
    from tinygiant_b200.engine import MoEModel
    from tinygiant_b200.ep import EPMoEModel
    L = 2
    full = MoEModel(H, I, E, K, L)
    full.fill_synthetic(77)
    ranks = [EPMoEModel(H, I, E, K, L, rank=r, size=G) for r in range(G)]
    for ep in ranks:
        ep.fill_synthetic(77)
    g = torch.Generator(device="cuda").manual_seed(T)
    X = torch.randn(T, H, generator=g, device="cuda")
    Xr = X.clone()
    full.decode_batched(Xr)
    Ys = [ep.y_buffer(T) for ep in ranks]
    for layer in range(L):
        for ep, Y in zip(ranks, Ys):
            ep.partial(layer, X, Y)
        total = Ys[0].clone()
        for Y in Ys[1:]:
            total += Y
        ranks[0].combine(X, total)
    torch.cuda.synchronize()
    assert torch.equal(X.view(torch.int32), Xr.view(torch.int32))
    # each rank's y is zero exactly where another rank holds the slot's expert
    nz = torch.stack([(Y.view(T, K, H) != 0).any(dim=2) for Y in Ys])
    assert int(nz.sum(dim=0).max()) <= 1
    for ep in ranks:
        ep.close()
    full.close()


def _emulate(ranks, X, L):
    """G ranks on one GPU: partial on each, an exact torch sum of y, combine."""
    T = X.shape[0]
    Ys = [ep.y_buffer(T) for ep in ranks]
    for layer in range(L):
        for ep, Y in zip(ranks, Ys):
            ep.partial(layer, X, Y)
        total = Ys[0].clone()
        for Y in Ys[1:]:
            total += Y
        ranks[0].combine(X, total)


@pytest.mark.parametrize("G,kernels", [(1, 1), (2, 1), (4, 1), (1, 2), (2, 2)])
def test_ep_shared_expert_matches_oracle(oracle, G, kernels):
    # host-made weights (oracle quantiser), a shared expert, two chained layers
    import numpy as np
    import torch
    from tinygiant_b200.ep import EPMoEModel
    h, i, e, k, L, T = 512, 256, 16, 4, 2, 6
    rng = np.random.default_rng(11)
    eb = oracle.expert_bytes(h, i)
    blobs = [oracle.quantize_q4_0(oracle.fill_normal(e * 3 * h * i, 30 + l, 0.05)) for l in range(L)]
    shared = [oracle.quantize_q4_0(oracle.fill_normal(3 * h * i, 60 + l, 0.05)) for l in range(L)]
    routers = [oracle.fill_normal(e * h, 90 + l, 0.05).reshape(e, h) for l in range(L)]
    norms = [rng.uniform(0.5, 1.5, h).astype(np.float32) for _ in range(L)]
    ranks = [EPMoEModel(h, i, e, k, L, rank=r, size=G, n_shared=1) for r in range(G)]
    for ep in ranks:
        ep.set_kernels(kernels)
        for l in range(L):
            ep.load_experts(l, ep.first, blobs[l][ep.first * eb:(ep.first + ep.n_local) * eb])
            ep.load_shared(l, shared[l])
            ep.set_router(l, routers[l])
            ep.set_ffn_norm(l, norms[l])
    X0 = rng.standard_normal((T, h)).astype(np.float32)
    X = torch.from_numpy(X0.copy()).cuda()
    _emulate(ranks, X, L)
    torch.cuda.synchronize()
    ref = X0.copy()
    for l in range(L):
        ref = oracle.moe_block_batched(blobs[l], routers[l], ref, k, h, i, normw=norms[l], shared=shared[l])
    assert np.array_equal(X.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    for ep in ranks:
        ep.close()


def test_ep_dsv3_width_matches_oracle(oracle):
    # DeepSeek-V3 widths (hidden 7168, intermediate 2048): 16-row gate/up units and the
    # separate Q8_0 pass over h; 16 routed experts + the shared one, 2 emulated ranks
    import numpy as np
    import torch
    from tinygiant_b200.ep import EPMoEModel
    h, i, e, k, L, T, G = 7168, 2048, 16, 8, 1, 2, 2
    rng = np.random.default_rng(5)
    R = (rng.standard_normal((e, h)) * 0.02).astype(np.float32)
    ranks = [EPMoEModel(h, i, e, k, L, rank=r, size=G, n_shared=1) for r in range(G)]
    for r, ep in enumerate(ranks):
        ep.fill_synthetic(123)
        ep.set_router(0, R)
        ep.set_kernels(1 + r % 2)          # dp4a on one rank, tensor cores on the other
    blob = np.concatenate([ranks[r].read_expert(0, x) for r in range(G)
                           for x in range(ranks[r].first, ranks[r].first + ranks[r].n_local)])
    shared = ranks[0].read_expert(0, e)
    assert np.array_equal(shared, ranks[1].read_expert(0, e))      # replicated
    X0 = rng.standard_normal((T, h)).astype(np.float32)
    X = torch.from_numpy(X0.copy()).cuda()
    _emulate(ranks, X, L)
    torch.cuda.synchronize()
    ref = oracle.moe_block_batched(blob, R, X0, k, h, i, shared=shared, n_threads=0)
    assert np.array_equal(X.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    for ep in ranks:
        ep.close()


def test_ep_fast_epilogue_same_bits_on_every_sharding():
    # kernels=3 (fast epilogue): each (row, token) sum is one fma chain over the blocks,
    # whatever the tile or rank, so 1, 2 and 4 emulated ranks give the same bits
    import numpy as np
    import torch
    from tinygiant_b200.ep import EPMoEModel
    h, i, e, k, L, T = 2048, 768, 16, 4, 2, 96
    rng = np.random.default_rng(3)
    X0 = rng.standard_normal((T, h)).astype(np.float32)
    outs = []
    for G in (1, 2, 4):
        ranks = [EPMoEModel(h, i, e, k, L, rank=r, size=G) for r in range(G)]
        for ep in ranks:
            ep.fill_synthetic(77)
            ep.set_kernels(3)
        X = torch.from_numpy(X0.copy()).cuda()
        _emulate(ranks, X, L)
        torch.cuda.synchronize()
        outs.append(X.cpu().numpy())
        for ep in ranks:
            ep.close()
    assert np.isfinite(outs[0]).all() and not np.array_equal(outs[0], X0)
    for o in outs[1:]:
        assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))


@pytest.mark.parametrize("T,kernels", [(1, 0), (7, 1), (300, 2)])
def test_ep_p2p_single_rank_matches_batched(T, kernels):
    # the NVLink-exchange entry point with one rank (its own region, its own flags):
    # chained layers (both buffer parities), eager and graph-replayed, against the
    # single-GPU batched path
    import torch
    from tinygiant_b200.engine import MoEModel
    from tinygiant_b200.ep import EPMoEModel
    L = 3
    full = MoEModel(H, I, E, K, L)
    full.fill_synthetic(31)
    ep = EPMoEModel(H, I, E, K, L, rank=0, size=1)
    ep.fill_synthetic(31)
    ep.set_kernels(kernels)
    ep.enable_p2p(512)
    X = torch.randn(T, H, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda")
    want = X.clone()
    full.decode_batched(want)
    got = X.clone()
    ep.decode(got)
    ep.p2p_status()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    graph = torch.cuda.CUDAGraph()
    Xg = X.clone()
    with torch.cuda.graph(graph):
        ep.decode(Xg)
    for _ in range(2):
        Xg.copy_(X)
        graph.replay()
        ep.p2p_status()
        assert torch.equal(Xg.view(torch.int32), want.view(torch.int32))
    del graph
    ep.close()
    full.close()


def test_ep_rejects_foreign_experts():
    import numpy as np
    from tinygiant_b200._lib import TinyGiantError
    from tinygiant_b200.ep import EPMoEModel
    ep = EPMoEModel(H, I, E, K, 1, rank=1, size=4)
    assert (ep.first, ep.n_local) == (32, 32)
    blob = np.zeros(ep.expert_bytes, np.uint8)
    ep.load_experts(0, 40, blob)
    with pytest.raises(TinyGiantError):
        ep.load_experts(0, 0, blob)          # expert 0 belongs to rank 0
    ep.close()


def _dispatch_emulated(ranks, shards, L):
    """Token dispatch of G ranks on one GPU: each rank's dispatch, the all-to-alls as
    tensor copies (records to their destinations in source-rank order, y rows back in
    each source's send order), the experts and the combine; no kernel waits on another."""
    import torch
    G = len(ranks)
    rb = ranks[0].record_bytes()
    for layer in range(L):
        sends = [ep.dispatch(layer, xs) for ep, xs in zip(ranks, shards)]
        counts = [c.cpu().tolist() for _, c in sends]          # counts[src][dst]
        ys = []
        for q, ep in enumerate(ranks):
            parts = [sends[src][0][sum(counts[src][:q]) * rb:(sum(counts[src][:q]) + counts[src][q]) * rb]
                     for src in range(G)]
            n = sum(counts[src][q] for src in range(G))
            ys.append(ep.dispatch_experts(layer, torch.cat(parts), n).clone())
        for src, ep in enumerate(ranks):
            parts = []
            for q in range(G):
                off = sum(counts[s2][q] for s2 in range(src))
                parts.append(ys[q][off:off + counts[src][q]])
            ep.dispatch_combine(shards[src], torch.cat(parts).reshape(-1))


@pytest.mark.parametrize("G,T,kernels", [(1, 5, 0), (2, 7, 1), (4, 64, 0), (8, 300, 2), (8, 41, 1)])
def test_ep_dispatch_emulated_matches_single_gpu(G, T, kernels):
    # every rank holds its own tokens; the (token, slot) pairs travel to their experts'
    # holders and back: the result must be the single-GPU batched path's, bit for bit
    import torch
    from tinygiant_b200.engine import MoEModel
    from tinygiant_b200.ep import EPMoEModel
    L = 2
    full = MoEModel(H, I, E, K, L)
    full.fill_synthetic(77)
    ranks = [EPMoEModel(H, I, E, K, L, rank=r, size=G) for r in range(G)]
    for ep in ranks:
        ep.fill_synthetic(77)
        ep.set_kernels(kernels)
    X = torch.randn(T, H, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda")
    want = X.clone()
    full.decode_batched(want)
    shards = [s.contiguous() for s in torch.tensor_split(X.clone(), G)]
    _dispatch_emulated(ranks, shards, L)
    for ep in ranks:
        ep.status()
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(shards).view(torch.int32), want.view(torch.int32))
    # a record is the 16-byte header and the Q8_0 row: 2,176 bytes at embed 2048
    assert ranks[0].record_bytes() == 16 + H // 32 * 34
    for ep in ranks:
        ep.close()
    full.close()


@pytest.mark.parametrize("G", [1, 2, 4])
def test_ep_dispatch_shared_expert_matches_oracle(oracle, G):
    # host-made weights, a shared expert (dispatched to the token's own rank), two layers
    import numpy as np
    import torch
    from tinygiant_b200.ep import EPMoEModel
    h, i, e, k, L, T = 512, 256, 16, 4, 2, 9
    rng = np.random.default_rng(12)
    eb = oracle.expert_bytes(h, i)
    blobs = [oracle.quantize_q4_0(oracle.fill_normal(e * 3 * h * i, 31 + l, 0.05)) for l in range(L)]
    shared = [oracle.quantize_q4_0(oracle.fill_normal(3 * h * i, 61 + l, 0.05)) for l in range(L)]
    routers = [oracle.fill_normal(e * h, 91 + l, 0.05).reshape(e, h) for l in range(L)]
    norms = [rng.uniform(0.5, 1.5, h).astype(np.float32) for _ in range(L)]
    ranks = [EPMoEModel(h, i, e, k, L, rank=r, size=G, n_shared=1) for r in range(G)]
    for ep in ranks:
        for l in range(L):
            ep.load_experts(l, ep.first, blobs[l][ep.first * eb:(ep.first + ep.n_local) * eb])
            ep.load_shared(l, shared[l])
            ep.set_router(l, routers[l])
            ep.set_ffn_norm(l, norms[l])
    X0 = rng.standard_normal((T, h)).astype(np.float32)
    shards = [torch.from_numpy(s.copy()).cuda() for s in np.array_split(X0, G)]
    _dispatch_emulated(ranks, shards, L)
    torch.cuda.synchronize()
    ref = X0.copy()
    for l in range(L):
        ref = oracle.moe_block_batched(blobs[l], routers[l], ref, k, h, i, normw=norms[l], shared=shared[l])
    got = torch.cat(shards).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    for ep in ranks:
        ep.close()


@pytest.mark.parametrize("T,kernels", [(1, 1), (9, 0), (300, 2)])
def test_ep_dispatch_p2p_single_rank_matches_batched(T, kernels):
    # the device-side dispatch with one rank (its own region and flags): chained layers
    # (both buffer halves), eager and graph-replayed, against the single-GPU batched path
    import torch
    from tinygiant_b200.engine import MoEModel
    from tinygiant_b200.ep import EPMoEModel
    L = 3
    full = MoEModel(H, I, E, K, L)
    full.fill_synthetic(33)
    ep = EPMoEModel(H, I, E, K, L, rank=0, size=1)
    ep.fill_synthetic(33)
    ep.set_kernels(kernels)
    ep.enable_dispatch_p2p(T)
    X = torch.randn(T, H, generator=torch.Generator(device="cuda").manual_seed(T + 1), device="cuda")
    want = X.clone()
    full.decode_batched(want)
    got = X.clone()
    ep.decode_dispatch_p2p(got)
    ep.dispatch_p2p_status()
    ep.status()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    assert ep.dispatch_p2p_counts() == (T * K, T * K)
    graph = torch.cuda.CUDAGraph()
    Xg = X.clone()
    with torch.cuda.graph(graph):
        ep.decode_dispatch_p2p(Xg)
    for _ in range(2):
        Xg.copy_(X)
        graph.replay()
        ep.dispatch_p2p_status()
        assert torch.equal(Xg.view(torch.int32), want.view(torch.int32))
    del graph
    ep.close()
    full.close()


def test_ep_dispatch_p2p_shared_expert_matches_oracle(oracle):
    # the device-side dispatch with a shared expert (its slot goes to the token's own rank),
    # one rank, host-made weights, two layers, against the oracle
    import numpy as np
    import torch
    from tinygiant_b200.ep import EPMoEModel
    h, i, e, k, L, T = 512, 256, 16, 4, 2, 7
    rng = np.random.default_rng(21)
    blobs = [oracle.quantize_q4_0(oracle.fill_normal(e * 3 * h * i, 41 + l, 0.05)) for l in range(L)]
    shared = [oracle.quantize_q4_0(oracle.fill_normal(3 * h * i, 71 + l, 0.05)) for l in range(L)]
    routers = [oracle.fill_normal(e * h, 81 + l, 0.05).reshape(e, h) for l in range(L)]
    norms = [rng.uniform(0.5, 1.5, h).astype(np.float32) for _ in range(L)]
    ep = EPMoEModel(h, i, e, k, L, rank=0, size=1, n_shared=1)
    for l in range(L):
        ep.load_experts(l, 0, blobs[l])
        ep.load_shared(l, shared[l])
        ep.set_router(l, routers[l])
        ep.set_ffn_norm(l, norms[l])
    ep.enable_dispatch_p2p(T)
    X0 = rng.standard_normal((T, h)).astype(np.float32)
    X = torch.from_numpy(X0.copy()).cuda()
    ep.decode_dispatch_p2p(X)
    ep.dispatch_p2p_status()
    ref = X0.copy()
    for l in range(L):
        ref = oracle.moe_block_batched(blobs[l], routers[l], ref, k, h, i, normw=norms[l], shared=shared[l])
    assert np.array_equal(X.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert ep.dispatch_p2p_counts() == (T * (k + 1), T * (k + 1))
    ep.close()


def test_ep_fused_single_rank_matches_decode_step():
    # the one-kernel EP step with one rank (every expert local, its own y buffer): odd and
    # even step counts (both buffer halves), a router changed after set-up, a graph replay,
    # against the one-GPU fused step
    import numpy as np
    import torch
    from tinygiant_b200.engine import MoEModel
    from tinygiant_b200.ep import EPMoEModel
    L = 3
    full = MoEModel(H, I, E, K, L)
    full.fill_synthetic(41)
    ep = EPMoEModel(H, I, E, K, L, rank=0, size=1)
    ep.fill_synthetic(41)
    ep.enable_fused()
    R = (np.random.default_rng(3).standard_normal((E, H)) * 0.02).astype(np.float32)
    full.set_router(1, R)
    ep.set_router(1, R)
    g = torch.Generator(device="cuda").manual_seed(5)
    for _ in range(3):
        x = torch.randn(H, generator=g, device="cuda")
        want = x.clone()
        full.decode_step(want, eager=True)
        got = x.clone()
        ep.decode_step(got)
        ep.fused_status()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32))
        for layer in range(L):
            idx, w = ep.fused_routing(layer)
            ridx, rw, _ = full.last_routing(layer)
            assert np.array_equal(idx, ridx) and np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    graph = torch.cuda.CUDAGraph()
    xg = torch.empty(H, device="cuda")
    with torch.cuda.graph(graph):
        ep.decode_step(xg)
    for _ in range(2):
        x = torch.randn(H, generator=g, device="cuda")
        want = x.clone()
        full.decode_step(want, eager=True)
        xg.copy_(x)
        graph.replay()
        ep.fused_status()
        assert torch.equal(xg.view(torch.int32), want.view(torch.int32))
    del graph
    ep.close()
    full.close()


@pytest.mark.parametrize("mode,layers,repeat,skip", [("nccl", 3, 1, "0"), ("p2p", 3, 1, "0"), ("p2p", 3, 4, "0"),
                                                     ("p2p", 1, 5, "0"), ("p2p", 3, 2, "1"),
                                                     ("fused", 3, 3, "0"), ("fused", 2, 2, "1"),
                                                     ("fused", 48, 1, "0"), ("dispatch", 3, 2, "0"),
                                                     ("dispatch_p2p", 3, 3, "0"), ("dispatch_p2p", 2, 1, "1")])
def test_ep_multi_gpu_matches_single_gpu(mode, layers, repeat, skip):
    # p2p: the exchange by direct NVLink stores and flags instead of the all-reduce; fused:
    # one kernel per rank and token; odd layer counts with several decodes back to back
    # reuse the receive buffers across decode boundaries; 48 layers is the benchmarked
    # model
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    # skip = 1: afterwards rank 1 skips one step and rank 0 must report TG_ETIMEOUT
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", EP_MODE=mode, EP_LAYERS=str(layers), EP_REPEAT=str(repeat),
               EP_SKIP=skip)
    port = 29531 + ("nccl", "p2p", "fused", "dispatch", "dispatch_p2p").index(mode) + 5 * layers + 200 * repeat + \
        1000 * int(skip)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           str(ROOT / "tests" / "ep_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    first = r.stderr.find("Traceback")                 # a worker's own error, ahead of torchrun's summary
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[max(0, first):][:3000]
    assert "bit-identical" in r.stdout
