"""GPU parity of the host tier: experts copied on demand from pinned host memory
into HBM slots (and a few pinned in HBM) give exactly the MoE block the oracle
computes for the same routing (tinygiant/engine.py:238-258 expert order), across
misses, hits, evictions and prefetches."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def oracle_block(oracle, blob, x, ids, w, H, I, normw):
    eb = oracle.expert_bytes(H, I)
    scale = oracle.rms_scale(x)
    normed = (x * np.float32(scale)) * normw
    moe = np.zeros(H, np.float32)
    for e, wj in zip(ids, w):
        oracle.expert_forward(blob[e * eb:(e + 1) * eb], normed, moe, float(wj), H, I, 1)
    return x + moe


@pytest.mark.parametrize("layout", ["ggml", "rows"])
def test_host_tier_matches_oracle(oracle, layout):
    """Host bytes as ggml blobs (repacked on the device after each copy) or as a
    version-4 row-split relayout holds them (copied as they are)."""
    import torch
    from tinygiant_b200 import relayout as R
    from tinygiant_b200.cache import HostTierCache
    from tinygiant_b200.engine import MoEModel
    H, I, E, k, L = 512, 256, 16, 4, 2
    rng = np.random.default_rng(21)
    m = MoEModel(H, I, E, k, L)
    eb = m.expert_bytes
    blobs, norms, host = [], [], []
    for l in range(L):
        b = oracle.quantize_q4_0((rng.standard_normal(E * 3 * H * I) * 0.02).astype(np.float32))
        nw = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        m.set_ffn_norm(l, nw)
        blobs.append(b)
        norms.append(nw)
        hb = b if layout == "ggml" else np.concatenate(
            [R.expert_convert(b[e * eb:(e + 1) * eb], H, I, True) for e in range(E)])
        host.append(torch.from_numpy(hb).pin_memory())
    cache = HostTierCache(m, host, cache_slots=6, layout=layout)
    cache.pin(0, [3])
    x = rng.standard_normal(H).astype(np.float32)
    xd = torch.from_numpy(x.copy()).cuda()
    xr = x.copy()
    for step in range(12):
        l = step % L
        ids = rng.choice(E, size=k, replace=False)
        w = rng.dirichlet(np.ones(k)).astype(np.float32)
        if step % 3 == 0:
            cache.prefetch(l, ids)
        cache.forward(l, ids, w, xd)
        xr = oracle_block(oracle, blobs[l], xr, ids, w, H, I, norms[l])
        torch.cuda.synchronize()
        assert np.array_equal(xd.cpu().numpy(), xr), f"step {step}"
    assert cache.misses > 0 and cache.hits > 0
    assert cache.hits + cache.misses == 12 * k
    m.close()


def test_host_tier_full_slots_error(oracle):
    import torch
    from tinygiant_b200.cache import HostTierCache
    from tinygiant_b200.engine import MoEModel
    H, I, E, k = 256, 256, 8, 4
    m = MoEModel(H, I, E, k, 1)
    b = oracle.quantize_q4_0((np.random.default_rng(1).standard_normal(E * 3 * H * I) * 0.02).astype(np.float32))
    cache = HostTierCache(m, [torch.from_numpy(b).pin_memory()], cache_slots=2)
    x = torch.zeros(H, device="cuda")
    with pytest.raises(RuntimeError):
        cache.forward(0, [0, 1, 2, 3], np.full(4, 0.25, np.float32), x)
    torch.cuda.synchronize()
    m.close()


def test_calibrated_pinned_tier_decode(oracle, tmp_path):
    """The reference's pinning flow on the HBM tier (tinygiant/cache.py:84-113,
    engine.py:154-186): calibrate request counts from the model's own routing, pin from
    usage with the relayout profile as backfill, then decode through the tier (pinned
    experts plus LRU slots) with that routing, bit-exact against the oracle and the
    all-resident model."""
    import torch
    from tests.test_gpu_parity import build_model
    from tinygiant_b200 import relayout as R
    from tinygiant_b200.cache import HostTierCache
    H, I, E, k, L = 512, 256, 16, 4, 2
    m, blobs, Rs, rng = build_model(oracle, H, I, E, k, L, seed=77)
    profile = {str(l): {"expert_ranking": [int(e) for e in rng.permutation(E)]} for l in range(L)}
    R.write_model(tmp_path, blobs, E, k, H, I, activation_profile=profile)
    rd = R.RelayoutReader(tmp_path)
    host = [torch.from_numpy(np.ascontiguousarray(rd.layer_bytes(l))).pin_memory() for l in range(L)]
    cache = HostTierCache(m, host, cache_slots=6, index=rd.index)

    def route(x, l):
        xd = torch.from_numpy(x.copy()).cuda()
        m.moe_layer(l, xd)
        idx, w, _ = m.last_routing(l)
        return idx, w, xd.cpu().numpy()

    # calibration: 5 tokens through both layers, counted per (layer, expert)
    for t in range(5):
        x = rng.standard_normal(H).astype(np.float32)
        for l in range(L):
            idx, w, x = route(x, l)
            cache.record(l, idx)
    counts = dict(cache.access_counts)
    assert sum(counts.values()) == 5 * L * k
    n = cache.pin_from_usage(3, L)
    assert n == 3 * L and cache.access_counts == {} and cache.hits == 0
    for l in range(L):
        top = sorted(((-c, e) for (ll, e), c in counts.items() if ll == l))[:3]
        assert all((l, e) in cache.pinned for _, e in top)
    # the tiered decode with the model's routing
    for t in range(6):
        x = rng.standard_normal(H).astype(np.float32)
        xt = torch.from_numpy(x.copy()).cuda()
        for l in range(L):
            idx, w, x_res = route(x, l)
            cache.forward(l, idx, w, xt)
            x = oracle_block(oracle, blobs[l], x, idx, w, H, I, m.norms[l])
            torch.cuda.synchronize()
            assert np.array_equal(xt.cpu().numpy(), x) and np.array_equal(x_res, x), f"token {t} layer {l}"
    assert cache.pinned_hits > 0 and cache.hits + cache.misses == 6 * L * k
    # get(): the resident expert, counted like a request
    e0 = int(rd.index["activation_profile"]["0"]["expert_ranking"][0])
    before = cache.access_counts.get((0, e0), 0)
    dev = cache.get(0, e0)
    assert dev.numel() == m.expert_bytes and cache.access_counts[(0, e0)] == before + 1
    torch.cuda.synchronize()
    file_expert = rd.layer_bytes(0)[e0 * m.expert_bytes:(e0 + 1) * m.expert_bytes]
    assert np.array_equal(dev.cpu().numpy(), R.expert_convert(file_expert, H, I, True))   # the kernels' layout
    m.close()
