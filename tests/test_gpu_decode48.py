"""Parity on the configuration the benchmark runs: the Qwen3-30B-A3B shape (H 2048,
I 768, 128 experts, top-8) through all 48 MoE layers, one token after another.

- 200 consecutive decode steps through tgx_decode_step (the fused kernel, replayed from
  its CUDA graph: the benchmark's path) are compared bit for bit with the oracle's
  48-layer decode (mirror order).  The experts of one 2-layer Q4_0 pool are loaded into
  every layer (layer l holds pool l % 2), so the oracle needs 680 MB, not 16 GB; routers
  and FFN norm weights differ per layer.
- The routing of > 10,000 (token, layer) pairs is compared with the reference engine's
  own expression in numpy fp32 (tinygiant/engine.py:229-236): RMSNorm, then
  argsort(R @ normed)[-8:].  The library ranks exact fixed-point router sums instead of
  an fp32 matvec of unspecified order; every pair whose top-8 set differs must be a near
  tie, which is asserted on the float64 logits.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, I, E, K, L = 2048, 768, 128, 8, 48
EPS = 1e-6
TIE_TOL = 1e-5   # |logit_a - logit_b| (float64) of two experts the two rankings swap


@pytest.fixture(scope="module")
def model48(oracle):
    import torch
    from tinygiant_b200.engine import MoEModel
    torch.cuda.set_device(0)
    pool_model = MoEModel(H, I, E, K, 2)
    pool_model.fill_synthetic(4242)
    pool = [pool_model.read_experts(l, 0, E) for l in range(2)]
    pool_model.close()
    rng = np.random.default_rng(48)
    routers = [(rng.standard_normal((E, H)) * 0.02).astype(np.float32) for _ in range(L)]
    norms = [(1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32) for _ in range(L)]
    m = MoEModel(H, I, E, K, L)
    for l in range(L):
        m.load_experts(l, pool[l % 2])
        m.set_router(l, routers[l])
        m.set_ffn_norm(l, norms[l])
    assert m.fused_info()[0] > 0, "the fused decode kernel must be the path under test"
    blobs = [pool[l % 2] for l in range(L)]
    yield m, blobs, routers, norms, rng
    m.close()


def test_decode_48_layers_200_tokens_bit_exact(oracle, model48):
    import torch
    m, blobs, routers, norms, rng = model48
    T = 200
    X = rng.standard_normal((T, H)).astype(np.float32)
    got = np.empty_like(X)
    xd = torch.empty(H, device="cuda")
    for t in range(T):                      # consecutive steps: epoch tags, recycled sums
        xd.copy_(torch.from_numpy(X[t]))
        m.decode_step(xd)
        got[t] = xd.cpu().numpy()
    m.sync_status()
    for t in range(T):
        want = oracle.decode_step_mt(blobs, routers, X[t].copy(), K, H, I, mode=oracle.TG_MIRROR, n_threads=0,
                                     norms=norms, eps=EPS)
        assert np.array_equal(got[t], want), f"token {t}: max |d| = {np.abs(got[t] - want).max():.3e}"


def reference_topk(R, x, w):
    """engine.py:229-236 in numpy fp32 (the C RMSNorm's sum of squares taken in float64)."""
    ss = np.float32(np.sum(x.astype(np.float64) ** 2))
    scale = np.float32(1.0) / np.sqrt(np.float32(ss / np.float32(x.size)) + np.float32(EPS))
    normed = (x * scale) * w
    logits = R @ normed
    return np.sort(np.argsort(logits)[-K:]), normed


def test_routing_agrees_with_reference_numpy(oracle, model48):
    import torch
    m, blobs, routers, norms, rng = model48
    T = 210                                 # 210 tokens x 48 layers = 10,080 pairs
    pairs = disagree = 0
    worst_gap = 0.0
    xd = torch.empty(H, device="cuda")
    for t in range(T):
        xd.copy_(torch.from_numpy(rng.standard_normal(H).astype(np.float32)))
        for l in range(L):
            x_in = xd.cpu().numpy()
            m.moe_layer(l, xd)
            gi = np.sort(m.last_routing(l)[0])
            ri, normed = reference_topk(routers[l], x_in, norms[l])
            pairs += 1
            if not np.array_equal(gi, ri):
                disagree += 1
                exact = routers[l].astype(np.float64) @ normed.astype(np.float64)
                only_gpu = np.setdiff1d(gi, ri)
                only_ref = np.setdiff1d(ri, gi)
                gap = float(np.max(np.abs(exact[only_gpu][:, None] - exact[only_ref][None, :])))
                worst_gap = max(worst_gap, gap)
                assert gap <= TIE_TOL, f"token {t} layer {l}: swapped experts {only_gpu} / {only_ref}, gap {gap:.3e}"
    m.sync_status()
    print(f"routing vs reference numpy fp32: {disagree} of {pairs} (token, layer) pairs differ "
          f"(rate {disagree / pairs:.2e}), largest float64 logit gap of a swap {worst_gap:.2e}")
    assert pairs >= 10000
    assert disagree <= pairs // 1000
