"""Pin the CPU oracle against the golden fixtures (gguf.quants + numpy float64).

These run on the CPU only.  They establish that the oracle, which the GPU
parity tests use as their checker, quantises exactly like gguf/ggml, computes
exact integer block dots, and follows the reference's expert-forward and
routing structure (csrc/libtinygiant.c:555-595, tinygiant/engine.py:231-258).
"""
import numpy as np
import pytest


def test_q8_0_bytes_match_gguf(oracle, golden):
    q = oracle.quantize_q8_0(golden["q8_x"])
    assert np.array_equal(q, golden["q8_q"])


def test_q8_0_dequant_matches_gguf(oracle, golden):
    assert np.array_equal(oracle.dequantize_q8_0(golden["q8_q"]), golden["q8_deq"])


def test_q4_0_bytes_match_gguf(oracle, golden):
    q = oracle.quantize_q4_0(golden["q4_w"])
    assert np.array_equal(q, golden["q4_q"])


def test_q4_0_dequant_matches_gguf(oracle, golden):
    assert np.array_equal(oracle.dequantize_q4_0(golden["q4_q"]), golden["q4_deq"])


def test_q8_0_random_sizes_match_gguf(oracle):
    from gguf import quants as Q
    from gguf.constants import GGMLQuantizationType as T
    rng = np.random.default_rng(7)
    for n in (32, 64 * 32, 2048, 7168):
        x = (rng.standard_normal(n) * rng.choice([1e-4, 1.0, 300.0])).astype(np.float32)
        assert np.array_equal(oracle.quantize_q8_0(x), Q.quantize(x.reshape(1, -1), T.Q8_0).ravel())
        w = (rng.standard_normal(n) * 0.02).astype(np.float32)
        assert np.array_equal(oracle.quantize_q4_0(w), Q.quantize(w.reshape(1, -1), T.Q4_0).ravel())


def test_block_dots_exact(oracle, golden):
    s = oracle.block_dots(golden["mv_W"], golden["mv_xq"], 96, 512)
    assert np.array_equal(s, golden["mv_sumi"])


@pytest.mark.parametrize("mode", [0, 1, 2])   # reference order, mirror order, fast tensor-core epilogue
def test_matvec_close_to_float64(oracle, golden, mode):
    y = oracle.matvec(golden["mv_W"], golden["mv_xq"], 96, 512, mode)
    y64 = golden["mv_y64"]
    # 16 fp32 block terms, each rounded twice, then 16 rounded adds
    bound = 64 * np.finfo(np.float32).eps * np.abs(y64).max()
    assert np.max(np.abs(y - y64)) <= bound


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_expert_forward_matches_float64_pipeline(oracle, golden, mode):
    H, I = int(golden["ex_H"]), int(golden["ex_I"])
    st = oracle.expert_stages(golden["ex_blob"], golden["ex_x"], H, I, mode)
    assert np.array_equal(st["xq"], golden["ex_xq"])
    g64, u64 = golden["ex_g64"], golden["ex_u64"]
    assert np.max(np.abs(st["g"] - g64)) <= 1e-5 * np.abs(g64).max()
    assert np.max(np.abs(st["u"] - u64)) <= 1e-5 * np.abs(u64).max()
    # requantised h: codes agree except for rare rounding-boundary flips of one step
    c_or = st["hq"].reshape(-1, 34)[:, 2:].view(np.int8).astype(int)
    c_gd = golden["ex_hq"].reshape(-1, 34)[:, 2:].view(np.int8).astype(int)
    diff = np.abs(c_or - c_gd)
    assert diff.max() <= 1 and (diff > 0).sum() <= 2
    y64 = golden["ex_y64"]
    assert np.max(np.abs(st["y"] - y64)) <= 2e-3 * np.abs(y64).max()


def test_routing_matches_float64(oracle, golden):
    R, x, k = golden["rt_R"], golden["rt_x"], int(golden["rt_k"])
    logits = oracle.router_logits(R, x)
    l64 = golden["rt_logits64"]
    assert np.max(np.abs(logits - l64)) <= 2e-6 * np.abs(l64).max()
    for mode in (0, 1):
        idx, w = oracle.topk_softmax(logits, k, mode)
        assert np.array_equal(idx, golden["rt_idx"])
        assert np.max(np.abs(w - golden["rt_w64"])) <= 1e-6


def test_topk_order_and_ties(oracle):
    l = np.array([0.5, 2.0, 2.0, -1.0, 3.0, 0.5], np.float32)
    idx, w = oracle.topk_softmax(l, 3, 1)
    # ascending-logit order (argsort(...)[-k:]), equal logits ordered by expert id
    assert list(idx) == [1, 2, 4]
    assert abs(float(w.sum()) - 1.0) < 1e-6


def test_expf_within_one_ulp(oracle):
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.uniform(-104, 89, 20000), rng.uniform(-1, 1, 20000),
                         np.array([0.0, -0.0, 1e-30, -1e-30, 88.7, -87.0, -100.0, 89.5, -105.0])]).astype(np.float32)
    mine = oracle.expf(xs)
    ref = np.exp(xs.astype(np.float64)).astype(np.float32)
    fin = np.isfinite(ref) & (ref > 0)
    ulp = np.abs(mine[fin].view(np.int32).astype(np.int64) - ref[fin].view(np.int32).astype(np.int64))
    assert ulp.max() <= 1
    assert mine[xs > 89].tolist() == [np.inf] * int((xs > 89).sum())
    assert (mine[xs < -104] == 0).all()


def test_silu_reference_vs_mirror(oracle):
    L = oracle.lib()
    rng = np.random.default_rng(5)
    g = rng.standard_normal(5000).astype(np.float32) * 4
    u = rng.standard_normal(5000).astype(np.float32)
    a = np.array([L.ref_silu_mul(float(a_), float(b_), 0) for a_, b_ in zip(g, u)], np.float32)
    b = np.array([L.ref_silu_mul(float(a_), float(b_), 1) for a_, b_ in zip(g, u)], np.float32)
    rel = np.abs(a - b) / np.maximum(np.abs(a), 1e-30)
    assert rel.max() < 4e-7


def test_moe_layer_and_decode_consistent(oracle):
    rng = np.random.default_rng(11)
    H, I, E, k, L = 256, 256, 16, 4, 3
    eb = oracle.expert_bytes(H, I)
    blobs = [oracle.quantize_q4_0((rng.standard_normal(E * 3 * H * I) * 0.02).astype(np.float32)) for _ in range(L)]
    assert blobs[0].size == E * eb
    Rs = [(rng.standard_normal((E, H)) * 0.02).astype(np.float32) for _ in range(L)]
    Ns = [(1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32) for _ in range(L)]
    x = rng.standard_normal(H).astype(np.float32)
    xs = x.copy()
    for l in range(L):
        xs, idx, w, logits = oracle.moe_block(blobs[l], Rs[l], xs, k, H, I, normw=Ns[l])
        assert len(set(idx.tolist())) == k
    xd, idx_all = oracle.decode_step(blobs, Rs, x, k, H, I, norms=Ns)
    assert np.array_equal(xd, xs)
    xm = x.copy()
    oracle.decode_step_mt(blobs, Rs, xm, k, H, I, 1, 4, norms=Ns)
    assert np.array_equal(xm, xs)


def test_rms_norm_block_matches_engine_order(oracle):
    """The MoE block's norm follows tg_rms_norm (csrc/libtinygiant.c:322-340):
    routing and expert input are RMSNorm(x) * w; the residual adds to raw x."""
    rng = np.random.default_rng(13)
    H, I, E, k = 256, 256, 8, 2
    blob = oracle.quantize_q4_0((rng.standard_normal(E * 3 * H * I) * 0.02).astype(np.float32))
    R = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    x = (3.0 * rng.standard_normal(H)).astype(np.float32)
    scale = oracle.rms_scale(x)
    assert abs(scale - 1.0 / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-6)) < 1e-6 * scale
    normed = (x * np.float32(scale)) * nw
    xn, idx, w, logits = oracle.moe_block(blob, R, x, k, H, I, normw=nw)
    l64 = R.astype(np.float64) @ normed.astype(np.float64)
    assert np.max(np.abs(logits - l64)) < 1e-5
    xl, idx2, w2, _ = oracle.moe_layer(blob, R, normed, k, H, I)   # same block on the pre-normed input
    assert np.array_equal(idx, idx2)
    assert np.array_equal(xn - x, (xl - normed)) or np.max(np.abs((xn - x) - (xl - normed))) < 1e-6


def test_engine_order_combine(oracle):
    """moe_layer == zeroed moe_out, tg_expert_forward per expert in idx order, x += moe_out
    (tinygiant/engine.py:240-258)."""
    rng = np.random.default_rng(12)
    H, I, E, k = 256, 256, 8, 3
    blob = oracle.quantize_q4_0((rng.standard_normal(E * 3 * H * I) * 0.02).astype(np.float32))
    R = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    xn, idx, w, _ = oracle.moe_layer(blob, R, x, k, H, I)
    eb = oracle.expert_bytes(H, I)
    moe = np.zeros(H, np.float32)
    for j in range(k):
        oracle.expert_forward(blob[idx[j] * eb:(idx[j] + 1) * eb], x, moe, w[j], H, I)
    assert np.array_equal(xn, x + moe)
