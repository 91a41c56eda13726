"""Pin the oracle's restatement of the reference's attention decode step
(csrc/libtinygiant.c:344-551: QKV projections, per-head RMSNorm, RoPE, KV append, GQA
softmax attention, output projection) against tests/golden/golden_attention.npz: the
reference package's own numpy path (engine.py:272-293 with tinygiant._math) and a
float64 restatement of the Q4 C path.
"""
from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import ROOT

gguf = pytest.importorskip("gguf")


@pytest.fixture(scope="module")
def ga():
    return dict(np.load(ROOT / "tests" / "golden" / "golden_attention.npz"))


def _shape(ga):
    return tuple(int(ga[k]) for k in ("embed", "n_heads", "n_kv", "head_dim", "kv_max", "pos"))


def _deq_q4k(b, rows, cols):
    from gguf import quants as Q
    from gguf.constants import GGMLQuantizationType as T
    return Q.dequantize(b.reshape(-1, 144), T.Q4_K).astype(np.float32).reshape(rows, cols)


def _rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / np.max(np.abs(b)))


def _run(oracle, ga, q4, mode, weights=None):
    E, NH, NKV, HD, KVM, POS = _shape(ga)
    kv_k, kv_v = ga["kv_k"].copy(), ga["kv_v"].copy()
    w = weights or (ga["wq"], ga["wk"], ga["wv"], ga["wo"])
    out = oracle.attention_decode(q4, *w, ga["q_norm"], ga["k_norm"], kv_k, kv_v, POS, ga["rope_cos"],
                                  ga["rope_sin"], ga["x"], E, NH, NKV, HD, POS, mode)
    return out, kv_k, kv_v


def _f32_weights(ga):
    E, NH, NKV, HD, _, _ = _shape(ga)
    return (_deq_q4k(ga["wq"], NH * HD, E), _deq_q4k(ga["wk"], NKV * HD, E),
            ga["wv"].view(np.float16).astype(np.float32).reshape(NKV * HD, E), _deq_q4k(ga["wo"], E, NH * HD))


def test_f32_variant_matches_reference_numpy_path(oracle, ga):
    """tg_attention_decode on fp32 weights against engine.py's numpy attention: only the
    float order differs."""
    out, kv_k, kv_v = _run(oracle, ga, False, oracle.TG_REF_ORDER, _f32_weights(ga))
    assert _rel(out, ga["out_np"]) < 1e-5
    _, _, NKV, _, _, POS = _shape(ga)
    assert _rel(kv_k[:, POS], ga["k_new"]) < 1e-5
    assert _rel(kv_v[:, POS], ga["v_new"]) < 1e-5
    # earlier rows untouched, later rows still zero
    assert np.array_equal(kv_k[:, :POS], ga["kv_k"][:, :POS]) and not kv_k[:, POS + 1:].any()


def test_q4_variant_matches_float64_restatement(oracle, ga):
    """tg_attention_decode_q4 (Q8(256) activations) against its float64 restatement, and
    within the reference test's matvec tolerance (rel 1e-2, csrc/test_libtinygiant.c
    Test 3) of the unquantised numpy path."""
    out, _, _ = _run(oracle, ga, True, oracle.TG_REF_ORDER)
    assert _rel(out, ga["out_q4_64"]) < 1e-5
    assert np.linalg.norm(out - ga["out_np"]) / np.linalg.norm(ga["out_np"]) < 1e-2


def test_mirror_mode_differs_only_in_exp(oracle, ga):
    a, _, _ = _run(oracle, ga, True, oracle.TG_REF_ORDER)
    b, _, _ = _run(oracle, ga, True, oracle.TG_MIRROR)
    assert _rel(b, a.astype(np.float64)) < 1e-5


def test_rope_identity_at_position_zero_and_rotation(oracle):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(4 * 64).astype(np.float32)
    assert np.array_equal(oracle.rope(x, np.ones(32, np.float32), np.zeros(32, np.float32), 4, 64), x)
    th = rng.uniform(-3, 3, 32).astype(np.float32)
    y = oracle.rope(x, np.cos(th), np.sin(th), 4, 64).reshape(4, 2, 32).astype(np.float64)
    xr = x.reshape(4, 2, 32).astype(np.float64)
    # each (i, i + half) pair is rotated: its length is kept
    assert np.allclose(np.hypot(y[:, 0], y[:, 1]), np.hypot(xr[:, 0], xr[:, 1]), rtol=1e-6)


def test_gqa_mapping_equals_repeated_kv_heads(oracle, ga):
    """Query head h reads kv head h // (n_heads / n_kv): with the kv heads repeated so
    that ratio = 1, the attention is the same computation."""
    E, NH, NKV, HD, KVM, POS = _shape(ga)
    wq, wk, wv, wo = _f32_weights(ga)
    ratio = NH // NKV
    wk1 = np.repeat(wk.reshape(NKV, HD, E), ratio, axis=0).reshape(NH * HD, E)
    wv1 = np.repeat(wv.reshape(NKV, HD, E), ratio, axis=0).reshape(NH * HD, E)
    kv_k1 = np.ascontiguousarray(np.repeat(ga["kv_k"], ratio, axis=0))
    kv_v1 = np.ascontiguousarray(np.repeat(ga["kv_v"], ratio, axis=0))
    a, _, _ = _run(oracle, ga, False, oracle.TG_MIRROR, (wq, wk, wv, wo))
    b = oracle.attention_decode(False, wq, wk1, wv1, wo, ga["q_norm"], ga["k_norm"], kv_k1, kv_v1, POS,
                                ga["rope_cos"], ga["rope_sin"], ga["x"], E, NH, NH, HD, POS, oracle.TG_MIRROR)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
