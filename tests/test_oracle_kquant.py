"""Pin the oracle's restatement of the reference's K-quant path (csrc/libtinygiant.c:
Q8(256) quantiser :61-89, Q4_K dot :104-169, Q6_K dot :194-243, f16/f32 matvec
:262-318, RMSNorm :322-340, expert forward :555-643) against the fixtures in
tests/golden/golden_kquant.npz (gguf dequantisation + numpy float64), with the
reference test's own tolerances where it has one (csrc/test_libtinygiant.c:108-293).
"""
from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import ROOT


@pytest.fixture(scope="module")
def gk():
    return dict(np.load(ROOT / "tests" / "golden" / "golden_kquant.npz"))


def _blocks(q8k_bytes):
    b = q8k_bytes.reshape(-1, 264)
    return b[:, 0:4].copy().view(np.float32).ravel(), b[:, 4:8].copy().view(np.int32).ravel(), b[:, 8:].view(np.int8)


def test_q8k_bytes_match_numpy_restatement(oracle, gk):
    sc, sm, codes = _blocks(oracle.quantize_q8k(gk["q8k_x"]))
    assert np.array_equal(sc.view(np.uint32), gk["q8k_scale"].view(np.uint32))
    assert np.array_equal(codes, gk["q8k_codes"].reshape(-1, 256))
    assert np.array_equal(sm, gk["q8k_sum"])


def test_q8k_rounds_half_to_even(oracle):
    # amax 127 -> inverse scale 1: x = k + 0.5 must round to the even neighbour (vcvtnq_s32_f32)
    x = np.zeros(256, np.float32)
    x[0] = 127.0
    x[1:9] = [0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, 126.5]
    _, _, codes = _blocks(oracle.quantize_q8k(x))
    assert codes[0, :9].tolist() == [127, 0, 2, 2, 0, -2, -2, 4, 126]


@pytest.mark.parametrize("fmt,key", [(0, "q4k"), (2, "q6k")])
def test_kquant_matvec_matches_gguf_dequant(oracle, gk, fmt, key):
    rows, cols = int(gk["mk_rows"]), int(gk["mk_cols"])
    y = oracle.matvec_k(gk[key + "_W"], fmt, gk["mk_x"], rows, cols)
    y64 = gk[key + "_y64"]
    # csrc/test_libtinygiant.c Test 1a bound (rel < 1e-4); a wrong nibble, scale or
    # sub-block order is off by O(1)
    assert np.max(np.abs(y - y64)) <= 1e-4 * np.max(np.abs(y64))


def test_q4k_matvec_close_to_unquantised(oracle, gk):
    # Test 3 of csrc/test_libtinygiant.c: quantised matvec vs float matvec, rel < 1e-2
    rows, cols = int(gk["mk_rows"]), int(gk["mk_cols"])
    y = oracle.matvec_k(gk["q4k_W"], 0, gk["mk_x"], rows, cols).astype(np.float64)
    ref = gk["q4k_yfloat64"]
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-2


def test_f16_and_f32_matvec(oracle, gk):
    rows, cols = int(gk["mk_rows"]), int(gk["mk_cols"])
    W = gk["f16_W"]
    y = oracle.matvec_k(W, 1, gk["mk_x"], rows, cols)
    assert np.max(np.abs(y - gk["f16_y64"])) <= 1e-5 * np.max(np.abs(gk["f16_y64"]))
    W32 = W.view(np.float16).astype(np.float32)
    y32 = oracle.matvec_k(W32, 4, gk["mk_x"], rows, cols)
    assert np.array_equal(y.view(np.uint32), y32.view(np.uint32))   # same values, same order


def test_f16_order_is_eight_chains(oracle):
    # the order is observable: eight running fused sums, folded (0+4, 1+5, 2+6, 3+7) pairwise
    cols = 64
    rng = np.random.default_rng(3)
    W = rng.standard_normal(cols).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    acc = [np.float32(0)] * 8
    for i in range(0, cols, 8):
        for v in range(8):
            acc[v] = np.float32(np.float64(W[i + v]) * np.float64(x[i + v]) + np.float64(acc[v]))
    t = [np.float32(acc[v] + acc[v + 4]) for v in range(4)]
    want = np.float32(np.float32(t[0] + t[1]) + np.float32(t[2] + t[3]))
    got = oracle.matvec_k(W, 4, x, 1, cols)[0]
    assert got.view(np.uint32) == want.view(np.uint32)


def test_rms_norm_reference_order(oracle):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(2048).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    out = oracle.rms_norm_k(x, w, 1e-6)
    ref = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-6) * w
    assert np.max(np.abs(out - ref)) <= 1e-5 * np.max(np.abs(ref))


@pytest.mark.parametrize("mode", [0, 1])
def test_expert_forward_q4k_matches_float64(oracle, gk, mode):
    H, I = int(gk["ex_H"]), int(gk["ex_I"])
    blob = gk["ex_blob"]
    gb = I * (H // 256) * 144
    out = np.zeros(H, np.float32)
    oracle.expert_forward_k(blob[:gb], blob[gb:2 * gb], blob[2 * gb:], 0, gk["ex_x"], out, 1.0, H, I, mode)
    y64 = gk["ex_y64"]
    assert np.all(np.isfinite(out))                       # Test 4 of the reference test
    # h is requantised from fp32 here and from float64 in the fixture: a code may move by one
    assert np.linalg.norm(out - y64) / np.linalg.norm(y64) < 2e-3


def test_expert_forward_accumulates_weighted(oracle, gk):
    H, I = int(gk["ex_H"]), int(gk["ex_I"])
    blob = gk["ex_blob"]
    gb = I * (H // 256) * 144
    base = np.linspace(-1, 1, H).astype(np.float32)
    y = np.zeros(H, np.float32)
    oracle.expert_forward_k(blob[:gb], blob[gb:2 * gb], blob[2 * gb:], 0, gk["ex_x"], y, 1.0, H, I)
    out = base.copy()
    oracle.expert_forward_k(blob[:gb], blob[gb:2 * gb], blob[2 * gb:], 0, gk["ex_x"], out, 0.375, H, I)
    assert np.array_equal(out, (base + np.float32(0.375) * y).astype(np.float32))
