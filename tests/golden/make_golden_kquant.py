"""Generate tests/golden/golden_kquant.npz: fixtures for the reference library's own
formats (csrc/libtinygiant.c: Q4_K and Q6_K super-blocks against 256-wide Q8
activation blocks, f16 rows).

    python tests/golden/make_golden_kquant.py

The reference ships no golden vectors and its library needs ARM NEON, so these pin
the oracle to independent arithmetic instead:
  * weight values from gguf.quants (gguf 0.19.0, the reference's dependency,
    pyproject.toml:13-16) dequantising Q4_K / Q6_K blocks;
  * the 256-wide Q8 activation codes from a numpy restatement of quantize_q8
    (libtinygiant.c:61-89: scale = amax/127 in fp32, codes = round-half-even of
    x * (127/amax) in fp32);
  * row dots sum_b scale_b * sum_i w_bi * code_bi, and f16 dots, in numpy float64;
  * one all-Q4_K expert forward (libtinygiant.c:555-595) in float64 on the gguf
    weights, x and h quantised by the numpy quantiser.
Weights are seeded random bytes (ql / qh / scale bytes / nibbles) with chosen fp16
d and dmin: gguf can dequantise K-quants but not quantise them.  Block 0 of the Q4_K
set uses the reference test's own fill constants (d = 0x3400, dmin = 0x2C00,
csrc/test_libtinygiant.c:63-78).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
from gguf import quants as Q
from gguf.constants import GGMLQuantizationType as T

OUT = Path(__file__).resolve().parent
SEED = 20261202


def f16_bits(v) -> np.ndarray:
    return np.asarray(v, np.float16).view(np.uint16)


def q4k_blocks(rng, n: int, ref_fill_first: bool = False) -> np.ndarray:
    b = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    d = f16_bits(rng.uniform(5e-4, 3e-3, n))
    dm = f16_bits(rng.uniform(2e-4, 2e-3, n))
    if ref_fill_first:
        d[0], dm[0] = 0x3400, 0x2C00
    b[:, 0:2] = d.view(np.uint8).reshape(n, 2)
    b[:, 2:4] = dm.view(np.uint8).reshape(n, 2)
    return b


def q6k_blocks(rng, n: int) -> np.ndarray:
    b = rng.integers(0, 256, size=(n, 210), dtype=np.uint8)
    b[:, 192:208] = rng.integers(-64, 64, size=(n, 16), dtype=np.int8).view(np.uint8)
    b[:, 208:210] = f16_bits(rng.uniform(5e-4, 2e-3, n)).view(np.uint8).reshape(n, 2)
    return b


def q8k(x: np.ndarray):
    """(scales f32[nb], codes int64[nb, 256]) of the reference's Q8 activation blocks."""
    xb = np.asarray(x, np.float32).reshape(-1, 256)
    amax = np.abs(xb).max(axis=1).astype(np.float32)
    sc = (amax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(amax > 0, np.float32(127) / amax, np.float32(0)).astype(np.float32)
    codes = np.rint((xb * inv[:, None]).astype(np.float32)).astype(np.int64)
    return sc, codes


def deq(blocks: np.ndarray, t) -> np.ndarray:
    return Q.dequantize(blocks.reshape(blocks.shape[0], -1), t).astype(np.float64).reshape(blocks.shape[0], 256)


def kdot64(wdeq_rows: np.ndarray, x: np.ndarray) -> np.ndarray:
    """float64 y[r] = sum_b scale_b * sum_i w[r, b, i] * code[b, i]."""
    sc, codes = q8k(x)
    rows = wdeq_rows.shape[0]
    w = wdeq_rows.reshape(rows, -1, 256)
    return (w * codes[None].astype(np.float64)).sum(axis=2) @ sc.astype(np.float64)


def main():
    rng = np.random.default_rng(SEED)
    fx = {}

    # Q8(256) activation quantiser: random, zero, half-way ties, one huge value.
    xs = [rng.standard_normal(256).astype(np.float32) * 3,
          np.zeros(256, np.float32),
          (np.arange(256, dtype=np.float32) % 9 - 4.5).astype(np.float32),   # equal +-amax pairs
          np.concatenate([np.full(255, 0.5, np.float32), [127.0]]).astype(np.float32),  # inv = 1: 0.5 -> 0
          np.concatenate([(np.arange(255, dtype=np.float32) - 127) + 0.5, [127.0]]).astype(np.float32),
          np.concatenate([np.full(255, 1e-3, np.float32), [-6e4]]).astype(np.float32)]
    qx = np.concatenate(xs)
    sc, codes = q8k(qx)
    fx["q8k_x"], fx["q8k_scale"], fx["q8k_codes"] = qx, sc, codes.astype(np.int8)
    fx["q8k_sum"] = codes.sum(axis=1).astype(np.int32)

    # Q4_K and Q6_K matrices: rows x cols, dequantised by gguf; y64 against Q8(256) of x.
    rows, cols = 24, 1024
    bpr = cols // 256
    w4 = q4k_blocks(rng, rows * bpr, ref_fill_first=True)
    w6 = q6k_blocks(rng, rows * bpr)
    x = rng.standard_normal(cols).astype(np.float32)
    d4 = deq(w4, T.Q4_K).reshape(rows, cols)
    d6 = deq(w6, T.Q6_K).reshape(rows, cols)
    fx["mk_rows"], fx["mk_cols"], fx["mk_x"] = np.int32(rows), np.int32(cols), x
    fx["q4k_W"], fx["q4k_y64"] = w4.ravel(), kdot64(d4, x)
    fx["q6k_W"], fx["q6k_y64"] = w6.ravel(), kdot64(d6, x)
    fx["q4k_yfloat64"] = d4 @ x.astype(np.float64)   # unquantised x: the reference test's matvec check

    # f16 rows.
    wf = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float16)
    fx["f16_W"] = wf.view(np.uint16)
    fx["f16_y64"] = wf.astype(np.float64) @ x.astype(np.float64)

    # One all-Q4_K expert (embed H, inter I) and its float64 forward.
    H, I = 512, 256
    gate = q4k_blocks(rng, I * H // 256)
    up = q4k_blocks(rng, I * H // 256)
    down = q4k_blocks(rng, H * I // 256)
    gd = deq(gate, T.Q4_K).reshape(I, H)
    ud = deq(up, T.Q4_K).reshape(I, H)
    dd = deq(down, T.Q4_K).reshape(H, I)
    xe = (rng.standard_normal(H) * 0.5).astype(np.float32)
    g64, u64 = kdot64(gd, xe), kdot64(ud, xe)
    h64 = g64 / (1.0 + np.exp(-g64)) * u64
    y64 = kdot64(dd, h64.astype(np.float32))
    fx["ex_H"], fx["ex_I"] = np.int32(H), np.int32(I)
    fx["ex_blob"] = np.concatenate([gate.ravel(), up.ravel(), down.ravel()])
    fx["ex_x"], fx["ex_h64"], fx["ex_y64"] = xe, h64, y64
    np.savez_compressed(OUT / "golden_kquant.npz", **fx)
    print("wrote", OUT / "golden_kquant.npz", sum(v.nbytes for v in fx.values()), "bytes")


if __name__ == "__main__":
    main()
