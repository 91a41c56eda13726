"""Generate the golden fixtures in tests/golden/ from gguf.quants and numpy.

    python tests/golden/make_golden.py

The reference (jerryjokesalot/tinygiant) stores no golden vectors, and its C
library needs ARM NEON, so its own outputs cannot be produced here.  These
fixtures pin the oracle and the GPU kernels to an independent implementation
instead:
  * Q8_0 / Q4_0 quantisation and dequantisation from gguf.quants (gguf 0.19.0,
    the package the reference depends on, pyproject.toml:13-16), whose Q8_0 is
    documented as bit-exact with ggml-quants.c;
  * exact int32 block dots computed in numpy int64 from the gguf nibble codes;
  * an expert forward (csrc/libtinygiant.c:555-595 structure) evaluated in
    numpy float64 on gguf-dequantised weights, with x and h quantised by gguf;
  * routing (tinygiant/engine.py:231-236) in float64.
Inputs are seeded numpy PCG64 draws plus hand-made edge blocks.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
from gguf import quants as Q
from gguf.constants import GGMLQuantizationType as T

OUT = Path(__file__).resolve().parent
SEED = 20261201


def q8_edge_blocks() -> np.ndarray:
    b = []
    b.append(np.zeros(32, np.float32))                                   # all zero: d = 0, codes 0
    t = np.arange(32, dtype=np.float32) - 15.5                            # .5 ties after scaling
    t[0] = 127.0
    b.append(t)
    b.append(-np.linspace(0, 3, 32, dtype=np.float32))                    # max magnitude negative
    b.append(np.full(32, 1e-6, np.float32) * np.arange(32, dtype=np.float32))  # fp16-subnormal scale
    b.append(np.array([0] * 31 + [5e4], np.float32))                      # one large value
    b.append(np.array([1.0, -1.0] * 16, np.float32) * 0.25)               # equal magnitudes
    v = np.zeros(32, np.float32)
    v[7] = -0.0
    v[9] = 3.0
    b.append(v)
    return np.stack(b)


def q4_edge_blocks() -> np.ndarray:
    b = []
    z = np.zeros(32, np.float32)
    z[0] = -0.0
    b.append(z)                                                           # all zero, first is -0.0
    t = np.linspace(-1, 1, 32, dtype=np.float32)
    b.append(t)                                                           # |max| tie: -1 first
    b.append(-t)                                                          # |max| tie: +1 first
    b.append(np.full(32, 3e-8, np.float32) * np.arange(32, dtype=np.float32))  # subnormal fp16 d
    b.append(np.array([0.5] * 32, np.float32))                            # constant block
    b.append(np.array([0] * 31 + [-2.0], np.float32))                     # negative max, last
    return np.stack(b)


def q4_codes(q4: np.ndarray) -> np.ndarray:
    """Signed Q4_0 codes (q - 8) of ggml blocks, shape (nblocks, 32)."""
    blk = q4.reshape(-1, 18)
    qs = blk[:, 2:]
    lo = (qs & 15).astype(np.int64) - 8
    hi = (qs >> 4).astype(np.int64) - 8
    return np.concatenate([lo, hi], axis=1)


def q8_codes(q8: np.ndarray) -> np.ndarray:
    return q8.reshape(-1, 34)[:, 2:].view(np.int8).astype(np.int64)


def quant(x: np.ndarray, t) -> np.ndarray:
    return Q.quantize(np.ascontiguousarray(x, np.float32).reshape(1, -1), t).ravel()


def deq(q: np.ndarray, t) -> np.ndarray:
    return Q.dequantize(q.reshape(1, -1), t).ravel().astype(np.float64)


def expert_f64(gate, up, down, x, H, I):
    """Expert forward in float64 on gguf-dequantised tensors; x and h go through gguf Q8_0."""
    xq = quant(x, T.Q8_0)
    xd = deq(xq, T.Q8_0)
    Wg = deq(gate, T.Q4_0).reshape(I, H)
    Wu = deq(up, T.Q4_0).reshape(I, H)
    Wd = deq(down, T.Q4_0).reshape(H, I)
    g = Wg @ xd
    u = Wu @ xd
    h = g / (1.0 + np.exp(-g)) * u
    hq = quant(h.astype(np.float32), T.Q8_0)
    y = Wd @ deq(hq, T.Q8_0)
    return xq, g, u, h, hq, y


def main():
    rng = np.random.default_rng(SEED)
    fx = {}

    # ---- Q8_0 quantiser
    x = rng.standard_normal(64 * 32).astype(np.float32)
    x = np.concatenate([x, q8_edge_blocks().ravel()])
    fx["q8_x"] = x
    fx["q8_q"] = quant(x, T.Q8_0)
    fx["q8_deq"] = Q.dequantize(fx["q8_q"].reshape(1, -1), T.Q8_0).ravel().astype(np.float32)

    # ---- Q4_0 quantiser
    w = (rng.standard_normal(128 * 32) * 0.02).astype(np.float32)
    w = np.concatenate([w, q4_edge_blocks().ravel()])
    fx["q4_w"] = w
    fx["q4_q"] = quant(w, T.Q4_0)
    fx["q4_deq"] = Q.dequantize(fx["q4_q"].reshape(1, -1), T.Q4_0).ravel().astype(np.float32)

    # ---- block dots and row dots (matvec 96 x 512)
    R, C = 96, 512
    Wm = (rng.standard_normal((R, C)) * 0.02).astype(np.float32)
    xm = rng.standard_normal(C).astype(np.float32)
    Wq = quant(Wm, T.Q4_0)
    xq = quant(xm, T.Q8_0)
    codes_w = q4_codes(Wq).reshape(R, C // 32, 32)
    codes_x = q8_codes(xq).reshape(C // 32, 32)
    fx["mv_W"] = Wq
    fx["mv_xq"] = xq
    fx["mv_x"] = xm
    fx["mv_sumi"] = np.einsum("rbj,bj->rb", codes_w, codes_x).astype(np.int32)
    fx["mv_y64"] = deq(Wq, T.Q4_0).reshape(R, C) @ deq(xq, T.Q8_0)

    # ---- expert forward, H=512, I=256
    H, I = 512, 256
    gate = quant(rng.standard_normal((I, H)) * 0.02, T.Q4_0)
    up = quant(rng.standard_normal((I, H)) * 0.02, T.Q4_0)
    down = quant(rng.standard_normal((H, I)) * 0.02, T.Q4_0)
    xe = rng.standard_normal(H).astype(np.float32)
    xq_e, g, u, h, hq, y = expert_f64(gate, up, down, xe, H, I)
    fx["ex_H"] = np.array(H)
    fx["ex_I"] = np.array(I)
    fx["ex_blob"] = np.concatenate([gate, up, down])
    fx["ex_x"] = xe
    fx["ex_xq"] = xq_e
    fx["ex_g64"] = g
    fx["ex_u64"] = u
    fx["ex_h64"] = h
    fx["ex_hq"] = hq
    fx["ex_y64"] = y

    # ---- routing, E=64, H=512, k=8
    E, k = 64, 8
    Rr = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    xr = rng.standard_normal(H).astype(np.float32)
    logits = Rr.astype(np.float64) @ xr.astype(np.float64)
    idx = np.argsort(logits, kind="stable")[-k:]
    wl = np.exp(logits[idx] - logits[idx].max())
    fx["rt_R"] = Rr
    fx["rt_x"] = xr
    fx["rt_k"] = np.array(k)
    fx["rt_logits64"] = logits
    fx["rt_idx"] = idx.astype(np.int32)
    fx["rt_w64"] = wl / wl.sum()

    np.savez_compressed(OUT / "golden_q4_0.npz", **fx)
    print("wrote", OUT / "golden_q4_0.npz", sum(v.nbytes for v in fx.values()), "bytes raw")


if __name__ == "__main__":
    main()
