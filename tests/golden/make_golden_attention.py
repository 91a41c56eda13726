"""Generate tests/golden/golden_attention.npz: fixtures for the reference's attention
decode step (csrc/libtinygiant.c:344-551 in C; engine.py:272-293 in numpy).

    PYTHONPATH=<the reference checkout> python tests/golden/make_golden_attention.py

The reference ships no attention test vectors and its C needs ARM NEON, so these pin
the oracle to the reference's own Python arithmetic instead:
  * out_np: the numpy engine path (engine.py:272-293: per-head rms_norm of q and k,
    apply_rope at pos, the new row appended to the cache, softmax(K q / sqrt(hd)) V per
    query head over kv head h // (n_heads / n_kv), then Wo) evaluated with the reference
    package's own tinygiant._math.rms_norm / build_rope_cache / apply_rope, imported from
    the reference checkout, on fp32 weights dequantised by gguf.quants (0.19.0);
  * out_q4_64: the same step the way tg_attention_decode_q4 computes it (Q4_K wq / wk /
    wo against the 256-wide Q8 blocks of their inputs, f16 wv against fp32 x) in
    float64, the Q8 blocks from make_golden_kquant's numpy restatement of quantize_q8.
head_dim is 128 because _math.apply_rope is written for HEAD_DIM = 128.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
from gguf.constants import GGMLQuantizationType as T

OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(OUT))
from make_golden_kquant import deq, kdot64, q4k_blocks  # noqa: E402

from tinygiant import _math as RM  # noqa: E402  (the reference package, from PYTHONPATH)

SEED = 20261203
EMBED, NH, NKV, HD, KV_MAX, POS = 256, 4, 2, 128, 8, 5


def numpy_attention(wq, wk, wv, wo, qn, kn, kv_k, kv_v, kv_len, cos, sin, x, pos):
    """engine.py:272-293 for one layer, through the reference's _math functions."""
    q = (wq @ x).reshape(NH, HD)
    k = (wk @ x).reshape(NKV, HD)
    v = (wv @ x).reshape(NKV, HD)
    q = RM.rms_norm(q, qn)
    k = RM.rms_norm(k, kn)
    q = RM.apply_rope(q, cos, sin, pos)
    k = RM.apply_rope(k, cos, sin, pos)
    K = np.concatenate([kv_k[:, :kv_len], k[:, None, :]], axis=1)
    V = np.concatenate([kv_v[:, :kv_len], v[:, None, :]], axis=1)
    out = np.zeros(NH * HD, dtype=np.float32)
    ratio = NH // NKV
    for h in range(NH):
        scores = (K[h // ratio] @ q[h]) / np.sqrt(HD)
        e = np.exp(scores - np.max(scores))
        out[h * HD:(h + 1) * HD] = (e / np.sum(e)) @ V[h // ratio]
    return (wo @ out).astype(np.float32), k.astype(np.float32), v.astype(np.float32)


def q4_path64(wq_d, wk_d, wv16, wo_d, qn, kn, kv_k, kv_v, kv_len, cos, sin, x, pos):
    """tg_attention_decode_q4's step in float64 (activations quantised as the C does)."""
    q = kdot64(wq_d, x).reshape(NH, HD)
    k = kdot64(wk_d, x).reshape(NKV, HD)
    v = (wv16.astype(np.float64) @ x.astype(np.float64)).reshape(NKV, HD)

    def norm(a, w):
        return a / np.sqrt(np.mean(a * a, axis=-1, keepdims=True) + 1e-6) * w.astype(np.float64)

    def rope(a):
        c, s = cos[pos].astype(np.float64), sin[pos].astype(np.float64)
        a1, a2 = a[:, :HD // 2], a[:, HD // 2:]
        return np.concatenate([a1 * c - a2 * s, a2 * c + a1 * s], axis=-1)

    q, k = rope(norm(q, qn)), rope(norm(k, kn))
    K = np.concatenate([kv_k[:, :kv_len].astype(np.float64), k[:, None, :]], axis=1)
    V = np.concatenate([kv_v[:, :kv_len].astype(np.float64), v[:, None, :]], axis=1)
    att = np.zeros(NH * HD)
    ratio = NH // NKV
    for h in range(NH):
        s = K[h // ratio] @ q[h] / np.sqrt(HD)
        e = np.exp(s - s.max())
        att[h * HD:(h + 1) * HD] = (e / e.sum()) @ V[h // ratio]
    return kdot64(wo_d, att.astype(np.float32))


def main():
    rng = np.random.default_rng(SEED)
    qd, kvd = NH * HD, NKV * HD
    wq = q4k_blocks(rng, qd * EMBED // 256)
    wk = q4k_blocks(rng, kvd * EMBED // 256)
    wo = q4k_blocks(rng, EMBED * qd // 256)
    wv = (rng.standard_normal((kvd, EMBED)) * 0.05).astype(np.float16)
    wq_d = deq(wq, T.Q4_K).reshape(qd, EMBED)
    wk_d = deq(wk, T.Q4_K).reshape(kvd, EMBED)
    wo_d = deq(wo, T.Q4_K).reshape(EMBED, qd)
    qn = (1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    x = rng.standard_normal(EMBED).astype(np.float32)
    kv_k = np.zeros((NKV, KV_MAX, HD), np.float32)
    kv_v = np.zeros((NKV, KV_MAX, HD), np.float32)
    kv_k[:, :POS] = rng.standard_normal((NKV, POS, HD)).astype(np.float32)
    kv_v[:, :POS] = rng.standard_normal((NKV, POS, HD)).astype(np.float32)
    cos, sin = RM.build_rope_cache(KV_MAX)

    out_np, k_new, v_new = numpy_attention(wq_d.astype(np.float32), wk_d.astype(np.float32),
                                           wv.astype(np.float32), wo_d.astype(np.float32), qn, kn, kv_k, kv_v,
                                           POS, cos, sin, x, POS)
    out64 = q4_path64(wq_d, wk_d, wv, wo_d, qn, kn, kv_k, kv_v, POS, cos, sin, x, POS)
    fx = dict(embed=np.int32(EMBED), n_heads=np.int32(NH), n_kv=np.int32(NKV), head_dim=np.int32(HD),
              kv_max=np.int32(KV_MAX), pos=np.int32(POS),
              wq=wq.ravel(), wk=wk.ravel(), wv=wv.view(np.uint16), wo=wo.ravel(), q_norm=qn, k_norm=kn, x=x,
              kv_k=kv_k, kv_v=kv_v, rope_cos=cos, rope_sin=sin,
              out_np=out_np, k_new=k_new, v_new=v_new, out_q4_64=out64)
    np.savez_compressed(OUT / "golden_attention.npz", **fx)
    print("wrote", OUT / "golden_attention.npz", sum(v.nbytes for v in fx.values()), "bytes")


if __name__ == "__main__":
    main()
