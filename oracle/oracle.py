"""ctypes wrapper around the CPU oracle (oracle/libtgref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, always as the checker.  The product package never
imports it.  See tg_ref.c for the reference file:line each routine follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libtgref.so"

TG_REF_ORDER = 0
TG_MIRROR = 1
TG_FAST_MMA = 2   # the tensor-core kernels' fast epilogue order (kernel mode 3)
QK = 32
Q4_0_BYTES = 18
Q8_0_BYTES = 34

_lib = None

VP = ctypes.c_void_p
CI = ctypes.c_int
CF = ctypes.c_float
I64 = ctypes.c_int64


def build() -> Path:
    """Compile the oracle from its sources with its Makefile (gcc; -B: always, never a
    stale library), returning the .so path."""
    subprocess.run(["make", "-s", "-B", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    L = ctypes.CDLL(str(LIB_PATH))
    sig = {
        "ref_f16_to_f32": (CF, [ctypes.c_uint16]),
        "ref_f32_to_f16": (ctypes.c_uint16, [CF]),
        "ref_expf": (CF, [CF]),
        "ref_quantize_q8_0": (None, [VP, VP, I64]),
        "ref_quantize_q4_0": (None, [VP, VP, I64]),
        "ref_dequantize_q8_0": (None, [VP, VP, I64]),
        "ref_dequantize_q4_0": (None, [VP, VP, I64]),
        "ref_block_dot_q4_0_q8_0": (ctypes.c_int32, [VP, VP]),
        "ref_block_dots": (None, [VP, VP, VP, CI, CI]),
        "ref_row_dot": (CF, [VP, VP, CI, CI]),
        "ref_matvec_q4_0": (None, [VP, VP, VP, CI, CI, CI]),
        "ref_silu_mul": (CF, [CF, CF, CI]),
        "ref_expert_forward": (None, [VP, VP, VP, VP, VP, CF, CI, CI, CI]),
        "ref_expert_forward_stages": (None, [VP, VP, VP, VP, VP, CF, CI, CI, CI,
                                             VP, VP, VP, VP, VP, VP]),
        "ref_router_logits": (None, [VP, VP, CI, CI, VP]),
        "ref_topk_softmax": (None, [VP, CI, CI, VP, VP, CI]),
        "ref_moe_layer": (None, [VP, ctypes.c_size_t, VP, VP, CI, CI, CI, CI, CI, VP, VP, VP]),
        "ref_rms_scale": (CF, [VP, CI, CF]),
        "ref_moe_block": (None, [VP, ctypes.c_size_t, VP, VP, CF, VP, CI, CI, CI, CI, CI, VP, VP, VP]),
        "ref_decode_step": (None, [VP, VP, VP, CF, CI, VP, CI, CI, CI, CI, CI, VP]),
        "ref_decode_step_mt": (None, [VP, VP, VP, CF, CI, VP, CI, CI, CI, CI, CI, CI]),
        "ref_moe_layer_batched": (None, [VP, ctypes.c_size_t, VP, VP, CI, CI, CI, CI, CI, CI, CI]),
        "ref_moe_block_batched": (None, [VP, ctypes.c_size_t, VP, VP, CF, VP, CI, CI, CI, CI, CI, CI, CI]),
        "ref_moe_block_batched_shared": (None, [VP, ctypes.c_size_t, VP, VP, CF, VP, CI, CI, CI, CI, CI, CI, CI,
                                                VP]),
        "ref_quantize_q8k": (None, [VP, VP, ctypes.c_int64]),
        "ref_matvec_k": (None, [VP, CI, VP, VP, CI, CI]),
        "ref_rms_norm_k": (None, [VP, VP, VP, CI, CF]),
        "ref_expert_forward_k": (None, [VP, VP, VP, CI, VP, VP, CF, CI, CI, CI]),
        "ref_rope": (None, [VP, CI, CI, VP, VP]),
        "ref_attention_decode": (None, [CI, VP, VP, VP, VP, VP, VP, VP, VP, CI, CI, VP, VP, VP, VP,
                                        CI, CI, CI, CI, CI, CI]),
        "ref_fill_normal": (None, [VP, I64, ctypes.c_uint64, CF]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data


# ---------------------------------------------------------------- quantisers

def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // QK * Q8_0_BYTES, dtype=np.uint8)
    lib().ref_quantize_q8_0(_p(x), _p(out), x.size)
    return out


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // QK * Q4_0_BYTES, dtype=np.uint8)
    lib().ref_quantize_q4_0(_p(x), _p(out), x.size)
    return out


def dequantize_q8_0(q: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    n = q.size // Q8_0_BYTES * QK
    out = np.empty(n, dtype=np.float32)
    lib().ref_dequantize_q8_0(_p(q), _p(out), n)
    return out


def dequantize_q4_0(q: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    n = q.size // Q4_0_BYTES * QK
    out = np.empty(n, dtype=np.float32)
    lib().ref_dequantize_q4_0(_p(q), _p(out), n)
    return out


def expf(x: np.ndarray) -> np.ndarray:
    f = lib().ref_expf
    return np.array([f(float(v)) for v in np.asarray(x, dtype=np.float32).ravel()], dtype=np.float32)


# ---------------------------------------------------------------- dots

def block_dots(W: np.ndarray, xq: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.empty((rows, cols // QK), dtype=np.int32)
    lib().ref_block_dots(_p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(xq)), _p(out), rows, cols)
    return out


def matvec(W: np.ndarray, xq: np.ndarray, rows: int, cols: int, mode: int = TG_MIRROR) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    lib().ref_matvec_q4_0(_p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(xq)), _p(y), rows, cols, mode)
    return y


# ---------------------------------------------------------------- expert / MoE

def expert_bytes(embed: int, inter: int) -> int:
    return 3 * inter * (embed // QK) * Q4_0_BYTES


def split_expert(blob: np.ndarray, embed: int, inter: int):
    t = inter * (embed // QK) * Q4_0_BYTES
    return blob[:t], blob[t:2 * t], blob[2 * t:3 * t]


def expert_forward(blob, x, out, w, embed, inter, mode=TG_MIRROR):
    g, u, d = split_expert(np.ascontiguousarray(blob), embed, inter)
    x = np.ascontiguousarray(x, dtype=np.float32)
    lib().ref_expert_forward(_p(g), _p(u), _p(d), _p(x), _p(out), float(w), embed, inter, mode)
    return out


def expert_stages(blob, x, embed, inter, mode=TG_MIRROR):
    g, u, d = split_expert(np.ascontiguousarray(blob), embed, inter)
    x = np.ascontiguousarray(x, dtype=np.float32)
    xq = np.empty(embed // QK * Q8_0_BYTES, np.uint8)
    hq = np.empty(inter // QK * Q8_0_BYTES, np.uint8)
    gg = np.empty(inter, np.float32)
    uu = np.empty(inter, np.float32)
    hh = np.empty(inter, np.float32)
    yy = np.empty(embed, np.float32)
    lib().ref_expert_forward_stages(_p(g), _p(u), _p(d), _p(x), None, 0.0, embed, inter, mode,
                                    _p(xq), _p(gg), _p(uu), _p(hh), _p(hq), _p(yy))
    return dict(xq=xq, g=gg, u=uu, h=hh, hq=hq, y=yy)


def router_logits(R: np.ndarray, x: np.ndarray) -> np.ndarray:
    R = np.ascontiguousarray(R, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    E, H = R.shape
    out = np.empty(E, np.float32)
    lib().ref_router_logits(_p(R), _p(x), E, H, _p(out))
    return out


def topk_softmax(logits: np.ndarray, k: int, mode=TG_MIRROR):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    idx = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    lib().ref_topk_softmax(_p(logits), logits.size, k, _p(idx), _p(w), mode)
    return idx, w


def moe_layer(layer_blob: np.ndarray, R: np.ndarray, x: np.ndarray, k: int, embed: int, inter: int,
              mode=TG_MIRROR):
    """Returns (x_new, idx, w, logits); x is not modified."""
    x = np.array(x, dtype=np.float32, copy=True)
    E = R.shape[0]
    idx = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    logits = np.empty(E, np.float32)
    lib().ref_moe_layer(_p(np.ascontiguousarray(layer_blob)), expert_bytes(embed, inter),
                        _p(np.ascontiguousarray(R, dtype=np.float32)), _p(x), E, k, embed, inter, mode,
                        _p(idx), _p(w), _p(logits))
    return x, idx, w, logits


RMS_EPS = 1e-6


def rms_scale(x: np.ndarray, eps: float = RMS_EPS) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return float(lib().ref_rms_scale(_p(x), x.size, eps))


def moe_block(layer_blob: np.ndarray, R: np.ndarray, x: np.ndarray, k: int, embed: int, inter: int,
              normw=None, eps: float = RMS_EPS, mode=TG_MIRROR):
    """The engine's MoE block with its FFN RMSNorm; returns (x_new, idx, w, logits)."""
    x = np.array(x, dtype=np.float32, copy=True)
    E = R.shape[0]
    idx = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    logits = np.empty(E, np.float32)
    nw = None if normw is None else np.ascontiguousarray(normw, dtype=np.float32)
    lib().ref_moe_block(_p(np.ascontiguousarray(layer_blob)), expert_bytes(embed, inter),
                        _p(np.ascontiguousarray(R, dtype=np.float32)), None if nw is None else _p(nw), eps,
                        _p(x), E, k, embed, inter, mode, _p(idx), _p(w), _p(logits))
    return x, idx, w, logits


def _ptr_array(arrs):
    return (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def decode_step(layer_blobs, routers, x, k, embed, inter, norms=None, eps: float = RMS_EPS, mode=TG_MIRROR):
    """Chained decode step over len(layer_blobs) MoE blocks; returns (x_new, idx[L,k])."""
    L = len(layer_blobs)
    blobs = [np.ascontiguousarray(b) for b in layer_blobs]
    rs = [np.ascontiguousarray(r, dtype=np.float32) for r in routers]
    ns = None if norms is None else [np.ascontiguousarray(n, dtype=np.float32) for n in norms]
    x = np.array(x, dtype=np.float32, copy=True)
    idx = np.empty((L, k), np.int32)
    lib().ref_decode_step(_ptr_array(blobs), _ptr_array(rs), None if ns is None else _ptr_array(ns), eps, L,
                          _p(x), rs[0].shape[0], k, embed, inter, mode, _p(idx))
    return x, idx


def decode_step_mt(layer_blobs, routers, x, k, embed, inter, mode=TG_MIRROR, n_threads=0, norms=None,
                   eps: float = RMS_EPS):
    L = len(layer_blobs)
    lib().ref_decode_step_mt(_ptr_array(layer_blobs), _ptr_array(routers),
                             None if norms is None else _ptr_array(norms), eps, L, _p(x), routers[0].shape[0],
                             k, embed, inter, mode, n_threads)
    return x


def moe_layer_batched(layer_blob, R, x, k, embed, inter, mode=TG_MIRROR, n_threads=0):
    x = np.array(x, dtype=np.float32, copy=True)
    T = x.shape[0]
    lib().ref_moe_layer_batched(_p(np.ascontiguousarray(layer_blob)), expert_bytes(embed, inter),
                                _p(np.ascontiguousarray(R, dtype=np.float32)), _p(x), T, R.shape[0], k,
                                embed, inter, mode, n_threads)
    return x


def moe_block_batched(layer_blob, R, x, k, embed, inter, normw=None, eps: float = RMS_EPS, mode=TG_MIRROR,
                      n_threads=0, shared=None):
    """moe_block for every row of x[T][embed] (independent tokens); returns the new x.
    shared: an optional shared-expert blob, added with weight 1 after the routed experts."""
    x = np.array(x, dtype=np.float32, copy=True)
    T = x.shape[0]
    nw = None if normw is None else np.ascontiguousarray(normw, dtype=np.float32)
    args = (_p(np.ascontiguousarray(layer_blob)), expert_bytes(embed, inter),
            _p(np.ascontiguousarray(R, dtype=np.float32)), None if nw is None else _p(nw), eps,
            _p(x), T, R.shape[0], k, embed, inter, mode, n_threads)
    if shared is None:
        lib().ref_moe_block_batched(*args)
    else:
        sh = np.ascontiguousarray(shared, dtype=np.uint8)
        lib().ref_moe_block_batched_shared(*args, _p(sh))
    return x


# ---------------------------------------------------------------- the reference's K-quant path

Q4K_BYTES, Q6K_BYTES, Q8K_BYTES = 144, 210, 264
FMT_Q4_K, FMT_F16, FMT_Q6_K, FMT_F32 = 0, 1, 2, 4


def quantize_q8k(x) -> np.ndarray:
    """The reference's 256-wide Q8 activation blocks (libtinygiant.c:55-89): per block
    fp32 scale, int32 sum of codes, 256 int8 codes; 264 bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 256 * Q8K_BYTES, np.uint8)
    lib().ref_quantize_q8k(_p(x), _p(out), x.size)
    return out


def matvec_k(W, fmt, x, rows, cols) -> np.ndarray:
    """y = W . x with W in Q4_K (fmt 0, on Q8(256) of x), f16 (1), Q6_K (2) or f32 (4)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, np.float32)
    lib().ref_matvec_k(_p(np.ascontiguousarray(W)), fmt, _p(x), _p(y), rows, cols)
    return y


def rms_norm_k(x, w, eps):
    """tg_rms_norm in the reference's order (libtinygiant.c:322-340)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().ref_rms_norm_k(_p(x), _p(w), _p(out), x.size, float(eps))
    return out


def expert_forward_k(gate, up, down, down_format, x, out, w, embed, inter, mode=TG_MIRROR):
    """tg_expert_forward_mixed (libtinygiant.c:599-643): out += w * expert(x), in place."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    lib().ref_expert_forward_k(_p(np.ascontiguousarray(gate)), _p(np.ascontiguousarray(up)),
                               _p(np.ascontiguousarray(down)), down_format, _p(x), _p(out), float(w),
                               embed, inter, mode)
    return out


def rope(x, cos_row, sin_row, n_heads, head_dim):
    """apply_rope_inplace (libtinygiant.c:344-360) on a copy of x[n_heads * head_dim]."""
    x = np.array(x, dtype=np.float32, copy=True)
    lib().ref_rope(_p(x), n_heads, head_dim, _p(np.ascontiguousarray(cos_row, np.float32)),
                   _p(np.ascontiguousarray(sin_row, np.float32)))
    return x


def attention_decode(q4, wq, wk, wv, wo, q_norm_w, k_norm_w, kv_k, kv_v, kv_len, rope_cos, rope_sin, x,
                     embed, n_heads, n_kv, head_dim, pos, mode=TG_MIRROR):
    """tg_attention_decode (q4 False: fp32 weights) / tg_attention_decode_q4 (q4 True: Q4_K
    wq / wk / wo bytes, f16 wv), libtinygiant.c:364-551.  kv_k / kv_v [n_kv][kv_max][head_dim]
    are updated in place (row kv_len); returns the output [embed]."""
    assert kv_k.dtype == np.float32 and kv_k.flags.c_contiguous and kv_v.flags.c_contiguous
    kv_max = kv_k.shape[1]
    out = np.empty(embed, np.float32)
    arrs = [np.ascontiguousarray(a) for a in (wq, wk, wv, wo)]
    qn = np.ascontiguousarray(q_norm_w, np.float32)
    kn = np.ascontiguousarray(k_norm_w, np.float32)
    rc = np.ascontiguousarray(rope_cos, np.float32)
    rs = np.ascontiguousarray(rope_sin, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    lib().ref_attention_decode(int(bool(q4)), *[_p(a) for a in arrs], _p(qn), _p(kn), _p(kv_k), _p(kv_v),
                               kv_len, kv_max, _p(rc), _p(rs), _p(x), _p(out), embed, n_heads, n_kv, head_dim,
                               pos, mode)
    return out


def fill_normal(n: int, seed: int, sigma: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().ref_fill_normal(_p(out), n, seed, sigma)
    return out


def nproc() -> int:
    return len(os.sched_getaffinity(0))
