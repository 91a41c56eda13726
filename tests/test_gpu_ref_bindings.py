"""Every function the reference's own loader registers (tinygiant/_lib.py:26-76, its
prototype table recorded in tests/golden/ref_bindings.json), called once through
exactly that registration (void results, as the reference binds them) on host buffers,
against the oracle: bit-exact for every output and KV-cache row.  tg_transformer_layer
(csrc/libtinygiant.c:662-702) runs a whole layer with experts of all three down
formats."""
import ctypes
import json

import numpy as np
import pytest

from tests.conftest import ROOT
from tests.test_gpu_attention import make_layer, rope_tables
from tests.test_gpu_kquant import FF16, FF32, FQ4K, FQ6K, matrix, q4k_blocks, same_bits

pytestmark = pytest.mark.gpu

TG_MIRROR = 1


@pytest.fixture(scope="module")
def reflib():
    from tinygiant_b200._lib import find_library
    table = json.loads((ROOT / "tests" / "golden" / "ref_bindings.json").read_text())["functions"]
    lib = ctypes.CDLL(str(find_library()))
    def ctype(name):   # the recorded ctypes class names (c_size_t is recorded as its alias's name)
        return None if name == "None" else getattr(ctypes, name)

    for name, proto in table.items():
        fn = getattr(lib, name)
        fn.restype = ctype(proto["restype"])
        fn.argtypes = [ctype(a) for a in proto["argtypes"]]
    lib.called = set()
    return lib, table


def P(a):
    return a.ctypes.data


def test_matvecs_and_norm(reflib, oracle):
    lib, _ = reflib
    rng = np.random.default_rng(31)
    rows, cols = 96, 2048
    x = rng.standard_normal(cols).astype(np.float32)
    for fmt, name in ((FQ4K, "tg_matmul_q4k"), (FQ6K, "tg_matmul_q6k"), (FF16, "tg_f16_matvec"),
                      (FF32, "tg_f32_matvec")):
        W = matrix(rng, fmt, rows, cols)
        y = np.empty(rows, np.float32)
        getattr(lib, name)(P(W), P(x), P(y), rows, cols)
        assert same_bits(y, oracle.matvec_k(W, fmt, x, rows, cols)), name
        lib.called.add(name)
    w = rng.uniform(0.5, 1.5, cols).astype(np.float32)
    out = np.empty(cols, np.float32)
    lib.tg_rms_norm(P(x), P(w), P(out), cols, 1e-6)
    assert same_bits(out, oracle.rms_norm_k(x, w, 1e-6))
    lib.called.add("tg_rms_norm")


def test_expert_calls(reflib, oracle):
    lib, _ = reflib
    rng = np.random.default_rng(32)
    H, I = 2048, 768
    x = rng.standard_normal(H).astype(np.float32)
    g, u, d = q4k_blocks(rng, I * H // 256), q4k_blocks(rng, I * H // 256), q4k_blocks(rng, H * I // 256)
    blob = np.concatenate([g, u, d])
    out = (rng.standard_normal(H) * 0.1).astype(np.float32)
    ref = out.copy()
    lib.tg_expert_forward(P(blob), P(x), P(out), 0.25, H, I)
    assert same_bits(out, oracle.expert_forward_k(g, u, d, FQ4K, x, ref, 0.25, H, I))
    d6 = matrix(rng, FQ6K, H, I)
    out2 = out.copy()
    lib.tg_expert_forward_mixed(P(g), P(u), P(d6), FQ6K, P(x), P(out2), 0.5, H, I)
    assert same_bits(out2, oracle.expert_forward_k(g, u, d6, FQ6K, x, out.copy(), 0.5, H, I))
    lib.called.update({"tg_expert_forward", "tg_expert_forward_mixed"})


@pytest.mark.parametrize("q4", [False, True])
def test_attention_calls(reflib, oracle, q4):
    lib, _ = reflib
    rng = np.random.default_rng(33 + q4)
    E, NH, NKV, HD, KVM, KL = 512, 8, 2, 64, 24, 9
    W, qn, kn = make_layer(rng, q4, E, NH, NKV, HD)
    kv_k = np.zeros((NKV, KVM, HD), np.float32)
    kv_v = np.zeros((NKV, KVM, HD), np.float32)
    kv_k[:, :KL] = rng.standard_normal((NKV, KL, HD))
    kv_v[:, :KL] = rng.standard_normal((NKV, KL, HD))
    cos, sin = rope_tables(32, HD)
    x = rng.standard_normal(E).astype(np.float32)
    kg, vg, ko, vo = kv_k.copy(), kv_v.copy(), kv_k.copy(), kv_v.copy()
    out = np.empty(E, np.float32)
    fn = lib.tg_attention_decode_q4 if q4 else lib.tg_attention_decode
    fn(*(P(w) for w in W), P(qn), P(kn), P(kg), P(vg), KL, KVM, P(cos), P(sin), P(x), P(out), E, NH, NKV, HD, KL)
    ref = oracle.attention_decode(q4, *W, qn, kn, ko, vo, KL, cos, sin, x, E, NH, NKV, HD, KL, TG_MIRROR)
    assert same_bits(out, ref) and same_bits(kg, ko) and same_bits(vg, vo)
    lib.called.add("tg_attention_decode_q4" if q4 else "tg_attention_decode")


def test_page_calls(reflib):
    lib, _ = reflib
    buf = np.zeros(1 << 20, np.uint8)
    lib.tg_prefetch(P(buf), buf.nbytes)
    addrs = (ctypes.c_void_p * 2)(P(buf), P(buf) + 4096)
    lens = (ctypes.c_size_t * 2)(4096, 8192)
    lib.tg_prefetch_batch(addrs, lens, 2)
    assert lib.tg_mlock(P(buf), buf.nbytes) in (0, -1)   # int, as the reference binds it
    lib.called.update({"tg_prefetch", "tg_prefetch_batch", "tg_mlock"})


def test_transformer_layer(reflib, oracle):
    lib, table = reflib
    rng = np.random.default_rng(34)
    E, NH, NKV, HD, KVM, KL, I = 512, 8, 2, 64, 24, 9, 256
    W, qn, kn = make_layer(rng, False, E, NH, NKV, HD)
    an = (1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    fn_ = (1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    kv_k = np.zeros((NKV, KVM, HD), np.float32)
    kv_v = np.zeros((NKV, KVM, HD), np.float32)
    kv_k[:, :KL] = rng.standard_normal((NKV, KL, HD))
    kv_v[:, :KL] = rng.standard_normal((NKV, KL, HD))
    cos, sin = rope_tables(32, HD)
    fmts = [FQ4K, FF16, FQ6K, FQ4K]
    experts = [(q4k_blocks(rng, I * E // 256), q4k_blocks(rng, I * E // 256), matrix(rng, f, E, I)) for f in fmts]
    wts = rng.dirichlet(np.ones(len(fmts))).astype(np.float32)
    x0 = rng.standard_normal(E).astype(np.float32)
    # the oracle, statement by statement as csrc/libtinygiant.c:662-702
    ko, vo = kv_k.copy(), kv_v.copy()
    xr = x0.copy()
    normed = oracle.rms_norm_k(xr, an, 1e-6)
    xr = xr + oracle.attention_decode(False, *W, qn, kn, ko, vo, KL, cos, sin, normed, E, NH, NKV, HD, KL, TG_MIRROR)
    normed = oracle.rms_norm_k(xr, fn_, 1e-6)
    moe = np.zeros(E, np.float32)
    for (g, u, d), f, w in zip(experts, fmts, wts):
        oracle.expert_forward_k(g, u, d, f, normed, moe, float(w), E, I)
    xr = xr + moe
    # this library through the reference's registration
    kg, vg, x = kv_k.copy(), kv_v.copy(), x0.copy()
    gp = (ctypes.c_void_p * len(fmts))(*[P(e[0]) for e in experts])
    up = (ctypes.c_void_p * len(fmts))(*[P(e[1]) for e in experts])
    dp = (ctypes.c_void_p * len(fmts))(*[P(e[2]) for e in experts])
    df = np.array(fmts, np.int32)
    lib.tg_transformer_layer(*(P(w) for w in W), P(an), P(qn), P(kn), P(fn_), P(kg), P(vg), KL, KVM, P(cos),
                             P(sin), gp, up, dp, P(df), P(wts), len(fmts), P(x), E, I, NH, NKV, HD, KL)
    assert same_bits(x, xr)
    assert same_bits(kg, ko) and same_bits(vg, vo)
    lib.called.add("tg_transformer_layer")


def test_every_registered_function_called(reflib):
    lib, table = reflib
    assert set(table) <= lib.called, f"not called: {sorted(set(table) - lib.called)}"
