"""GPU parity of the reference's attention decode step (csrc/libtinygiant.c:344-551:
tg_attention_decode, tg_attention_decode_q4) through the C ABI: outputs and KV caches
bit-exact against the oracle's restatement, which tests/test_oracle_attention.py pins
to the reference package's own numpy path; plus the golden fixture's float64 value
within the 1e-5 relative tolerance."""
from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import ROOT
from tests.test_gpu_kquant import q4k_blocks, same_bits

pytestmark = pytest.mark.gpu

TG_MIRROR = 1


def rope_tables(max_pos, hd, base=1_000_000.0):
    """build_rope_cache's recipe (tinygiant/_math.py): fp32 inverse frequencies, outer
    product with the positions, fp32 cos / sin."""
    inv = (1.0 / (base ** (np.arange(0, hd, 2, dtype=np.float32) / hd))).astype(np.float32)
    f = np.outer(np.arange(max_pos, dtype=np.float32), inv)
    return np.cos(f).astype(np.float32), np.sin(f).astype(np.float32)


def make_layer(rng, q4, E, NH, NKV, HD):
    qd, kvd = NH * HD, NKV * HD
    if q4:
        wq, wk, wo = q4k_blocks(rng, qd * E // 256), q4k_blocks(rng, kvd * E // 256), q4k_blocks(rng, E * qd // 256)
        wv = (rng.standard_normal(kvd * E) * 0.05).astype(np.float16).view(np.uint16)
    else:
        wq, wk, wv, wo = [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in (qd * E, kvd * E, kvd * E, E * qd)]
    qn = (1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    return (wq, wk, wv, wo), qn, kn


def host_call(lib, q4, W, qn, kn, kv_k, kv_v, kv_len, cos, sin, x, E, NH, NKV, HD, pos):
    out = np.empty(E, np.float32)
    fn = lib.tg_attention_decode_q4 if q4 else lib.tg_attention_decode
    rc = fn(*(w.ctypes.data for w in W), qn.ctypes.data, kn.ctypes.data, kv_k.ctypes.data, kv_v.ctypes.data,
            kv_len, kv_k.shape[1], cos.ctypes.data, sin.ctypes.data, x.ctypes.data, out.ctypes.data, E, NH, NKV, HD,
            pos)
    assert rc == 0, lib.tg_last_error()
    return out


class DeviceLayer:
    """One layer's weights, norms, rope tables and caches resident on cuda:0."""

    def __init__(self, lib, q4, W, qn, kn, kv_k, kv_v, cos, sin, E, NH, NKV, HD):
        import torch
        self.torch, self.lib, self.q4 = torch, lib, q4
        dev = torch.device("cuda:0")

        def t(a):
            a = np.ascontiguousarray(a)
            return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).to(dev)

        self.W = [t(w) for w in W]
        self.qn, self.kn, self.cos, self.sin = t(qn), t(kn), t(cos), t(sin)
        self.kv_k, self.kv_v = t(kv_k), t(kv_v)
        self.shape = (E, NH, NKV, HD)
        self.kv_max = kv_k.shape[1]
        self.sb = lib.tgx_attention_scratch_bytes(NH, NKV, HD, self.kv_max)
        self.scratch = torch.empty(self.sb, dtype=torch.uint8, device=dev)
        self.out = torch.empty(E, dtype=torch.float32, device=dev)

    def step(self, x, kv_len, pos):
        import ctypes
        torch = self.torch
        xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        E, NH, NKV, HD = self.shape
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        rc = self.lib.tgx_attention_decode(int(self.q4), *(P(w) for w in self.W), P(self.qn), P(self.kn),
                                           P(self.kv_k), P(self.kv_v), kv_len, self.kv_max, P(self.cos), P(self.sin),
                                           P(xd), P(self.out), E, NH, NKV, HD, pos, P(self.scratch), self.sb, None)
        assert rc == 0, self.lib.tg_last_error()
        torch.cuda.synchronize()
        return self.out.cpu().numpy()

    def caches(self):
        return self.kv_k.cpu().numpy(), self.kv_v.cpu().numpy()


def test_host_entry_q4_golden_bit_exact(lib, oracle):
    ga = dict(np.load(ROOT / "tests" / "golden" / "golden_attention.npz"))
    E, NH, NKV, HD, POS = (int(ga[k]) for k in ("embed", "n_heads", "n_kv", "head_dim", "pos"))
    W = (ga["wq"], ga["wk"], ga["wv"], ga["wo"])
    kg, vg = ga["kv_k"].copy(), ga["kv_v"].copy()
    ko, vo = ga["kv_k"].copy(), ga["kv_v"].copy()
    got = host_call(lib, True, W, ga["q_norm"], ga["k_norm"], kg, vg, POS, ga["rope_cos"], ga["rope_sin"], ga["x"],
                    E, NH, NKV, HD, POS)
    ref = oracle.attention_decode(True, *W, ga["q_norm"], ga["k_norm"], ko, vo, POS, ga["rope_cos"], ga["rope_sin"],
                                  ga["x"], E, NH, NKV, HD, POS, TG_MIRROR)
    assert same_bits(got, ref)
    assert same_bits(kg, ko) and same_bits(vg, vo)
    y64 = ga["out_q4_64"]
    assert np.max(np.abs(got - y64)) <= 1e-5 * np.max(np.abs(y64))


@pytest.mark.parametrize("q4", [True, False])
def test_host_entry_random_bit_exact(lib, oracle, q4):
    rng = np.random.default_rng(7 + q4)
    E, NH, NKV, HD, KVM, L = 512, 8, 2, 64, 40, 17
    W, qn, kn = make_layer(rng, q4, E, NH, NKV, HD)
    kv_k = np.zeros((NKV, KVM, HD), np.float32)
    kv_v = np.zeros((NKV, KVM, HD), np.float32)
    kv_k[:, :L] = rng.standard_normal((NKV, L, HD))
    kv_v[:, :L] = rng.standard_normal((NKV, L, HD))
    cos, sin = rope_tables(64, HD)
    x = rng.standard_normal(E).astype(np.float32)
    kg, vg, ko, vo = kv_k.copy(), kv_v.copy(), kv_k.copy(), kv_v.copy()
    got = host_call(lib, q4, W, qn, kn, kg, vg, L, cos, sin, x, E, NH, NKV, HD, 33)
    ref = oracle.attention_decode(q4, *W, qn, kn, ko, vo, L, cos, sin, x, E, NH, NKV, HD, 33, TG_MIRROR)
    assert same_bits(got, ref) and same_bits(kg, ko) and same_bits(vg, vo)


@pytest.mark.parametrize("kv_len", [0, 1, 31, 32, 33, 257, 1023])
def test_device_entry_qwen_shape(lib, oracle, kv_len):
    """Qwen3-30B-A3B attention (embed 2048, 32 query heads, 4 kv heads, head_dim 128)
    with Q4_K / f16 weights, the caches [4][1024][128] on the device."""
    rng = np.random.default_rng(kv_len + 11)
    E, NH, NKV, HD, KVM = 2048, 32, 4, 128, 1024
    W, qn, kn = make_layer(rng, True, E, NH, NKV, HD)
    kv_k = np.zeros((NKV, KVM, HD), np.float32)
    kv_v = np.zeros((NKV, KVM, HD), np.float32)
    kv_k[:, :kv_len] = rng.standard_normal((NKV, kv_len, HD))
    kv_v[:, :kv_len] = rng.standard_normal((NKV, kv_len, HD))
    cos, sin = rope_tables(KVM, HD)
    x = rng.standard_normal(E).astype(np.float32)
    dl = DeviceLayer(lib, True, W, qn, kn, kv_k, kv_v, cos, sin, E, NH, NKV, HD)
    got = dl.step(x, kv_len, kv_len)
    ref = oracle.attention_decode(True, *W, qn, kn, kv_k, kv_v, kv_len, cos, sin, x, E, NH, NKV, HD, kv_len,
                                  TG_MIRROR)
    gk, gv = dl.caches()
    assert same_bits(got, ref)
    assert same_bits(gk, kv_k) and same_bits(gv, kv_v)


@pytest.mark.parametrize("q4,E,NH,NKV,HD", [
    (True, 256, 4, 4, 64),      # no grouping
    (False, 512, 32, 1, 32),    # 32 query heads on one kv head
    (True, 512, 2, 1, 256),     # the widest head
    (False, 200, 5, 5, 40),     # odd head count, head_dim 40
    (False, 96, 3, 1, 8),       # the narrowest head
])
def test_device_entry_shapes(lib, oracle, q4, E, NH, NKV, HD):
    rng = np.random.default_rng(E + NH * 7 + HD)
    KVM, L = 100, 70
    W, qn, kn = make_layer(rng, q4, E, NH, NKV, HD)
    kv_k = np.zeros((NKV, KVM, HD), np.float32)
    kv_v = np.zeros((NKV, KVM, HD), np.float32)
    kv_k[:, :L] = rng.standard_normal((NKV, L, HD))
    kv_v[:, :L] = rng.standard_normal((NKV, L, HD))
    cos, sin = rope_tables(128, HD)
    x = rng.standard_normal(E).astype(np.float32)
    dl = DeviceLayer(lib, q4, W, qn, kn, kv_k, kv_v, cos, sin, E, NH, NKV, HD)
    got = dl.step(x, L, 90)
    ref = oracle.attention_decode(q4, *W, qn, kn, kv_k, kv_v, L, cos, sin, x, E, NH, NKV, HD, 90, TG_MIRROR)
    gk, gv = dl.caches()
    assert same_bits(got, ref) and same_bits(gk, kv_k) and same_bits(gv, kv_v)


def test_decode_sequence_grows_cache(lib, oracle):
    """Twelve tokens in a row from an empty cache (the engine's kv_len = pos), each fed
    the previous output: every output and the final caches bit-exact."""
    rng = np.random.default_rng(5)
    E, NH, NKV, HD, KVM = 1024, 16, 4, 64, 16
    W, qn, kn = make_layer(rng, True, E, NH, NKV, HD)
    kv_k = np.zeros((NKV, KVM, HD), np.float32)
    kv_v = np.zeros((NKV, KVM, HD), np.float32)
    cos, sin = rope_tables(KVM, HD)
    dl = DeviceLayer(lib, True, W, qn, kn, kv_k, kv_v, cos, sin, E, NH, NKV, HD)
    x = rng.standard_normal(E).astype(np.float32)
    for pos in range(12):
        got = dl.step(x, pos, pos)
        ref = oracle.attention_decode(True, *W, qn, kn, kv_k, kv_v, pos, cos, sin, x, E, NH, NKV, HD, pos, TG_MIRROR)
        assert same_bits(got, ref), pos
        x = (ref / np.max(np.abs(ref))).astype(np.float32)
    gk, gv = dl.caches()
    assert same_bits(gk, kv_k) and same_bits(gv, kv_v)


def _oracle_token(oracle, x, layers, moe, caches, pos, cos, sin, shape):
    """One decode token through the oracle: per layer x += attention(rms_norm(x) * attn_norm)
    (engine.py:203-226), then the MoE block (engine.py:229-258)."""
    E, NH, NKV, HD, I, k = shape
    for l, (W, qn, kn, an) in enumerate(layers):
        normed = oracle.rms_norm_k(x, an, 1e-6)
        out = oracle.attention_decode(True, *W, qn, kn, caches[l][0], caches[l][1], pos, cos, sin, normed, E, NH, NKV,
                                      HD, pos, TG_MIRROR)
        x = (x + out).astype(np.float32)
        if moe is not None:
            blobs, Rs, norms = moe
            x = oracle.moe_block(blobs[l], Rs[l], x, k, E, I, normw=norms[l])[0]
    return x


def _attention_model(rng, E, NH, NKV, HD, L, kv_max):
    from tinygiant_b200.engine import AttentionModel
    am = AttentionModel(E, NH, NKV, HD, L, kv_max=kv_max, q4=True)
    layers = []
    for l in range(L):
        W, qn, kn = make_layer(rng, True, E, NH, NKV, HD)
        an = (1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        am.set_layer(l, *W, qn, kn, an)
        layers.append((W, qn, kn, an))
    return am, layers


def test_decode_token_whole_layers_bit_exact(oracle):
    """Whole decode layers (attention, then the fused MoE block) for six tokens from an
    empty cache, replayed from one CUDA graph with the position read on the device (one
    token eager): every token's hidden state and the final caches bit-exact; a reset
    then replays the first token exactly."""
    import torch
    from tests.test_gpu_parity import build_model
    E, I, NE, k, L, NH, NKV, HD, KVM = 1024, 512, 64, 8, 2, 16, 4, 64, 16
    m, blobs, Rs, rng = build_model(oracle, E, I, NE, k, L, seed=77)
    am, layers = _attention_model(rng, E, NH, NKV, HD, L, KVM)
    cos, sin = rope_tables(KVM, HD)
    caches = [(np.zeros((NKV, KVM, HD), np.float32), np.zeros((NKV, KVM, HD), np.float32)) for _ in range(L)]
    shape = (E, NH, NKV, HD, I, k)
    x = (rng.standard_normal(E) * 0.5).astype(np.float32)
    x0 = x.copy()
    xd = torch.from_numpy(x.copy()).cuda()
    first = None
    for pos in range(6):
        am.decode_token(xd, m, eager=(pos == 2))
        x = _oracle_token(oracle, x, layers, (blobs, Rs, m.norms), caches, pos, cos, sin, shape)
        got = xd.cpu().numpy()
        assert same_bits(got, x), pos
        first = got.copy() if pos == 0 else first
    assert am.status() == 6
    for l in range(L):
        gk, gv = am.read_kv(l)
        assert same_bits(gk, caches[l][0]) and same_bits(gv, caches[l][1])
    am.reset(0)
    xd.copy_(torch.from_numpy(x0))
    am.decode_token(xd, m)
    assert same_bits(xd.cpu().numpy(), first) and am.status() == 1
    am.close()
    m.close()


def test_attention_layer_calls_and_full_cache(oracle):
    """tgx_attn_layer per layer plus tgx_attn_advance equals the oracle; a cache of
    kv_max rows takes exactly kv_max tokens, and the next one is refused."""
    import torch
    E, NH, NKV, HD, L, KVM = 512, 8, 2, 64, 3, 3
    rng = np.random.default_rng(13)
    am, layers = _attention_model(rng, E, NH, NKV, HD, L, KVM)
    cos, sin = rope_tables(KVM, HD)
    caches = [(np.zeros((NKV, KVM, HD), np.float32), np.zeros((NKV, KVM, HD), np.float32)) for _ in range(L)]
    x = rng.standard_normal(E).astype(np.float32)
    xd = torch.from_numpy(x.copy()).cuda()
    for pos in range(KVM):
        if pos == 1:
            am.decode_token(xd)            # attention-only token through the graph
        else:
            for l in range(L):
                am.layer(l, xd)
            am.advance()
        x = _oracle_token(oracle, x, layers, None, caches, pos, cos, sin, (E, NH, NKV, HD, 0, 0))
        assert same_bits(xd.cpu().numpy(), x), pos
    assert am.status() == KVM
    with pytest.raises(RuntimeError):
        am.decode_token(xd)
    with pytest.raises(RuntimeError):
        am.layer(0, xd)
    am.close()
