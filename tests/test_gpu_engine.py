"""The reference engine's token loop on the device (tinygiant/engine.py:188-266,
378-409) against the same loop through the oracle: embedding row, attention and MoE
block per layer, final RMSNorm, output projection.  Logits bit-exact at every prefill
and decode position; greedy and sampled generation pick the same tokens."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TG_MIRROR = 1


class OracleEngine:
    """engine.py:188-266 through the oracle, with its own caches."""

    def __init__(self, oracle, layers, moe, embd, onorm, head, head_fmt, shape, cos, sin):
        self.o, self.layers, self.moe = oracle, layers, moe
        self.embd, self.onorm, self.head, self.head_fmt = embd, onorm, head, head_fmt
        self.shape, self.cos, self.sin = shape, cos, sin
        E, NH, NKV, HD, I, k, KVM = shape
        self.caches = [(np.zeros((NKV, KVM, HD), np.float32), np.zeros((NKV, KVM, HD), np.float32))
                       for _ in layers]
        self.routes = []   # (layer, top-k ids) of every MoE block evaluated

    def forward(self, token, pos):
        o, (E, NH, NKV, HD, I, k, KVM) = self.o, self.shape
        x = self.embd[token].copy()
        blobs, Rs, norms = self.moe
        for l, (W, qn, kn, an) in enumerate(self.layers):
            normed = o.rms_norm_k(x, an, 1e-6)
            att = o.attention_decode(True, *W, qn, kn, self.caches[l][0], self.caches[l][1], pos, self.cos, self.sin,
                                     normed, E, NH, NKV, HD, pos, TG_MIRROR)
            x = (x + att).astype(np.float32)
            x, idx = o.moe_block(blobs[l], Rs[l], x, k, E, I, normw=norms[l])[:2]
            self.routes.append((l, idx))
        final = o.rms_norm_k(x, self.onorm, 1e-6)
        return o.matvec_k(self.head, self.head_fmt, final, self.head.shape[0], E)

    def generate(self, prompt, n, temperature, top_p, rng):
        from tinygiant_b200.engine import sample_token
        for i, t in enumerate(prompt):
            logits = self.forward(t, i)
        out, nxt = [], None
        for step in range(n):
            if step > 0:
                logits = self.forward(nxt, len(prompt) + step - 1)
            nxt = sample_token(logits, temperature, top_p, rng)
            out.append(nxt)
        return out


def _build(oracle, head_f16):
    import torch
    from tests.test_gpu_attention import make_layer, rope_tables
    from tests.test_gpu_parity import build_model
    from tinygiant_b200.engine import AttentionModel, DecodeEngine
    E, I, NE, k, L, NH, NKV, HD, KVM, V = 1024, 512, 64, 8, 2, 16, 4, 64, 32, 1000
    m, blobs, Rs, rng = build_model(oracle, E, I, NE, k, L, seed=31 + head_f16)
    am = AttentionModel(E, NH, NKV, HD, L, kv_max=KVM, q4=True)
    layers = []
    for l in range(L):
        W, qn, kn = make_layer(rng, True, E, NH, NKV, HD)
        an = (1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        am.set_layer(l, *W, qn, kn, an)
        layers.append((W, qn, kn, an))
    embd = (rng.standard_normal((V, E)) * 0.5).astype(np.float32)
    onorm = (1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    head = (rng.standard_normal((V, E)) * 0.05).astype(np.float32)
    head_dev = torch.from_numpy(head).cuda()
    if head_f16:
        head = head.astype(np.float16)
        head_dev = head_dev.half()
    eng = DecodeEngine(m, am, torch.from_numpy(embd).cuda(), torch.from_numpy(onorm).cuda(), head_dev)
    cos, sin = rope_tables(KVM, HD)
    ref = OracleEngine(oracle, layers, (blobs, Rs, m.norms), embd, onorm,
                       head.view(np.uint16) if head_f16 else head, 1 if head_f16 else 4,
                       (E, NH, NKV, HD, I, k, KVM), cos, sin)
    return eng, ref, m, am


def _same(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("head_f16", [False, True])
def test_forward_one_token_logits_bit_exact(oracle, head_f16):
    eng, ref, m, am = _build(oracle, head_f16)
    eng.reset()
    for pos, tok in enumerate([5, 17, 300, 999, 0]):
        got = eng.forward_one_token(tok, pos).cpu().numpy()
        assert _same(got, ref.forward(tok, pos)), pos
    # a new sequence after reset replays the first token exactly
    ref2 = OracleEngine(ref.o, ref.layers, ref.moe, ref.embd, ref.onorm, ref.head, ref.head_fmt, ref.shape, ref.cos,
                        ref.sin)
    eng.reset()
    assert _same(eng.forward_one_token(5, 0).cpu().numpy(), ref2.forward(5, 0))
    am.close()
    m.close()


def test_generate_stream_greedy_and_sampled(oracle):
    eng, ref, m, am = _build(oracle, False)
    prompt = [11, 42, 7]
    eng.reset()
    greedy = list(eng.generate_stream(prompt, n_tokens=4, temperature=0.0))
    assert greedy == ref.generate(prompt, 4, 0.0, 0.9, None)
    eng.reset()
    ref_s = OracleEngine(ref.o, ref.layers, ref.moe, ref.embd, ref.onorm, ref.head, ref.head_fmt, ref.shape, ref.cos,
                         ref.sin)
    sampled = list(eng.generate_stream(prompt, n_tokens=4, temperature=0.8, top_p=0.9,
                                       rng=np.random.RandomState(7)))
    assert sampled == ref_s.generate(prompt, 4, 0.8, 0.9, np.random.RandomState(7))
    am.close()
    m.close()


def test_calibrate_and_pin_experts(oracle):
    """engine.py:154-186 on the device: calibrate() counts every layer's routing of the
    prompt and the greedy tokens (the oracle's routing of the same tokens), then
    pin_experts() pins each layer's most requested experts in a host-tier cache."""
    import torch
    from tinygiant_b200.cache import HostTierCache
    eng, ref, m, am = _build(oracle, False)
    prompt = [3, 141, 59]
    eng.reset()
    counts = eng.calibrate(prompt, n_tokens=2)
    # the oracle's routing of the same tokens: the prompt, then two greedy steps
    logits = None
    for i, t in enumerate(prompt):
        logits = ref.forward(t, i)
    nxt = int(np.argmax(logits))
    for step in range(2):
        logits = ref.forward(nxt, len(prompt) + step)
        nxt = int(np.argmax(logits))
    want = {}
    for l, idx in ref.routes:
        for e in idx:
            want[(l, int(e))] = want.get((l, int(e)), 0) + 1
    assert counts == want
    host = [torch.from_numpy(m.read_experts(l, 0, m.n_experts)).pin_memory() for l in range(m.n_layers)]
    cache = HostTierCache(m, host, cache_slots=4)
    eng.reset()
    n = eng.pin_experts(cache, 2, calibrate_tokens=2, prompt_tokens=prompt)
    assert n == 2 * m.n_layers and cache.access_counts == {}
    for l in range(m.n_layers):
        top = sorted((-c, e) for (ll, e), c in want.items() if ll == l)[:2]
        assert all((l, e) in cache.pinned for _, e in top)
    am.close()
    m.close()
