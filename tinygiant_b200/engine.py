"""Device-resident MoE expert path: the reference engine's per-layer MoE block
(tinygiant/engine.py:229-258: router -> top-k -> softmax -> expert forwards ->
weighted combine -> residual) run by libtinygiant.so on a B200.

PyTorch is used only for device/pinned buffers and streams; all arithmetic is
in the library's CUDA kernels.  There is no CPU fallback: a missing library or
device raises.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _constants as C
from ._lib import TGX_EAGER, TGX_MULTI, TgxShape, check, get_lib


def _stream_handle(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def _dev_ptr(t) -> int:
    import torch
    assert isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
    return t.data_ptr()


class MoEModel:
    """L MoE layers of E Q4_0 experts (gate | up | down) plus their fp32 routers, in HBM."""

    def __init__(self, embed=C.EMBED_DIM, inter=C.EXPERT_INTERMEDIATE, n_experts=C.N_EXPERTS,
                 top_k=C.N_EXPERTS_USED, n_layers=C.N_LAYERS, device=0):
        self.lib = get_lib()
        self.shape = TgxShape(embed, inter, n_experts, top_k, n_layers, C.RMS_EPS)
        self.embed, self.inter, self.n_experts, self.top_k, self.n_layers = embed, inter, n_experts, top_k, n_layers
        self.device = device
        h = ctypes.c_void_p()
        check(self.lib.tgx_ctx_create(device, ctypes.byref(self.shape), ctypes.byref(h)), self.lib)
        self._ctx = h
        self.expert_bytes = int(self.lib.tgx_expert_bytes(h))
        assert self.expert_bytes == C.expert_bytes(embed, inter)

    # ---------------------------------------------------------------- lifetime
    def close(self):
        if self._ctx:
            self.lib.tgx_ctx_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._ctx

    # ---------------------------------------------------------------- weights
    def load_experts(self, layer: int, blob: np.ndarray, first: int = 0):
        """blob: uint8 ggml Q4_0 experts, expert-contiguous (a layer_NNN.q4.bin slice)."""
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        n = blob.size // self.expert_bytes
        assert n * self.expert_bytes == blob.size
        check(self.lib.tgx_load_experts(self._ctx, layer, first, n, blob.ctypes.data, 0), self.lib)

    def load_experts_rows(self, layer: int, blob: np.ndarray, first: int = 0):
        """blob: experts already in the row-split layout (a version-4 "rows" relayout):
        copied as they are."""
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        n = blob.size // self.expert_bytes
        assert n * self.expert_bytes == blob.size
        check(self.lib.tgx_load_experts_rows(self._ctx, layer, first, n, blob.ctypes.data, 0), self.lib)

    def load_experts_device(self, layer: int, ptr: int, n: int, first: int = 0):
        check(self.lib.tgx_load_experts(self._ctx, layer, first, n, ptr, 1), self.lib)

    def read_experts(self, layer: int, first: int, n: int) -> np.ndarray:
        out = np.empty(n * self.expert_bytes, np.uint8)
        check(self.lib.tgx_read_experts(self._ctx, layer, first, n, out.ctypes.data), self.lib)
        return out

    def set_router(self, layer: int, R: np.ndarray):
        R = np.ascontiguousarray(R, dtype=np.float32)
        assert R.shape == (self.n_experts, self.embed)
        check(self.lib.tgx_set_router(self._ctx, layer, R.ctypes.data, 0), self.lib)

    def set_ffn_norm(self, layer: int, w: np.ndarray):
        """FFN RMSNorm weight of `layer` (engine.py:229, default all ones)."""
        w = np.ascontiguousarray(w, dtype=np.float32)
        assert w.shape == (self.embed,)
        check(self.lib.tgx_set_ffn_norm(self._ctx, layer, w.ctypes.data, 0), self.lib)

    def fill_synthetic(self, seed: int, w_sigma: float = 0.02, r_sigma: float = 0.02):
        check(self.lib.tgx_fill_synthetic(self._ctx, seed, w_sigma, r_sigma), self.lib)

    # ---------------------------------------------------------------- compute
    def expert_forward(self, layer: int, expert: int, x, out, weight: float, stream=None):
        """out (cuda f32[embed]) += weight * expert(x): one resident expert, the reference's
        tg_expert_forward on device memory."""
        check(self.lib.tgx_expert_forward(self._ctx, layer, expert, _dev_ptr(x), _dev_ptr(out), weight,
                                          _stream_handle(stream)), self.lib)

    def moe_layer(self, layer: int, x, stream=None):
        """MoE block `layer` on x (cuda f32[embed]) in place:
        x += sum_j w_j * expert_j(RMSNorm(x) * ffn_norm)."""
        check(self.lib.tgx_moe_layer(self._ctx, layer, _dev_ptr(x), _stream_handle(stream)), self.lib)

    def decode_step(self, x, stream=None, eager: bool = False, multi: bool = False):
        """All layers chained on x in place: one fused kernel per step (or three
        kernels per layer with multi=True), replayed from a CUDA graph unless eager."""
        flags = (TGX_EAGER if eager else 0) | (TGX_MULTI if multi else 0)
        check(self.lib.tgx_decode_step(self._ctx, _dev_ptr(x), _stream_handle(stream), flags), self.lib)

    def moe_batched(self, layer: int, X, stream=None):
        """MoE block `layer` for T tokens at once on X (cuda f32[T][embed]) in place;
        each row gets exactly what moe_layer gives it."""
        assert X.dim() == 2 and X.shape[1] == self.embed
        check(self.lib.tgx_moe_batched(self._ctx, layer, _dev_ptr(X), X.shape[0], _stream_handle(stream)), self.lib)

    def decode_batched(self, X, stream=None):
        """All layers chained for T tokens on X (cuda f32[T][embed]) in place."""
        assert X.dim() == 2 and X.shape[1] == self.embed
        check(self.lib.tgx_decode_batched(self._ctx, _dev_ptr(X), X.shape[0], _stream_handle(stream)), self.lib)

    def set_batched_kernels(self, kernels: int):
        """Expert matmuls of the batched path: 0 auto, 1 dp4a, 2 tensor cores (same bits);
        3 tensor cores with the fast epilogue (within the accumulation-order tolerance)."""
        check(self.lib.tgx_set_batched_kernels(self._ctx, kernels), self.lib)

    def sync_status(self):
        """Synchronise; raise if a bounded wait inside the fused kernel expired."""
        check(self.lib.tgx_sync_status(self._ctx), self.lib)

    def set_wait_limit(self, cycles: int = 0):
        """Limit of every bounded wait in the fused kernel, in SM cycles (0: the default)."""
        check(self.lib.tgx_set_wait_limit(self._ctx, cycles), self.lib)

    def inject_missing(self, n: int):
        """Test hook: make the fused kernel wait for n router-sum contributions that never
        come (n = 0: normal), so its first routing wait runs out."""
        check(self.lib.tgx_fused_inject_missing(self._ctx, n), self.lib)

    def fused_info(self):
        ctas, smem, arena = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(self.lib.tgx_fused_info(self._ctx, ctypes.byref(ctas), ctypes.byref(smem), ctypes.byref(arena)),
              self.lib)
        return ctas.value, smem.value, arena.value

    def last_routing(self, layer: int):
        idx = np.empty(self.top_k, np.int32)
        w = np.empty(self.top_k, np.float32)
        logits = np.empty(self.n_experts, np.float32)
        check(self.lib.tgx_last_routing(self._ctx, layer, idx.ctypes.data, w.ctypes.data, logits.ctypes.data),
              self.lib)
        return idx, w, logits


def expert_forward(lib, q4: np.ndarray, x: np.ndarray, out: np.ndarray, weight: float, embed: int, inter: int):
    """Host-pointer expert forward, the reference engine's per-expert call
    (engine.py:249-257) on an all-Q4_0 expert."""
    eb = C.expert_bytes(embed, inter)
    t = inter * (embed // C.QK) * C.Q4_0_BYTES
    q4 = np.ascontiguousarray(q4, np.uint8)
    assert q4.size == eb
    check(lib.tg_expert_forward_mixed(q4.ctypes.data, q4.ctypes.data + t, q4.ctypes.data + 2 * t, 3,
                                      x.ctypes.data, out.ctypes.data, ctypes.c_float(weight), embed, inter), lib)
    return out


def rope_cache(max_pos: int, head_dim: int = C.HEAD_DIM, base: float = C.ROPE_BASE):
    """The reference's build_rope_cache (tinygiant/_math.py:11-17): fp32 inverse
    frequencies 1 / base^(2i / head_dim), their outer product with the fp32 positions,
    fp32 cos and sin, each [max_pos][head_dim / 2]."""
    inv = (1.0 / (base ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))).astype(np.float32)
    f = np.outer(np.arange(max_pos, dtype=np.float32), inv)
    return np.cos(f).astype(np.float32), np.sin(f).astype(np.float32)


def _host_or_dev(a):
    """(pointer, on_device) of a numpy array (kept alive by the caller) or a cuda tensor."""
    if a is None:
        return None, 0
    if isinstance(a, np.ndarray):
        assert a.flags.c_contiguous
        return a.ctypes.data, 0
    assert a.is_cuda and a.is_contiguous()
    return a.data_ptr(), 1


class AttentionModel:
    """The attention half of every decode layer, resident in HBM (engine.py:199-226):
    x += attention(RMSNorm(x) * attn_norm) with the reference's tg_attention_decode(_q4)
    step, KV caches [n_layers][2][n_kv][kv_max][head_dim] fp32 and a device position.

    With a MoEModel, decode_token runs whole decode layers (attention, then the MoE
    block) for one token, replayed from a CUDA graph."""

    def __init__(self, embed=C.EMBED_DIM, n_heads=C.N_HEADS, n_kv_heads=C.N_KV_HEADS, head_dim=C.HEAD_DIM,
                 n_layers=C.N_LAYERS, kv_max=4096, q4=True, device=0, eps=C.RMS_EPS):
        self.lib = get_lib()
        self.embed, self.n_heads, self.n_kv_heads, self.head_dim = embed, n_heads, n_kv_heads, head_dim
        self.n_layers, self.kv_max, self.q4, self.device = n_layers, kv_max, bool(q4), device
        h = ctypes.c_void_p()
        check(self.lib.tgx_attn_create(device, int(self.q4), n_layers, embed, n_heads, n_kv_heads, head_dim, kv_max,
                                       float(eps), ctypes.byref(h)), self.lib)
        self._a = h
        cos, sin = rope_cache(kv_max, head_dim)
        self.set_rope(cos, sin)

    def close(self):
        if self._a:
            self.lib.tgx_attn_destroy(self._a)
            self._a = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._a

    def matrix_bytes(self):
        """Bytes of wq, wk, wv, wo in this model's formats (Q4_K / f16, or fp32)."""
        qd, kvd, E = self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim, self.embed
        if self.q4:
            return qd * E // 256 * 144, kvd * E // 256 * 144, kvd * E * 2, E * qd // 256 * 144
        return qd * E * 4, kvd * E * 4, kvd * E * 4, E * qd * 4

    def set_layer(self, layer: int, wq=None, wk=None, wv=None, wo=None, q_norm=None, k_norm=None, attn_norm=None):
        """Weights of one layer (numpy host arrays or cuda tensors, all of one kind); None keeps a part."""
        parts = [_host_or_dev(a) for a in (wq, wk, wv, wo, q_norm, k_norm, attn_norm)]
        kinds = {d for p, d in parts if p is not None}
        assert len(kinds) <= 1, "pass host arrays or device tensors, not both"
        on_dev = kinds.pop() if kinds else 0
        check(self.lib.tgx_attn_set_layer(self._a, layer, *(p for p, _ in parts), on_dev), self.lib)

    def set_rope(self, cos: np.ndarray, sin: np.ndarray):
        cos = np.ascontiguousarray(cos, np.float32)
        sin = np.ascontiguousarray(sin, np.float32)
        check(self.lib.tgx_attn_set_rope(self._a, cos.ctypes.data, sin.ctypes.data, cos.shape[0], 0), self.lib)

    def fill_synthetic(self, seed: int):
        """Random weights generated on the device: Q4_K blocks of random bytes with fp16
        scales d in [5e-5, 1.5e-4] and dmin = 7.5 d (near zero-mean weights), f16 wv of
        N(0, 0.02) (fp32 N(0, 0.02) matrices when q4 is off), norm weights 1."""
        import torch
        gen = torch.Generator(device="cuda").manual_seed(seed)
        dev = torch.device("cuda", self.device)
        sizes = self.matrix_bytes()
        for l in range(self.n_layers):
            mats = []
            for i, n in enumerate(sizes):
                if self.q4 and i != 2:
                    b = torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=gen).view(-1, 144)
                    d = torch.empty(b.shape[0], device=dev).uniform_(5e-5, 1.5e-4, generator=gen)
                    b[:, 0:2] = d.half().view(torch.uint8).view(-1, 2)
                    b[:, 2:4] = (d * 7.5).half().view(torch.uint8).view(-1, 2)
                    mats.append(b.view(-1))
                else:
                    v = torch.randn(n // (2 if self.q4 else 4), device=dev, generator=gen) * 0.02
                    mats.append((v.half() if self.q4 else v).view(torch.uint8))
            self.set_layer(l, *mats)
        torch.cuda.synchronize()

    def reset(self, pos: int = 0):
        """Start a sequence at `pos` rows cached (engine.py:145-148's kv_len = 0)."""
        check(self.lib.tgx_attn_set_pos(self._a, pos), self.lib)

    def status(self) -> int:
        """Synchronise; the device position; raises if a step ran past the cache."""
        p = ctypes.c_int()
        check(self.lib.tgx_attn_status(self._a, ctypes.byref(p)), self.lib)
        return p.value

    def read_kv(self, layer: int):
        shape = (self.n_kv_heads, self.kv_max, self.head_dim)
        k, v = np.empty(shape, np.float32), np.empty(shape, np.float32)
        check(self.lib.tgx_attn_read_kv(self._a, layer, k.ctypes.data, v.ctypes.data), self.lib)
        return k, v

    def layer(self, layer: int, x, stream=None):
        """x (cuda f32[embed]) += attention of `layer` at the current position."""
        check(self.lib.tgx_attn_layer(self._a, layer, _dev_ptr(x), _stream_handle(stream)), self.lib)

    def advance(self, stream=None):
        check(self.lib.tgx_attn_advance(self._a, _stream_handle(stream)), self.lib)

    def decode_token(self, x, moe: "MoEModel | None" = None, stream=None, eager: bool = False):
        """One token through every layer (attention, then moe's MoE block when given),
        then the position moves on; x (cuda f32[embed]) in place."""
        check(self.lib.tgx_decode_token(self._a, moe.handle if moe is not None else None, _dev_ptr(x),
                                        _stream_handle(stream), TGX_EAGER if eager else 0), self.lib)


def sample_token(logits: np.ndarray, temperature: float, top_p: float, rng=np.random) -> int:
    """The reference's choice of the next token (engine.py:344-360, 395-407): the argmax
    when temperature is 0, else top-p sampling of softmax(logits / temperature): the
    most probable tokens whose cumulative probability first reaches top_p (plus the one
    that crosses it), renormalised, drawn with rng.choice (np.random, the reference's
    generator, by default)."""
    if temperature <= 0:
        return int(np.argmax(logits))
    p = np.exp((logits - np.max(logits)) / temperature)
    p /= np.sum(p)
    order = np.argsort(p)[::-1]
    keep = order[:np.searchsorted(np.cumsum(p[order]), top_p) + 1]
    q = p[keep]
    q /= np.sum(q)
    return int(rng.choice(keep, p=q))


class DecodeEngine:
    """The reference engine's token loop on the device (tinygiant/engine.py:188-266,
    378-409): the token's embedding row, then for every layer x += attention(x) and the
    MoE block (one CUDA graph per token, AttentionModel.decode_token), then the final
    RMSNorm (tg_rms_norm's order) and the output projection (tg_f32_matvec /
    tg_f16_matvec's order; the reference evaluates it with numpy, equal within fp32
    rounding).  Positions follow the reference: forward_one_token(token, pos) caches
    row pos; generate_stream prefills the prompt at 0 .. P-1."""

    def __init__(self, moe: MoEModel, attn: AttentionModel, token_embd, output_norm, output_weight,
                 eps: float = C.RMS_EPS):
        import torch
        assert moe.embed == attn.embed and moe.n_layers == attn.n_layers
        assert token_embd.is_cuda and token_embd.dtype == torch.float32 and token_embd.dim() == 2
        assert output_weight.is_cuda and output_weight.dtype in (torch.float32, torch.float16)
        self.torch, self.lib, self.moe, self.attn = torch, moe.lib, moe, attn
        self.embd, self.norm, self.head = token_embd.contiguous(), output_norm.contiguous(), output_weight.contiguous()
        self.vocab, self.embed, self.eps = token_embd.shape[0], moe.embed, float(eps)
        assert self.head.shape == (self.vocab, self.embed) and self.norm.shape == (self.embed,)
        self.fmt = 1 if self.head.dtype == torch.float16 else 4   # tg_f16_matvec / tg_f32_matvec
        dev = token_embd.device
        self.x = torch.empty(self.embed, dtype=torch.float32, device=dev)
        self.normed = torch.empty(self.embed, dtype=torch.float32, device=dev)
        self.logits = torch.empty(self.vocab, dtype=torch.float32, device=dev)
        self.next_pos = None

    @classmethod
    def synthetic(cls, moe: MoEModel, attn: AttentionModel, vocab: int, seed: int, head_f16: bool = True):
        """Random embeddings and output weights N(0, 0.02), output norm weights 1."""
        import torch
        gen = torch.Generator(device="cuda").manual_seed(seed)
        dev = torch.device("cuda", moe.device)
        embd = torch.randn(vocab, moe.embed, generator=gen, device=dev) * 0.02
        head = torch.randn(vocab, moe.embed, generator=gen, device=dev) * 0.02
        return cls(moe, attn, embd, torch.ones(moe.embed, device=dev), head.half() if head_f16 else head)

    def reset(self):
        """A new sequence (engine.py:143-151): the caches are empty again."""
        self.attn.reset(0)
        self.next_pos = 0

    def calibrate(self, prompt_tokens, n_tokens: int = 10, counts: dict | None = None) -> dict:
        """engine.py:154-161: run the prompt and n_tokens greedy tokens, then start a new
        sequence.  Every layer's routing of every token is added to counts[(layer,
        expert)] (a cache's access_counts, so that pin_from_usage follows it); returns the
        counts."""
        counts = {} if counts is None else counts

        def record():
            for layer in range(self.moe.n_layers):
                for e in self.moe.last_routing(layer)[0]:
                    key = (layer, int(e))
                    counts[key] = counts.get(key, 0) + 1

        logits = None
        for i, tok in enumerate(prompt_tokens):
            logits = self.forward_one_token(tok, i)
            record()
        nxt = int(self.torch.argmax(logits).item())
        for step in range(n_tokens):
            logits = self.forward_one_token(nxt, len(prompt_tokens) + step)
            record()
            nxt = int(self.torch.argmax(logits).item())
        self.reset()
        return counts

    def pin_experts(self, cache, n_per_layer: int, calibrate_tokens: int | None = None, prompt_tokens=None) -> int:
        """engine.py:163-186 on a HostTierCache: with calibrate_tokens and prompt_tokens,
        calibrate into the cache's request counts and pin from usage (backfilled from the
        relayout profile); else pin the static profile's hot experts.  Returns the count."""
        if calibrate_tokens and prompt_tokens:
            self.calibrate(prompt_tokens, n_tokens=calibrate_tokens, counts=cache.access_counts)
            return cache.pin_from_usage(n_per_layer, self.moe.n_layers)
        return cache.pin_hot_experts(n_per_layer)

    def forward_one_token(self, token_id: int, pos: int, stream=None):
        """Logits [vocab] (a cuda tensor, overwritten by the next call) of token_id at pos."""
        if pos != self.next_pos:
            self.attn.reset(pos)
        s = _stream_handle(stream)
        torch = self.torch
        st = stream if stream is None or isinstance(stream, torch.cuda.Stream) else torch.cuda.ExternalStream(s)
        with torch.cuda.stream(st):   # the row copy goes on the same stream as the kernels
            self.x.copy_(self.embd[int(token_id)])
        self.attn.decode_token(self.x, self.moe, stream)
        check(self.lib.tgx_rms_norm(_dev_ptr(self.x), _dev_ptr(self.norm), _dev_ptr(self.normed), self.embed,
                                    self.eps, s), self.lib)
        check(self.lib.tgx_kq_matvec(self.fmt, self.head.data_ptr(), _dev_ptr(self.normed), _dev_ptr(self.logits),
                                     self.vocab, self.embed, s), self.lib)
        self.next_pos = pos + 1
        return self.logits

    def generate_stream(self, prompt_tokens, n_tokens: int = 128, temperature: float = 0.7, top_p: float = 0.9,
                        rng=np.random):
        """Yield n_tokens generated after the prompt (engine.py:378-409): greedy on the
        device when temperature is 0, else sample_token on the host."""
        logits = None
        for i, tok in enumerate(prompt_tokens):
            logits = self.forward_one_token(tok, i)
        nxt = None
        for step in range(n_tokens):
            pos = len(prompt_tokens) + step
            if step > 0:
                logits = self.forward_one_token(nxt, pos - 1)
            if temperature <= 0:
                nxt = int(self.torch.argmax(logits).item())
            else:
                nxt = sample_token(logits.cpu().numpy(), temperature, top_p, rng)
            yield nxt
