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
        """Expert matmuls of the batched path: 0 auto, 1 dp4a, 2 tensor cores; same bits."""
        check(self.lib.tgx_set_batched_kernels(self._ctx, kernels), self.lib)

    def sync_status(self):
        """Synchronise; raise if a bounded wait inside the fused kernel expired."""
        check(self.lib.tgx_sync_status(self._ctx), self.lib)

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
