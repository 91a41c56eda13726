"""ctypes bindings of libtinygiant.so (the B200 build), mirroring the reference's
tinygiant/_lib.py: find_library() looks next to the package and in the repo
root, load_tinygiant_lib() registers the prototypes and returns the CDLL (or
None when no library is found, as the reference does).

Differences from the reference (tinygiant/_lib.py:26-76): every entry point
returns an int status (0 = TG_OK, negative = error) instead of void, and the
device-resident tgx_* API is registered as well.  check() turns a status into a
TinyGiantError carrying tg_last_error().
"""
from __future__ import annotations

import ctypes
from pathlib import Path

VP = ctypes.c_void_p
CI = ctypes.c_int
CF = ctypes.c_float
SZ = ctypes.c_size_t
LL = ctypes.c_longlong
U64 = ctypes.c_uint64

TG_OK = 0
TG_EINVAL = -1
TG_ECUDA = -2
TG_ENOMEM = -3
TG_EUNSUPPORTED = -4
TG_ENODEV = -5
TG_ETIMEOUT = -6

TG_FMT_Q4_K = 0
TG_FMT_F16 = 1
TG_FMT_Q6_K = 2
TG_FMT_Q4_0 = 3

TG_NOALLOC_SCRATCH_BYTES = 4194304  # include/tinygiant.h

TGX_KQ_CHAINED = 1

TGX_EAGER = 1
TGX_MULTI = 2

LIB_NAME = "libtinygiant.so"


class TinyGiantError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"tinygiant error {code}: {msg}")
        self.code = code


class TgxShape(ctypes.Structure):
    _fields_ = [("embed", CI), ("inter", CI), ("n_experts", CI), ("top_k", CI), ("n_layers", CI),
                ("rms_eps", CF)]


# name -> (restype, argtypes); the order follows include/tinygiant.h
PROTOTYPES = {
    "tg_last_error": (ctypes.c_char_p, []),
    "tg_version": (CI, []),
    "tg_device_count": (CI, []),
    "tg_quantize_q8_0": (CI, [VP, VP, CI]),
    "tg_quantize_q4_0": (CI, [VP, VP, LL]),
    "tg_block_dots_q4_0": (CI, [VP, VP, VP, CI, CI]),
    "tg_matmul_q4_0": (CI, [VP, VP, VP, CI, CI]),
    "tg_expert_forward_q4_0": (CI, [VP, VP, VP, CF, CI, CI]),
    "tg_expert_forward_mixed": (CI, [VP, VP, VP, CI, VP, VP, CF, CI, CI]),
    "tg_moe_forward_q4_0": (CI, [VP, VP, CI, VP, VP, CI, CI]),
    "tg_matmul_q4k": (CI, [VP, VP, VP, CI, CI]),
    "tg_matmul_q6k": (CI, [VP, VP, VP, CI, CI]),
    "tg_f16_matvec": (CI, [VP, VP, VP, CI, CI]),
    "tg_f32_matvec": (CI, [VP, VP, VP, CI, CI]),
    "tg_rms_norm": (CI, [VP, VP, VP, CI, CF]),
    "tg_attention_decode": (CI, [VP, VP, VP, VP, VP, VP, VP, VP, CI, CI, VP, VP, VP, VP, CI, CI, CI, CI, CI]),
    "tg_attention_decode_q4": (CI, [VP, VP, VP, VP, VP, VP, VP, VP, CI, CI, VP, VP, VP, VP, CI, CI, CI, CI, CI]),
    "tg_transformer_layer": (CI, [VP] * 10 + [CI, CI] + [VP] * 7 + [CI, VP] + [CI] * 6),
    "tgx_attention_scratch_bytes": (SZ, [CI, CI, CI, CI]),
    "tgx_attn_create": (CI, [CI, CI, CI, CI, CI, CI, CI, CI, CF, VP]),
    "tgx_attn_destroy": (CI, [VP]),
    "tgx_attn_layer_bytes": (SZ, [VP]),
    "tgx_attn_set_layer": (CI, [VP, CI, VP, VP, VP, VP, VP, VP, VP, CI]),
    "tgx_attn_set_rope": (CI, [VP, VP, VP, CI, CI]),
    "tgx_attn_set_pos": (CI, [VP, CI]),
    "tgx_attn_status": (CI, [VP, VP]),
    "tgx_attn_kv": (CI, [VP, CI, VP, VP]),
    "tgx_load_experts_rows": (CI, [VP, CI, CI, CI, VP, CI]),
    "tgx_rms_norm": (CI, [VP, VP, VP, CI, CF, VP]),
    "tgx_attn_read_kv": (CI, [VP, CI, VP, VP]),
    "tgx_attn_layer": (CI, [VP, CI, VP, VP]),
    "tgx_attn_advance": (CI, [VP, VP]),
    "tgx_decode_token": (CI, [VP, VP, VP, VP, CI]),
    "tgx_attention_decode": (CI, [CI, VP, VP, VP, VP, VP, VP, VP, VP, CI, CI, VP, VP, VP, VP, CI, CI, CI, CI, CI,
                                  VP, SZ, VP]),
    "tg_expert_forward": (CI, [VP, VP, VP, CF, CI, CI]),
    "tg_moe_forward": (CI, [VP, VP, CI, VP, VP, CI, CI]),
    "tgx_kq_matrix_bytes": (SZ, [CI, ctypes.c_longlong, CI]),
    "tgx_kq_prepare": (CI, [CI, VP, VP, ctypes.c_longlong, CI, VP]),
    "tgx_kq_matvec": (CI, [CI, VP, VP, VP, CI, CI, VP]),
    "tgx_ep_create": (CI, [CI, ctypes.POINTER(TgxShape), CI, CI, CI, ctypes.POINTER(VP)]),
    "tgx_ep_load_shared": (CI, [VP, CI, VP, CI]),
    "tgx_ep_read_expert": (CI, [VP, CI, CI, VP]),
    "tgx_ep_destroy": (CI, [VP]),
    "tgx_ep_expert_range": (CI, [VP, ctypes.POINTER(CI), ctypes.POINTER(CI)]),
    "tgx_ep_load_experts": (CI, [VP, CI, CI, CI, VP, CI]),
    "tgx_ep_set_router": (CI, [VP, CI, VP, CI]),
    "tgx_ep_set_ffn_norm": (CI, [VP, CI, VP, CI]),
    "tgx_ep_fill_synthetic": (CI, [VP, U64, CF, CF]),
    "tgx_ep_y_floats": (SZ, [VP, CI]),
    "tgx_ep_moe_partial": (CI, [VP, CI, VP, CI, VP, VP]),
    "tgx_ep_combine": (CI, [VP, VP, CI, VP, VP]),
    "tgx_ep_set_kernels": (CI, [VP, CI]),
    "tgx_ep_status": (CI, [VP, VP]),
    "tgx_ep_p2p_handle_bytes": (SZ, []),
    "tgx_ep_p2p_init": (CI, [VP, CI, VP]),
    "tgx_ep_p2p_connect": (CI, [VP, VP]),
    "tgx_ep_moe_layer_p2p": (CI, [VP, CI, VP, CI, VP]),
    "tgx_ep_p2p_status": (CI, [VP, VP]),
    "tgx_ep_p2p_disconnect": (CI, [VP]),
    "tgx_ep_fused_init": (CI, [VP, VP]),
    "tgx_ep_fused_connect": (CI, [VP, VP]),
    "tgx_ep_decode_step": (CI, [VP, VP, VP]),
    "tgx_ep_fused_trace": (CI, [VP, VP, VP, VP]),
    "tgx_ep_fused_info": (CI, [VP, ctypes.POINTER(CI), ctypes.POINTER(CI)]),
    "tgx_ep_set_wait_limit": (CI, [VP, ctypes.c_longlong]),
    "tgx_ep_fused_last_routing": (CI, [VP, CI, VP, VP]),
    "tgx_ep_fused_status": (CI, [VP, VP]),
    "tgx_ep_fused_epoch": (CI, [VP, ctypes.POINTER(ctypes.c_uint)]),
    "tgx_ep_fused_reset": (CI, [VP, ctypes.c_uint]),
    "tgx_ep_record_bytes": (SZ, [VP]),
    "tgx_ep_dispatch": (CI, [VP, CI, VP, CI, VP, VP, VP]),
    "tgx_ep_dispatch_experts": (CI, [VP, CI, VP, CI, VP, VP]),
    "tgx_ep_dispatch_combine": (CI, [VP, VP, CI, VP, VP]),
    "tgx_ep_dispatch_p2p_init": (CI, [VP, CI, VP]),
    "tgx_ep_dispatch_p2p_connect": (CI, [VP, VP]),
    "tgx_ep_moe_layer_dispatch_p2p": (CI, [VP, CI, VP, CI, VP]),
    "tgx_ep_dispatch_p2p_counts": (CI, [VP, ctypes.POINTER(CI), ctypes.POINTER(CI)]),
    "tgx_ep_dispatch_p2p_status": (CI, [VP, VP]),
    "tgx_set_batched_kernels": (CI, [VP, CI]),
    "tgx_kq_scratch_bytes": (SZ, [CI, CI, CI]),
    "tgx_kq_experts_forward": (CI, [VP, VP, VP, CI, CI, VP, VP, VP, CI, CI, CI, VP, SZ, CI, VP]),
    "tg_expert_forward_q4_0_noalloc": (CI, [VP, VP, VP, CF, CI, CI, VP]),
    "tg_mlock": (CI, [VP, SZ]),
    "tg_prefetch": (CI, [VP, SZ]),
    "tg_prefetch_batch": (CI, [VP, VP, CI]),
    "tgx_ctx_create": (CI, [CI, ctypes.POINTER(TgxShape), ctypes.POINTER(VP)]),
    "tgx_ctx_destroy": (CI, [VP]),
    "tgx_expert_bytes": (SZ, [VP]),
    "tgx_load_experts": (CI, [VP, CI, CI, CI, VP, CI]),
    "tgx_read_experts": (CI, [VP, CI, CI, CI, VP]),
    "tgx_set_router": (CI, [VP, CI, VP, CI]),
    "tgx_set_ffn_norm": (CI, [VP, CI, VP, CI]),
    "tgx_fill_synthetic": (CI, [VP, U64, CF, CF]),
    "tgx_moe_layer": (CI, [VP, CI, VP, VP]),
    "tgx_decode_step": (CI, [VP, VP, VP, CI]),
    "tgx_moe_batched": (CI, [VP, CI, VP, CI, VP]),
    "tgx_decode_batched": (CI, [VP, VP, CI, VP]),
    "tgx_experts_forward": (CI, [VP, CI, VP, VP, CI, VP, VP]),
    "tgx_repack_experts": (CI, [VP, VP, VP, CI, VP]),
    "tgx_sync_status": (CI, [VP]),
    "tgx_expert_forward": (CI, [VP, CI, CI, VP, VP, CF, VP]),
    "tgx_set_wait_limit": (CI, [VP, ctypes.c_longlong]),
    "tgx_fused_inject_missing": (CI, [VP, CI]),
    "tgx_fused_info": (CI, [VP, VP, VP, VP]),
    "tgx_fused_debug": (CI, [VP, VP, VP, SZ]),
    "tgx_fused_trace": (CI, [VP, VP, VP, VP]),
    "tgx_last_routing": (CI, [VP, CI, VP, VP, VP]),
}


def find_library():
    """Find libtinygiant.so next to this package or in the repository root."""
    pkg_dir = Path(__file__).parent
    repo_dir = pkg_dir.parent
    for path in (pkg_dir / LIB_NAME, repo_dir / LIB_NAME):
        if path.exists():
            return path
    return None


def load_tinygiant_lib(lib_path=None):
    """Load the B200 library and register its prototypes; None if not found."""
    if lib_path is None:
        lib_path = find_library()
    if lib_path is None:
        return None
    lib = ctypes.CDLL(str(lib_path))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None


def get_lib():
    """The loaded library; raises if it has not been built (no silent fallback)."""
    global _LIB
    if _LIB is None:
        _LIB = load_tinygiant_lib()
        if _LIB is None:
            raise RuntimeError(
                "libtinygiant.so not found: build it with `python -m tinygiant_b200.build`")
    return _LIB


def check(rc: int, lib=None) -> int:
    if rc != TG_OK:
        lib = lib or get_lib()
        msg = lib.tg_last_error()
        raise TinyGiantError(rc, msg.decode() if msg else "")
    return rc
