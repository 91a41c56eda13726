"""The C-ABI library loads and exports every symbol include/*.h declares, and its
argument checks work without a GPU (no compute calls)."""
import ctypes
import re
from pathlib import Path

import numpy as np

from tinygiant_b200 import _lib as L

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(tgx?_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("tg_expert_forward_mixed", "tg_moe_forward_q4_0", "tg_quantize_q8_0", "tgx_decode_step"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(L.find_library()))
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_prototypes_cover_header():
    assert declared_symbols() <= set(L.PROTOTYPES)


def test_argument_errors_without_device():
    lib = L.load_tinygiant_lib()
    assert lib.tg_quantize_q8_0(None, None, 0) == L.TG_EINVAL
    assert b"bad arguments" in lib.tg_last_error()
    x = np.zeros(48, np.float32)
    out = np.zeros(64, np.uint8)
    assert lib.tg_quantize_q8_0(x.ctypes.data, out.ctypes.data, 48) == L.TG_EINVAL  # not a multiple of 32
    assert lib.tg_expert_forward_q4_0(out.ctypes.data, x.ctypes.data, x.ctypes.data, 1.0, 2000, 768) == L.TG_EINVAL
    assert lib.tg_expert_forward_mixed(out.ctypes.data, out.ctypes.data, out.ctypes.data, 7,
                                       x.ctypes.data, x.ctypes.data, 1.0, 2048, 768) == L.TG_EINVAL
    assert lib.tg_matmul_q4k(out.ctypes.data, x.ctypes.data, x.ctypes.data, 4, 300) == L.TG_EINVAL
    assert lib.tg_matmul_q6k(out.ctypes.data, x.ctypes.data, x.ctypes.data, 0, 256) == L.TG_EINVAL
    assert lib.tg_f16_matvec(out.ctypes.data, x.ctypes.data, x.ctypes.data, 4, 12) == L.TG_EINVAL
    assert lib.tg_rms_norm(x.ctypes.data, x.ctypes.data, x.ctypes.data, 6, 1e-6) == L.TG_EINVAL
    assert lib.tgx_kq_matrix_bytes(2, 4, 300) == 0 and lib.tgx_kq_matrix_bytes(2, 4, 512) == 4 * 2 * 210
    assert lib.tgx_kq_experts_forward(None, None, None, 0, 1, None, None, None, 2048, 768, 0, None, 0, 0,
                                      None) == L.TG_EINVAL
    assert lib.tgx_kq_scratch_bytes(8, 2048, 768) >= 8 * (768 + 2048) * 4
    assert lib.tgx_kq_scratch_bytes(0, 2048, 768) == 0
    # attention decode: head_dim not a multiple of 8, kv_len outside the cache, null pointers
    p = x.ctypes.data
    assert lib.tg_attention_decode(p, p, p, p, p, p, p, p, 0, 4, p, p, p, p, 48, 4, 2, 12, 0) == L.TG_EINVAL
    assert lib.tg_attention_decode_q4(p, p, p, p, p, p, p, p, 4, 4, p, p, p, p, 256, 2, 1, 128, 0) == L.TG_EINVAL
    assert lib.tg_attention_decode_q4(None, p, p, p, p, p, p, p, 0, 4, p, p, p, p, 256, 2, 1, 128, 0) == L.TG_EINVAL
    assert lib.tgx_attention_decode(1, p, p, p, p, p, p, p, p, 0, 8, p, p, p, p, 2048, 32, 5, 128, 0, p, 1 << 20,
                                    None) == L.TG_EINVAL   # 32 query heads over 5 kv heads
    assert lib.tgx_attention_scratch_bytes(32, 4, 128, 4096) == 4 * ((4096 + 1024) + 4096 + 32 * 4096 + 4096)
    assert lib.tgx_attention_scratch_bytes(32, 4, 128, 4097) == 4 * ((4096 + 1024) + 4096 + 32 * 4100 + 4096)
    assert lib.tgx_attention_scratch_bytes(0, 4, 128, 4096) == 0
    sb = lib.tgx_attention_scratch_bytes(32, 4, 128, 64)
    assert lib.tgx_attention_decode(1, p, p, p, p, p, p, p, p, 0, 64, p, p, p, p, 2048, 32, 4, 128, 0, p, sb - 16,
                                    None) == L.TG_EINVAL   # scratch too small
    ah = ctypes.c_void_p()
    assert lib.tgx_attn_create(0, 1, 48, 2048, 32, 4, 12, 4096, 1e-6, ctypes.byref(ah)) == L.TG_EINVAL  # head_dim
    assert lib.tgx_attn_create(0, 1, 0, 2048, 32, 4, 128, 4096, 1e-6, ctypes.byref(ah)) == L.TG_EINVAL   # layers
    assert lib.tgx_attn_create(0, 1, 48, 2048, 32, 4, 128, 40000, 1e-6, ctypes.byref(ah)) == L.TG_EINVAL  # kv_max
    assert lib.tgx_decode_token(None, None, None, None, 0) == L.TG_EINVAL
    assert lib.tgx_attn_set_pos(None, 0) == L.TG_EINVAL
    assert lib.tgx_load_experts_rows(None, 0, 0, 1, p, 0) == L.TG_EINVAL
    shape = L.TgxShape(2048, 768, 128, 8, 48, 1e-6)
    h = ctypes.c_void_p()
    bad = L.TgxShape(2048, 768, 128, 200, 48, 1e-6)
    assert lib.tgx_ctx_create(0, ctypes.byref(bad), ctypes.byref(h)) == L.TG_EINVAL
    if lib.tg_device_count() == 0:
        assert lib.tgx_ctx_create(0, ctypes.byref(shape), ctypes.byref(h)) == L.TG_ENODEV
        assert lib.tgx_attn_create(0, 1, 48, 2048, 32, 4, 128, 4096, 1e-6, ctypes.byref(ah)) == L.TG_ENODEV
        xs = np.zeros(64, np.float32)
        assert lib.tg_quantize_q8_0(xs.ctypes.data, out.ctypes.data, 64) == L.TG_ENODEV
        assert lib.tg_expert_forward_mixed(out.ctypes.data, out.ctypes.data, out.ctypes.data, L.TG_FMT_Q6_K,
                                           x.ctypes.data, x.ctypes.data, 1.0, 2048, 768) == L.TG_ENODEV


def test_mlock_matches_reference_semantics():
    lib = L.load_tinygiant_lib()
    buf = np.zeros(1 << 16, np.uint8)
    rc = lib.tg_mlock(buf.ctypes.data, buf.nbytes)
    assert rc in (0, -1)  # mlock's own result, as csrc/libtinygiant.c:761-766 returns it


def test_prefetch_hints_match_reference_semantics():
    # csrc/libtinygiant.c:745-759: page-aligned WILLNEED advice, no effect on the data
    lib = L.load_tinygiant_lib()
    buf = np.arange(1 << 16, dtype=np.uint8)
    assert lib.tg_prefetch(buf.ctypes.data + 123, 40000) == 0
    addrs = (ctypes.c_void_p * 2)(buf.ctypes.data, buf.ctypes.data + 5000)
    lens = (ctypes.c_size_t * 2)(100, 20000)
    assert lib.tg_prefetch_batch(addrs, lens, 2) == 0
    assert lib.tg_prefetch_batch(addrs, lens, 0) == 0
    assert np.array_equal(buf, np.arange(1 << 16, dtype=np.uint8))
