"""GPU parity: the CUDA path, called through the C ABI, against the CPU oracle.

Bar: bit-exact for quantisation, integer block dots, and (in the oracle's
mirror order) for every fp32 output; within max-abs-rel 1e-5 of the oracle's
reference order (sequential block sums, libm expf) for expert outputs, where
the only differences are fp32 accumulation order and rare one-step requant
flips, which are counted.
"""
import ctypes

import numpy as np
import pytest

from order_check import check_reference_order
from tinygiant_b200 import _constants as C
from tinygiant_b200._lib import TG_EINVAL, check

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5  # max-abs-rel tolerance for fp32 expert outputs vs the reference order


def max_abs_rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def p(a):
    return a.ctypes.data


def rand_expert(rng, oracle, H, I, sigma=0.02):
    w = (rng.standard_normal(3 * H * I) * sigma).astype(np.float32)
    return oracle.quantize_q4_0(w)


# ------------------------------------------------------------------ quantisers

def test_q8_0_golden(lib, golden):
    x = golden["q8_x"]
    out = np.zeros(x.size // 32 * 34, np.uint8)
    check(lib.tg_quantize_q8_0(p(x), p(out), x.size), lib)
    assert np.array_equal(out, golden["q8_q"])


def test_q4_0_golden(lib, golden):
    w = golden["q4_w"]
    out = np.zeros(w.size // 32 * 18, np.uint8)
    check(lib.tg_quantize_q4_0(p(w), p(out), w.size), lib)
    assert np.array_equal(out, golden["q4_q"])


@pytest.mark.parametrize("n,scale", [(32, 1.0), (2048, 1.0), (7168, 1e-3), (1 << 20, 50.0)])
def test_q8_0_random(lib, oracle, n, scale):
    x = (np.random.default_rng(n).standard_normal(n) * scale).astype(np.float32)
    out = np.zeros(n // 32 * 34, np.uint8)
    check(lib.tg_quantize_q8_0(p(x), p(out), n), lib)
    assert np.array_equal(out, oracle.quantize_q8_0(x))


def test_q4_0_random_large(lib, oracle):
    w = (np.random.default_rng(9).standard_normal(C.expert_bytes() // 18 * 32) * 0.02).astype(np.float32)
    out = np.zeros(w.size // 32 * 18, np.uint8)
    check(lib.tg_quantize_q4_0(p(w), p(out), w.size), lib)
    assert np.array_equal(out, oracle.quantize_q4_0(w))


# ------------------------------------------------------------------ dots

def test_block_dots_golden(lib, golden):
    out = np.zeros((96, 16), np.int32)
    check(lib.tg_block_dots_q4_0(p(golden["mv_W"]), p(golden["mv_xq"]), p(out), 96, 512), lib)
    assert np.array_equal(out, golden["mv_sumi"])


@pytest.mark.parametrize("rows,cols", [(768, 2048), (2048, 768), (5, 7168), (1, 256)])
def test_block_dots_exact(lib, oracle, rows, cols):
    rng = np.random.default_rng(rows * 31 + cols)
    W = oracle.quantize_q4_0((rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    xq = oracle.quantize_q8_0(rng.standard_normal(cols).astype(np.float32) * 3)
    out = np.zeros((rows, cols // 32), np.int32)
    check(lib.tg_block_dots_q4_0(p(W), p(xq), p(out), rows, cols), lib)
    assert np.array_equal(out, oracle.block_dots(W, xq, rows, cols))


def test_block_dots_extreme_codes(lib, oracle):
    # all nibbles 0 or 15 and all activations +-127: the int32 range edges of a block dot
    rows, cols = 4, 256
    W = np.zeros(rows * cols // 32 * 18, np.uint8).reshape(-1, 18)
    W[:, 0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    W[0::2, 2:] = 0x00
    W[1::2, 2:] = 0xFF
    W = W.ravel()
    xq = np.zeros(cols // 32 * 34, np.uint8).reshape(-1, 34)
    xq[:, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    xq[0::2, 2:] = np.uint8(127)
    xq[1::2, 2:] = np.int8(-127).view(np.uint8)
    xq = xq.ravel()
    out = np.zeros((rows, cols // 32), np.int32)
    check(lib.tg_block_dots_q4_0(p(W), p(xq), p(out), rows, cols), lib)
    ref = oracle.block_dots(W, xq, rows, cols)
    assert np.array_equal(out, ref)
    assert np.abs(ref).max() == 32 * 8 * 127


@pytest.mark.parametrize("rows,cols", [(768, 2048), (2048, 768), (3, 7168)])
def test_matvec_bit_exact(lib, oracle, rows, cols):
    rng = np.random.default_rng(rows + cols)
    W = oracle.quantize_q4_0((rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    x = rng.standard_normal(cols).astype(np.float32)
    y = np.zeros(rows, np.float32)
    check(lib.tg_matmul_q4_0(p(W), p(x), p(y), rows, cols), lib)
    ym = oracle.matvec(W, oracle.quantize_q8_0(x), rows, cols, 1)
    assert np.array_equal(y, ym)
    yr = oracle.matvec(W, oracle.quantize_q8_0(x), rows, cols, 0)
    assert max_abs_rel(y, yr) <= REL_TOL


# ------------------------------------------------------------------ expert forward

def flips(hq_a, hq_b):
    a = hq_a.reshape(-1, 34)[:, 2:].view(np.int8).astype(int)
    b = hq_b.reshape(-1, 34)[:, 2:].view(np.int8).astype(int)
    return int((a != b).sum())


@pytest.mark.parametrize("H,I", [(C.EMBED_DIM, C.EXPERT_INTERMEDIATE), (512, 256), (256, 2048)])
def test_expert_forward_bit_exact(lib, oracle, H, I):
    rng = np.random.default_rng(H * 7 + I)
    blob = rand_expert(rng, oracle, H, I)
    x = rng.standard_normal(H).astype(np.float32)
    out0 = (rng.standard_normal(H) * 0.1).astype(np.float32)
    out = out0.copy()
    check(lib.tg_expert_forward_q4_0(p(blob), p(x), p(out), ctypes.c_float(0.125), H, I), lib)
    ref = oracle.expert_forward(blob, x, out0.copy(), 0.125, H, I, 1)
    assert np.array_equal(out, ref)
    # against the reference order (sequential block sums, libm expf): the stage-wise
    # bound of tests/order_check.py, on the GPU's own expert output
    st_m = oracle.expert_stages(blob, x, H, I, 1)
    st_r = oracle.expert_stages(blob, x, H, I, 0)
    y_gpu = np.zeros(H, np.float32)
    check(lib.tg_expert_forward_q4_0(p(blob), p(x), p(y_gpu), ctypes.c_float(1.0), H, I), lib)
    assert np.array_equal(y_gpu, st_m["y"])
    nflip, err = check_reference_order(st_m, st_r, y_gpu)
    print(f"H={H} I={I}: requant flips vs reference order = {nflip}, max-abs-rel = {err:.2e}")


def test_expert_forward_golden(lib, golden):
    H, I = int(golden["ex_H"]), int(golden["ex_I"])
    blob, x = golden["ex_blob"], golden["ex_x"]
    out = np.zeros(H, np.float32)
    check(lib.tg_expert_forward_q4_0(p(blob), p(x), p(out), ctypes.c_float(1.0), H, I), lib)
    y64 = golden["ex_y64"]
    assert np.max(np.abs(out - y64)) <= 2e-3 * np.abs(y64).max()


def test_expert_forward_mixed_and_formats(lib, oracle):
    H, I = C.EMBED_DIM, C.EXPERT_INTERMEDIATE
    rng = np.random.default_rng(77)
    blob = rand_expert(rng, oracle, H, I)
    x = rng.standard_normal(H).astype(np.float32)
    t = I * (H // 32) * 18
    a = np.zeros(H, np.float32)
    b = np.zeros(H, np.float32)
    check(lib.tg_expert_forward_q4_0(p(blob), p(x), p(a), ctypes.c_float(0.3), H, I), lib)
    g, u, d = blob[:t].copy(), blob[t:2 * t].copy(), blob[2 * t:].copy()
    check(lib.tg_expert_forward_mixed(p(g), p(u), p(d), 3, p(x), p(b), ctypes.c_float(0.3), H, I), lib)
    assert np.array_equal(a, b)
    # down formats 0 / 1 / 2 are the reference's own (tests/test_gpu_kquant.py); others are rejected
    assert lib.tg_expert_forward_mixed(p(g), p(u), p(d), 9, p(x), p(b), ctypes.c_float(0.3), H, I) == TG_EINVAL


def test_expert_forward_zero_input(lib, oracle):
    H, I = C.EMBED_DIM, C.EXPERT_INTERMEDIATE
    blob = rand_expert(np.random.default_rng(1), oracle, H, I)
    x = np.zeros(H, np.float32)
    out = np.full(H, 0.5, np.float32)
    check(lib.tg_expert_forward_q4_0(p(blob), p(x), p(out), ctypes.c_float(1.0), H, I), lib)
    assert np.array_equal(out, np.full(H, 0.5, np.float32))


@pytest.mark.parametrize("sigma,xscale,finite", [(0.1, 30.0, True), (0.5, 100.0, False)])
def test_expert_forward_large_inputs(lib, oracle, sigma, xscale, finite):
    """Large activations.  With sigma=0.5, x ~ N(0, 100^2) the intermediate h reaches ~3e7,
    so its Q8_0 scale (amax/127) overflows fp16 to inf, exactly as ggml's Q8_0 does; the
    GPU must then produce the same non-finite outputs as the oracle."""
    H, I = C.EMBED_DIM, C.EXPERT_INTERMEDIATE
    rng = np.random.default_rng(2)
    blob = rand_expert(rng, oracle, H, I, sigma=sigma)
    x = (rng.standard_normal(H) * xscale).astype(np.float32)
    out = np.zeros(H, np.float32)
    check(lib.tg_expert_forward_q4_0(p(blob), p(x), p(out), ctypes.c_float(1.0), H, I), lib)
    ref = oracle.expert_forward(blob, x, np.zeros(H, np.float32), 1.0, H, I, 1)
    assert bool(np.isfinite(ref).all()) == finite
    assert np.array_equal(out, ref, equal_nan=True)


@pytest.mark.parametrize("k", [1, 8])
def test_moe_forward_bit_exact(lib, oracle, k):
    H, I = C.EMBED_DIM, C.EXPERT_INTERMEDIATE
    rng = np.random.default_rng(100 + k)
    blobs = [rand_expert(rng, oracle, H, I) for _ in range(k)]
    w = rng.dirichlet(np.ones(k)).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    out = np.full(H, 9.0, np.float32)
    ptrs = (ctypes.c_void_p * k)(*[b.ctypes.data for b in blobs])
    check(lib.tg_moe_forward_q4_0(ptrs, p(w), k, p(x), p(out), H, I), lib)
    ref = np.zeros(H, np.float32)
    for j in range(k):
        oracle.expert_forward(blobs[j], x, ref, w[j], H, I, 1)
    assert np.array_equal(out, ref)


# ------------------------------------------------------------------ device-resident MoE

def build_model(oracle, H, I, E, k, L, seed):
    """A random L-layer model loaded through the C ABI, with its host copy:
    Q4_0 experts, fp32 routers and FFN RMSNorm weights ~ 1 + N(0, 0.1)."""
    import torch  # noqa: F401
    from tinygiant_b200.engine import MoEModel
    rng = np.random.default_rng(seed)
    m = MoEModel(H, I, E, k, L)
    blobs, Rs, Ns = [], [], []
    for l in range(L):
        b = oracle.quantize_q4_0((rng.standard_normal(E * 3 * H * I) * 0.02).astype(np.float32))
        R = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
        nw = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        m.load_experts(l, b)
        m.set_router(l, R)
        m.set_ffn_norm(l, nw)
        blobs.append(b)
        Rs.append(R)
        Ns.append(nw)
    m.norms = Ns
    return m, blobs, Rs, rng


def test_load_read_roundtrip(oracle):
    m, blobs, Rs, _ = build_model(oracle, 512, 256, 8, 2, 2, 5)
    for l in range(2):
        assert np.array_equal(m.read_experts(l, 0, 8), blobs[l])
    m.close()


@pytest.mark.parametrize("H,I,E,k,L", [(512, 256, 16, 4, 3), (C.EMBED_DIM, C.EXPERT_INTERMEDIATE, 128, 8, 2),
                                       (1024, 512, 64, 6, 2)])
def test_moe_layer_and_decode_bit_exact(oracle, H, I, E, k, L):
    import torch
    m, blobs, Rs, rng = build_model(oracle, H, I, E, k, L, seed=H + E)
    x0 = rng.standard_normal(H).astype(np.float32)
    # layer by layer
    xd = torch.from_numpy(x0.copy()).cuda()
    xr = x0.copy()
    for l in range(L):
        m.moe_layer(l, xd)
        xr, idx, w, logits = oracle.moe_block(blobs[l], Rs[l], xr, k, H, I, normw=m.norms[l])
        gi, gw, gl = m.last_routing(l)
        assert np.array_equal(gl, logits)
        assert np.array_equal(gi, idx)
        assert np.array_equal(gw, w)
        assert np.array_equal(xd.cpu().numpy(), xr)
    # whole step, eager and graph
    xref, idx_all = oracle.decode_step(blobs, Rs, x0, k, H, I, norms=m.norms)
    for eager in (True, False, False):
        xd = torch.from_numpy(x0.copy()).cuda()
        m.decode_step(xd, eager=eager)
        torch.cuda.synchronize()
        assert np.array_equal(xd.cpu().numpy(), xref)
        for l in range(L):
            assert np.array_equal(m.last_routing(l)[0], idx_all[l])
    m.close()


def test_fused_path_active_and_repeated_steps(oracle, lib):
    """The fused kernel is the default for these shapes; many consecutive steps
    (epoch tags, router accumulators recycled between launches) stay bit-exact,
    interleaved with single-layer calls and the multi-kernel path."""
    import torch
    from tinygiant_b200._lib import TGX_EAGER, TGX_MULTI
    H, I, E, k, L = 1024, 512, 64, 8, 3
    m, blobs, Rs, rng = build_model(oracle, H, I, E, k, L, seed=91)
    ctas, smem, arena = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(lib.tgx_fused_info(m.handle, ctypes.byref(ctas), ctypes.byref(smem), ctypes.byref(arena)), lib)
    assert ctas.value > 0 and smem.value > arena.value > 0
    for step in range(6):
        x0 = rng.standard_normal(H).astype(np.float32)
        xref, idx_all = oracle.decode_step(blobs, Rs, x0, k, H, I, norms=m.norms)
        xd = torch.from_numpy(x0.copy()).cuda()
        flags = [0, TGX_EAGER, TGX_MULTI, TGX_MULTI | TGX_EAGER, 0, 0][step]
        check(lib.tgx_decode_step(m.handle, xd.data_ptr(), torch.cuda.current_stream().cuda_stream, flags), lib)
        torch.cuda.synchronize()
        assert np.array_equal(xd.cpu().numpy(), xref), f"step {step} flags {flags}"
        assert lib.tgx_sync_status(m.handle) == 0
        # one single layer in between
        l = step % L
        xs = torch.from_numpy(x0.copy()).cuda()
        m.moe_layer(l, xs)
        xr, idx, w, logits = oracle.moe_block(blobs[l], Rs[l], x0, k, H, I, normw=m.norms[l])
        assert np.array_equal(xs.cpu().numpy(), xr)
        assert np.array_equal(m.last_routing(l)[0], idx)
    m.close()


def test_fused_extreme_inputs_complete(oracle, lib):
    """Activations of 1e30 overflow x^2 and the router products; the fixed-point
    sums clamp per element, so the fused kernel still completes (no wait expires)
    and matches the oracle."""
    import torch
    H, I, E, k, L = 512, 256, 16, 4, 2
    m, blobs, Rs, rng = build_model(oracle, H, I, E, k, L, seed=17)
    x0 = rng.standard_normal(H).astype(np.float32)
    x0[::7] = 1e30
    x0[3::11] = -1e30
    xd = torch.from_numpy(x0.copy()).cuda()
    m.decode_step(xd)
    assert lib.tgx_sync_status(m.handle) == 0
    xref, _ = oracle.decode_step(blobs, Rs, x0, k, H, I, norms=m.norms)
    assert np.array_equal(xd.cpu().numpy(), xref, equal_nan=True)
    m.close()


def test_synthetic_model_layer_parity(oracle):
    """Full Qwen3-shape synthetic model generated on the device: pull the
    experts back and check one chained 2-layer step against the oracle."""
    import torch
    from tinygiant_b200.engine import MoEModel
    H, I, E, k, L = C.EMBED_DIM, C.EXPERT_INTERMEDIATE, C.N_EXPERTS, C.N_EXPERTS_USED, 2
    m = MoEModel(H, I, E, k, L)
    m.fill_synthetic(1234)
    blobs = [m.read_experts(l, 0, E) for l in range(L)]
    # routers: regenerate by reading logits is not possible; set known ones instead
    rng = np.random.default_rng(4)
    Rs = [(rng.standard_normal((E, H)) * 0.02).astype(np.float32) for _ in range(L)]
    for l in range(L):
        m.set_router(l, Rs[l])
    w = oracle.dequantize_q4_0(blobs[0][: 18 * 4096])
    assert 0.015 < w.std() < 0.025
    x0 = np.random.default_rng(5).standard_normal(H).astype(np.float32)
    xd = torch.from_numpy(x0.copy()).cuda()
    m.decode_step(xd)
    xref, _ = oracle.decode_step(blobs, Rs, x0, k, H, I)
    assert np.array_equal(xd.cpu().numpy(), xref)
    m.close()
