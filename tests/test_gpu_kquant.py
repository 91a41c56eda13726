"""GPU parity of the reference's own formats (csrc/libtinygiant.c: Q4_K, Q6_K, f16,
f32, RMSNorm, the expert forward and tg_moe_forward) through the C ABI, bit-exact
against the oracle's restatement (which tests/test_oracle_kquant.py pins to gguf
dequantisation and float64), plus the golden fixtures at the reference test's
tolerance."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu

FQ4K, FF16, FQ6K, FF32 = 0, 1, 2, 4


def q4k_blocks(rng, n, bounded=False):
    b = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    if bounded:   # near zero-mean weights (dmin ~ 7.5 d): activations stay bounded over chained layers
        d = rng.uniform(5e-5, 1.5e-4, n)
        b[:, 0:2] = np.asarray(d, np.float16).view(np.uint8).reshape(n, 2)
        b[:, 2:4] = np.asarray(7.5 * d, np.float16).view(np.uint8).reshape(n, 2)
        return b.ravel()
    b[:, 0:2] = np.asarray(rng.uniform(5e-4, 3e-3, n), np.float16).view(np.uint8).reshape(n, 2)
    b[:, 2:4] = np.asarray(rng.uniform(2e-4, 2e-3, n), np.float16).view(np.uint8).reshape(n, 2)
    return b.ravel()


def q6k_blocks(rng, n):
    b = rng.integers(0, 256, size=(n, 210), dtype=np.uint8)
    b[:, 192:208] = rng.integers(-64, 64, size=(n, 16), dtype=np.int8).view(np.uint8)
    b[:, 208:210] = np.asarray(rng.uniform(5e-4, 2e-3, n), np.float16).view(np.uint8).reshape(n, 2)
    return b.ravel()


def matrix(rng, fmt, rows, cols):
    if fmt == FQ4K:
        return q4k_blocks(rng, rows * cols // 256)
    if fmt == FQ6K:
        return q6k_blocks(rng, rows * cols // 256)
    w = (rng.standard_normal(rows * cols) * 0.05).astype(np.float32)
    return w.astype(np.float16).view(np.uint16) if fmt == FF16 else w


MATVEC = {FQ4K: "tg_matmul_q4k", FQ6K: "tg_matmul_q6k", FF16: "tg_f16_matvec", FF32: "tg_f32_matvec"}


def gpu_matvec(lib, fmt, W, x, rows, cols):
    y = np.empty(rows, np.float32)
    rc = getattr(lib, MATVEC[fmt])(W.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols)
    assert rc == 0, lib.tg_last_error()
    return y


def same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("fmt", [FQ4K, FQ6K, FF16, FF32])
@pytest.mark.parametrize("rows,cols", [(1, 256), (37, 512), (768, 2048), (2048, 768), (64, 7168), (9, 16384)])
def test_matvec_bit_exact(lib, oracle, fmt, rows, cols):
    rng = np.random.default_rng(rows * 131 + cols + fmt)
    W = matrix(rng, fmt, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    assert same_bits(gpu_matvec(lib, fmt, W, x, rows, cols), oracle.matvec_k(W, fmt, x, rows, cols))


@pytest.mark.parametrize("fmt,key", [(FQ4K, "q4k"), (FQ6K, "q6k")])
def test_matvec_golden(lib, fmt, key):
    gk = np.load(ROOT / "tests" / "golden" / "golden_kquant.npz")
    rows, cols = int(gk["mk_rows"]), int(gk["mk_cols"])
    y = gpu_matvec(lib, fmt, gk[key + "_W"], gk["mk_x"], rows, cols)
    y64 = gk[key + "_y64"]
    assert np.max(np.abs(y - y64)) <= 1e-4 * np.max(np.abs(y64))


def test_matvec_edge_inputs(lib, oracle):
    rng = np.random.default_rng(11)
    rows, cols = 40, 1024
    for fmt in (FQ4K, FQ6K):
        W = matrix(rng, fmt, rows, cols)
        x = np.zeros(cols, np.float32)                  # amax 0: scale 0, codes 0
        x[300:310] = [0.5, 1.5, -2.5, 127, 3.5, -0.5, 0, 1e-30, -127, 2.5]   # ties after scaling by 1
        x[512:768] = 0.0
        x[768:] = 1e-30                                  # tiny scale, large inverse
        assert same_bits(gpu_matvec(lib, fmt, W, x, rows, cols), oracle.matvec_k(W, fmt, x, rows, cols))


def test_rms_norm_bit_exact(lib, oracle):
    rng = np.random.default_rng(2)
    for dim in (4, 1024, 2048, 7168):
        x = rng.standard_normal(dim).astype(np.float32)
        w = rng.uniform(0.5, 1.5, dim).astype(np.float32)
        out = np.empty(dim, np.float32)
        assert lib.tg_rms_norm(x.ctypes.data, w.ctypes.data, out.ctypes.data, dim, 1e-6) == 0, lib.tg_last_error()
        assert same_bits(out, oracle.rms_norm_k(x, w, 1e-6))


def expert(rng, fmt_down, H, I):
    return q4k_blocks(rng, I * H // 256), q4k_blocks(rng, I * H // 256), matrix(rng, fmt_down, H, I)


@pytest.mark.parametrize("fmt", [FQ4K, FF16, FQ6K])
@pytest.mark.parametrize("H,I", [(512, 256), (2048, 768), (7168, 2048)])
def test_expert_forward_mixed_bit_exact(lib, oracle, fmt, H, I):
    rng = np.random.default_rng(H + I + fmt)
    g, u, d = expert(rng, fmt, H, I)
    x = rng.standard_normal(H).astype(np.float32)
    base = (rng.standard_normal(H) * 0.1).astype(np.float32)
    out = base.copy()
    rc = lib.tg_expert_forward_mixed(g.ctypes.data, u.ctypes.data, d.ctypes.data, fmt, x.ctypes.data,
                                     out.ctypes.data, 0.625, H, I)
    assert rc == 0, lib.tg_last_error()
    ref = base.copy()
    oracle.expert_forward_k(g, u, d, fmt, x, ref, 0.625, H, I)
    assert same_bits(out, ref)


def test_expert_forward_blob_and_golden(lib, oracle):
    gk = np.load(ROOT / "tests" / "golden" / "golden_kquant.npz")
    H, I = int(gk["ex_H"]), int(gk["ex_I"])
    blob, x = gk["ex_blob"], gk["ex_x"]           # held: an NpzFile lookup returns a fresh array
    out = np.zeros(H, np.float32)
    assert lib.tg_expert_forward(blob.ctypes.data, x.ctypes.data, out.ctypes.data, 1.0, H, I) == 0
    gb = I * (H // 256) * 144
    ref = np.zeros(H, np.float32)
    oracle.expert_forward_k(blob[:gb], blob[gb:2 * gb], blob[2 * gb:], FQ4K, x, ref, 1.0, H, I)
    assert same_bits(out, ref)
    y64 = gk["ex_y64"]
    assert np.linalg.norm(out - y64) / np.linalg.norm(y64) < 2e-3


@pytest.mark.parametrize("n", [1, 8])
def test_moe_forward_bit_exact(lib, oracle, n):
    H, I = 2048, 768
    rng = np.random.default_rng(40 + n)
    blobs = [np.concatenate(expert(rng, FQ4K, H, I)) for _ in range(n)]
    w = rng.dirichlet(np.ones(n)).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    out = np.full(H, 7.0, np.float32)                   # overwritten, not accumulated
    ptrs = (ctypes.c_void_p * n)(*[b.ctypes.data for b in blobs])
    assert lib.tg_moe_forward(ptrs, w.ctypes.data, n, x.ctypes.data, out.ctypes.data, H, I) == 0, lib.tg_last_error()
    gb = I * (H // 256) * 144
    ref = np.zeros(H, np.float32)
    for e in range(n):
        b = blobs[e]
        oracle.expert_forward_k(b[:gb], b[gb:2 * gb], b[2 * gb:], FQ4K, x, ref, float(w[e]), H, I)
    assert same_bits(out, ref)


@pytest.mark.parametrize("fmt", [FQ4K, FF16, FQ6K])
def test_device_experts_forward(lib, oracle, fmt):
    import torch
    H, I, n = 2048, 768, 8
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(90 + fmt)
    experts = [expert(rng, fmt, H, I) for _ in range(n)]
    s = torch.cuda.current_stream().cuda_stream
    keep, ptr = [], {"g": [], "u": [], "d": []}
    for g, u, d in experts:
        for key, m, f, rows, cols in (("g", g, FQ4K, I, H), ("u", u, FQ4K, I, H), ("d", d, fmt, H, I)):
            raw = torch.from_numpy(m.view(np.uint8).copy()).to(dev)
            nb = lib.tgx_kq_matrix_bytes(f, rows, cols)
            assert nb == raw.numel()
            dst = torch.empty(nb, dtype=torch.uint8, device=dev)
            assert lib.tgx_kq_prepare(f, ctypes.c_void_p(raw.data_ptr()), ctypes.c_void_p(dst.data_ptr()), rows,
                                      cols, ctypes.c_void_p(s)) == 0, lib.tg_last_error()
            keep += [raw, dst]
            ptr[key].append(dst.data_ptr())
    parr = {k: torch.tensor(v, dtype=torch.int64, device=dev) for k, v in ptr.items()}
    w = rng.dirichlet(np.ones(n)).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    base = (rng.standard_normal(H) * 0.1).astype(np.float32)
    wd, xd, od = (torch.from_numpy(a.copy()).to(dev) for a in (w, x, base))
    sb = lib.tgx_kq_scratch_bytes(n, H, I)
    scratch = torch.zeros(sb, dtype=torch.uint8, device=dev)

    def run(out, flags):
        rc = lib.tgx_kq_experts_forward(*(ctypes.c_void_p(parr[k].data_ptr()) for k in "gud"), fmt, n,
                                        ctypes.c_void_p(wd.data_ptr()), ctypes.c_void_p(xd.data_ptr()),
                                        ctypes.c_void_p(out.data_ptr()), H, I, 1, ctypes.c_void_p(scratch.data_ptr()),
                                        sb, flags, ctypes.c_void_p(s))
        assert rc == 0, lib.tg_last_error()

    run(od, 0)
    od2 = torch.from_numpy(base.copy()).to(dev)
    run(od2, 1)                               # chained behind the previous call: same result
    torch.cuda.synchronize()
    ref = base.copy()
    for e, (g, u, d) in enumerate(experts):
        oracle.expert_forward_k(g, u, d, fmt, x, ref, float(w[e]), H, I)
    assert same_bits(od.cpu().numpy(), ref)
    assert same_bits(od2.cpu().numpy(), ref)
    # the row-block counters (the first 16 KB) are left at zero for the next call
    assert int(scratch[:16384].count_nonzero()) == 0


def test_device_scratch_across_shapes(lib, oracle):
    # one scratch, a large shape then a small one: the small call finds its counters zero
    import torch
    dev = torch.device("cuda", 0)
    s = torch.cuda.current_stream().cuda_stream
    sb = lib.tgx_kq_scratch_bytes(2, 7168, 2048)
    scratch = torch.zeros(sb, dtype=torch.uint8, device=dev)
    rng = np.random.default_rng(5)
    for H, I in ((7168, 2048), (512, 256), (2048, 768)):
        ex = [expert(rng, FQ4K, H, I) for _ in range(2)]
        keep = [[torch.from_numpy(m.copy()).to(dev) for m in e3] for e3 in ex]
        tab = [torch.tensor([k[j].data_ptr() for k in keep], dtype=torch.int64, device=dev) for j in range(3)]
        w = np.array([0.25, 0.75], np.float32)
        x = rng.standard_normal(H).astype(np.float32)
        wd, xd = torch.from_numpy(w).to(dev), torch.from_numpy(x).to(dev)
        od = torch.zeros(H, dtype=torch.float32, device=dev)
        rc = lib.tgx_kq_experts_forward(*(ctypes.c_void_p(t.data_ptr()) for t in tab), 0, 2,
                                        ctypes.c_void_p(wd.data_ptr()), ctypes.c_void_p(xd.data_ptr()),
                                        ctypes.c_void_p(od.data_ptr()), H, I, 0, ctypes.c_void_p(scratch.data_ptr()),
                                        sb, 0, ctypes.c_void_p(s))
        assert rc == 0, lib.tg_last_error()
        torch.cuda.synchronize()
        ref = np.zeros(H, np.float32)
        for e, (g, u, d) in enumerate(ex):
            oracle.expert_forward_k(g, u, d, FQ4K, x, ref, float(w[e]), H, I)
        assert same_bits(od.cpu().numpy(), ref), (H, I)


def test_device_chain_in_place(lib, oracle):
    # x_{l+1} = x_l + sum_e w_e expert_e(x_l) over 6 chained layers, out == x, in one
    # CUDA graph of chained calls: bit-exact to the oracle's sequence
    import torch
    H, I, n, L = 2048, 768, 8, 6
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(123)
    layers = [[tuple(q4k_blocks(rng, I * H // 256, bounded=True) for _ in range(2)) +
               (q4k_blocks(rng, H * I // 256, bounded=True),) for _ in range(n)] for _ in range(L)]
    keep, tabs = [], []
    for lay in layers:
        ptr = {"g": [], "u": [], "d": []}
        for g, u, d in lay:
            for key, m in (("g", g), ("u", u), ("d", d)):
                t = torch.from_numpy(m.copy()).to(dev)
                keep.append(t)
                ptr[key].append(t.data_ptr())
        tabs.append({k: torch.tensor(v, dtype=torch.int64, device=dev) for k, v in ptr.items()})
    w = rng.dirichlet(np.ones(n)).astype(np.float32)
    x0 = (rng.standard_normal(H) * 0.05).astype(np.float32)
    wd = torch.from_numpy(w).to(dev)
    xd = torch.from_numpy(x0.copy()).to(dev)
    sb = lib.tgx_kq_scratch_bytes(n, H, I)
    scratch = torch.zeros(sb, dtype=torch.uint8, device=dev)

    def token(stream):
        for l in range(L):
            rc = lib.tgx_kq_experts_forward(*(ctypes.c_void_p(tabs[l][k].data_ptr()) for k in "gud"), 0, n,
                                            ctypes.c_void_p(wd.data_ptr()), ctypes.c_void_p(xd.data_ptr()),
                                            ctypes.c_void_p(xd.data_ptr()), H, I, 1,
                                            ctypes.c_void_p(scratch.data_ptr()), sb, 1 if l else 0,
                                            ctypes.c_void_p(stream))
            assert rc == 0, lib.tg_last_error()

    token(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    eager = xd.cpu().numpy().copy()
    xd.copy_(torch.from_numpy(x0))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        token(torch.cuda.current_stream().cuda_stream)
    xd.copy_(torch.from_numpy(x0))
    graph.replay()
    torch.cuda.synchronize()
    replayed = xd.cpu().numpy().copy()
    del graph
    ref = x0.copy()
    for lay in layers:
        acc = ref.copy()
        for e, (g, u, d) in enumerate(lay):
            oracle.expert_forward_k(g, u, d, FQ4K, ref, acc, float(w[e]), H, I)
        ref = acc
    assert np.all(np.isfinite(ref))
    assert same_bits(eager, ref)
    assert same_bits(replayed, ref)


def test_expert_forward_ref_order_within_tolerance(lib, oracle):
    # the reference's libm expf in place of the mirror exp: h may differ in the last bit,
    # which can move a code of its Q8 requantisation by one
    H, I = 2048, 768
    rng = np.random.default_rng(77)
    g, u, d = expert(rng, FQ4K, H, I)
    x = rng.standard_normal(H).astype(np.float32)
    out = np.zeros(H, np.float32)
    assert lib.tg_expert_forward_mixed(g.ctypes.data, u.ctypes.data, d.ctypes.data, FQ4K, x.ctypes.data,
                                       out.ctypes.data, 1.0, H, I) == 0
    ref = np.zeros(H, np.float32)
    oracle.expert_forward_k(g, u, d, FQ4K, x, ref, 1.0, H, I, mode=oracle.TG_REF_ORDER)
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 1e-3
