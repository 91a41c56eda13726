"""tg_expert_forward_q4_0_noalloc: the expert forward on device pointers with a
fixed static scratch, checked against tg_expert_forward_q4_0 (the host-pointer
entry point) and against the CPU oracle on two calls in a row.  Collected last, so
it also runs after every other test in the same process; it must pass alone in a
fresh process too."""
import ctypes

import numpy as np
import pytest

from tinygiant_b200 import _lib as L


def p(a):
    return a.ctypes.data


def rand_case(rng, oracle, H, I):
    blob = oracle.quantize_q4_0((rng.standard_normal(3 * H * I) * 0.02).astype(np.float32))
    x = rng.standard_normal(H).astype(np.float32)
    out0 = (rng.standard_normal(H) * 0.1).astype(np.float32)
    return blob, x, out0


def test_noalloc_rejects_oversize_and_bad_args():
    lib = L.load_tinygiant_lib()
    x = np.zeros(4096, np.float32)
    assert lib.tg_expert_forward_q4_0_noalloc(p(x), p(x), p(x), ctypes.c_float(1.0), 4096, 1024, None) == L.TG_EINVAL
    msg = lib.tg_last_error().decode()
    assert "scratch" in msg and str(L.TG_NOALLOC_SCRATCH_BYTES) in msg
    assert lib.tg_expert_forward_q4_0_noalloc(None, p(x), p(x), ctypes.c_float(1.0), 2048, 768, None) == L.TG_EINVAL
    assert lib.tg_expert_forward_q4_0_noalloc(p(x), p(x), p(x), ctypes.c_float(1.0), 2000, 768, None) == L.TG_EINVAL


@pytest.mark.gpu
def test_noalloc_matches_host_entry_point_twice(lib, oracle):
    import torch

    rng = np.random.default_rng(2024)
    stream = torch.cuda.current_stream()
    # two calls in a row with different shapes and data: a stale scratch would show
    for H, I, wt in ((2048, 768, 0.375), (512, 256, -1.25)):
        blob, x, out0 = rand_case(rng, oracle, H, I)
        want = out0.copy()
        L.check(lib.tg_expert_forward_q4_0(p(blob), p(x), p(want), ctypes.c_float(wt), H, I), lib)

        d_blob = torch.from_numpy(blob).cuda()
        d_x = torch.from_numpy(x).cuda()
        d_out = torch.from_numpy(out0).cuda()
        torch.cuda.synchronize()
        L.check(lib.tg_expert_forward_q4_0_noalloc(d_blob.data_ptr(), d_x.data_ptr(), d_out.data_ptr(),
                                                   ctypes.c_float(wt), H, I, stream.cuda_stream), lib)
        stream.synchronize()
        got = d_out.cpu().numpy()
        assert np.array_equal(got, want), (H, I, float(np.max(np.abs(got - want))))
        # and, independently of the other CUDA path, the oracle's mirror order
        ref = oracle.expert_forward(blob, x, out0.copy(), wt, H, I, 1)
        assert np.array_equal(got, ref), (H, I, float(np.max(np.abs(got - ref))))


@pytest.mark.gpu
def test_noalloc_rejects_host_pointers(lib):
    x = np.zeros(2048, np.float32)
    blob = np.zeros(2048 * 768 * 3 // 32 * 18, np.uint8)
    assert lib.tg_expert_forward_q4_0_noalloc(p(blob), p(x), p(x), ctypes.c_float(1.0), 2048, 768,
                                              None) == L.TG_EINVAL
    assert b"device memory" in lib.tg_last_error()
