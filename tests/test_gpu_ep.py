"""GPU parity of expert parallelism (tgx_ep_*): the sharded path must equal the
single-GPU batched path with all experts (itself bit-exact to the CPU oracle) bit for
bit.  On one GPU, G ranks are emulated by G contexts on the same device whose y
buffers are summed with torch (each element has one nonzero term, so the sum is
exact); no kernel waits on another.  With two or more GPUs, a torchrun job runs the
real NCCL exchange (tests/ep_worker.py)."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8


@pytest.mark.parametrize("G", [2, 4, 8])
@pytest.mark.parametrize("T", [1, 5, 64])
def test_ep_emulated_matches_single_gpu(G, T):
    import torch
    from tinygiant_b200.engine import MoEModel
    from tinygiant_b200.ep import EPMoEModel
    L = 2
    full = MoEModel(H, I, E, K, L)
    full.fill_synthetic(77)
    ranks = [EPMoEModel(H, I, E, K, L, rank=r, size=G) for r in range(G)]
    for ep in ranks:
        ep.fill_synthetic(77)
    g = torch.Generator(device="cuda").manual_seed(T)
    X = torch.randn(T, H, generator=g, device="cuda")
    Xr = X.clone()
    full.decode_batched(Xr)
    Ys = [ep.y_buffer(T) for ep in ranks]
    for layer in range(L):
        for ep, Y in zip(ranks, Ys):
            ep.partial(layer, X, Y)
        total = Ys[0].clone()
        for Y in Ys[1:]:
            total += Y
        ranks[0].combine(X, total)
    torch.cuda.synchronize()
    assert torch.equal(X.view(torch.int32), Xr.view(torch.int32))
    # each rank's y is zero exactly where another rank holds the slot's expert
    nz = torch.stack([(Y.view(T, K, H) != 0).any(dim=2) for Y in Ys])
    assert int(nz.sum(dim=0).max()) <= 1
    for ep in ranks:
        ep.close()
    full.close()


def test_ep_rejects_foreign_experts():
    import numpy as np
    from tinygiant_b200._lib import TinyGiantError
    from tinygiant_b200.ep import EPMoEModel
    ep = EPMoEModel(H, I, E, K, 1, rank=1, size=4)
    assert (ep.first, ep.n_local) == (32, 32)
    blob = np.zeros(ep.expert_bytes, np.uint8)
    ep.load_experts(0, 40, blob)
    with pytest.raises(TinyGiantError):
        ep.load_experts(0, 0, blob)          # expert 0 belongs to rank 0
    ep.close()


def test_ep_nccl_matches_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531", str(ROOT / "tests" / "ep_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "bit-identical" in r.stdout
