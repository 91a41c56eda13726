"""The fused decode kernel's bounded waits, made to run out without faulting anything:
a short per-context wait limit (tgx_set_wait_limit) and a router-sum contribution that
no block sends (tgx_fused_inject_missing, a stand-in for a block that never arrives).
The launch must end on its own, tgx_sync_status must report TG_ETIMEOUT, and the same
context must then decode bit-exact against the oracle, eager and from its graph."""
import numpy as np
import pytest

from tests.test_gpu_parity import build_model

pytestmark = pytest.mark.gpu


def test_wait_runs_out_then_context_recovers(oracle):
    import torch
    from tinygiant_b200._lib import TG_ETIMEOUT, TinyGiantError
    H, I, E, k, L = 512, 256, 16, 4, 2
    m, blobs, Rs, rng = build_model(oracle, H, I, E, k, L, seed=606)
    assert m.fused_info()[0] > 0
    x0 = rng.standard_normal(H).astype(np.float32)
    xref, _ = oracle.decode_step(blobs, Rs, x0, k, H, I, norms=m.norms)

    m.set_wait_limit(200_000)                    # ~0.1 ms at the B200's clock
    m.inject_missing(1)
    for eager in (True, False):                  # the direct launch, then the recaptured graph
        xd = torch.from_numpy(x0.copy()).cuda()
        m.decode_step(xd, eager=eager)
        with pytest.raises(TinyGiantError) as err:
            m.sync_status()
        assert err.value.code == TG_ETIMEOUT
        assert "bounded device wait expired" in str(err.value)
        m.sync_status()                          # reported once; the state is reset

    m.inject_missing(0)
    m.set_wait_limit(0)
    for eager in (True, False, False):
        xd = torch.from_numpy(x0.copy()).cuda()
        m.decode_step(xd, eager=eager)
        m.sync_status()
        assert np.array_equal(xd.cpu().numpy(), xref)
    m.close()
