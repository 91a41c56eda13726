"""The oracle's mirror order (the GPU's, bit for bit) against the reference order
(sequential block sums and libm expf, csrc/libtinygiant.c:555-595) over many random
Qwen3-shape experts: the stage-wise bound of order_check.py holds for every expert, and
requantisation flips of h stay rare."""
import numpy as np

from order_check import check_reference_order


def test_reference_order_bound_qwen3_shape(oracle):
    H, I, n = 2048, 768, 40
    flipped = 0
    worst_clean = 0.0
    for s in range(n):
        rng = np.random.default_rng(5000 + s)
        blob = oracle.quantize_q4_0((rng.standard_normal(3 * H * I) * 0.02).astype(np.float32))
        x = rng.standard_normal(H).astype(np.float32)
        nflip, err = check_reference_order(oracle.expert_stages(blob, x, H, I, 1),
                                           oracle.expert_stages(blob, x, H, I, 0))
        flipped += nflip > 0
        if nflip == 0:
            worst_clean = max(worst_clean, err)
    # measured at this shape: about 2% of experts have one flipped h code or scale
    assert flipped <= 4, f"{flipped} of {n} experts with requantisation flips"
    assert worst_clean <= 1e-6
