"""The bound that north_star's "max-abs-rel 1e-5 after accumulation-order differences"
becomes for an expert forward whose intermediate h is requantised to Q8_0.

The GPU sums in the oracle's mirror order (lane-strided block partials met in an xor
tree, this library's exp).  The reference sums blocks sequentially with libm expf
(csrc/libtinygiant.c:555-595).  The two orders give fp32 gate, up and h values within a
few ulps.  The Q8_0 requantisation of h then maps them to codes and fp16 scales, and
a value or an amax that lands on a rounding boundary can take the neighbouring code or
the neighbouring fp16 scale in one order and not the other.  So the check is stage-wise:
  - g, u and h: max-abs-rel <= 1e-5;
  - Q8_0 of h: every code that differs differs by one step, every scale by one fp16 ulp;
  - y: max-abs-rel <= 1e-5 when no code and no scale differs, else <= FLIP_BOUND per
    differing code or scale (measured: at most 1.3e-3 for one flip at the Qwen3 shape).
"""
import numpy as np

REL_TOL = 1e-5
FLIP_BOUND = 2e-3


def max_abs_rel(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def requant_flips(hq_a, hq_b):
    """(differing codes, differing scales, largest code step, largest scale step in fp16 ulps)."""
    a, b = hq_a.reshape(-1, 34), hq_b.reshape(-1, 34)
    ca, cb = a[:, 2:].view(np.int8).astype(int), b[:, 2:].view(np.int8).astype(int)
    sa, sb = a[:, :2].copy().view(np.uint16).astype(int), b[:, :2].copy().view(np.uint16).astype(int)
    return (int((ca != cb).sum()), int((sa != sb).sum()), int(np.abs(ca - cb).max(initial=0)),
            int(np.abs(sa - sb).max(initial=0)))


def check_reference_order(st_mirror, st_ref, y_got=None):
    """Assert the stage-wise bound between the mirror-order stages (or y_got, an output
    bit-identical to them) and the reference-order stages; returns (flips, y error)."""
    for name in ("g", "u", "h"):
        err = max_abs_rel(st_mirror[name], st_ref[name])
        assert err <= REL_TOL, f"{name}: max-abs-rel {err:.3e} > {REL_TOL}"
    ncode, nscale, dcode, dscale = requant_flips(st_mirror["hq"], st_ref["hq"])
    assert dcode <= 1 and dscale <= 1, f"requant steps: code {dcode}, scale {dscale} fp16 ulps"
    y = st_mirror["y"] if y_got is None else y_got
    err = max_abs_rel(y, st_ref["y"])
    nflip = ncode + nscale
    bound = REL_TOL if nflip == 0 else FLIP_BOUND * nflip
    assert err <= bound, f"y: max-abs-rel {err:.3e} > {bound:.1e} with {ncode} code and {nscale} scale flips"
    return nflip, err
