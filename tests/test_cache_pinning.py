"""The reference's ExpertCache pinning rules (tinygiant/cache.py:72-152) as this build
chooses them, without a GPU: driven from a relayout's index.json activation profile
and from request counts, and, where the reference checkout is present, compared with
the reference's own ExpertCache run on the same relayout directory."""
import sys
from pathlib import Path

import numpy as np
import pytest

from tinygiant_b200 import relayout as R
from tinygiant_b200.cache import select_hot, select_pins

REF = Path("/root/reference")
H, I, E, L = 256, 256, 8, 3


def make_relayout(tmp_path):
    rng = np.random.default_rng(12)
    eb = 3 * H * I // 32 * 18
    blobs = [rng.integers(0, 256, E * eb, dtype=np.uint8) for _ in range(L)]
    profile = {}
    for l in range(L):
        ranking = [int(e) for e in rng.permutation(E)]
        profile[str(l)] = {"expert_ranking": ranking, "activation_counts": {str(e): E - i for i, e in
                                                                             enumerate(ranking)}}
    R.write_model(tmp_path, blobs, E, 2, H, I, activation_profile=profile)
    return R.RelayoutReader(tmp_path)


def usage():
    # calibration requests: layer 0 has a tie (experts 2 and 6, three each), layer 1 has
    # one requested expert (backfill from the profile), layer 2 none
    counts = {}
    for layer, e, n in ((0, 6, 3), (0, 2, 3), (0, 4, 5), (0, 1, 1), (1, 7, 2)):
        counts[(layer, e)] = n
    return counts


def test_static_profile_pins(tmp_path):
    rd = make_relayout(tmp_path)
    prof = rd.index["activation_profile"]
    got = select_hot(prof, 3)
    assert got == [(l, e) for l in range(L) for e in prof[str(l)]["expert_ranking"][:3]]


def test_usage_pins_with_backfill(tmp_path):
    rd = make_relayout(tmp_path)
    prof = rd.index["activation_profile"]
    got = select_pins(usage(), prof, {0: 3, 1: 3, 2: 2}, L)
    # layer 0: by count, ties by the smaller id: 4 (5), 2 (3), 6 (3)
    assert got[:3] == [(0, 4), (0, 2), (0, 6)]
    # layer 1: 7, then the profile's order without 7
    rank1 = [e for e in prof["1"]["expert_ranking"] if e != 7]
    assert got[3:6] == [(1, 7), (1, rank1[0]), (1, rank1[1])]
    # layer 2: the profile only
    assert got[6:] == [(2, e) for e in prof["2"]["expert_ranking"][:2]]
    # a layer asked for zero pins is skipped
    assert all(l != 2 for l, _ in select_pins(usage(), prof, {0: 1, 1: 1}, L))


@pytest.mark.skipif(not (REF / "tinygiant" / "cache.py").exists(), reason="reference checkout not present")
def test_matches_the_reference_expert_cache(tmp_path):
    sys.path.insert(0, str(REF))
    try:
        from tinygiant.cache import ExpertCache
    finally:
        sys.path.remove(str(REF))
    rd = make_relayout(tmp_path)
    prof = rd.index["activation_profile"]

    def ref_pins(run):
        ec = ExpertCache(tmp_path, rd.index)
        order = []
        real = ec._lock_expert

        def lock(layer, e):
            order.append((layer, int(e)))
            real(layer, e)
        ec._lock_expert = lock
        run(ec)
        return order

    assert ref_pins(lambda ec: ec.pin_hot_experts(2)) == select_hot(prof, 2)

    def usage_run(ec):
        for (layer, e), n in usage().items():
            for _ in range(n):
                ec.get(layer, e)
        ec.pin_from_usage(3, L)
    assert ref_pins(usage_run) == select_pins(usage(), prof, {l: 3 for l in range(L)}, L)

    def nonuniform_run(ec):
        for (layer, e), n in usage().items():
            for _ in range(n):
                ec.get(layer, e)
        ec.pin_nonuniform({0: 2, 2: 4}, L)
    assert ref_pins(nonuniform_run) == select_pins(usage(), prof, {0: 2, 2: 4}, L)
