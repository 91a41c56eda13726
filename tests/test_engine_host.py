"""The host side of the device engine's token choice (tinygiant/engine.py:344-360,
395-407), without a GPU."""
import numpy as np

from tinygiant_b200.engine import sample_token


def test_greedy_is_the_first_argmax():
    logits = np.array([0.5, 2.0, -1.0, 2.0], np.float32)
    assert sample_token(logits, 0.0, 0.9) == 1


def test_top_p_keeps_the_smallest_prefix_reaching_p():
    logits = np.log(np.array([0.05, 0.6, 0.3, 0.05], np.float32))
    # p = 0.5: only the most probable token (0.6 already reaches it)
    picks = {sample_token(logits, 1.0, 0.5, np.random.RandomState(s)) for s in range(50)}
    assert picks == {1}
    # p = 0.85: the two most probable (0.6, then 0.9 crosses it)
    picks = {sample_token(logits, 1.0, 0.85, np.random.RandomState(s)) for s in range(200)}
    assert picks == {1, 2}


def test_seeded_sampling_is_repeatable():
    rng = np.random.default_rng(0)
    logits = rng.standard_normal(5000).astype(np.float32)
    a = [sample_token(logits, 0.7, 0.9, np.random.RandomState(3)) for _ in range(3)]
    b = [sample_token(logits, 0.7, 0.9, np.random.RandomState(3)) for _ in range(3)]
    assert a == b
