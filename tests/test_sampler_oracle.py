"""Sampling oracle on hand-checked cases (CPU): the kept-set rules of
vllm/sampler.py:7-42 (top-k with lower-index-first ties, top-p keeping
cum <= p plus the first token, both over bf16(logits / T))."""
import numpy as np

from oracle import sampler as osm


def _kept(logits, T=1.0, k=0, p=1.0):
    keep, _, _ = osm.kept_mask(np.asarray(logits, np.float32), T, k, p)
    return set(np.flatnonzero(keep).tolist())


def test_top_k_ties_take_lower_indices():
    assert _kept([3, 1, 2, 2, 0], k=3) == {0, 2, 3}
    assert _kept([3, 1, 2, 2, 0], k=2) == {0, 2}
    assert _kept([1, 1, 1, 1], k=2) == {0, 1}
    assert _kept([0, 5, 5, 1], k=1) == {1}


def test_top_p_keeps_cumulative_at_most_p_and_the_first():
    # logits exact in bf16: probabilities 0.610, 0.224, 0.083, 0.083
    # (cumulative 0.610, 0.835, 0.917, 1.0)
    lg = [0.0, -1.0, -2.0, -2.0]
    assert _kept(lg, p=0.84) == {0, 1}
    assert _kept(lg, p=0.83) == {0}
    assert _kept(lg, p=0.3) == {0}          # the first token always stays
    assert _kept(lg, p=0.99) == {0, 1, 2}   # the token that crosses p is dropped


def test_top_p_after_top_k_renormalises():
    lg = [0.0, -0.5, -1.0, -2.0]
    # top_k=2 -> probs 0.622, 0.378; top_k=3 -> cum 0.506, 0.813, 1.0
    assert _kept(lg, k=2, p=0.6) == {0}
    assert _kept(lg, k=2, p=0.99) == {0}
    assert _kept(lg, k=3, p=0.9) == {0, 1}


def test_temperature_scales_in_bf16():
    x = osm.scaled(np.array([1.0, 3.0], np.float32), 0.7)
    assert x.dtype == np.float32
    # bf16 values only (low 16 bits zero)
    assert not (x.view(np.uint32) & 0xFFFF).any()
    pr = osm.probs(np.array([0.0, np.log(3.0)], np.float32), 1.0, 0, 1.0)
    assert abs(pr[1] - 0.75) < 2e-3
