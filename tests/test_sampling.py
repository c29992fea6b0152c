"""CPU checks of the sampling restatement (oracle) that the device sampler is tested against.

* the Philox-4x32-10 restatement reproduces the generator's published known-answer
  vectors (Random123 kat_vectors: zero counter/key, all-ones, and the pi digits);
* the top-k / top-p distribution follows model.py:414-424: top-k by value with ties to
  the lower index, the (cumsum - p) < top_p mask keeps at least the best token, and the
  inverse-CDF draw at u returns kept tokens only, the best one for u = 0;
* temperature <= 0 is the greedy argmax (first index of the maximum).
"""
import numpy as np
import torch

from oracle.reference_model import philox4x32_10, philox_uniform, sample_token, sampling_distribution


def test_philox_known_answers():
    assert philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    ones = 0xFFFFFFFF
    assert philox4x32_10((ones,) * 4, (ones,) * 2) == (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == (
        0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


def test_uniform_range_and_spread():
    u = np.array([philox_uniform(7, p) for p in range(4000)])
    assert u.min() >= 0.0 and u.max() < 1.0
    assert abs(u.mean() - 0.5) < 0.02


def test_topk_topp_rules():
    logits = torch.tensor([1.0, 3.0, 3.0, 2.0, -1.0, 0.5])
    ids, probs, kept = sampling_distribution(logits, 1.0, 3, 1.0)
    assert ids.tolist() == [1, 2, 3]  # tie between 1 and 2 -> lower index first
    assert abs(float(probs.sum()) - float(kept)) < 1e-6
    ids, probs, _ = sampling_distribution(logits, 1.0, 6, 1e-9)  # top-p keeps the best only
    assert ids.tolist() == [1]
    assert sample_token(logits, 1.0, 6, 0.95, 0.0) == 1
    for u in np.linspace(0, 0.999, 50):
        assert sample_token(logits, 0.8, 4, 0.9, float(u)) in (1, 2, 3, 0)
    assert sample_token(logits, 0.0, 6, 0.9, 0.3) == 1  # greedy: first index of the max
