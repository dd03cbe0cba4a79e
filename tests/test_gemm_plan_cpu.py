"""The checked GEMM's split-K policy (host arithmetic, no GPU): decode-sized outputs fill the SMs once; long-K
outputs take the split count whose waves are best balanced over the resident CTAs or pairs; limits on the count."""
import pytest

from sdcguard_b200 import _native


@pytest.fixture(scope="module")
def choose():
    return _native.lib().sdc_gemm_choose_split


def test_split_policy(choose):
    # training dW GEMMs on CTA pairs (74 resident pairs, K = 16384 -> 256 K blocks)
    assert choose(36, 74, 256, 0, 0) == 2          # 2304 x 768: 9 pair units x 4 tiles: two waves of half K
    assert choose(48, 74, 256, 0, 0) == 3          # 3072 x 768: 96 units would need two waves; 144 in two is better
    # single CTAs: 168 tiles on 148 SMs would take two waves unsplit; seven splits pack them into eight
    assert choose(168, 148, 256, 0, 0) == 7
    # a full GPU with many tiles: no split
    assert choose(1000, 74, 16, 0, 0) == 1
    # decode-sized outputs on single CTAs: as many splits as fill the SMs once, at most a quarter of the K blocks
    assert choose(66, 148, 16, 1, 0) == 2
    assert choose(10, 148, 16, 1, 0) == 4
    # forced counts keep the limits (8 splits, a quarter of the K blocks)
    assert choose(36, 74, 256, 0, 5) == 5
    assert choose(36, 74, 256, 0, 20) == 8
    assert choose(36, 74, 12, 0, 20) == 3
    assert choose(0, 74, 256, 0, 0) == 1
