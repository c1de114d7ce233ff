"""The test-side Philox4x32-10 against the generator's published known-answer
vectors (Random123 kat_vectors, philox4x32 with 10 rounds)."""
import numpy as np
import pytest

from philox import dropout_keep, philox4x32_10

KAT = [
    ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
     (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
    ((0xffffffff, 0xffffffff, 0xffffffff, 0xffffffff), (0xffffffff, 0xffffffff),
     (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
    ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
     (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1)),
]


@pytest.mark.parametrize("ctr,key,want", KAT)
def test_philox_known_answers(ctr, key, want):
    got = philox4x32_10(*[np.array([c], dtype=np.uint32) for c in ctr], *key)
    assert tuple(int(g[0]) for g in got) == want


def test_keep_rate():
    keep = dropout_keep(np.arange(1 << 18), 0.3, seed=12345)
    assert abs(keep.mean() - 0.7) < 0.005
