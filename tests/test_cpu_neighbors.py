"""
Host side of the neighbour search of the rate model's preparation: the bitstream order (Morton curve of the coarse positions, then of the
fine ones) that decides which Gaussians are "earlier" equals the oracle's restatement on the fixtures' positions and on edge cases.
"""
import os

import numpy as np
import pytest

from igs_b200 import neighbors as nb
from oracle import neighbors as on

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("name", ["cfg2_480p_yuv", "rgb_subgreen_320x200"])
@pytest.mark.parametrize("refine_bits", [0, 3])
def test_bitstream_order_matches_oracle(name, refine_bits):
    q = np.load(os.path.join(GOLDEN, f"py_{name}.npz"))["q_xy"].astype(np.int64)
    np.testing.assert_array_equal(nb.bitstream_order(q, refine_bits), on.bitstream_order(q, refine_bits))


def test_bitstream_order_edge_cases():
    rng = np.random.default_rng(3)
    dup = np.repeat(rng.integers(0, 5, size=(20, 2)), 3, axis=0)  # equal positions keep their index order (stable)
    for q in (dup, np.zeros((1, 2), np.int64), rng.integers(-(2 ** 31), 2 ** 31, size=(300, 2))):
        for bits in (0, 2):
            np.testing.assert_array_equal(nb.bitstream_order(q, bits), on.bitstream_order(q, bits))
    with pytest.raises(ValueError):
        nb.bitstream_order(np.array([[0, 0], [2 ** 33, 0]], np.int64))


def test_morton_interleave():
    x = np.array([0, 1, 0, 3, 0xFFFFFFFF], np.uint64)
    y = np.array([0, 0, 1, 3, 0], np.uint64)
    np.testing.assert_array_equal(nb.morton_encode(x, y), np.array([0, 1, 2, 15, 0x5555555555555555], np.uint64))
