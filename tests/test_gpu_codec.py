"""
The size estimate of the training loop's rate decisions (compress.estimate_bits / compress.rans_codec.estimate_stream_bits) with its
token histograms built on the GPU (igs_estimate_stream_bits): equal, to the last bit of the double, to the reference's own estimates in
tests/golden/py_codec.npz, per stream and per set of attributes.
"""
import os

import numpy as np
import pytest

from igs_b200 import bitstream, codec

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "py_codec.npz")


@pytest.mark.parametrize("name", ["p500", "p3000_refine3", "p1", "p64_const", "p800_big"])
def test_estimates_match_reference(name):
    z = np.load(GOLDEN)
    attrs = [z[f"{name}/attr{k}/indices"] for k in range(int(z[f"{name}/num_attributes"]))]
    refs = [None if row[0] == -2 else [int(r) for r in row if r != -2] for row in z[f"{name}/refs"]]
    streams = [a[:, c].copy() for a in attrs for c in range(a.shape[1])]
    got = codec.estimate_stream_bits(streams)
    assert np.array_equal(np.array(got), z[f"{name}/stream_estimates"])
    assert codec.estimate_stream_bits(streams[0]) == z[f"{name}/stream_estimates"][0]
    assert bitstream.estimate_bits(attrs, channel_refs=refs) == float(z[f"{name}/estimate_bits"])
