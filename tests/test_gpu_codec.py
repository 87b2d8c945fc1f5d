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


def _reference_rans():
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import build_ref

    try:
        return build_ref.load_cpp_module(build_ref.RANS)
    except ImportError:
        return None


@pytest.mark.skipif(_reference_rans() is None, reason="the reference's igs_rans module (oracle/build_ref.py) is not built")
def test_full_size_streams_match_reference_coder():
    """The 2160p workload's 80,000 Gaussians as the bitstream codes them (position gaps in Morton order, log-scales, rotation, features
    after rounding to their steps): the GPU size estimates equal the reference coder's (built from source) to the last bit, and the
    library's payload is the reference coder's, byte for byte."""
    import torch

    from igs_b200 import workloads

    wl = workloads.get_workload("cfg4_2160p")
    inp = workloads.make_inputs(wl)
    q = torch.round(inp["means"].double() * torch.tensor([wl.width, wl.height], dtype=torch.float64) / 0.125).long().numpy()
    _, order, codes = bitstream.bitstream_order(q, 3)
    rot = np.round(inp["rotations"].numpy()[:, :1] / (np.pi / 256)).astype(np.int64)
    scale = np.round(np.log2(np.abs(inp["scales"].numpy())) / 0.03125).astype(np.int64)
    feat = np.round(inp["features"].numpy() * 64).astype(np.int64)
    streams = [np.diff(codes, prepend=np.uint64(0)).astype(np.int64)] + [a[order][:, c].copy() for a in (scale, rot, feat)
                                                                          for c in range(a.shape[1])]
    rans = _reference_rans()
    assert codec.estimate_stream_bits(streams) == [rans.estimate_stream_bits(s) for s in streams]

    class Writer:
        num_bits = 0

        def write(self, *a):
            pass

        write_se = write_ue = write

    payload, _ = codec.encode_streams([streams], Writer())
    ref_payload, _ = rans.encode_streams(streams)
    assert payload == bytes(ref_payload)
