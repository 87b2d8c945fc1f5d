"""
The IGS1 bitstream container and its rANS coder (igs_b200.bitstream over igs_rans_encode / igs_rans_decode, host code) against golden
vectors of the reference's own encoder (tests/golden/py_codec.npz, made by tests/golden/make_golden_codec.py with the reference's
compress package and its C++ modules built from source): bit-identical bitstreams, the same order and estimated attribute sizes, and
decoding that reproduces the attributes, for one-stage and two-stage positions, channel transforms, a single Gaussian, constant streams
and values of 41 bits (raw bits in several chunks). Plus round trips of larger seeded attributes and the rejection of truncated payloads.
"""
import os

import numpy as np
import pytest

from igs_b200 import bitstream, codec

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "py_codec.npz")
CASES = ["p500", "p3000_refine3", "p1", "p64_const", "p800_big"]


def load(z, name):
    attrs = [(z[f"{name}/attr{k}/indices"], z[f"{name}/attr{k}/steps"], z[f"{name}/attr{k}/origins"])
             for k in range(int(z[f"{name}/num_attributes"]))]
    refs = [None if row[0] == -2 else [int(r) for r in row if r != -2] for row in z[f"{name}/refs"]]
    refine_bits = int(z[f"{name}/refine_bits"])
    exps = z[f"{name}/exponents"]
    return attrs, refs, refine_bits, (exps if len(exps) else None), z[f"{name}/meta"].tobytes()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name", CASES)
def test_encode_matches_reference_bytes(golden, name):
    attrs, refs, refine_bits, exps, meta = load(golden, name)
    data, order, nbytes = bitstream.encode_bitstream(attrs, meta, codec="rans", channel_refs=refs, refine_bits=refine_bits,
                                                     refine_exponents=exps)
    want = golden[f"{name}/bitstream"].tobytes()
    assert len(data) == len(want) and data == want
    assert np.array_equal(order, golden[f"{name}/order"])
    assert np.array_equal(np.array(nbytes), golden[f"{name}/attribute_bytes"])


@pytest.mark.parametrize("name", CASES)
def test_decode_reference_bitstream(golden, name):
    attrs, refs, refine_bits, exps, meta = load(golden, name)
    order = golden[f"{name}/order"]
    reconstruct = (lambda a: (a, exps[order])) if refine_bits else None
    decoded, got_meta = bitstream.decode_bitstream(golden[f"{name}/bitstream"].tobytes(), reconstruct=reconstruct)
    assert got_meta == meta
    for (want, steps, origins), (got, got_steps, got_origins) in zip(attrs, decoded):
        assert np.array_equal(got, want[order])
        assert np.array_equal(got_steps, steps) and np.array_equal(got_origins, origins)


@pytest.mark.parametrize("p,seed", [(20000, 1), (4097, 2)])
def test_round_trip(p, seed):
    rng = np.random.default_rng(seed)
    f32 = lambda *v: np.array(v, dtype=np.float32).astype(np.float64)  # noqa: E731
    attrs = [(rng.integers(0, 1 << 16, size=(p, 2), dtype=np.int64), f32(1.0, 1.0), f32(0, 0)),
             (rng.integers(-300, 300, size=(p, 2), dtype=np.int64), f32(0.5, 0.25), f32(1, 1)),
             (rng.geometric(0.05, size=(p, 3)).astype(np.int64), f32(1 / 64, 1 / 64, 1 / 64), f32(0, 0, 0))]
    data, order, _ = bitstream.encode_bitstream(attrs, b"", channel_refs=[None, None, [1, -1, 1]])
    decoded, _ = bitstream.decode_bitstream(data)
    for (want, _, _), (got, _, _) in zip(attrs, decoded):
        assert np.array_equal(got, want[order])


def test_truncated_payload_is_rejected(golden):
    data = golden["p500/bitstream"].tobytes()
    with pytest.raises(ValueError):
        bitstream.decode_bitstream(data[:len(data) - 40])


def _reference_rans():
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from oracle import build_ref

    try:
        return build_ref.load_cpp_module(build_ref.RANS)
    except ImportError:
        return None


def _stream_sets():
    """Seeded stream sets that reach the encoder's edge cases: wide and narrow ranges, 40-bit values (raw bits in three chunks), even
    and odd lengths (the median of two middle values in different buckets), constant and two-valued streams, one value."""
    rng = np.random.default_rng(11)
    yield [rng.integers(-(1 << 40), 1 << 40, 1000, dtype=np.int64), rng.integers(-3, 4, 1000, dtype=np.int64)]
    yield [np.sort(rng.integers(0, 1 << 30, 4096, dtype=np.int64)), rng.normal(0, 40, 4096).astype(np.int64)]
    yield [np.r_[np.zeros(500, np.int64), np.full(500, 1 << 33, np.int64)], rng.geometric(0.001, 1000).astype(np.int64)]
    yield [np.full(333, -7, np.int64), (rng.standard_cauchy(333) * 1000).astype(np.int64).clip(-(1 << 50), 1 << 50)]
    yield [np.array([123456789], np.int64), np.array([-5], np.int64)]
    yield [rng.integers(0, 2, 20001, dtype=np.int64) * (1 << 20) + rng.integers(0, 3, 20001, dtype=np.int64)]


@pytest.mark.skipif(_reference_rans() is None, reason="the reference's igs_rans module (oracle/build_ref.py) is not built")
@pytest.mark.parametrize("k", range(6))
def test_payload_matches_reference_coder(k):
    """The library's encoder against the reference's C++ coder (built from source into oracle/_ref) on the same streams: the same
    payload bytes, the same mapping and model per stream, and the library decodes the payload to the mapped values."""
    streams = list(_stream_sets())[k]
    rans = _reference_rans()
    ref_payload, ref_models = rans.encode_streams(streams)

    class Writer:
        num_bits = 0

        def write(self, *a):
            pass

        write_se = write_ue = write

    payload, _ = codec.encode_streams([streams], Writer())
    assert payload == bytes(ref_payload)
    count = len(streams[0])
    rows = np.zeros((len(streams), codec.MODEL_FIELDS), dtype=np.int64)
    table = np.zeros((len(streams), codec.MAX_TOKENS), dtype=np.int64)
    for j, m in enumerate(ref_models):
        rows[j, 3:7] = (m[3], m[4], m[5], len(m[6]))
        table[j, :len(m[6])] = m[6]
    buf = np.frombuffer(payload, dtype=np.uint8).copy()
    values = np.zeros((len(streams), count), dtype=np.int64)
    lib = codec._lib.load()
    p = lambda a: codec.ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    assert lib.igs_rans_decode(len(streams), count, p(rows), p(table), p(buf), buf.size, p(values)) == 0
    ref_values = rans.decode_streams(bytes(ref_payload), [(m[3], m[4], m[5], np.asarray(m[6], dtype=np.int64)) for m in ref_models],
                                     count)
    for j in range(len(streams)):
        assert np.array_equal(values[j], np.asarray(ref_values[j]))
