"""
Golden vectors of the IGS1 bitstream container and its rANS coder: the reference's own compress.encode_bitstream, compress.estimate_bits
and compress.rans_codec.estimate_stream_bits run on seeded quantized attributes, with its C++ modules (igs_rans, igs_prediction) built
from its sources into oracle/_ref by oracle/build_ref.py. Writes tests/golden/py_codec.npz: per case the inputs, the bitstream bytes, the
order, the estimated bytes per attribute and the size estimates.

Usage: python tests/golden/make_golden_codec.py [REFERENCE_ROOT] [OUT_DIR]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def cases():
    """(name, attributes, channel_refs, refine_bits, exponents or None, meta) of seeded quantized Gaussians."""
    out = []
    rng = np.random.default_rng(2024)

    def attrs(p, pos_range, refine_bits=0, big=False):
        pos = rng.integers(0, pos_range, size=(p, 2), dtype=np.int64)
        scale = np.round(rng.normal(0, 20, size=(p, 2))).astype(np.int64)
        rot = rng.integers(0, 64, size=(p, 1), dtype=np.int64)
        feat = np.round(rng.normal(30, 12, size=(p, 3))).astype(np.int64)
        if big:
            feat[:, 0] = rng.integers(-(1 << 40), 1 << 40, size=p, dtype=np.int64)
        f32 = lambda *v: np.array(v, dtype=np.float32).astype(np.float64)  # noqa: E731
        return [(pos, f32(1 / 4096, 1 / 4096), f32(0, 0)), (scale, f32(0.25, 0.25), f32(-2, -2)), (rot, f32(np.pi / 64), f32(0)),
                (feat, f32(1 / 64, 1 / 64, 1 / 32), f32(0, 0.5, 0))]

    out.append(("p500", attrs(500, 4096), [None, None, None, [1, -1, 1]], 0, None, b"meta-500"))
    a = attrs(3000, 1 << 14)
    exps = rng.integers(0, 4, size=(3000, 2), dtype=np.int64)
    a[0] = ((a[0][0] >> exps) << exps, a[0][1], a[0][2])  # positions multiples of 2^exponent
    out.append(("p3000_refine3", a, [None, None, None, None], 3, exps, b""))
    out.append(("p1", attrs(1, 16), None, 0, None, b""))
    const = attrs(64, 4)
    const[1] = (np.zeros_like(const[1][0]), const[1][1], const[1][2])
    out.append(("p64_const", const, None, 0, None, b"x"))
    out.append(("p800_big", attrs(800, 1 << 20, big=True), [None, None, None, [-1, 0, 0]], 0, None, b""))
    return out


def main(reference_root, out_dir):
    sys.path[:0] = [os.path.join(ROOT, "oracle", "_ref"), reference_root]
    import compress
    from compress import rans_codec

    arrays = {}
    for name, attributes, refs, refine_bits, exps, meta in cases():
        data, order, nbytes = compress.encode_bitstream(attributes, meta, codec="rans", channel_refs=refs, refine_bits=refine_bits,
                                                        refine_exponents=exps)
        est = compress.estimate_bits([a[0] for a in attributes], channel_refs=refs)
        stream_est = [rans_codec.estimate_stream_bits(a[0][:, c].copy()) for a in attributes for c in range(a[0].shape[1])]
        for k, (indices, steps, origins) in enumerate(attributes):
            arrays[f"{name}/attr{k}/indices"] = indices
            arrays[f"{name}/attr{k}/steps"] = steps
            arrays[f"{name}/attr{k}/origins"] = origins
        arrays[f"{name}/num_attributes"] = np.array(len(attributes))
        arrays[f"{name}/refs"] = np.array([[-2] * 3 if r is None else list(r) + [-2] * (3 - len(r)) for r in (refs or [None] * 4)])
        arrays[f"{name}/refine_bits"] = np.array(refine_bits)
        arrays[f"{name}/exponents"] = exps if exps is not None else np.zeros((0, 2), dtype=np.int64)
        arrays[f"{name}/meta"] = np.frombuffer(meta, dtype=np.uint8)
        arrays[f"{name}/bitstream"] = np.frombuffer(data, dtype=np.uint8)
        arrays[f"{name}/order"] = order
        arrays[f"{name}/attribute_bytes"] = np.array(nbytes)
        arrays[f"{name}/estimate_bits"] = np.array(est)
        arrays[f"{name}/stream_estimates"] = np.array(stream_est)
        print(name, len(data), "bytes")
    np.savez_compressed(os.path.join(out_dir, "py_codec.npz"), **arrays)


if __name__ == "__main__":
    sys.path.insert(0, ROOT)
    from oracle.build_ref import reference_root

    main(reference_root(sys.argv[1] if len(sys.argv) > 1 else None), sys.argv[2] if len(sys.argv) > 2 else HERE)
