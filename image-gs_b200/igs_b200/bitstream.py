"""
The IGS1 bitstream container of quantized Gaussian attributes (compress/__init__.py:104-225 with compress/common.py), byte for byte:
a packed header (magic, codec and refinement bits, number of Gaussians, metadata length, number of attributes), then per attribute its
channel count, quantization steps and origins, and either the position offsets (first attribute) or the channels' reference channels;
the optional position refinement bits; the streams' models (igs_b200.codec); the rANS payload. Gaussians are in the Morton order of their
(coarse) positions, positions are coded as gaps between sorted Morton codes, other attributes after the lossless channel transform.

Same functions, arguments and results as compress: bitstream_order, encode_bitstream, decode_bitstream, estimate_bits. The entropy coder
is the library's (igs_rans_encode / igs_rans_decode); the size estimate's histograms run on the GPU.
"""
import struct

import numpy as np

from . import codec as _codec
from .neighbors import morton_encode

MAGIC = b"IGS1"
HEADER = "<4sBIBB"
CODECS = {"rans": 1}


class BitWriter:
    """Big-endian bit fields, Exp-Golomb codes and float32 fields, as compress.common.BitWriter writes them."""

    def __init__(self):
        self.value, self.num_bits = 0, 0

    def write(self, value, num_bits):
        if num_bits > 0:
            if value < 0 or value >> num_bits:
                raise ValueError(f"Value {value} does not fit in {num_bits} bits")
            self.value = (self.value << num_bits) | value
            self.num_bits += num_bits

    def write_ue(self, value):
        self.write(value + 1, 2 * (value + 1).bit_length() - 1)

    def write_se(self, value):
        self.write_ue(2 * value if value >= 0 else -2 * value - 1)

    def write_f32(self, value):
        self.write(struct.unpack("<I", struct.pack("<f", value))[0], 32)

    def to_bytes(self):
        pad = -self.num_bits % 8
        return (self.value << pad).to_bytes((self.num_bits + pad) // 8, "big")


class BitReader:
    def __init__(self, data, pos=0):
        self.data, self.bit_pos = data, 8 * pos

    def read(self, num_bits):
        value = 0
        for _ in range(num_bits):
            value = (value << 1) | ((self.data[self.bit_pos >> 3] >> (7 - (self.bit_pos & 7))) & 1)
            self.bit_pos += 1
        return value

    def read_ue(self, max_zeros=64):
        zeros = 0
        while self.read(1) == 0:
            zeros += 1
            if zeros > max_zeros:
                raise ValueError("Invalid Exp-Golomb code")
        return ((1 << zeros) | self.read(zeros)) - 1

    def read_se(self):
        v = self.read_ue()
        return v >> 1 if v % 2 == 0 else -(v >> 1) - 1

    def read_f32(self):
        return struct.unpack("<f", struct.pack("<I", self.read(32)))[0]

    def byte_pos(self):
        return (self.bit_pos + 7) // 8


def _compact(x):
    # the even bits of x [uint64] gathered into the lower 32 (inverse of the Morton interleave)
    x = x & np.uint64(0x5555555555555555)
    for shift, mask in ((1, 0x3333333333333333), (2, 0x0F0F0F0F0F0F0F0F), (4, 0x00FF00FF00FF00FF), (8, 0x0000FFFF0000FFFF),
                        (16, 0x00000000FFFFFFFF)):
        x = (x | (x >> np.uint64(shift))) & np.uint64(mask)
    return x


def morton_decode(codes):
    return _compact(codes), _compact(codes >> np.uint64(1))


def _check_refs(refs, num_channels):
    if len(refs) != num_channels or any(not -1 <= r < num_channels or r == c or (r >= 0 and refs[r] >= 0) for c, r in enumerate(refs)):
        raise ValueError(f"Invalid reference channels {list(refs)} for {num_channels} channels")


def subtract_channels(values, refs):
    """Channel c replaced by its difference with channel refs[c] (-1 keeps it)."""
    _check_refs(refs, values.shape[1])
    out = values.copy()
    for c, r in enumerate(refs):
        if r >= 0:
            out[:, c] -= values[:, r]
    return out


def add_channels(values, refs):
    _check_refs(refs, values.shape[1])
    out = values.copy()
    for c, r in enumerate(refs):
        if r >= 0:
            out[:, c] += values[:, r]
    return out


def _morton_order(positions):
    offsets = positions.min(axis=0)
    values = positions - offsets
    if values.max() >= 2 ** 32:
        raise ValueError("The position must have at most 2^32 quantization levels per coordinate")
    codes = morton_encode(values[:, 0], values[:, 1])
    order = np.argsort(codes, kind="stable")
    return offsets, order, codes[order]


def bitstream_order(positions, refine_bits=0):
    """(offsets of the coarse positions, the order of the Gaussians, their sorted Morton codes): along the Morton curve of the coarse
    positions (positions >> refine_bits), within a coarse cell by the Morton code of the positions."""
    positions = np.asarray(positions, dtype=np.int64)
    if refine_bits == 0:
        return _morton_order(positions)
    coarse = positions >> refine_bits
    offsets = coarse.min(axis=0)
    if (coarse - offsets).max() >= 2 ** 32:
        raise ValueError("The position must have at most 2^32 quantization levels per coordinate")
    codes = morton_encode(*(coarse - offsets).T)
    fine = morton_encode(*(positions - positions.min(axis=0)).T)
    order = np.lexsort((fine, codes))
    return offsets, order, codes[order]


def _write_params(writer, steps, origins):
    if np.any(np.float32(steps) != steps) or np.any(np.float32(origins) != origins):
        raise ValueError("Quantization steps and origins must be single-precision values")
    shared = bool(np.all(steps == steps[0]) and np.all(origins == origins[0]))
    writer.write(int(shared), 1)
    for step, origin in zip(steps[:1] if shared else steps, origins[:1] if shared else origins):
        writer.write_f32(float(step))
        writer.write_f32(float(origin))


def _read_params(reader, num_channels):
    shared = reader.read(1)
    params = [(reader.read_f32(), reader.read_f32()) for _ in range(1 if shared else num_channels)]
    params = params * num_channels if shared else params
    return np.array([s for s, _ in params], dtype=np.float64), np.array([o for _, o in params], dtype=np.float64)


def _pack_bits(values, lengths):
    """Concatenated big-endian fields of the given lengths as one integer, and its number of bits."""
    total = int(lengths.sum())
    if total == 0:
        return 0, 0
    starts = np.cumsum(lengths) - lengths
    bits = np.zeros(total, dtype=np.uint8)
    for j in range(int(lengths.max())):
        has = lengths > j
        bits[starts[has] + j] = (values[has] >> (lengths[has] - 1 - j)) & 1
    packed = np.packbits(bits)
    return int.from_bytes(packed.tobytes(), "big") >> (8 * len(packed) - total), total


def _unpack_bits(data, bit_pos, lengths):
    total = int(lengths.sum())
    first = bit_pos // 8
    bits = np.unpackbits(np.frombuffer(data[first:(bit_pos + total + 7) // 8], dtype=np.uint8))[bit_pos - 8 * first:][:total]
    if len(bits) != total:
        raise ValueError("Truncated position refinement")
    starts = np.cumsum(lengths) - lengths
    values = np.zeros(len(lengths), dtype=np.int64)
    for j in range(int(lengths.max(initial=0))):
        has = lengths > j
        values[has] = (values[has] << 1) | bits[starts[has] + j]
    return values


def encode_bitstream(attributes, meta=b"", codec="rans", channel_refs=None, refine_bits=0, refine_exponents=None):
    """compress.encode_bitstream: attributes is a list of (indices [P, C] int64, steps [C], origins [C]), the first the positions (C = 2);
    channel_refs per attribute (None or [C] reference channels); refine_bits two-stage positions with refine_exponents [P, 2] low bits
    omitted. Returns (bitstream bytes, order of the Gaussians in it, estimated bytes per attribute)."""
    name = codec
    if name not in CODECS:
        raise ValueError(f"Unsupported bitstream codec '{name}', valid values include {', '.join(repr(n) for n in CODECS)}")
    if not 0 <= refine_bits < 16:
        raise ValueError(f"Refinement bits must be between 0 and 15 but got: {refine_bits}")
    channel_refs = [None] * len(attributes) if channel_refs is None else channel_refs
    if len(channel_refs) != len(attributes) or channel_refs[0] is not None:
        raise ValueError("Channel references must be given per attribute, and the position cannot be transformed")
    writer, groups, header_bits, order = BitWriter(), [], [], None
    for idx, ((indices, steps, origins), refs) in enumerate(zip(attributes, channel_refs)):
        start = writer.num_bits
        num_channels = indices.shape[1]
        writer.write_ue(num_channels - 1)
        _write_params(writer, steps, origins)
        if idx == 0:
            if num_channels != 2:
                raise ValueError("The first attribute must be the position")
            offsets, order, codes = bitstream_order(indices, refine_bits)
            for offset in offsets:
                writer.write_se(int(offset))
            groups.append([np.diff(codes, prepend=np.uint64(0)).astype(np.int64)])
        else:
            refs = [-1] * num_channels if refs is None else list(refs)
            for ref in refs:
                writer.write_ue(ref + 1)
            values = subtract_channels(indices[order], refs)
            groups.append([values[:, c] for c in range(num_channels)])
        header_bits.append(writer.num_bits - start)
    if refine_bits > 0:
        exponents = np.zeros_like(attributes[0][0]) if refine_exponents is None else refine_exponents
        if np.any(exponents < 0) or np.any(exponents > refine_bits):
            raise ValueError(f"Refinement exponents must be between 0 and {refine_bits}")
        start = writer.num_bits
        low = attributes[0][0][order] & ((1 << refine_bits) - 1)
        exps = exponents[order]
        if np.any(low & ((1 << exps) - 1)):
            raise ValueError("Position indices must be multiples of 2^exponent")
        value, total = _pack_bits((low >> exps).reshape(-1), (refine_bits - exps).reshape(-1))
        writer.write_ue(total)
        writer.write(value, total)
        header_bits[0] += writer.num_bits - start
    payload, group_bits = _codec.encode_streams(groups, writer)
    header = struct.pack(HEADER, MAGIC, CODECS[name] | refine_bits << 4, len(order), len(meta), len(attributes)) + meta
    return header + writer.to_bytes() + payload, order, [(b + c) / 8.0 for b, c in zip(header_bits, group_bits)]


def estimate_bits(indices, channel_refs=None):
    """compress.estimate_bits: the estimated coded size in bits of the attributes' streams without the header, with the estimates of
    all streams from one GPU launch."""
    channel_refs = [None] * len(indices) if channel_refs is None else channel_refs
    _, order, codes = _morton_order(indices[0])
    streams = [np.diff(codes, prepend=np.uint64(0)).astype(np.int64)]
    for values, refs in zip(indices[1:], channel_refs[1:]):
        values = values[order] if refs is None else subtract_channels(values[order], refs)
        streams += [values[:, c] for c in range(values.shape[1])]
    return sum(_codec.estimate_stream_bits([np.ascontiguousarray(s) for s in streams]))


def decode_bitstream(data, reconstruct=None):
    """compress.decode_bitstream: (attributes with the Gaussians in bitstream order, metadata); reconstruct(attributes) -> (attributes,
    refine_exponents) as the reference's, required for two-stage positions."""
    magic, codec_byte, num_gaussians, meta_len, num_attributes = struct.unpack_from(HEADER, data)
    codec_id, refine_bits = codec_byte & 15, codec_byte >> 4
    if magic != MAGIC or codec_id not in CODECS.values():
        raise ValueError("Not an Image-GS bitstream")
    pos = struct.calcsize(HEADER)
    meta = data[pos:pos + meta_len]
    reader = BitReader(data, pos + meta_len)
    params = []
    for idx in range(num_attributes):
        num_channels = reader.read_ue() + 1
        steps, origins = _read_params(reader, num_channels)
        if idx == 0:
            extra = np.array([reader.read_se() for _ in range(num_channels)], dtype=np.int64)
        else:
            extra = [reader.read_ue() - 1 for _ in range(num_channels)]
        params.append((num_channels, steps, origins, extra))
    if refine_bits > 0:
        refine_total = reader.read_ue()
        refine_pos = reader.bit_pos
        reader.bit_pos += refine_total
    num_streams = [1] + [num_channels for num_channels, _, _, _ in params[1:]]
    groups = _codec.decode_streams(reader, data, num_streams, num_gaussians)
    attributes = []
    for idx, ((_, steps, origins, extra), streams) in enumerate(zip(params, groups)):
        if idx == 0:
            codes = np.cumsum(streams[0].astype(np.uint64), dtype=np.uint64)
            values = (np.stack(morton_decode(codes), axis=1).astype(np.int64) + extra) << refine_bits
        else:
            values = add_channels(np.stack(streams, axis=1), extra)
        attributes.append((values, steps, origins))
    exponents = None
    if reconstruct is not None:
        attributes, exponents = reconstruct(attributes)
    if refine_bits > 0:
        if reconstruct is None:
            raise ValueError("Decoding two-stage positions requires reconstruct (the refinement exponents)")
        exponents = np.zeros((num_gaussians, 2), dtype=np.int64) if exponents is None else np.asarray(exponents, dtype=np.int64)
        lengths = (refine_bits - exponents).reshape(-1)
        if lengths.sum() != refine_total:
            raise ValueError("The refinement exponents do not match the bitstream")
        low = _unpack_bits(data, refine_pos, lengths).reshape(-1, 2) << exponents
        positions, steps, origins = attributes[0]
        attributes = [(positions + low, steps, origins)] + list(attributes[1:])
    return attributes, meta


_ROUTES = {"compress": ("bitstream_order", "encode_bitstream", "decode_bitstream", "estimate_bits"),
           "model": ("bitstream_order", "encode_bitstream", "decode_bitstream"),  # bound at import, model.py:19
           "compress.quantization": ("estimate_bits",)}                              # bound at import, compress/quantization.py:15


def install(*module_names):
    """Route the reference's calls of compress.bitstream_order, encode_bitstream, decode_bitstream and estimate_bits to these functions
    (same signatures and results; the bytes written are the reference's): the names are replaced in each named module that is imported
    or importable (default: compress, and model and compress.quantization, which bind them when imported). Returns {(module, name):
    original} for restore()."""
    import importlib

    ours = {"bitstream_order": bitstream_order, "encode_bitstream": encode_bitstream, "decode_bitstream": decode_bitstream,
            "estimate_bits": estimate_bits}
    replaced = {}
    for name in module_names or tuple(_ROUTES):
        try:
            module = importlib.import_module(name)
        except ImportError:
            continue
        for attr in _ROUTES.get(name, tuple(ours)):
            if hasattr(module, attr):
                replaced[(name, attr)] = getattr(module, attr)
                setattr(module, attr, ours[attr])
    return replaced


def restore(replaced):
    """Undo install()."""
    import importlib

    for (name, attr), original in replaced.items():
        setattr(importlib.import_module(name), attr, original)
