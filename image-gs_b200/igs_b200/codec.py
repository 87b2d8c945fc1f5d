"""
Entropy coding of the bitstream's integer streams with the reference's format (compress/rans_codec.py): the per-stream headers written
here, the payload and its models by the library (igs_rans_encode / igs_rans_decode, host code with the reference's model search), and the
size estimate of the training loop's rate decisions on the GPU (igs_estimate_stream_bits). Same names, arguments and results as
compress.rans_codec: encode_streams(groups, writer), decode_streams(reader, data, num_streams, count), estimate_stream_bits(values).
"""
import ctypes

import numpy as np
import torch

from . import _lib

MAX_TOKENS = 4608  # include/igs_b200.h: IGS_RANS_MAX_TOKENS
MODEL_FIELDS = 8   # IGS_RANS_MODEL_FIELDS


def _zigzag(values):
    values = np.asarray(values, dtype=np.int64)
    return (values << 1) ^ (values >> 63)


def _unzigzag(values):
    values = np.asarray(values, dtype=np.int64)
    return (values >> 1) ^ -(values & 1)


def bit_length(values):
    """Bit lengths of non-negative integers below 2^53 [int64]."""
    return np.frexp(np.asarray(values, dtype=np.float64))[1].astype(np.int64)


def ue_bits(values):
    """Lengths of the order-0 Exp-Golomb codes of non-negative integers [int64]."""
    return 2 * bit_length(np.asarray(values, dtype=np.int64) + 1) - 1


def _table_layout(codes):
    """(cost after the length and mantissa bits, whether the differences' Exp-Golomb codes are cheaper than fixed-width codes)."""
    fixed = 5 + len(codes) * int(bit_length(codes.max()))
    delta = int(ue_bits(_zigzag(np.diff(codes, prepend=0))).sum())
    return 1 + min(fixed, delta), delta < fixed


def write_table(writer, codes, mantissa_bits):
    writer.write_ue(len(codes) - 1)
    writer.write(mantissa_bits, 2)
    _, use_delta = _table_layout(codes)
    writer.write(int(use_delta), 1)
    if use_delta:
        for d in np.diff(codes, prepend=0):
            writer.write_se(int(d))
    else:
        width = int(bit_length(codes.max()))
        writer.write(width, 5)
        for c in codes:
            writer.write(int(c), width)


def read_table(reader):
    """(count codes [int64], mantissa_bits) of one stream's token model."""
    num = reader.read_ue() + 1
    mantissa_bits = reader.read(2)
    if reader.read(1):
        codes = np.cumsum([reader.read_se() for _ in range(num)]).astype(np.int64)
    else:
        width = reader.read(5)
        codes = np.array([reader.read(width) for _ in range(num)], dtype=np.int64)
    return codes, mantissa_bits


def encode_streams(groups, writer):
    """Encode groups (attributes) of integer streams [P] int64 (all of one length) with one rANS state; each stream's model goes to
    writer. Returns the payload (bytes) and the estimated size in bits of each group (its headers and payload share)."""
    lib = _lib.load()
    flat = [np.asarray(s, dtype=np.int64) for streams in groups for s in streams]
    if not flat or any(s.ndim != 1 or len(s) == 0 or len(s) != len(flat[0]) for s in flat):
        raise ValueError("Streams must be non-empty one-dimensional arrays of one length")
    num, count = len(flat), len(flat[0])
    streams = np.ascontiguousarray(np.stack(flat))
    capacity = lib.igs_rans_payload_bound(num, count)
    payload = np.empty(capacity, dtype=np.uint8)
    size = ctypes.c_size_t(0)
    models = np.zeros((num, MODEL_FIELDS), dtype=np.int64)
    codes = np.zeros((num, MAX_TOKENS), dtype=np.int64)
    payload_bits = np.zeros(num, dtype=np.float64)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    _lib.check(lib.igs_rans_encode(num, count, p(streams), 0, p(payload), capacity, ctypes.byref(size), p(models), p(codes),
                                   p(payload_bits)), "igs_rans_encode")
    rows = iter(range(num))
    group_bits = []
    for streams_of_group in groups:
        start, bits = writer.num_bits, 0.0
        for _ in streams_of_group:
            k = next(rows)
            delta, zigzag_mapped, param, split_exp, msb_bits, mantissa_bits, num_codes = (int(x) for x in models[k, :7])
            writer.write(delta, 1)
            writer.write(zigzag_mapped, 1)
            writer.write_se(param)
            writer.write(split_exp, 4)
            writer.write(msb_bits, 2)
            write_table(writer, codes[k, :num_codes].copy(), mantissa_bits)
            bits += float(payload_bits[k])
        group_bits.append(writer.num_bits - start + bits)
    return payload[:size.value].tobytes(), group_bits


def decode_streams(reader, data, num_streams, count):
    """Decode groups of num_streams[i] streams of count values: their models from reader, the payload after them in data."""
    lib = _lib.load()
    heads = []
    for num in num_streams:
        for _ in range(num):
            delta, zigzag_mapped, param = reader.read(1), reader.read(1), reader.read_se()
            split_exp, msb_bits = reader.read(4), reader.read(2)
            codes, mantissa_bits = read_table(reader)
            heads.append((delta, zigzag_mapped, param, split_exp, msb_bits, mantissa_bits, codes))
    total = len(heads)
    models = np.zeros((total, MODEL_FIELDS), dtype=np.int64)
    table = np.zeros((total, MAX_TOKENS), dtype=np.int64)
    for k, (_, _, _, split_exp, msb_bits, mantissa_bits, codes) in enumerate(heads):
        if len(codes) > MAX_TOKENS:
            raise ValueError("Invalid token model")
        models[k, 3:7] = (split_exp, msb_bits, mantissa_bits, len(codes))
        table[k, :len(codes)] = codes
    payload = np.frombuffer(bytes(data[reader.byte_pos():]), dtype=np.uint8).copy()
    values = np.zeros((total, count), dtype=np.int64)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    status = lib.igs_rans_decode(total, count, p(models), p(table), p(payload), payload.size, p(values))
    if status != _lib.IGS_OK:
        raise ValueError(lib.igs_last_error().decode())
    groups, k = [], 0
    for num in num_streams:
        groups.append([])
        for _ in range(num):
            delta, zigzag_mapped, param = heads[k][:3]
            v = (_unzigzag(values[k]) if zigzag_mapped else values[k]) + param
            groups[-1].append(np.cumsum(v) if delta else v)
            k += 1
    return groups


def estimate_stream_bits(values, device="cuda"):
    """Estimated coded size in bits of a stream of integers [int64] (a numpy array or a tensor): compress.rans_codec's estimate, with the
    token histograms on the GPU. A list of streams of one length gives a list of estimates from one launch."""
    many = isinstance(values, (list, tuple))
    streams = [torch.as_tensor(np.asarray(v, dtype=np.int64)) if not isinstance(v, torch.Tensor) else v for v in
               (values if many else [values])]
    if any(s.ndim != 1 or s.numel() == 0 or s.numel() != streams[0].numel() for s in streams):
        raise ValueError("Streams must be non-empty one-dimensional arrays of one length")
    dev = streams[0].device if streams[0].is_cuda else torch.device(device)
    stacked = torch.stack([s.to(dev, torch.int64) for s in streams]).contiguous()
    lib = _lib.load()
    ws_bytes = lib.igs_estimate_bits_workspace(len(streams))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    bits = np.zeros(len(streams), dtype=np.float64)
    with torch.cuda.device(dev):
        _lib.check(lib.igs_estimate_stream_bits(len(streams), stacked.size(1), _lib.ptr(stacked), ctypes.c_void_p(bits.ctypes.data),
                                                _lib.ptr(ws), ws_bytes, ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)),
                   "estimate_stream_bits")
    return [float(b) for b in bits] if many else float(bits[0])
