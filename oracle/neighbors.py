"""
ORACLE (test infrastructure): brute-force restatement of the neighbour search of the rate model's preparation
(compress/csrc/prediction.cpp:69-166 nearest_neighbors, causal_neighbors) and of compress.rate.bitstream_neighbors (compress/rate.py:56-66)
with the bitstream order of compress/__init__.py:43-58 and the Morton codes of compress/common.py:87-131. O(P^2) numpy: small cases only.
"""
import numpy as np

NUM_NEIGHBORS = 8


def nearest_neighbors(positions, causal=True):
    """(indices [P, 8], squared distances [P, 8]) int64, ordered by squared distance then index, -1 where there are fewer."""
    pos = np.asarray(positions, dtype=np.int64)
    num = len(pos)
    ids = np.full((num, NUM_NEIGHBORS), -1, dtype=np.int64)
    d2 = np.full((num, NUM_NEIGHBORS), -1, dtype=np.int64)
    for i in range(num):
        cand = np.arange(i) if causal else np.delete(np.arange(num), i)
        if len(cand) == 0:
            continue
        diff = pos[cand] - pos[i]
        dist = diff[:, 0] * diff[:, 0] + diff[:, 1] * diff[:, 1]
        order = np.lexsort((cand, dist))[:NUM_NEIGHBORS]
        ids[i, :len(order)] = cand[order]
        d2[i, :len(order)] = dist[order]
    return ids, d2


def _part1by1(x):
    x = x & np.uint64(0x00000000FFFFFFFF)
    x = (x | (x << np.uint64(16))) & np.uint64(0x0000FFFF0000FFFF)
    x = (x | (x << np.uint64(8))) & np.uint64(0x00FF00FF00FF00FF)
    x = (x | (x << np.uint64(4))) & np.uint64(0x0F0F0F0F0F0F0F0F)
    x = (x | (x << np.uint64(2))) & np.uint64(0x3333333333333333)
    x = (x | (x << np.uint64(1))) & np.uint64(0x5555555555555555)
    return x


def morton_encode(x, y):
    return _part1by1(x.astype(np.uint64)) | (_part1by1(y.astype(np.uint64)) << np.uint64(1))


def bitstream_order(positions, refine_bits=0):
    positions = np.asarray(positions, dtype=np.int64)
    if refine_bits == 0:
        values = positions - positions.min(axis=0)
        return np.argsort(morton_encode(values[:, 0], values[:, 1]), kind="stable")
    coarse = positions >> refine_bits
    codes = morton_encode(*(coarse - coarse.min(axis=0)).T)
    fine = morton_encode(*(positions - positions.min(axis=0)).T)
    return np.lexsort((fine, codes))


def bitstream_neighbors(q_xy, refine_bits=0):
    q_xy = np.asarray(q_xy, dtype=np.int64)
    order = bitstream_order(q_xy, refine_bits)
    sorted_neighbors, _ = nearest_neighbors(q_xy[order], causal=True)
    out = np.full((len(q_xy), NUM_NEIGHBORS), -1, dtype=np.int64)
    out[order] = np.where(sorted_neighbors >= 0, order[sorted_neighbors.clip(min=0)], -1)
    return out
