"""
Tile-row bands on one GPU: each band of a 1-, 2-, 3- and 4-way split is binned, rendered and back-propagated alone, as one rank of a
multi-GPU step does, with the fused step kernel and with the two separate kernels. The band's tile lists, render (and, with the separate
kernels, its 16-bit top-K lists) equal the matching rows of the whole-image step bit for bit, and the band gradients summed over the bands
(what the NCCL all-reduce computes) equal the whole-image gradients.
"""
import numpy as np
import pytest
import torch

from common import assert_close_grad, make_case, np_, to_dev
from igs_b200 import bands, pipeline

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_bands_reassemble_the_whole_image(world, fused, device):
    wl, inp = make_case(150, 210, 900, seed=71)  # 10 tile rows, the last one partial
    d = to_dev(inp, device)
    h, w = wl.height, wl.width
    full = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], fused=fused)
    full.launch()
    torch.cuda.synchronize()
    tiles_x, tiles_y = full.tb[0], full.tb[1]
    fb, fids = np_(full.bins), np_(full.ids)
    sums = {k: torch.zeros_like(getattr(full, k)) for k in ("v_xy", "v_conic", "v_colors")}
    loss = 0.0
    for rank in range(world):
        r0, r1 = bands.band_rows(tiles_y, world, rank)
        step = bands.BandStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], h, w, r0, r1,
                              capacity=full.capacity, fused=fused)
        step.launch()
        torch.cuda.synchronize()
        t0, t1 = r0 * tiles_x, r1 * tiles_x
        # tile lists: the band's tiles hold exactly the whole image's lists for those tiles
        bb, bids = np_(step.bins)[: t1 - t0], np_(step.ids)
        for t in range(t0, t1):
            a = fids[fb[t, 0]:fb[t, 1]] if fb[t, 1] > fb[t, 0] else np.zeros(0, np.int32)
            b = bids[bb[t - t0, 0]:bb[t - t0, 1]] if bb[t - t0, 1] > bb[t - t0, 0] else np.zeros(0, np.int32)
            np.testing.assert_array_equal(a, b)
        assert torch.equal(step.image, full.image[:, 16 * r0:16 * r0 + step.band_h])
        if not fused:  # the fused kernel keeps its top-K lists in shared memory
            assert torch.equal(step.topk[: t1 - t0], full.topk[t0:t1])
        for k in sums:
            sums[k] += getattr(step, k)
        loss += float(step.loss)
    for k in sums:
        assert_close_grad(sums[k], getattr(full, k), what=k)
    assert abs(loss - float(full.loss)) <= 1e-5 * float(full.loss)


def test_band_rows_balance_by_weight():
    assert bands.band_rows(10, 3, 0) == (0, 3) and bands.band_rows(10, 3, 2) == (6, 10)
    weights = [1, 1, 1, 1, 10, 10, 1, 1, 1, 1]
    parts = [bands.band_rows(10, 2, r, weights) for r in range(2)]
    assert parts[0][0] == 0 and parts[-1][1] == 10 and parts[0][1] == parts[1][0]
    assert 4 <= parts[0][1] <= 6
