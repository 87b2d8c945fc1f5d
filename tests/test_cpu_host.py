"""
Host logic without a GPU: tile-row band splits (contiguous, covering, balanced by weight), the tile grid, and the seeded workloads
(deterministic, with the configurations' shapes).
"""
import numpy as np
import pytest

from igs_b200 import bands, ops, workloads


@pytest.mark.parametrize("seed", range(20))
def test_band_rows_split_is_contiguous_covering_and_balanced(seed):
    rng = np.random.default_rng(seed)
    tiles_y = int(rng.integers(1, 200))
    world = int(rng.integers(1, 9))
    weights = rng.exponential(1.0, tiles_y) * (rng.random(tiles_y) < 0.8)  # some empty rows
    for w in (None, weights.tolist()):
        parts = [bands.band_rows(tiles_y, world, r, w) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == tiles_y
        for (a0, a1), (b0, b1) in zip(parts, parts[1:]):
            assert a1 == b0 and a0 <= a1
        if w is not None and weights.sum() > 0:
            # no band exceeds its share by more than one row's weight
            share, biggest = weights.sum() / world, weights.max()
            for a0, a1 in parts:
                assert weights[a0:a1].sum() <= share + biggest + 1e-9


def test_band_rows_rejects_bad_arguments():
    with pytest.raises(ValueError):
        bands.band_rows(10, 2, 2)
    with pytest.raises(ValueError):
        bands.band_rows(10, 2, 0, [1.0] * 9)


def test_tile_grid():
    assert ops.tile_grid(1080, 1920) == (120, 68, 1)
    assert ops.tile_grid(1, 1) == (1, 1, 1)
    assert ops.tile_grid(17, 33) == (3, 2, 1)


def test_workloads_are_seeded_and_shaped():
    wl = workloads.get_workload("cfg1_256")
    a, b = workloads.make_inputs(wl), workloads.make_inputs(wl)
    assert workloads.input_digest(a) == workloads.input_digest(b)
    assert a["target"].shape == (3, 256, 256) and a["means"].shape == (1000, 2) and a["features"].shape == (1000, 3)
    assert float(a["target"].min()) >= 0.0 and float(a["target"].max()) <= 1.0
    yuv = workloads.make_inputs(workloads.get_workload("cfg2_480p_yuv"))
    assert yuv["loss_target"].shape == (3, 480, 854) and yuv["loss_transform"].shape == (3, 3)
    tex = workloads.get_workload("cfg5_tex9")
    assert tex.channels == 9 and tex.images == 64 and workloads.get_workload("cfg4_2160p").sharding == "bands"


def test_roofline_bytes_of_the_raster_kernels():
    """bench.py's roofline entry: the fused step kernel moves the target, the image, the list IDs, each Gaussian's parameters once and its
    gradients once; the separate kernels also move the [H, W, 10] lists and the image gradient."""
    import bench

    p, c, n, k, isect, tiles = 2_073_600, 3, 20_000, 10, 178_298, 8_160
    fwd = p * (4 * c + 4 * k) + isect * 4 + n * 4 * (5 + c) + 12 * c * p
    bwd = p * (4 * c + 4 * k) + n * 4 * ((5 + c) + (2 + 3 + c))
    fused = bench.raster_roofline({"raster": 0.2}, p, c, n, k, isect, tiles, 6540.2, "measured", "cfg3_1080p")
    assert fused["kernel"] == "raster_step"
    assert fused["algorithmic_bytes"] == fwd + bwd  # the operator surface of forward, loss and backward
    assert fused["moved_bytes"] == p * 8 * c + isect * 4 + n * 4 * (5 + c) * 2 + tiles * 8
    assert fused["achieved"] == pytest.approx(fused["algorithmic_bytes"] / 0.2e-3 / 1e9)
    assert fused["frac"] == pytest.approx(fused["achieved"] / 6540.2)
    assert fused["traffic"] > 0 and 0 < fused["issue_active"] <= 1
    split = bench.raster_roofline({"forward": 0.11, "backward": 0.13}, p, c, n, k, isect, tiles, 6540.2, "measured", "cfg3_1080p")
    assert split["kernel"] == "raster_backward" and split["kernel_ms"] == 0.13
    assert split["algorithmic_bytes"] == bwd == split["moved_bytes"]
    other = bench.raster_roofline({"raster": 0.5}, p, c, n, k, isect, tiles, 6540.2, "measured", "cfg4_2160p")
    assert other["traffic"] is None and other["issue_active"] is None  # no capture of that workload


def test_rate_model_install_replaces_and_restores(monkeypatch):
    """igs_b200.rate_model.install routes a module's rate_model / bitstream_neighbors to the GPU versions, what they do not handle to the
    module's own functions, and restore undoes it."""
    import sys
    import types

    import numpy as np
    import torch

    from igs_b200 import neighbors, rate_model

    fake = types.ModuleType("fake_compress_rate")
    fake.rate_model, fake.bitstream_neighbors, fake.other = "ref_rate_model", "ref_neighbors", "untouched"
    monkeypatch.setitem(sys.modules, "fake_compress_rate", fake)
    calls = []
    fake.rate_model = lambda *a: calls.append(("rate_model", a)) or "reference"
    fake.bitstream_neighbors = lambda *a: calls.append(("bitstream_neighbors", a)) or "reference"
    originals = (fake.rate_model, fake.bitstream_neighbors)
    replaced = rate_model.install("fake_compress_rate", "no_such_module_here")
    assert fake.rate_model.original is originals[0] and fake.bitstream_neighbors.original is originals[1]
    assert fake.other == "untouched" and len(replaced) == 2
    # what the GPU versions do not handle goes to the reference's functions: here no GPU, a CPU device, 13 channels
    feat13 = torch.zeros(4, 13)
    args = (np.zeros((4, 2), np.int64), feat13, torch.zeros(4, 2), torch.zeros(4), [-1] * 13, [-1] * 13, torch.ones(13), torch.ones(13),
            torch.float32, torch.device("cpu"))
    assert fake.rate_model(*args) == "reference" and calls[-1][0] == "rate_model" and calls[-1][1][-1] == 0
    assert fake.bitstream_neighbors(np.zeros((4, 2), np.int64)) == "reference"
    assert not rate_model.runs_on_gpu(feat13, "cuda:0") and not rate_model.runs_on_gpu(torch.zeros(4, 3), "cpu")
    # installing twice wraps the reference's functions, not the routes
    again = rate_model.install("fake_compress_rate")
    assert fake.rate_model.original is originals[0]
    rate_model.restore(again)
    rate_model.restore(replaced)
    assert (fake.rate_model, fake.bitstream_neighbors) == originals


@pytest.mark.parametrize("n,c", [(1, 1), (20000, 3), (50000, 9), (63, 12)])
def test_packed_parameter_layout(n, c):
    """RasterStep.packed_layout: means, scales, rotations, features back to back, each on a 256-byte boundary, in a buffer that holds
    them all and no more than the alignment padding."""
    from igs_b200 import pipeline

    offsets, length = pipeline.RasterStep.packed_layout(n, c)
    sizes = (2 * n, 2 * n, n, c * n)
    align = pipeline.RasterStep.PACK_ALIGN
    assert offsets[0] == 0 and all(o % align == 0 for o in offsets) and align * 4 % 256 == 0
    for k in range(3):
        assert offsets[k] + sizes[k] <= offsets[k + 1] < offsets[k] + sizes[k] + align
    assert offsets[3] + sizes[3] <= length < offsets[3] + sizes[3] + align
