"""
Top-K lists that our forward pass did not write. The kernels that read them treat a slot they cannot address as empty instead of
reading out of bounds: a Gaussian ID outside [0, N) in [H, W, 10] lists (the backward operator, the leave-one-out kernel and the feature
weights), a list position at or past the end of its tile's list in the 16-bit tile lists (the training step's backward). Each result
equals the one computed from the same lists with those slots emptied.
"""
import pytest
import torch

from common import make_case, ours_stages, to_dev
from igs_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def case(device):
    h, w = 72, 104
    _, inp = make_case(h, w, n=250, seed=21)
    d = to_dev(inp, device)
    return h, w, d, ours_stages(d, h, w)


def test_ids_outside_the_gaussians_count_as_empty(case, device):
    h, w, d, st = case
    n = d["means"].shape[0]
    topk = st["pixel_topk"]
    g = torch.Generator().manual_seed(5)
    mask = (torch.rand(topk.shape, generator=g) < 0.2).to(device)
    bad = torch.randint(n, n + 100_000, topk.shape, generator=g, dtype=torch.int32)
    bad.view(-1)[::5] = 2**31 - 1
    bad.view(-1)[1::5] = -7  # other negative IDs are empty slots already, as in the reference
    corrupted = torch.where(mask, bad.to(device), topk)
    cleaned = torch.where(mask, torch.full_like(topk, -1), topk)
    xys, conics, feats = st["xys"], st["conics"], d["features"]

    grads_bad = ops.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, feats, st["v_output"], corrupted)
    grads_ok = ops.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, feats, st["v_output"], cleaned)
    for a, b in zip(grads_bad, grads_ok):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-9)  # float atomics: summation order only

    loo_bad = ops.topk_norm_loo_loss_increase(h, w, xys, conics, feats, corrupted, d["target"], False, 1e-4)
    loo_ok = ops.topk_norm_loo_loss_increase(h, w, xys, conics, feats, cleaned, d["target"], False, 1e-4)
    torch.testing.assert_close(loo_bad, loo_ok, rtol=1e-5, atol=1e-6)

    assert torch.equal(ops.topk_feature_weights_fixed(h, w, xys, conics, corrupted),
                       ops.topk_feature_weights_fixed(h, w, xys, conics, cleaned))  # integer atomics: exact
    torch.cuda.synchronize()


def test_tile_list_positions_past_the_list_count_as_empty(case, device):
    h, w, d, st = case
    tb = ops.tile_grid(h, w)
    ids, bins = st["gaussian_ids_sorted"], st["tile_bins"]
    xys, conics, feats = st["xys"], st["conics"], d["features"]
    lens = (bins[:, 1] - bins[:, 0]).long()
    _, tile_topk = ops.nd_rasterize_forward_topk_norm_tiles(tb, (w, h, 1), int(lens.max()), ids, bins, xys, conics, feats)
    positions = tile_topk.to(torch.int32) & 0xFFFF  # the uint16 values
    g = torch.Generator().manual_seed(6)
    mask = (torch.rand(positions.shape, generator=g) < 0.2).to(device)
    # a position in [len, 65534] of the tile's list, stored as the uint16 bit pattern
    span = (65535 - lens)[:, None, None].cpu()
    past = (lens[:, None, None].cpu() + (torch.rand(positions.shape, generator=g) * span).long()).clamp(max=65534).to(device)
    corrupted = torch.where(mask, past.to(torch.int32), positions)
    cleaned = torch.where(mask, torch.full_like(positions, 0xFFFF), positions)
    as_u16 = lambda t: (t - 65536 * (t >= 32768).to(torch.int32)).to(torch.int16)

    grads_bad = ops.nd_rasterize_backward_topk_norm_tiles(h, w, ids, bins, xys, conics, feats, st["v_output"], as_u16(corrupted))
    grads_ok = ops.nd_rasterize_backward_topk_norm_tiles(h, w, ids, bins, xys, conics, feats, st["v_output"], as_u16(cleaned))
    for a, b in zip(grads_bad, grads_ok):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-9)
    torch.cuda.synchronize()
