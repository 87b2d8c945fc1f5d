"""
The GPU neighbour search of the rate model's preparation (igs_nearest_neighbors; compress/csrc/prediction.cpp:69-166 and
compress/rate.py:56-66): exact equality with the brute-force oracle on random, duplicate-heavy, degenerate and wide-range positions, causal
and not, and with the neighbours the reference's own rate_model computed for the 480p YUV workload and a small RGB one.
"""
import os

import numpy as np
import pytest
import torch

from igs_b200 import neighbors as nb
from oracle import neighbors as on

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cases():
    rng = np.random.default_rng(5)
    yield "tiny", rng.integers(0, 50, size=(5, 2))
    yield "nine", rng.integers(0, 50, size=(9, 2))
    yield "random", rng.integers(0, 4000, size=(3000, 2))
    yield "duplicates", rng.integers(0, 12, size=(1500, 2))  # many equal positions and distances: ties by index
    yield "line", np.stack([rng.integers(0, 10 ** 6, size=1200), np.full(1200, 7)], axis=1)
    yield "wide", rng.integers(-2 ** 29, 2 ** 29, size=(1000, 2))  # squared distances up to 2^61: no int64 overflow
    yield "clustered", np.concatenate([rng.integers(0, 20, size=(800, 2)), rng.integers(10 ** 5, 10 ** 5 + 3000, size=(800, 2))])


@pytest.mark.parametrize("causal", [True, False])
def test_nearest_neighbors_match_brute_force(causal, device):
    for name, pos in cases():
        pos = pos.astype(np.int64)
        ids, d2 = nb.nearest_neighbors(torch.from_numpy(pos).to(device), causal=causal, return_dist2=True)
        ref_ids, ref_d2 = on.nearest_neighbors(pos, causal=causal)
        np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids, err_msg=name)
        np.testing.assert_array_equal(d2.cpu().numpy(), ref_d2, err_msg=name)


@pytest.mark.parametrize("name", ["cfg2_480p_yuv", "rgb_subgreen_320x200"])
def test_bitstream_neighbors_match_reference(name, device):
    z = np.load(os.path.join(GOLDEN, f"py_{name}.npz"))
    q = z["q_xy"].astype(np.int64)
    got = nb.bitstream_neighbors(q, 3, device=device)
    np.testing.assert_array_equal(got, on.bitstream_neighbors(q, 3))
    np.testing.assert_array_equal(got.clip(min=0), z["neighbors"])  # the reference's rate model stores them clamped to 0
    np.testing.assert_array_equal(got >= 0, z["weights"] > 0)


def test_empty_and_single(device):
    assert nb.bitstream_neighbors(np.zeros((0, 2), np.int64), device=device).shape == (0, 8)
    one = nb.nearest_neighbors(torch.zeros(1, 2, dtype=torch.int64, device=device))
    assert bool((one == -1).all())


def test_matches_reference_search_at_80k(device):
    """The 2160p workload's 80,000 positions (1/8-pixel steps, bitstream order): identical to the reference's own C++ causal_neighbors
    (compress/csrc/prediction.cpp, built from source into oracle/_ref)."""
    from igs_b200 import workloads
    from oracle import build_ref

    try:
        ref = build_ref.load_prediction()
    except ImportError as e:
        pytest.skip(str(e))
    wl = workloads.get_workload("cfg4_2160p")
    inp = workloads.make_inputs(wl)
    q = torch.round(inp["means"].double() * torch.tensor([wl.width, wl.height], dtype=torch.float64) / 0.125).long().numpy()
    ordered = np.ascontiguousarray(q[nb.bitstream_order(q, 3)])
    got = nb.causal_neighbors(torch.from_numpy(ordered).to(device)).cpu().numpy()
    np.testing.assert_array_equal(got, ref.causal_neighbors(ordered))


@pytest.mark.parametrize("refine_bits", [0, 3])
@pytest.mark.parametrize("case", ["small", "ragged", "large", "duplicates", "negative", "one_point", "all_equal"])
def test_bitstream_order_on_the_gpu_equals_the_host_sort(case, refine_bits, device):
    """igs_bitstream_order (Morton keys, stable radix sort) gives the host sort's order (numpy, the reference's definition) exactly."""
    rng = np.random.default_rng(7 * ["small", "ragged", "large", "duplicates", "negative", "one_point", "all_equal"].index(case) + refine_bits)
    n = {"small": 100, "ragged": 2048 * 3 + 17, "large": 100_000, "duplicates": 5000, "negative": 3000, "one_point": 1,
         "all_equal": 700}[case]
    span = 30720 if case != "small" else 64
    q = rng.integers(0, span, size=(n, 2), dtype=np.int64)
    if case == "duplicates":
        q = q[rng.integers(0, 50, size=n)]  # fifty distinct positions, many ties broken by index
    if case == "negative":
        q -= 20000
    if case == "all_equal":
        q[:] = 1234
    got = nb.bitstream_order_device(torch.from_numpy(q).to(device), refine_bits)
    assert got is not None
    np.testing.assert_array_equal(got.cpu().numpy(), nb.bitstream_order(q, refine_bits))


def test_bitstream_order_falls_back_for_wide_keys(device):
    rng = np.random.default_rng(4)
    q = rng.integers(0, 2**30, size=(1000, 2), dtype=np.int64)  # coarse and fine codes together wider than 64 bits
    assert nb.bitstream_order_device(torch.from_numpy(q).to(device), 2) is None
    got = nb.bitstream_neighbors(q, 2, device=device)  # the host sort then gives the order
    np.testing.assert_array_equal(got, on.bitstream_neighbors(q, 2))
    with pytest.raises(ValueError, match="2\\^32"):
        nb.bitstream_order_device(torch.tensor([[0, 0], [2**33, 0]], dtype=torch.int64, device=device), 0)
