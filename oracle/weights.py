"""
ORACLE (test infrastructure): PyTorch restatement of the per-Gaussian feature weights, compress.quantization.feature_weights
(compress/quantization.py:218-230) over model._iter_topk_weights (model.py:1404-1421): per pixel, the weights exp(-sigma) of its top-K
Gaussians recomputed in float32 from pixel_topk, normalized in float64 with eps, squared, scaled by 2^40, rounded and summed per Gaussian
in int64. Device-agnostic: the tests run it on the CPU and on CUDA tensors (ATen's own GPU arithmetic, the reference's).
"""
import torch


def iter_topk_weights(xy, conics, pixel_topk, img_h, img_w, chunk_size=2 ** 18):
    """(first pixel, ids [P, K] with empty entries as 0, valid [P, K], weights before normalization [P, K]) per chunk of pixels."""
    topk = pixel_topk.shape[-1]
    pixel_topk = pixel_topk.reshape(-1, topk).long()
    rows, cols = torch.meshgrid(torch.arange(img_h, device=xy.device), torch.arange(img_w, device=xy.device), indexing="ij")
    pixels = torch.stack([cols, rows], dim=-1).reshape(-1, 1, 2).to(xy.dtype)
    for begin in range(0, len(pixel_topk), chunk_size):
        ids = pixel_topk[begin:begin + chunk_size]
        valid = ids >= 0
        ids = ids.clamp(min=0)
        delta = xy[ids] - pixels[begin:begin + chunk_size]
        conic = conics[ids]
        sigma = 0.5 * (conic[..., 0] * delta[..., 0] ** 2 + conic[..., 2] * delta[..., 1] ** 2) + conic[..., 1] * delta[..., 0] * delta[..., 1]
        yield begin, ids, valid, torch.exp(-sigma) * valid


def feature_weights_fixed(topk_weights, num_gaussians, eps, device):
    """The int64 fixed-point sums (40 fractional bits) of feature_weights."""
    fixed_point = torch.zeros(num_gaussians, dtype=torch.int64, device=device)
    for _, ids, valid, weights in topk_weights:
        weights = weights.to(torch.float64)
        normalized = weights / (weights.sum(dim=1, keepdim=True) + eps)
        fixed_point.index_add_(0, ids[valid], torch.round(normalized[valid].square() * 2.0 ** 40).to(torch.int64))
    return fixed_point


def feature_weights(xy, conics, pixel_topk, img_h, img_w, eps=1e-4):
    """[N] float64 feature weights."""
    fixed = feature_weights_fixed(iter_topk_weights(xy, conics, pixel_topk, img_h, img_w), len(xy), eps, xy.device)
    return fixed.to(torch.float64) / 2.0 ** 40
