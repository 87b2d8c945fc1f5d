"""
Seeded synthetic workloads of the Image-GS rasterization step: target images and 2D Gaussian models with the shapes and value
distributions of the five benchmark configurations (one 256x256 RGB case runnable on CPU, 480p YUV with the rate term, 1080p/20k RGB,
2160p/80k RGB for tile-row bands, and 2048x2048 nine-channel texture stacks).

Everything is generated on the CPU with torch.Generator(seed), so the CPU oracle, the reference kernels and ours see bit-identical inputs on
any machine; callers move the tensors to the GPU themselves.

Gaussian parameters follow the operator surface of project_gaussians_2d_scale_rot (gsplat/gsplat/project_gaussians_2d_scale_rot.py:12-28):
means in [0, 1) normalized image coordinates, scales in pixels (standard deviations; here exp of normally distributed log-scales, with the
log-axis difference shrunk symmetrically to a maximum anisotropy), rotations in radians, features [N, C].
"""
import math
from dataclasses import dataclass, field
from typing import Optional

import torch

TILE = 16


@dataclass(frozen=True)
class Workload:
    name: str
    height: int
    width: int
    num_gaussians: int
    channels: int
    log_scale_mean: float  # natural log of pixels
    log_scale_std: float
    max_anisotropy: Optional[float] = None  # ratio of the two scales; None leaves them independent
    color_space: str = "rgb"  # "yuv": features and target in BT.601 YUV, loss through the luma-weighted transform
    rate_term: bool = False
    seed: int = 1000
    images: int = 1  # independent images of this shape (texture stacks)
    sharding: str = "images"  # across GPUs: "images" (one independent image per GPU) or "bands" (tile-row bands of one image)
    notes: str = field(default="", compare=False)

    @property
    def tile_bounds(self):
        return ((self.width + TILE - 1) // TILE, (self.height + TILE - 1) // TILE, 1)

    @property
    def num_tiles(self):
        tx, ty, _ = self.tile_bounds
        return tx * ty

    @property
    def num_pixels(self):
        return self.height * self.width


# The five configurations; seed = 1000 + their 1-based index
CONFIGS = {
    "cfg1_256": Workload("cfg1_256", 256, 256, 1000, 3, math.log(2.0), 0.5, seed=1001,
                         notes="256x256 RGB, 1k Gaussians; one forward + L1 backward, CPU-runnable"),
    "cfg2_480p_yuv": Workload("cfg2_480p_yuv", 480, 854, 4000, 3, math.log(2.5), 0.5, max_anisotropy=6.0, color_space="yuv",
                              rate_term=True, seed=1002, notes="854x480 YUV, 4k Gaussians, luma-weighted L1 + rate term, feature step 1/64"),
    "cfg3_1080p": Workload("cfg3_1080p", 1080, 1920, 20000, 3, math.log(3.0), 0.6, seed=1003,
                           notes="1920x1080 RGB, 20k Gaussians; headline fwd+bwd steps/s"),
    "cfg4_2160p": Workload("cfg4_2160p", 2160, 3840, 80000, 3, math.log(3.0), 0.7, max_anisotropy=8.0, seed=1004, sharding="bands",
                           notes="3840x2160 RGB, 80k Gaussians; tile-row bands across GPUs with a gradient all-reduce"),
    "cfg5_tex9": Workload("cfg5_tex9", 2048, 2048, 50000, 9, math.log(3.0), 0.6, seed=1005, images=64,
                          notes="64 independent 2048x2048 9-channel texture stacks, 50k Gaussians each; one image per GPU"),
}


def get_workload(name: str) -> Workload:
    if name not in CONFIGS:
        raise KeyError(f"unknown workload {name!r}; known: {', '.join(CONFIGS)}")
    return CONFIGS[name]


def custom_workload(height, width, num_gaussians, channels=3, log_scale_mean=math.log(2.0), log_scale_std=0.5,
                    max_anisotropy=None, seed=7, name="custom") -> Workload:
    """A workload of any shape (parity tests use small and ragged ones)."""
    return Workload(name, height, width, num_gaussians, channels, log_scale_mean, log_scale_std, max_anisotropy, seed=seed)


def sinusoid_target(generator, channels, height, width, num_waves=8, noise_std=0.02):
    """[C, H, W] float32 in [0, 1]: per channel a sum of num_waves random oriented 2D sinusoids rescaled to [0, 1], plus N(0, noise_std)
    noise, clipped to [0, 1]."""
    ys = torch.arange(height, dtype=torch.float64)[:, None] / max(height, 1)
    xs = torch.arange(width, dtype=torch.float64)[None, :] / max(width, 1)
    planes = []
    for _ in range(channels):
        freq = 1.0 + 15.0 * torch.rand(num_waves, generator=generator, dtype=torch.float64)
        angle = math.pi * torch.rand(num_waves, generator=generator, dtype=torch.float64)
        phase = 2.0 * math.pi * torch.rand(num_waves, generator=generator, dtype=torch.float64)
        amp = 0.2 + torch.rand(num_waves, generator=generator, dtype=torch.float64)
        plane = torch.zeros(height, width, dtype=torch.float64)
        for w in range(num_waves):
            u = torch.cos(angle[w]) * xs + torch.sin(angle[w]) * ys
            plane += amp[w] * torch.sin(2.0 * math.pi * freq[w] * u + phase[w])
        lo, hi = plane.min(), plane.max()
        plane = (plane - lo) / (hi - lo) if hi > lo else torch.zeros_like(plane)
        planes.append(plane)
    target = torch.stack(planes).to(torch.float32)
    target += noise_std * torch.randn(target.shape, generator=generator, dtype=torch.float32)
    return target.clamp_(0.0, 1.0).contiguous()


# Full-range BT.601 RGB -> YUV without chroma offset (utils/color_utils.py:8-10 of the reference), a published colour-space matrix
RGB_TO_YUV = torch.tensor([[0.299, 0.587, 0.114],
                           [-0.168736, -0.331264, 0.5],
                           [0.5, -0.418688, -0.081312]], dtype=torch.float64)


def loss_transform_yuv(uv_weight=0.25):
    """[3, 3] float32 map of YUV features to the loss space: the RGB image of (Y, uv_weight U, uv_weight V)
    (utils/color_utils.py:29-39 of the reference)."""
    inverse = torch.linalg.inv(RGB_TO_YUV)
    weights = torch.tensor([1.0, uv_weight, uv_weight], dtype=torch.float64)
    return (inverse * weights[None, :]).to(torch.float32)


def gaussians(generator, wl: Workload):
    """Model of wl: means [N, 2] in [0, 1), scales [N, 2] in pixels, rotations [N, 1] in [0, pi), features [N, C] ~ N(0.5, 0.2)."""
    n = wl.num_gaussians
    means = torch.rand(n, 2, generator=generator, dtype=torch.float32)
    log_scales = wl.log_scale_mean + wl.log_scale_std * torch.randn(n, 2, generator=generator, dtype=torch.float32)
    if wl.max_anisotropy is not None:
        limit = math.log(wl.max_anisotropy)
        diff = log_scales[:, 0] - log_scales[:, 1]
        excess = (diff.abs() - limit).clamp(min=0.0) * diff.sign()
        log_scales = log_scales - torch.stack([0.5 * excess, -0.5 * excess], dim=1)
    scales = torch.exp(log_scales)
    rotations = math.pi * torch.rand(n, 1, generator=generator, dtype=torch.float32)
    features = 0.5 + 0.2 * torch.randn(n, wl.channels, generator=generator, dtype=torch.float32)
    return means.contiguous(), scales.contiguous(), rotations.contiguous(), features.contiguous()


def make_inputs(wl: Workload, image_index: int = 0):
    """Seeded CPU tensors of one image of wl: dict with target [C, H, W] (in the feature colour space), means, scales, rotations, features,
    and for YUV the loss transform and the loss-space target."""
    generator = torch.Generator().manual_seed(wl.seed * 1000 + image_index)
    target = sinusoid_target(generator, wl.channels, wl.height, wl.width)
    means, scales, rotations, features = gaussians(generator, wl)
    out = dict(target=target, means=means, scales=scales, rotations=rotations, features=features)
    if wl.color_space == "yuv":
        rgb = target
        yuv = torch.einsum("dc,chw->dhw", RGB_TO_YUV.to(torch.float32), rgb).contiguous()
        transform = loss_transform_yuv()
        out.update(target=yuv, loss_transform=transform,
                   loss_target=torch.einsum("dc,chw->dhw", transform, yuv).contiguous())
    return out


def input_digest(inputs):
    """Short hash of the generated tensors, so fixtures can check that a machine regenerates the same inputs."""
    import hashlib

    h = hashlib.sha256()
    for key in sorted(inputs):
        h.update(key.encode())
        h.update(inputs[key].contiguous().numpy().tobytes())
    return h.hexdigest()[:16]


def quant_settings(wl: Workload, device):
    """Step quantization settings of the reference's defaults (cfgs/default.yaml: pos_step 0.125 px, scale_step 1/32 octave, rot_step
    0.703125 degrees, feature step 1/64) as the tensors of model.quant_steps (model.py:300-305)."""
    return dict(pos_steps=(0.125 / torch.tensor([wl.width, wl.height], dtype=torch.float32)).to(device),
                scale_step=float(torch.tensor(0.03125, dtype=torch.float32)), rot_step=float(torch.tensor(math.radians(0.703125),
                                                                                                             dtype=torch.float32)),
                feat_steps=torch.full((wl.channels,), 0.015625, dtype=torch.float32, device=device))


class RateModelTensors:
    """The fields of the reference's compress.rate.RateModel that the rate operators read, from a dict of arrays."""

    def __init__(self, arrays, device):
        t = lambda k, dt=torch.float32: torch.as_tensor(arrays[k]).to(device=device, dtype=dt).contiguous()  # noqa: E731
        self.neighbors = t("neighbors", torch.int32)
        self.weights, self.slope, self.inv_steps = t("weights"), t("slope"), t("inv_steps")
        self.feat_coeffs, self.inv_rot = t("feat_coeffs"), t("inv_rot")
        self.offsets, self.sources, self.source_weights = t("offsets", torch.int32), t("sources", torch.int32), t("source_weights")
        self.color_refs = tuple(int(v) for v in arrays["color_refs"])
        self.pred_channels = tuple(int(v) for v in arrays["pred_channels"])
