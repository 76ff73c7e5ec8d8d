"""Seeded synthetic inputs for the benchmark configurations (no datasets are needed or used).

Constructions (one per benchmark configuration of the port):
  blurred_pair   : target = N(0,1) (seed 0) Gaussian-blurred (sigma, radius ceil(3 sigma), zero
                   'same' padding, normalised taps), min-max scaled to [0,1];
                   pred = target + noise * N(0,1) (seed 1).            configs 1, 2, 4
  mri_pair       : target = blurred noise sigma=3 in [0,1]; pred = target warped by a smooth
                   displacement (3-channel N(0,1), seed 2, blurred sigma=8, scaled to max |u| = 4
                   voxels, trilinear grid_sample, align_corners=True, border padding)
                   + 0.05 * N(0,1) (seed 3); computed in fp32, cast last.   config 3
  gigavoxel_pair : target = blurred noise sigma=4 in [0,1]; pred = 0.8 target + 0.2 * independent
                   blurred noise (seed 2) in [0,1].                        config 5
Random numbers come from a torch.Generator on the requested device, so CPU and CUDA inputs differ
for the same seed; `sha256_of` fingerprints a tensor for the records.
"""
import hashlib
import math

import torch
import torch.nn.functional as F


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def gaussian_taps(sigma, device, dtype=torch.float32):
    r = int(math.ceil(3.0 * sigma))
    x = torch.arange(-r, r + 1, device=device, dtype=torch.float64)
    w = torch.exp(-0.5 * (x / sigma) ** 2)
    return (w / w.sum()).to(dtype)


def gaussian_blur3d(x, sigma):
    """Separable Gaussian blur of (B, 1, D, H, W) with zero 'same' padding, plane-chunked along D
    for the W and H passes so that gigavoxel volumes need little temporary memory."""
    w = gaussian_taps(sigma, x.device, x.dtype)
    k = w.numel()
    r = k // 2
    out = x
    for shape, pad in (((1, 1, 1, 1, k), (0, 0, r)), ((1, 1, 1, k, 1), (0, r, 0))):
        res = torch.empty_like(out)
        step = max(1, (1 << 26) // max(1, out.shape[-1] * out.shape[-2]))
        for z in range(0, out.shape[2], step):
            res[:, :, z:z + step] = F.conv3d(out[:, :, z:z + step], w.view(shape), padding=pad)
        out = res
    res = torch.empty_like(out)
    step = max(1, (1 << 24) // max(1, out.shape[-1]))
    for y in range(0, out.shape[3], step):
        res[:, :, :, y:y + step] = F.conv3d(out[:, :, :, y:y + step], w.view(1, 1, k, 1, 1),
                                            padding=(r, 0, 0))
    return res


def _minmax_(x):
    lo, hi = x.min(), x.max()
    x.sub_(lo).div_(hi - lo)
    return x


def blurred_noise(shape, sigma, seed, device="cpu"):
    """N(0,1) of `shape` (N, C, D, H, W), blurred per volume, min-max scaled to [0,1] (fp32)."""
    n, c, d, h, w = shape
    x = torch.randn((n * c, 1, d, h, w), generator=_gen(device, seed), device=device)
    x = gaussian_blur3d(x, sigma)
    return _minmax_(x).view(shape)


def blurred_pair(shape, sigma=2.0, noise=0.1, seed=0, device="cpu", dtype=torch.float32):
    """Configs 1, 2 and 4: (pred, target)."""
    target = blurred_noise(shape, sigma, seed, device)
    pred = target + noise * torch.randn(shape, generator=_gen(device, seed + 1), device=device)
    return pred.to(dtype).contiguous(), target.to(dtype).contiguous()


def mri_pair(shape=(8, 1, 160, 192, 224), device="cpu", dtype=torch.bfloat16):
    """Config 3: a smooth random warp of blurred noise (see module docstring)."""
    n, c, d, h, w = shape
    target = blurred_noise(shape, 3.0, 0, device)
    disp = torch.randn((n * 3, 1, d, h, w), generator=_gen(device, 2), device=device)
    disp = gaussian_blur3d(disp, 8.0).view(n, 3, d, h, w)
    disp = disp * (4.0 / disp.abs().amax().clamp_min(1e-12))
    zz, yy, xx = torch.meshgrid(torch.arange(d, device=device, dtype=torch.float32),
                                torch.arange(h, device=device, dtype=torch.float32),
                                torch.arange(w, device=device, dtype=torch.float32), indexing="ij")
    # disp channels are (dz, dy, dx) in voxels; grid_sample wants (x, y, z) in [-1, 1]
    gx = (xx + disp[:, 2]) * (2.0 / max(w - 1, 1)) - 1.0
    gy = (yy + disp[:, 1]) * (2.0 / max(h - 1, 1)) - 1.0
    gz = (zz + disp[:, 0]) * (2.0 / max(d - 1, 1)) - 1.0
    grid = torch.stack((gx, gy, gz), dim=-1)
    del disp, gx, gy, gz
    warped = F.grid_sample(target.view(n, c, d, h, w), grid, mode="bilinear", padding_mode="border",
                           align_corners=True)
    del grid
    pred = warped + 0.05 * torch.randn(shape, generator=_gen(device, 3), device=device)
    return pred.to(dtype).contiguous(), target.to(dtype).contiguous()


def gigavoxel_pair(shape=(1, 1, 1024, 1024, 1024), device="cpu", dtype=torch.float32):
    """Config 5: pred = 0.8 target + 0.2 independent blurred noise."""
    target = blurred_noise(shape, 4.0, 0, device)
    other = blurred_noise(shape, 4.0, 2, device)
    pred = other.mul_(0.2).add_(target, alpha=0.8)
    return pred.to(dtype).contiguous(), target.to(dtype).contiguous()


def sha256_of(t):
    """SHA-256 of a tensor's bytes (moved to CPU), for input fingerprints in records."""
    a = t.detach().contiguous().cpu()
    if a.dtype == torch.bfloat16:
        a = a.view(torch.int16)
    return hashlib.sha256(a.numpy().tobytes()).hexdigest()
