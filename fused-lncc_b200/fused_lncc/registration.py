"""Dense 3-D registration driven by the fused LNCC loss: the caller side of the loss in its main use.

A displacement field is optimised with Adam so that warp(moving) matches fixed, under
loss = LNCC(warped, fixed) + lam * diffusion(disp). This is the loop of the reference's
examples/registration_demo.py:45-92 (trilinear `grid_sample` warp with border padding, a
finite-difference diffusion regulariser, Adam on the field), written for this package so that an
integration check runs the loss where it is optimised rather than evaluated. The reference compares
against MONAI, which is not installed here; the GPU test compares against the reference's PyTorch
LNCC instead.

    python -m fused_lncc.registration --size 96 --iters 150
"""
import argparse
import json

import torch
import torch.nn.functional as F

from . import fused_lncc_loss


def identity_grid(D, H, W, device):
    """(1, D, H, W, 3) sampling grid of the identity map, in grid_sample's (x, y, z) order."""
    z, y, x = torch.meshgrid(torch.linspace(-1, 1, D, device=device), torch.linspace(-1, 1, H, device=device),
                             torch.linspace(-1, 1, W, device=device), indexing="ij")
    return torch.stack([x, y, z], dim=-1)[None]


def warp(vol, disp, base):
    """vol (1, C, D, H, W) sampled at base + disp; disp (1, 3, D, H, W) in normalised coordinates."""
    grid = base + disp.permute(0, 2, 3, 4, 1)
    return F.grid_sample(vol, grid, mode="bilinear", padding_mode="border", align_corners=True)


def smooth_field(shape, amp, generator, ksz=11, device="cuda"):
    """Gaussian-like random field: N(0,1) noise through three k^3 mean filters, scaled to std `amp`."""
    f = torch.randn(shape, generator=generator, device=device)
    g = torch.full((1, 1, ksz, ksz, ksz), 1.0 / ksz ** 3, device=device)
    for _ in range(3):
        f = F.conv3d(f.reshape(-1, 1, *shape[2:]), g, padding=ksz // 2).reshape(shape)
    return amp * f / (f.std() + 1e-6)


def diffusion(disp):
    """Mean squared forward differences of the field along D, H and W."""
    dz = disp[:, :, 1:] - disp[:, :, :-1]
    dy = disp[:, :, :, 1:] - disp[:, :, :, :-1]
    dx = disp[:, :, :, :, 1:] - disp[:, :, :, :, :-1]
    return dz.pow(2).mean() + dy.pow(2).mean() + dx.pow(2).mean()


def make_pair(size, device="cuda", seed=0, amp=0.06):
    """(fixed, moving, base): a structured [0, 1] volume and its warp by a known smooth field."""
    gen = torch.Generator(device=device).manual_seed(seed)
    shape = (1, 1, size, size, size)
    fixed = smooth_field(shape, 1.0, gen, ksz=7, device=device).clamp(-3, 3)
    fixed = (fixed - fixed.min()) / (fixed.max() - fixed.min())
    base = identity_grid(size, size, size, device)
    true_disp = smooth_field((1, 3, size, size, size), amp, gen, device=device)
    moving = warp(fixed, true_disp, base).detach()
    return fixed.contiguous(), moving.contiguous(), base


def register(loss_fn, fixed, moving, base, iters=150, lr=0.02, lam=0.5):
    """Adam on the displacement field; returns per-iteration losses, ms/iter, peak memory and the
    final MSE and LNCC similarity (1 - fused loss) of the warped volume."""
    D, H, W = fixed.shape[2:]
    disp = torch.zeros(1, 3, D, H, W, device=fixed.device, requires_grad=True)
    opt = torch.optim.Adam([disp], lr=lr)
    losses = []
    torch.cuda.synchronize(fixed.device)
    torch.cuda.reset_peak_memory_stats(fixed.device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(iters):
        opt.zero_grad(set_to_none=True)
        warped = warp(moving, disp, base)
        loss = loss_fn(warped, fixed) + lam * diffusion(disp)
        loss.backward()
        opt.step()
        losses.append(loss.detach())
    t1.record()
    torch.cuda.synchronize(fixed.device)
    with torch.no_grad():
        warped = warp(moving, disp, base)
        mse = F.mse_loss(warped, fixed).item()
        sim = 1.0 - fused_lncc_loss(warped, fixed, 7).item()
    return {"losses": torch.stack(losses).float().cpu().tolist(), "ms_per_iter": t0.elapsed_time(t1) / iters,
            "peak_gb": torch.cuda.max_memory_allocated(fixed.device) / 1e9, "mse": mse, "sim": sim,
            "disp": disp.detach()}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--size", type=int, default=96)
    ap.add_argument("--iters", type=int, default=150)
    ap.add_argument("--kernel-size", type=int, default=7)
    a = ap.parse_args(argv)
    fixed, moving, base = make_pair(a.size)
    with torch.no_grad():
        mse0 = F.mse_loss(moving, fixed).item()
        sim0 = 1.0 - fused_lncc_loss(moving, fixed, a.kernel_size).item()
    r = register(lambda w, f: fused_lncc_loss(w, f, a.kernel_size), fixed, moving, base, iters=a.iters)
    r.pop("disp")
    losses = r.pop("losses")
    print(json.dumps({"size": a.size, "iters": a.iters, "before": {"mse": mse0, "sim": sim0},
                      "after": {"mse": r["mse"], "sim": r["sim"]}, "ms_per_iter": r["ms_per_iter"],
                      "peak_gb": r["peak_gb"], "loss_first": losses[0], "loss_last": losses[-1]}))


if __name__ == "__main__":
    main()
