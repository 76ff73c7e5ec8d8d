"""GPU: seeded random shapes, kernel sizes and dtypes against the fp64 C oracle.

Mirrors the reference's shape sweep (reference tests/test_robust.py:36-43) with generated cases: D, H, W
in 1 .. 300 (W % 4 == 0 and not), B = N*C in 1 .. 6, k in {3, 5, 7, 9}, fp32 and bf16, the automatic
kernel choice and the general sweep kernel, the companion launch on and off. Volumes are capped at
~1.5 M voxels per case so that the whole file runs in well under a minute on one B200. The cases are
drawn once from a fixed seed, so a failure names a reproducible case.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from fused_lncc import _lib, lncc_fused
from oracle import c_oracle

pytestmark = pytest.mark.gpu


def _cases(n=48, seed=20261202):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        k = int(rng.choice([3, 5, 7, 9]))
        H = int(rng.integers(1, 301))
        W = int(rng.integers(1, 301))
        if rng.random() < 0.6:
            W = max(4, W // 4 * 4)  # the warp-specialised kernel's shapes
        D = int(rng.integers(1, max(2, min(300, 1_500_000 // (H * W)) + 1)))
        B = int(rng.integers(1, 7))
        while B > 1 and B * D * H * W > 1_500_000:
            B -= 1
        dtype = "bf16" if rng.random() < 0.3 else "fp32"
        kernel = "sweep" if rng.random() < 0.25 else "auto"
        companion = bool(rng.random() < 0.5)
        out.append((i, B, D, H, W, k, dtype, kernel, companion))
    return out


@pytest.mark.parametrize("case", _cases(), ids=lambda c: "c{}-B{}D{}H{}W{}-k{}-{}-{}-comp{}".format(*c))
def test_fuzz_matches_oracle(case):
    i, B, D, H, W, k, dtype, kernel, companion = case
    g = torch.Generator().manual_seed(1000 + i)
    p = torch.randn(B, D, H, W, generator=g)
    t = 0.6 * p + 0.8 * torch.randn(B, D, H, W, generator=g)
    tdt = torch.float32 if dtype == "fp32" else torch.bfloat16
    p, t = p.to("cuda", tdt), t.to("cuda", tdt)
    prev = _lib.set_companion(companion)
    _lib.select_kernel(_lib.KERNEL_SWEEP if kernel == "sweep" else _lib.KERNEL_AUTO)
    try:
        cs = torch.zeros((), dtype=torch.float64, device="cuda")
        _, gr = lncc_fused(p, t, k, grad_scale=1.0, cc_sum_out=cs)
        torch.cuda.synchronize()
    finally:
        _lib.select_kernel(_lib.KERNEL_AUTO)
        _lib.set_companion(prev)
    o = c_oracle.lncc(p.float().cpu().numpy(), t.float().cpu().numpy(), k, grad_scale=1.0)
    n = o["count"]
    loss_tol = 1e-5 if dtype == "fp32" else 1e-3
    assert abs((1 - cs.item() / n) - o["loss"]) < loss_tol, (cs.item() / n, 1 - o["loss"])
    ref = torch.from_numpy(o["grad"]).double().flatten()
    gd = gr.double().cpu().flatten()
    if ref.norm() > 0:
        rel = ((gd - ref).norm() / ref.norm()).item()
        cos = F.cosine_similarity(gd, ref, dim=0).item()
        if dtype == "fp32":
            assert cos > 0.9999 and rel < 1e-3, (cos, rel)
        else:
            assert rel < 1e-2, rel
    assert gr.dtype == tdt and gr.shape == p.shape
