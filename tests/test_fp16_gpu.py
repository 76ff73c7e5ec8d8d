"""GPU: fp16 inputs (not in the reference, which lists fp16 as open: BENCHMARKS.md:177-178).

fp16 is handled like bf16: loaded into fp32, all arithmetic in fp32, the gradient rounded to fp16 on
store. The oracle sees the fp16 values as fp64. Tolerances: fp16 keeps 11 significant bits against
bf16's 8, so the bf16 contract's figures (|loss| < 1e-3, rel < 1e-2) are used as upper bounds and the
tighter ones the format allows are asserted where they hold (loss 2e-4, rel 2e-3).

The gradient of 1 - mean(cc) is of order 1/M, below fp16's normal range (6.1e-5) for large volumes;
the C-ABI cases therefore ask for d(sum cc)/dpred (grad_scale = 1, values of order 1), and the
autograd cases scale the loss as torch.amp.GradScaler does. The autograd path folds grad_out into the
fp32 scale before the fp16 rounding.
"""
import pytest
import torch
import torch.nn.functional as F

from fused_lncc import _lib, fused_lncc_loss, lncc_fused
from oracle import c_oracle

pytestmark = pytest.mark.gpu

LOSS_TOL = 2e-4
REL = 2e-3


def _pair(shape, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    p = torch.rand(shape, generator=g)
    t = 0.7 * p + 0.3 * torch.rand(shape, generator=g)
    return p.to("cuda", dtype), t.to("cuda", dtype)


def _rel(g, ref):
    g = g.double().cpu().flatten()
    ref = ref.double().cpu().flatten()
    return ((g - ref).norm() / ref.norm()).item(), F.cosine_similarity(g, ref, dim=0).item()


@pytest.mark.parametrize("kernel", ["auto", "sweep"])
@pytest.mark.parametrize("k", [3, 5, 7, 9])
@pytest.mark.parametrize("shape", [(2, 20, 24, 32), (1, 33, 17, 40), (3, 12, 40, 21)])
def test_fp16_cabi_matches_oracle(kernel, k, shape):
    p, t = _pair(shape, seed=k * 100 + shape[1])
    _lib.select_kernel(_lib.KERNEL_SWEEP if kernel == "sweep" else _lib.KERNEL_AUTO)
    try:
        cs = torch.zeros((), dtype=torch.float64, device="cuda")
        _, gr = lncc_fused(p, t, k, grad_scale=1.0, cc_sum_out=cs)
        torch.cuda.synchronize()
    finally:
        _lib.select_kernel(_lib.KERNEL_AUTO)
    o = c_oracle.lncc(p.float().cpu().numpy(), t.float().cpu().numpy(), k, grad_scale=1.0)
    assert abs((1 - cs.item() / o["count"]) - o["loss"]) < LOSS_TOL
    rel, cos = _rel(gr, torch.from_numpy(o["grad"]))
    assert gr.dtype == torch.float16 and torch.isfinite(gr).all()
    assert rel < REL and cos > 0.9999, (rel, cos)


@pytest.mark.parametrize("shape,k", [((2, 16, 64, 64, 64), 7), ((1, 1, 96, 200, 136), 9)])
def test_fp16_companion_and_tiles(shape, k):
    """Shapes that take the companion launch and row/column tiles, with the companion on and off."""
    p, t = _pair(shape, seed=7)
    outs = []
    for comp in (True, False):
        prev = _lib.set_companion(comp)
        try:
            cs = torch.zeros((), dtype=torch.float64, device="cuda")
            _, gr = lncc_fused(p, t, k, grad_scale=1.0, cc_sum_out=cs)
            torch.cuda.synchronize()
        finally:
            _lib.set_companion(prev)
        outs.append((cs.item(), gr))
    assert abs(outs[0][0] - outs[1][0]) / abs(outs[1][0]) < 1e-6
    rel, _ = _rel(outs[0][1], outs[1][1])
    assert rel < 1e-3
    # the fp16 result against the fp32 kernel on the same (fp16-exact) values
    cs32 = torch.zeros((), dtype=torch.float64, device="cuda")
    _, g32 = lncc_fused(p.float(), t.float(), k, grad_scale=1.0, cc_sum_out=cs32)
    torch.cuda.synchronize()
    assert abs(outs[0][0] - cs32.item()) / abs(cs32.item()) < 1e-6
    rel, cos = _rel(outs[0][1], g32)
    assert rel < REL and cos > 0.9999, (rel, cos)


def test_fp16_autograd_scaled_loss_matches_oracle():
    """GradScaler-style: backward of scale * loss; the gradient / scale matches d(1 - mean cc)/dpred,
    although most of its values are below fp16's normal range unscaled."""
    p, t = _pair((2, 1, 24, 40, 48), seed=3)
    scale = 65536.0
    pg = p.clone().requires_grad_(True)
    loss = fused_lncc_loss(pg, t, 7)
    (loss * scale).backward()
    torch.cuda.synchronize()
    assert loss.dtype == torch.float32 and pg.grad.dtype == torch.float16
    o = c_oracle.lncc(p.float().cpu().numpy(), t.float().cpu().numpy(), 7)
    assert abs(loss.item() - o["loss"]) < LOSS_TOL
    rel, cos = _rel(pg.grad.float() / scale, torch.from_numpy(o["grad"]))
    assert rel < REL and cos > 0.9999, (rel, cos)


def test_fp16_retain_graph_and_sum_reduction():
    p, t = _pair((1, 2, 20, 24, 32), seed=5)
    pg = p.clone().requires_grad_(True)
    loss = fused_lncc_loss(pg, t, 5, reduction="sum")
    loss.backward(torch.tensor(2.0, device="cuda"), retain_graph=True)
    g1 = pg.grad.clone()
    pg.grad = None
    loss.backward(torch.tensor(2.0, device="cuda"))
    assert torch.equal(g1, pg.grad)
    o = c_oracle.lncc(p.float().cpu().numpy(), t.float().cpu().numpy(), 5, grad_scale=-1.0)
    rel, _ = _rel(g1.float() / 2.0, torch.from_numpy(o["grad"]))
    assert rel < REL, rel
    assert abs(loss.item() - o["count"] * o["loss"]) / (o["count"] * o["loss"]) < 1e-3


def test_fp16_loss_only_and_none_map():
    p, t = _pair((1, 1, 16, 24, 28), seed=9)
    with torch.no_grad():
        loss = fused_lncc_loss(p, t, 7)
    o = c_oracle.lncc(p.float().cpu().numpy(), t.float().cpu().numpy(), 7)
    assert abs(loss.item() - o["loss"]) < LOSS_TOL
    m = fused_lncc_loss(p, t, 7, reduction="none")
    assert m.dtype == torch.float32 and m.shape == p.shape
    assert abs(m.double().mean().item() - o["loss"]) < LOSS_TOL
