"""GPU parity of the `reduction` argument ('sum', 'none'), an addition the reference lists as open
(reference BENCHMARKS.md:177-178). Checked against the fp64 C oracle: 'sum' is count - sum(cc) with
the gradient of -sum(cc); 'none' is the map 1 - ncc, and its gradient for an upstream map G is the
reference's backward formula (lncc3d.cu:166-235) applied to the oracle's adjoint maps weighted by G:
-(box(G*A) + 2p*box(G*B) + t*box(G*C)).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from fused_lncc import fused_lncc_loss
from oracle import c_oracle

pytestmark = pytest.mark.gpu


def _cos_rel(g, ref):
    g = g.detach().float().cpu().flatten().double()
    ref = torch.as_tensor(ref).float().flatten().double()
    cos = F.cosine_similarity(g, ref, dim=0).item()
    rel = ((g - ref).norm() / ref.norm().clamp_min(1e-300)).item()
    return cos, rel


def _pair(shape, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    p = torch.randn(*shape, generator=g)
    t = 0.7 * p + 0.5 * torch.randn(*shape, generator=g)
    return p.to("cuda", dtype), t.to("cuda", dtype)


@pytest.mark.parametrize("k", [3, 7, 9])
def test_sum_matches_oracle(k):
    p, t = _pair((2, 1, 12, 20, 24), 10 + k)
    pg = p.clone().requires_grad_(True)
    loss = fused_lncc_loss(pg, t, k, reduction="sum")
    loss.backward()
    o = c_oracle.lncc(p.cpu().numpy(), t.cpu().numpy(), k, grad_scale=-1.0)
    ref = o["count"] - o["cc_sum"]
    assert loss.dtype == torch.float32 and loss.dim() == 0
    assert abs(loss.item() - ref) < 1e-5 * o["count"], (loss.item(), ref)
    cos, rel = _cos_rel(pg.grad, o["grad"])
    assert cos > 0.9999 and rel < 1e-3, (cos, rel)
    # 'sum' is 'mean' times the voxel count, gradient included
    pm = p.clone().requires_grad_(True)
    lm = fused_lncc_loss(pm, t, k)
    lm.backward()
    assert abs(lm.item() * o["count"] - loss.item()) < 1e-4 * o["count"]
    torch.testing.assert_close(pm.grad * o["count"], pg.grad, rtol=1e-4, atol=1e-6)


def _oracle_map_grad(p, t, G, k):
    o = c_oracle.lncc(p, t, k, grad=False, maps=True)
    box = lambda x: c_oracle.box3d(x.astype(np.float32), k).astype(np.float64)
    g = -(box(G * o["A"]) + 2.0 * p * box(G * o["B"]) + t * box(G * o["C"]))
    return 1.0 - o["ncc"], g


@pytest.mark.parametrize("k,shape", [(3, (1, 2, 9, 11, 13)), (7, (2, 1, 14, 18, 20)), (9, (1, 1, 12, 24, 16))])
def test_none_map_and_weighted_grad_match_oracle(k, shape):
    p, t = _pair(shape, 40 + k)
    G = torch.randn(*shape, generator=torch.Generator().manual_seed(7)).cuda()
    pg = p.clone().requires_grad_(True)
    m = fused_lncc_loss(pg, t, k, reduction="none")
    assert m.dtype == torch.float32 and m.shape == p.shape
    (m * G).sum().backward()
    ref_map, ref_g = _oracle_map_grad(p.cpu().numpy().astype(np.float64), t.cpu().numpy().astype(np.float64),
                                      G.cpu().numpy().astype(np.float64), k)
    assert np.abs(m.detach().cpu().numpy() - ref_map).max() < 1e-4
    cos, rel = _cos_rel(pg.grad, ref_g)
    assert cos > 0.9999 and rel < 1e-3, (cos, rel)
    assert pg.grad.dtype == p.dtype


def test_none_with_unit_upstream_equals_sum():
    p, t = _pair((1, 2, 16, 24, 32), 3)
    a = p.clone().requires_grad_(True)
    fused_lncc_loss(a, t, 7, reduction="none").sum().backward()
    b = p.clone().requires_grad_(True)
    fused_lncc_loss(b, t, 7, reduction="sum").backward()
    cos, rel = _cos_rel(a.grad, b.grad.cpu())
    assert cos > 0.99999 and rel < 1e-4, (cos, rel)


def test_none_bf16_and_mean_of_map():
    p, t = _pair((1, 1, 20, 16, 24), 5, torch.bfloat16)
    m = fused_lncc_loss(p, t, 5, reduction="none")
    with torch.no_grad():
        mean = fused_lncc_loss(p, t, 5)
    assert abs(m.mean().item() - mean.item()) < 1e-4


def test_reduction_compiles_without_graph_break():
    p, t = _pair((1, 1, 10, 12, 16), 9)

    def f(x, y):
        return fused_lncc_loss(x, y, 5, reduction="sum") + fused_lncc_loss(x, y, 5, reduction="none").mean()

    cf = torch.compile(f, fullgraph=True)
    pg = p.clone().requires_grad_(True)
    cf(pg, t).backward()
    pe = p.clone().requires_grad_(True)
    f(pe, t).backward()
    torch.testing.assert_close(pg.grad, pe.grad, rtol=1e-4, atol=1e-7)


def test_bad_reduction_raises():
    p, t = _pair((1, 1, 8, 8, 8), 1)
    with pytest.raises(ValueError):
        fused_lncc_loss(p, t, 3, reduction="max")
