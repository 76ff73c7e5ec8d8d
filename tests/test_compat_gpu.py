"""GPU: the materialising compat path (fused_lncc.compat, the reference extension's entry points) and
graph capture / compilation of the fused loss.

Checks mirror the reference's own:
  * ncc map against a box-sum reference map, max |diff| < 1e-3 (reference tests/verify_fwd.py:27-34);
  * the backward from maps equals the box-scatter formula sc*(box(A) + 2p*box(Bc) + t*box(Cc)),
    max |diff| < 1e-8 (reference tests/test_pytest.py:38-51);
  * loss 1 - mean(ncc) and grad at the port's fp32 / bf16 tolerances.
The checker is the fp64 C oracle (maps, box3d and grad), and, where built, the reference's CUDA kernels.
"""
import pytest
import torch
import torch.nn.functional as F

from fused_lncc import compat, fused_lncc_loss
from oracle import c_oracle, ref_cuda

pytestmark = pytest.mark.gpu


def rand_pair(shape, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    p = torch.randn(*shape, generator=g)
    t = torch.randn(*shape, generator=g)
    return p.to("cuda", dtype), t.to("cuda", dtype)


def oracle_maps(p, t, k, dr=1e-5):
    o = c_oracle.lncc(p.float().cpu().numpy(), t.float().cpu().numpy(), k, dr, grad=True, maps=True)
    return {name: torch.from_numpy(o[name]) for name in ("ncc", "A", "B", "C")}, o


def rel(a, b):
    a, b = a.double().flatten().cpu(), b.double().flatten().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-300)).item()


@pytest.mark.parametrize("k", [3, 5, 7, 9])
@pytest.mark.parametrize("shape", [(8, 24, 24, 24), (8, 32, 40, 48), (3, 13, 11, 9)])
def test_maps_match_oracle(k, shape):
    p, t = rand_pair(shape, seed=k)
    ncc, A, Bc, Cc = compat.lncc_forward(p, t, k, 1e-5)
    assert all(m.dtype == torch.float32 and m.shape == p.shape for m in (ncc, A, Bc, Cc))
    om, _ = oracle_maps(p, t, k)
    assert (ncc.cpu() - om["ncc"]).abs().max().item() < 1e-3
    assert rel(ncc, om["ncc"]) < 1e-4
    for got, name in ((A, "A"), (Bc, "B"), (Cc, "C")):
        assert rel(got, om[name]) < 1e-3, name


def test_maps_bf16_match_oracle_on_bf16_values():
    p, t = rand_pair((4, 20, 24, 28), seed=3, dtype=torch.bfloat16)
    ncc, A, Bc, Cc = compat.lncc_forward(p, t, 7, 1e-5)
    assert ncc.dtype == torch.float32
    om, _ = oracle_maps(p, t, 7)
    assert (ncc.cpu() - om["ncc"]).abs().max().item() < 1e-3
    assert rel(Cc, om["C"]) < 1e-2


@pytest.mark.parametrize("k", [3, 5, 7, 9])
def test_backward_from_maps_matches_oracle_grad(k):
    p, t = rand_pair((6, 24, 20, 28), seed=10 + k)
    ncc, A, Bc, Cc = compat.lncc_forward(p, t, k, 1e-5)
    sc = -1.0 / ncc.numel()
    g = compat.lncc_backward(A, Bc, Cc, p, t, k, sc)
    _, o = oracle_maps(p, t, k)
    gr = torch.from_numpy(o["grad"])
    assert F.cosine_similarity(g.double().flatten().cpu(), gr.double().flatten(), dim=0).item() > 0.9999
    assert rel(g, gr) < 1e-3


@pytest.mark.parametrize("k", [3, 5, 7, 9])
def test_fused_backward_matches_scatter(k):
    """Reference tests/test_pytest.py:38-51 on the compat entry points."""
    p, t = rand_pair((6, 24, 20, 28), seed=0)
    ncc, A, Bc, Cc = compat.lncc_forward(p, t, k, 1e-5)
    sc = -1.0 / ncc.numel()
    box = lambda x: compat.box3d_sep_forward(x.contiguous(), k)
    ref = sc * (box(A) + 2.0 * p * box(Bc) + t * box(Cc))
    got = compat.lncc_backward(A, Bc, Cc, p, t, k, sc)
    assert (ref - got).abs().max().item() < 1e-8


@pytest.mark.parametrize("k", [3, 5, 7, 9])
@pytest.mark.parametrize("shape", [(2, 33, 17, 45), (1, 1, 1, 1), (3, 2, 5, 3), (1, 70, 9, 130)])
def test_box3d_matches_oracle(k, shape):
    g = torch.Generator().manual_seed(7)
    x = torch.randn(*shape, generator=g)
    y = compat.box3d_sep_forward(x.cuda(), k).cpu()
    yo = torch.from_numpy(c_oracle.box3d(x.numpy(), k))
    assert (y - yo).abs().max().item() <= 1e-5 * max(1.0, yo.abs().max().item())


@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (2, 1, 1, 7), (1, 3, 1, 1), (2, 2, 3, 2)])
def test_maps_tiny_volumes(shape):
    p, t = rand_pair(shape, seed=1)
    ncc, A, Bc, Cc = compat.lncc_forward(p, t, 7, 1e-5)
    om, _ = oracle_maps(p, t, 7)
    assert torch.isfinite(ncc).all()
    assert (ncc.cpu() - om["ncc"]).abs().max().item() < 1e-3


def test_nan_propagates_with_zero_adjoints():
    p, t = rand_pair((1, 12, 12, 12), seed=2)
    p[0, 6, 6, 6] = float("nan")
    ncc, A, Bc, Cc = compat.lncc_forward(p, t, 3, 1e-5)
    assert torch.isnan(ncc[0, 6, 6, 6])
    assert A[0, 6, 6, 6] == 0 and Bc[0, 6, 6, 6] == 0 and Cc[0, 6, 6, 6] == 0
    assert torch.isfinite(ncc[0, 0, 0, 0])


def test_reference_ops_reproduce_reference_glue():
    """torch.ops.fused_lncc.forward/backward driven as the reference's _FusedLNCC drives them
    (fused_lncc/__init__.py:50-74) give the fused loss and gradient."""
    p, t = rand_pair((2, 3, 20, 24, 28), seed=5)
    pf, tf = p.reshape(6, 20, 24, 28), t.reshape(6, 20, 24, 28)
    ncc, A, Bc, Cc = torch.ops.fused_lncc.forward(pf, tf, 7, 1e-5)
    loss_ref = 1.0 - ncc.mean()
    g_ref = torch.ops.fused_lncc.backward(A, Bc, Cc, pf, tf, 7, 1.0) * (-1.0 / ncc.numel())
    pr = p.clone().requires_grad_(True)
    loss = fused_lncc_loss(pr, t, 7)
    loss.backward()
    assert abs(loss.item() - loss_ref.item()) < 1e-5
    assert F.cosine_similarity(pr.grad.flatten(), g_ref.flatten(), dim=0).item() > 0.9999
    assert rel(pr.grad, g_ref.reshape(p.shape)) < 1e-3


@pytest.mark.skipif(ref_cuda.built_path() is None, reason="oracle/_ref not built")
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_maps_and_box_match_reference_cuda(dtype):
    p, t = rand_pair((4, 40, 48, 56), seed=9, dtype=dtype)
    ours = compat.lncc_forward(p, t, 7, 1e-5)
    theirs = ref_cuda.forward_maps(p.unsqueeze(1), t.unsqueeze(1), 7)  # (N, C=1, D, H, W)
    assert (ours[0] - theirs[0]).abs().max().item() < 1e-3
    for a, b in zip(ours[1:], theirs[1:]):
        assert rel(a, b) < 1e-3
    sc = -1.0 / p.numel()
    g_ours = compat.lncc_backward(*theirs[1:], p, t, 7, sc)
    g_theirs = ref_cuda.load().lncc_backward(*theirs[1:], p, t, 7, sc)
    assert rel(g_ours, g_theirs) < (1e-2 if dtype == torch.bfloat16 else 1e-5)
    x = theirs[1]
    assert rel(compat.box3d_sep_forward(x, 7), ref_cuda.box3d(x, 7)) < 1e-5


# ---- compilation and graph capture of the fused loss ------------------------------------------------
def test_torch_compile_fullgraph_no_graph_break():
    """The custom ops trace with no graph break (the reference's reason for its ops,
    fused_lncc/__init__.py:22-24). aot_eager: traced by Dynamo/AOTAutograd, run eagerly."""
    p, t = rand_pair((1, 2, 24, 24, 24), seed=4)
    fn = torch.compile(lambda a, b: fused_lncc_loss(a, b, 7), fullgraph=True, backend="aot_eager")
    pc = p.clone().requires_grad_(True)
    lc = fn(pc, t)
    lc.backward()
    pe = p.clone().requires_grad_(True)
    le = fused_lncc_loss(pe, t, 7)
    le.backward()
    assert lc.dtype == torch.float32
    assert abs(lc.item() - le.item()) < 1e-7
    assert torch.equal(pc.grad, pe.grad)


def test_cuda_graph_capture_and_replay():
    """fwd + bwd captured into one CUDA graph and replayed on new inputs gives the eager results."""
    p, t = rand_pair((2, 4, 32, 32, 32), seed=6)
    sp = p.clone().requires_grad_(True)
    st = t.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):  # warm-up outside capture (kernel attributes, allocator pools)
            sp.grad = None
            fused_lncc_loss(sp, st, 7).backward()
    torch.cuda.current_stream().wait_stream(s)
    sp.grad = None
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        loss_g = fused_lncc_loss(sp, st, 7)
        loss_g.backward()
    for seed in (11, 12):
        p2, t2 = rand_pair((2, 4, 32, 32, 32), seed=seed)
        with torch.no_grad():
            sp.copy_(p2)
            st.copy_(t2)
        g.replay()
        torch.cuda.synchronize()
        pe = p2.clone().requires_grad_(True)
        le = fused_lncc_loss(pe, t2, 7)
        le.backward()
        assert abs(loss_g.item() - le.item()) < 1e-7
        assert torch.equal(sp.grad, pe.grad)
    del g
