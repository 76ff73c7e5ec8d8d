"""GPU parity: the sm_100a kernels against the CPU oracle and the reference's golden vectors.

Assertions mirror the reference's own suites (tests/test_pytest.py, test_robust.py, test_fixes.py,
test_bf16.py, verify_bwd.py) at the tolerances of the port's contract:
  fp32: |loss - oracle| < 1e-5, grad cosine > 0.9999 and relative L2 error < 1e-3;
  bf16: |loss - oracle(bf16 values)| < 1e-3, grad relative L2 error < 1e-2.
"""
import json
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from fused_lncc import fused_lncc_loss, lncc_fused
from oracle import c_oracle

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FP32_LOSS_TOL = 1e-5
FP32_COS = 0.9999
FP32_REL = 1e-3
BF16_LOSS_TOL = 1e-3
BF16_REL = 1e-2


def fused(p, t, k, dr=1e-5):
    p = p.detach().clone().requires_grad_(True)
    loss = fused_lncc_loss(p, t, k, dr)
    loss.backward()
    torch.cuda.synchronize()
    return loss.item(), p.grad


def oracle(p, t, k, dr=1e-5):
    o = c_oracle.lncc(p.detach().float().cpu().numpy(), t.detach().float().cpu().numpy(), k, dr)
    return o["loss"], torch.from_numpy(o["grad"])


def cos_rel(g, ref):
    g = g.detach().float().cpu().flatten().double()
    ref = ref.detach().float().cpu().flatten().double()
    cos = F.cosine_similarity(g, ref, dim=0).item()
    rel = ((g - ref).norm() / ref.norm().clamp_min(1e-300)).item()
    return cos, rel


def assert_fp32_parity(p, t, k, loss_tol=FP32_LOSS_TOL):
    lf, gf = fused(p, t, k)
    lo, go = oracle(p, t, k)
    assert abs(lf - lo) < loss_tol, (lf, lo)
    cos, rel = cos_rel(gf, go)
    assert cos > FP32_COS and rel < FP32_REL, (cos, rel)
    assert gf.dtype == p.dtype and gf.shape == p.shape


# ---- golden vectors from the reference's own oracle -------------------------------------------------
def test_golden_cases():
    arr = np.load(os.path.join(GOLD, "golden.npz"))
    meta = json.load(open(os.path.join(GOLD, "golden.json")))
    for name, c in meta["cases"].items():
        p = torch.from_numpy(arr[name + "/pred"]).cuda()
        t = torch.from_numpy(arr[name + "/target"]).cuda()
        lf, gf = fused(p, t, c["k"])
        assert abs(lf - c["loss_f64"]) < FP32_LOSS_TOL, (name, lf, c["loss_f64"])
        cos, rel = cos_rel(gf, torch.from_numpy(arr[name + "/grad"]))
        assert cos > FP32_COS and rel < FP32_REL, (name, cos, rel)


def test_golden_config1():
    from fused_lncc import synth
    arr = np.load(os.path.join(GOLD, "golden.npz"))
    c1 = json.load(open(os.path.join(GOLD, "golden.json")))["config1"]
    pred, target = synth.blurred_pair((1, 1, 64, 64, 64), device="cpu")
    assert synth.sha256_of(pred) == c1["sha256_pred"]
    lf, gf = fused(pred.cuda(), target.cuda(), 7)
    assert abs(lf - c1["loss_f64"]) < FP32_LOSS_TOL
    flat = gf.cpu().flatten().double()
    idx = torch.from_numpy(arr["config1/sample_idx"])
    ref = torch.from_numpy(arr["config1/sample_grad"])
    rel = ((flat[idx] - ref).norm() / ref.norm()).item()
    assert rel < FP32_REL
    assert abs(flat.norm().item() / c1["grad_l2"] - 1) < FP32_REL


# ---- reference tests/test_pytest.py --------------------------------------------------------------
@pytest.mark.parametrize("k", [3, 5, 7, 9])
def test_forward_backward_matches_oracle(k):
    torch.manual_seed(0)
    p = torch.randn(2, 4, 32, 32, 32, device="cuda")
    t = torch.randn_like(p)
    assert_fp32_parity(p, t, k)


def test_bf16_runs():
    p = torch.randn(1, 2, 16, 16, 16, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    t = torch.randn_like(p)
    loss = fused_lncc_loss(p, t, 7)
    loss.backward()
    assert loss.dtype == torch.float32
    assert p.grad.dtype == torch.bfloat16 and torch.isfinite(p.grad).all()


def test_degenerate_zero_in_range():
    p = torch.zeros(1, 1, 16, 16, 16, device="cuda")
    loss = fused_lncc_loss(p, p, 7)
    assert torch.isfinite(loss) and 0.0 <= loss.item() <= 1.001


def test_unsupported_dtype_and_kernel_raise():
    p = torch.randn(1, 1, 16, 16, 16, device="cuda", dtype=torch.float64)
    with pytest.raises(RuntimeError):
        fused_lncc_loss(p, p, 7)
    q = torch.randn(1, 1, 16, 16, 16, device="cuda")
    with pytest.raises(RuntimeError):
        fused_lncc_loss(q, q, 11)
    with pytest.raises(RuntimeError):
        fused_lncc_loss(q, q.bfloat16(), 7)


# ---- reference tests/test_robust.py ---------------------------------------------------------------
@pytest.mark.parametrize("k", [3, 5, 7, 9])
def test_regression_28cube(k):
    torch.manual_seed(0)
    p = torch.randn(2, 4, 28, 28, 28, device="cuda")
    t = torch.randn(2, 4, 28, 28, 28, device="cuda")
    assert_fp32_parity(p, t, k)


@pytest.mark.parametrize("name,p,t,exact", [
    ("zeros", torch.zeros(2, 2, 32, 32, 32), torch.zeros(2, 2, 32, 32, 32), True),
    ("const5", torch.full((2, 2, 32, 32, 32), 5.0), torch.full((2, 2, 32, 32, 32), 5.0), True),
    ("const1e4", torch.full((1, 1, 32, 32, 32), 1e4), torch.full((1, 1, 32, 32, 32), 1e4), False),
    ("near_const", torch.full((1, 2, 24, 24, 24), 3.0) + 1e-3 * torch.randn(1, 2, 24, 24, 24,
                                                                             generator=torch.Generator().manual_seed(5)),
     torch.full((1, 2, 24, 24, 24), 3.0), False),
])
def test_degenerate_inputs(name, p, t, exact):
    """reference tests/test_robust.py:23-34: finite, in [0, 1.0001], finite grad. For small-integer
    constants the window sums are exact in fp32, so the loss must also equal the fp64 oracle (and
    an all-zero input must give an all-zero gradient). The gradient of a constant input is a
    difference of nearly equal terms of size ~25*m*(n-m) (border windows have cc = 1 - O(dr)), which
    no fp32 kernel, the reference's included, resolves; for 1e4 constants and near-constant windows
    even the loss is below fp32 resolution. There only the reference's own assertions apply."""
    p, t = p.cuda(), t.cuda()
    lf, gf = fused(p, t, 7)
    assert np.isfinite(lf) and 0.0 <= lf <= 1.0001, (name, lf)
    assert torch.isfinite(gf).all(), name
    if exact:
        lo, go = oracle(p, t, 7)
        assert abs(lf - lo) < FP32_LOSS_TOL, (name, lf, lo)
        if go.abs().max() == 0:
            assert gf.abs().max().item() == 0.0, name


@pytest.mark.parametrize("shape", [(1, 1, 2, 2, 2), (1, 1, 2, 40, 40), (1, 3, 7, 9, 11), (3, 5, 13, 17, 19),
                                   (1, 1, 128, 1, 1), (1, 1, 1, 1, 1), (2, 1, 1, 33, 65), (1, 1, 9, 1, 70)])
@pytest.mark.parametrize("k", [3, 7, 9])
def test_shape_edge_cases(shape, k):
    """reference tests/test_robust.py:36-43 compares the loss only; the gradient is checked too,
    except for a 1-voxel volume, where every window holds the same single voxel and the gradient is
    a difference of two nearly equal terms (relative error ~ var/dr * eps in any fp32 kernel)."""
    g = torch.Generator().manual_seed(hash((shape, k)) % (2 ** 31))
    p = torch.randn(*shape, generator=g).cuda()
    t = torch.randn(*shape, generator=g).cuda()
    if shape[2] * shape[3] * shape[4] == 1:
        lf, gf = fused(p, t, k)
        lo, _ = oracle(p, t, k)
        assert abs(lf - lo) < FP32_LOSS_TOL and torch.isfinite(gf).all()
        return
    assert_fp32_parity(p, t, k)


def test_large_shape_runs():
    p = torch.randn(2, 32, 128, 128, 128, device="cuda", requires_grad=True)
    t = torch.randn_like(p)
    fused_lncc_loss(p, t, 7).backward()
    assert torch.isfinite(p.grad).all()


# ---- reference tests/test_fixes.py ----------------------------------------------------------------
def test_many_volumes_deep():
    p = torch.randn(2080, 1, 128, 8, 8, device="cuda", requires_grad=True)
    t = torch.randn_like(p)
    loss = fused_lncc_loss(p, t, 7)
    loss.backward()
    assert torch.isfinite(loss) and torch.isfinite(p.grad).all()
    # spot-check parity on a few of the volumes
    sel = [0, 1037, 2079]
    o = c_oracle.lncc(p.detach()[sel].cpu().numpy(), t[sel].cpu().numpy(), 7, grad_scale=-1.0 / p.numel())
    cos, rel = cos_rel(p.grad[sel], torch.from_numpy(o["grad"]))
    assert cos > FP32_COS and rel < FP32_REL


@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_nonfinite_input_gives_nonfinite_loss(bad):
    t = torch.randn(1, 1, 16, 16, 16, device="cuda")
    p = torch.randn(1, 1, 16, 16, 16, device="cuda")
    p[0, 0, 8, 8, 8] = bad
    assert not torch.isfinite(fused_lncc_loss(p, t, 7))


@pytest.mark.parametrize("k", [3, 5, 7, 9])
def test_regression_40cube(k):
    torch.manual_seed(1)
    p = torch.randn(2, 8, 40, 40, 40, device="cuda")
    t = torch.randn_like(p)
    assert_fp32_parity(p, t, k)


# ---- reference tests/test_bf16.py -----------------------------------------------------------------
@pytest.mark.parametrize("k", [3, 7, 9])
def test_bf16_matches_fp32_of_bf16_values(k):
    torch.manual_seed(0)
    pb = torch.randn(2, 4, 40, 40, 40, device="cuda", dtype=torch.bfloat16)
    tb = torch.randn(2, 4, 40, 40, 40, device="cuda", dtype=torch.bfloat16)
    lb, gb = fused(pb, tb, k)
    lo, go = oracle(pb, tb, k)
    assert abs(lb - lo) < BF16_LOSS_TOL
    _, rel = cos_rel(gb, go)
    assert gb.dtype == torch.bfloat16 and torch.isfinite(gb).all() and rel < BF16_REL


# ---- autograd glue ---------------------------------------------------------------------------------
def test_grad_out_scaling_and_retain_graph():
    torch.manual_seed(2)
    p = torch.randn(1, 2, 20, 20, 20, device="cuda", requires_grad=True)
    t = torch.randn_like(p)
    loss = fused_lncc_loss(p, t, 5)
    (3.0 * loss).backward(retain_graph=True)
    g1 = p.grad.clone()
    p.grad = None
    loss.backward()                       # second backward recomputes
    g2 = p.grad.clone()
    torch.testing.assert_close(g1, 3.0 * g2, rtol=1e-5, atol=1e-12)
    lo, go = oracle(p, t, 5)
    cos, rel = cos_rel(g2, go)
    assert cos > FP32_COS and rel < FP32_REL


def test_no_grad_path_loss_only():
    torch.manual_seed(3)
    p = torch.randn(2, 1, 24, 24, 24, device="cuda")
    t = torch.randn_like(p)
    with torch.no_grad():
        l0 = fused_lncc_loss(p, t, 7).item()
    l1, _ = fused(p, t, 7)
    assert l0 == l1


def test_deterministic():
    torch.manual_seed(4)
    p = torch.randn(2, 3, 33, 35, 37, device="cuda")
    t = torch.randn_like(p)
    l1, g1 = fused(p, t, 7)
    l2, g2 = fused(p, t, 7)
    assert l1 == l2 and torch.equal(g1, g2)


def test_plane_range_matches_whole_volume():
    torch.manual_seed(5)
    p = torch.randn(2, 1, 40, 19, 23, device="cuda")
    t = torch.randn_like(p)
    _, g_full = lncc_fused(p, t, 7, grad_scale=1.0)
    s_full = torch.zeros(1, dtype=torch.float64, device="cuda")
    s_part = torch.zeros(1, dtype=torch.float64, device="cuda")
    lncc_fused(p, t, 7, grad=False, cc_sum_out=s_full)
    parts = 0.0
    for z0, z1 in [(0, 13), (13, 29), (29, 40)]:
        _, g = lncc_fused(p, t, 7, grad_scale=1.0, z_range=(z0, z1), cc_sum_out=s_part)
        parts += s_part.item()
        torch.testing.assert_close(g, g_full[:, :, z0:z1], rtol=1e-4, atol=1e-5)
    assert abs(parts - s_full.item()) < 1e-6 * max(1.0, abs(s_full.item()))


# ---- every kernel: the warp-specialised cluster kernel (default) and the general sweep -----------------
@pytest.fixture(params=["sweep", "ws"])
def kernel(request):
    from fused_lncc import _lib
    _lib.select_kernel({"sweep": _lib.KERNEL_SWEEP, "ws": _lib.KERNEL_WS}[request.param])
    yield request.param
    _lib.select_kernel(_lib.KERNEL_AUTO)


@pytest.mark.parametrize("shape,k", [((2, 3, 20, 32, 64), 7), ((1, 2, 40, 48, 128), 9), ((2, 1, 9, 16, 8), 3),
                                     ((1, 1, 33, 130, 16), 5), ((3, 1, 70, 17, 20), 7), ((1, 1, 6, 256, 16), 3)])
def test_both_kernels_match_oracle(kernel, shape, k):
    g = torch.Generator().manual_seed(sum(shape) * 31 + k)
    p = torch.randn(*shape, generator=g).cuda()
    t = torch.randn(*shape, generator=g).cuda()
    assert_fp32_parity(p, t, k)


@pytest.mark.parametrize("k", [3, 5, 7, 9])
def test_ws_equals_sweep_blurred(k):
    from fused_lncc import _lib, synth
    pred, target = synth.blurred_pair((2, 2, 48, 64, 128), device="cuda")
    outs = []
    for which in (_lib.KERNEL_SWEEP, _lib.KERNEL_WS):
        _lib.select_kernel(which)
        try:
            outs.append(fused(pred, target, k))
        finally:
            _lib.select_kernel(_lib.KERNEL_AUTO)
    (l1, g1) = outs[0]
    for l2, g2 in outs[1:]:
        assert abs(l1 - l2) < 1e-6
        cos, rel = cos_rel(g2, g1)
        assert cos > 0.999999 and rel < 1e-4, (cos, rel)


# tiled planes (W > 128 or H > 128: overlapping spans) and odd sizes through the warp-specialised kernel
# (W % 8 == 0 takes 8-column global accesses, W % 8 == 4 the 4-column ones)
@pytest.mark.parametrize("shape,k", [((1, 1, 20, 40, 224), 9), ((1, 1, 24, 200, 200), 7), ((1, 1, 33, 130, 16), 5),
                                     ((1, 1, 6, 256, 16), 3), ((1, 1, 3, 2, 4), 7), ((2, 1, 17, 260, 12), 3),
                                     ((1, 2, 24, 40, 132), 7), ((1, 1, 30, 48, 252), 9),
                                     # 129 - 256 rows: one tile in a cluster of up to 16 CTAs
                                     ((1, 1, 20, 256, 136), 9), ((1, 2, 12, 250, 64), 7), ((1, 1, 9, 144, 32), 5)])
def test_ws_tiled_matches_sweep(shape, k):
    from fused_lncc import _lib
    g = torch.Generator().manual_seed(sum(shape) * 7 + k)
    p = torch.randn(*shape, generator=g).cuda()
    t = torch.randn(*shape, generator=g).cuda()
    outs = []
    for which in (_lib.KERNEL_SWEEP, _lib.KERNEL_WS):
        _lib.select_kernel(which)
        try:
            s = torch.zeros((), dtype=torch.float64, device="cuda")
            _, gr = lncc_fused(p, t, k, grad_scale=1.0, cc_sum_out=s)
            torch.cuda.synchronize()
            outs.append((s.item(), gr.float()))
        finally:
            _lib.select_kernel(_lib.KERNEL_AUTO)
    (s1, g1), (s2, g2) = outs
    assert abs(s1 - s2) < 1e-6 * max(1.0, abs(s1)) + 1e-9 * p.numel(), (s1, s2)
    cos, rel = cos_rel(g2, g1)
    assert cos > 0.999999 and rel < 1e-5, (cos, rel)


def test_ws_repeat_bitwise():
    """Many launches of the mbarrier-paced kernel give bitwise identical loss and gradient."""
    from fused_lncc import _lib, synth
    pred, target = synth.blurred_pair((2, 2, 48, 128, 128), device="cuda")
    _lib.select_kernel(_lib.KERNEL_WS)
    try:
        s0 = torch.zeros((), dtype=torch.float64, device="cuda")
        _, g0 = lncc_fused(pred, target, 7, cc_sum_out=s0)
        s = torch.zeros_like(s0)
        g = torch.empty_like(g0)
        for _ in range(50):
            lncc_fused(pred, target, 7, cc_sum_out=s, out=g)
        torch.cuda.synchronize()
        assert s.item() == s0.item() and torch.equal(g, g0)
    finally:
        _lib.select_kernel(_lib.KERNEL_AUTO)


# Companion launch: in a call with enough volumes the last ones (too few: the last planes of each) run in
# clusters of 2 CTAs on the SMs that the main clusters leave idle, concurrently on a second stream. The
# result must not depend on it.
@pytest.mark.parametrize("shape,k,dtype", [((1, 8, 64, 128, 128), 7, torch.float32),
                                           ((3, 3, 64, 128, 128), 5, torch.float32),
                                           ((2, 8, 48, 128, 136), 9, torch.bfloat16),
                                           # too few volumes for a share of whole ones (one
                                           # volume, or four): the companion takes the last planes
                                           ((1, 1, 512, 128, 128), 5, torch.float32),
                                           ((1, 4, 128, 128, 128), 7, torch.float32),
                                           # 256 rows: one cluster of 16 CTAs, bf16
                                           ((1, 2, 128, 256, 128), 7, torch.bfloat16),
                                           ((1, 1, 160, 256, 256), 7, torch.float32)])
def test_ws_companion_matches_single_launch(shape, k, dtype):
    from fused_lncc import _lib, synth
    pred, target = synth.blurred_pair(shape, device="cuda", dtype=dtype)
    lib = _lib.load()
    B, (D, H, W) = shape[0] * shape[1], shape[2:]
    dt = 0 if dtype == torch.float32 else 1
    outs = []
    for on in (True, False):
        prev = _lib.set_companion(on)
        try:
            assert lib.lncc_launch_count(B, D, H, W, k, dt, 0, D, 1) == (2 if on else 1)
            s = torch.zeros((), dtype=torch.float64, device="cuda")
            _, g = lncc_fused(pred, target, k, grad_scale=1.0, cc_sum_out=s)
            torch.cuda.synchronize()
            outs.append((s.item(), g.float()))
        finally:
            _lib.set_companion(prev)
    (s1, g1), (s2, g2) = outs
    # the companion ran: it computes the last volume on its own row tiling, so that volume's gradient
    # differs in the last bits (the kernel is deterministic: one plan gives identical bits)
    assert not torch.equal(g1.reshape(-1, *shape[2:])[-1], g2.reshape(-1, *shape[2:])[-1])
    assert abs(s1 - s2) < 1e-6 * max(1.0, abs(s1)), (s1, s2)
    cos, rel = cos_rel(g1, g2)
    assert cos > 0.99999 and rel < (1e-5 if dtype == torch.float32 else 5e-3), (cos, rel)


@pytest.mark.parametrize("shape,k", [((1, 8, 64, 128, 128), 7), ((1, 1, 512, 128, 128), 5)])
def test_ws_companion_loss_only(shape, k):
    """Loss without gradient (the D group then only boxes its W-box share): the same sum with and
    without the companion launch, and the companion runs for these shapes (volume split, plane split)."""
    from fused_lncc import _lib, synth
    pred, target = synth.blurred_pair(shape, device="cuda")
    lib = _lib.load()
    B, (D, H, W) = shape[0] * shape[1], shape[2:]
    sums = []
    for on in (True, False):
        prev = _lib.set_companion(on)
        try:
            assert lib.lncc_launch_count(B, D, H, W, k, 0, 0, D, 0) == (2 if on else 1)
            s = torch.zeros((), dtype=torch.float64, device="cuda")
            lncc_fused(pred, target, k, grad=False, cc_sum_out=s)
            torch.cuda.synchronize()
            sums.append(s.item())
        finally:
            _lib.set_companion(prev)
    assert abs(sums[0] - sums[1]) < 1e-6 * max(1.0, abs(sums[1])), sums


def test_ws_companion_under_graph_capture():
    """The fork to the companion's stream and the join are captured like any stream work: a replay
    gives the eager result bit for bit (the stream and events were made by the eager call)."""
    from fused_lncc import synth
    pred, target = synth.blurred_pair((1, 8, 64, 128, 128), device="cuda")
    s_e = torch.zeros((), dtype=torch.float64, device="cuda")
    _, g_e = lncc_fused(pred, target, 7, cc_sum_out=s_e)
    s = torch.zeros_like(s_e)
    g = torch.empty_like(g_e)
    lncc_fused(pred, target, 7, cc_sum_out=s, out=g)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        lncc_fused(pred, target, 7, cc_sum_out=s, out=g)
    s.zero_()
    g.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert s.item() == s_e.item() and torch.equal(g, g_e)
    del graph


def test_ws_companion_two_host_threads():
    """Two host threads, each on a stream of its own, call the companion path concurrently and each
    captures and replays a graph of it: the library's second stream and events are per (thread,
    device), so neither thread's fork or join orders the other's work, and every result equals the
    single-threaded one bit for bit."""
    import threading
    from fused_lncc import synth
    shapes = [(1, 8, 64, 128, 128), (1, 1, 512, 128, 128)]
    inputs = [synth.blurred_pair(sh, device="cuda") for sh in shapes]
    ref = []
    for p, t in inputs:
        s = torch.zeros((), dtype=torch.float64, device="cuda")
        _, g = lncc_fused(p, t, 7, cc_sum_out=s)
        ref.append((s.clone(), g.clone()))
    torch.cuda.synchronize()
    errors = []
    capture_lock = threading.Lock()

    def work(idx):
        try:
            p, t = inputs[idx]
            stream = torch.cuda.Stream()
            with torch.cuda.stream(stream):
                s = torch.zeros((), dtype=torch.float64, device="cuda")
                g = torch.empty_like(p)
                for _ in range(6):
                    s.zero_()
                    lncc_fused(p, t, 7, cc_sum_out=s, out=g)
                    if not (torch.equal(s, ref[idx][0]) and torch.equal(g, ref[idx][1])):
                        errors.append((idx, "eager"))
                stream.synchronize()
                graph = torch.cuda.CUDAGraph()
                # torch.cuda.graph() empties the allocator cache and synchronises the device on entry,
                # which CUDA refuses while the other thread's capture is open: one capture at a time
                # (the other thread's eager calls and replays still run alongside)
                with capture_lock:
                    with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
                        lncc_fused(p, t, 7, cc_sum_out=s, out=g)
                for _ in range(4):
                    s.zero_()
                    g.zero_()
                    graph.replay()
                    if not (torch.equal(s, ref[idx][0]) and torch.equal(g, ref[idx][1])):
                        errors.append((idx, "replay"))
                stream.synchronize()
                del graph
        except Exception as e:  # noqa: BLE001 - reported by the main thread
            errors.append((idx, repr(e)))

    threads = [threading.Thread(target=work, args=(i,)) for i in range(2)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=120)
    assert not any(th.is_alive() for th in threads)
    assert not errors, errors


def test_bf16_k9_and_loss_only():
    from fused_lncc import synth
    pred, target = synth.blurred_pair((2, 2, 40, 64, 64), device="cuda", dtype=torch.bfloat16)
    lb, gb = fused(pred, target, 9)
    lo, go = oracle(pred, target, 9)
    assert abs(lb - lo) < BF16_LOSS_TOL
    _, rel = cos_rel(gb, go)
    assert gb.dtype == torch.bfloat16 and rel < BF16_REL
    with torch.no_grad():
        assert abs(fused_lncc_loss(pred, target, 9).item() - lb) < 1e-7


def test_wait_timeout_is_reported_as_status():
    """A bounded wait that runs out is recorded in the workspace and read back as LNCC_ERR_ABORTED;
    the context stays usable, and a normal call afterwards clears the record."""
    from fused_lncc import _lib, synth
    lib = _lib.load()
    ws = torch.zeros(64, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.lncc_wait_timeout_selftest(ws.data_ptr(), ws.numel(), 20000, stream) == 0
    assert lib.lncc_check_abort(ws.data_ptr(), stream) == 9  # LNCC_ERR_ABORTED
    pred, target = synth.blurred_pair((1, 2, 24, 32, 64), device="cuda")
    B, D, H, W = 2, 24, 32, 64
    nb = lib.lncc_workspace_bytes(B, D, H, W, 7, 0, 0, D)
    ws2 = torch.full((nb,), 0xFF, dtype=torch.uint8, device="cuda")  # garbage header
    g = torch.empty_like(pred)
    st = lib.lncc_fused_forward(pred.data_ptr(), target.data_ptr(), 0, B, D, H, W, 7, 1e-5, 0, D, g.data_ptr(),
                                1.0, None, None, None, 1.0, ws2.data_ptr(), nb, stream)
    assert st == 0
    assert lib.lncc_check_abort(ws2.data_ptr(), stream) == 0
    lf, _ = fused(pred, target, 7)
    lo, _ = oracle(pred, target, 7)
    assert abs(lf - lo) < FP32_LOSS_TOL
