"""GPU: the bounds-checked build (liblncc_sm100_checked.so, LNCC_CHECKED=1) reports no out-of-range
access and keeps parity, on the shapes of the reference's compute-sanitizer drivers
(reference tests/_sanitize2.py:6, tests/_sanitize_bf16.py:5-6) plus tiled, 16-CTA, companion and
odd-W shapes, through both fused kernels, the compat entry points and the per-voxel loss map.
compute-sanitizer is closed on this pool; this build is its stand-in.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import c_oracle

pytestmark = pytest.mark.gpu

ST_OK = 0
SANITIZE_SHAPES = [((3, 5, 13, 17, 11), 7, torch.float32), ((2, 4, 16, 16, 16), 7, torch.float32),
                   ((1, 1, 2, 2, 2), 7, torch.float32), ((3, 5, 13, 17, 11), 7, torch.bfloat16),
                   ((1, 2, 16, 16, 16), 7, torch.bfloat16)]
# warp-specialised kernel corner cases: tiled spans, a cluster of 16, the companion launch, W % 8 == 4
WS_SHAPES = [((1, 1, 20, 40, 224), 9, torch.float32), ((1, 1, 24, 200, 200), 7, torch.float32),
             ((1, 1, 20, 256, 136), 9, torch.float32), ((1, 2, 12, 250, 64), 7, torch.float32),
             ((1, 8, 40, 128, 128), 7, torch.float32), ((2, 1, 17, 260, 12), 3, torch.bfloat16),
             ((1, 1, 3, 2, 4), 5, torch.float32)]


@pytest.fixture(scope="module")
def clib():
    from fused_lncc import _lib
    path = os.path.join(os.path.dirname(_lib.LIB_PATH), "liblncc_sm100_checked.so")
    if not os.path.exists(path):
        import importlib.util
        spec = importlib.util.spec_from_file_location(
            "_b", os.path.join(os.path.dirname(os.path.dirname(_lib.LIB_PATH)), "build.py"))
        b = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(b)
        b.build_library(checked=True)
    lib = ctypes.CDLL(path)
    for name, (res, args) in _lib.SIGNATURES.items():
        f = getattr(lib, name)
        f.restype, f.argtypes = res, args
    assert lib.lncc_checked_build() == 1
    return lib


def _pair(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    p = torch.randn(*shape, generator=g)
    t = torch.randn(*shape, generator=g)
    return p.to("cuda", dtype).contiguous(), t.to("cuda", dtype).contiguous()


def _fused(lib, p, t, k):
    B = int(np.prod(p.shape[:-3]))
    D, H, W = p.shape[-3:]
    dt = 0 if p.dtype == torch.float32 else 1
    nb = lib.lncc_workspace_bytes(B, D, H, W, k, dt, 0, D)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    g = torch.empty_like(p)
    s = torch.zeros((), dtype=torch.float64, device="cuda")
    st = lib.lncc_fused_forward(p.data_ptr(), t.data_ptr(), dt, B, D, H, W, k, 1e-5, 0, D, g.data_ptr(), 1.0, None,
                                s.data_ptr(), None, 1.0, ws.data_ptr(), nb, torch.cuda.current_stream().cuda_stream)
    return st, s.item(), g


def _check_against_oracle(p, t, k, cc_sum, g):
    o = c_oracle.lncc(p.float().cpu().numpy(), t.float().cpu().numpy(), k, grad_scale=1.0)
    n = o["count"]
    tol = 1e-5 if p.dtype == torch.float32 else 1e-3
    assert abs(cc_sum - o["cc_sum"]) < tol * n, (cc_sum, o["cc_sum"])
    ref = torch.from_numpy(o["grad"]).double().flatten()
    gd = g.double().cpu().flatten()
    rel = ((gd - ref).norm() / ref.norm().clamp_min(1e-300)).item()
    assert rel < (1e-3 if p.dtype == torch.float32 else 1e-2), rel


@pytest.mark.parametrize("kernel", [1, 3])  # the general sweep kernel, the warp-specialised kernel
@pytest.mark.parametrize("shape,k,dtype", SANITIZE_SHAPES + WS_SHAPES)
def test_checked_fused_no_violation_and_parity(clib, kernel, shape, k, dtype):
    assert clib.lncc_select_kernel(kernel) == ST_OK
    try:
        p, t = _pair(shape, dtype, sum(shape) + k)
        st, cc, g = _fused(clib, p, t, k)
        assert st == ST_OK, clib.lncc_strerror(st)
        _check_against_oracle(p, t, k, cc, g)
    finally:
        clib.lncc_select_kernel(0)


@pytest.mark.parametrize("shape,k,dtype", SANITIZE_SHAPES[:3] + [((1, 2, 9, 40, 33), 9, torch.bfloat16)])
def test_checked_compat_and_loss_map_no_violation(clib, shape, k, dtype):
    p, t = _pair(shape, dtype, 3 + k)
    B = int(np.prod(shape[:-3]))
    D, H, W = shape[-3:]
    dt = 0 if dtype == torch.float32 else 1
    stream = torch.cuda.current_stream().cuda_stream
    maps = [torch.empty(shape, dtype=torch.float32, device="cuda") for _ in range(4)]
    st = clib.lncc_maps_forward(p.data_ptr(), t.data_ptr(), dt, B, D, H, W, k, 1e-5, *[m.data_ptr() for m in maps], stream)
    assert st == ST_OK, clib.lncc_strerror(st)
    g = torch.empty_like(p)
    st = clib.lncc_maps_backward(maps[1].data_ptr(), maps[2].data_ptr(), maps[3].data_ptr(), p.data_ptr(), t.data_ptr(),
                                 dt, B, D, H, W, k, 1.0, g.data_ptr(), stream)
    assert st == ST_OK, clib.lncc_strerror(st)
    y = torch.empty(shape, dtype=torch.float32, device="cuda")
    st = clib.lncc_box3d(maps[0].data_ptr(), y.data_ptr(), B, D, H, W, k, stream)
    assert st == ST_OK, clib.lncc_strerror(st)
    lm = torch.empty(shape, dtype=torch.float32, device="cuda")
    st = clib.lncc_loss_map_forward(p.data_ptr(), t.data_ptr(), dt, B, D, H, W, k, 1e-5, lm.data_ptr(), stream)
    assert st == ST_OK, clib.lncc_strerror(st)
    nb = clib.lncc_loss_map_scratch_bytes(B, D, H, W)
    scratch = torch.empty(nb // 4, dtype=torch.float32, device="cuda")
    st = clib.lncc_loss_map_backward(torch.ones(shape, device="cuda").data_ptr(), p.data_ptr(), t.data_ptr(), dt,
                                     B, D, H, W, k, 1e-5, g.data_ptr(), scratch.data_ptr(), nb, stream)
    assert st == ST_OK, clib.lncc_strerror(st)
    torch.testing.assert_close(lm, 1.0 - maps[0], rtol=0, atol=1e-6, equal_nan=True)


def test_product_library_is_not_the_checked_build():
    from fused_lncc import _lib
    assert _lib.load().lncc_checked_build() == 0
