"""GPU: lncc_fused_forward_noalloc, the entry point for callers that cannot allocate device memory
(a framework that owns the allocator, a pool that must not grow, a loop where allocating is not
allowed). It must give what lncc_fused_forward gives with a caller-allocated workspace, call after
call, although every call reuses one fixed scratch array inside the library.

This file is collected last on purpose, and passes both alone and after the rest of the suite."""
import pytest
import torch

pytestmark = pytest.mark.gpu
FP32_LOSS_TOL = 1e-5
FP32_REL = 1e-3


def _call(lib, fn_name, p, t, k, with_workspace):
    B = p.shape[0] * p.shape[1]
    D, H, W = p.shape[2:]
    g = torch.empty_like(p)
    loss = torch.empty((), dtype=torch.float32, device=p.device)
    csum = torch.zeros(1, dtype=torch.float64, device=p.device)
    M = float(p.numel())
    stream = torch.cuda.current_stream().cuda_stream
    args = [p.data_ptr(), t.data_ptr(), 0, B, D, H, W, k, 1e-5, 0, D, g.data_ptr(), -1.0 / M, None,
            csum.data_ptr(), loss.data_ptr(), M]
    if with_workspace:
        n = lib.lncc_workspace_bytes(B, D, H, W, k, 0, 0, D)
        ws = torch.empty(n, dtype=torch.uint8, device=p.device)
        args += [ws.data_ptr(), n, stream]
    else:
        args += [stream]
    st = getattr(lib, fn_name)(*args)
    torch.cuda.synchronize()
    assert st == 0, st
    return loss.item(), csum.item(), g


# the last shape is large enough for the regular entry point to add its companion launch; this one
# stays a single launch on the caller's stream
@pytest.mark.parametrize("shape,k", [((2, 3, 24, 20, 28), 7), ((1, 2, 40, 64, 128), 5), ((1, 8, 64, 128, 128), 7)])
def test_noalloc_matches_workspace_entry_point_twice(shape, k):
    from fused_lncc import _lib
    lib = _lib.load()
    gen = torch.Generator().manual_seed(11)
    for call in range(2):  # two calls in a row share the library's scratch array
        p = torch.randn(*shape, generator=gen).cuda()
        t = torch.randn(*shape, generator=gen).cuda()
        l0, s0, g0 = _call(lib, "lncc_fused_forward", p, t, k, True)
        l1, s1, g1 = _call(lib, "lncc_fused_forward_noalloc", p, t, k, False)
        assert abs(l1 - l0) < FP32_LOSS_TOL, (call, l0, l1)
        # a call this size may run in two launches through the regular entry point, whose different
        # row tilings round the sum differently: the suite's 1e-6 relative bound for cc sums
        assert abs(s1 - s0) <= 1e-6 * max(1.0, abs(s0)), (call, s0, s1)
        rel = ((g1.double() - g0.double()).norm() / g0.double().norm()).item()
        assert rel < FP32_REL, (call, rel)


def test_noalloc_rejects_oversize_request():
    from fused_lncc import _lib
    lib = _lib.load()
    # 65536 fp64 partials is the fixed limit; a workload that needs more must be refused up front
    B, D, H, W = 300000, 16, 16, 16
    need = lib.lncc_workspace_bytes(B, D, H, W, 7, 0, 0, D)
    assert need > 65536 * 8
    # null inputs: even if the size check were skipped, argument validation stops before any launch
    st = lib.lncc_fused_forward_noalloc(None, None, 0, B, D, H, W, 7, 1e-5, 0, D, None, 1.0, None, None, None,
                                        1.0, None)
    assert st == 8, st  # LNCC_ERR_TOO_LARGE
