"""CPU: the Python API raises the reference's exception types before any GPU work
(reference fused_lncc/__init__.py:81-82 asserts; lncc3d.cu:128-129,158 TORCH_CHECKs)."""
import pytest
import torch

from fused_lncc import fused_lncc_loss, lncc_fused


def test_non_5d_asserts():
    x = torch.zeros(1, 8, 8, 8)
    with pytest.raises(AssertionError):
        fused_lncc_loss(x, x, 7)


def test_shape_mismatch_asserts():
    with pytest.raises(AssertionError):
        fused_lncc_loss(torch.zeros(1, 1, 8, 8, 8), torch.zeros(1, 1, 8, 8, 9), 7)


def test_even_kernel_asserts():
    x = torch.zeros(1, 1, 8, 8, 8)
    with pytest.raises(AssertionError):
        fused_lncc_loss(x, x, 4)


def test_cpu_tensor_raises_runtime_error():
    x = torch.zeros(1, 1, 8, 8, 8)
    with pytest.raises(RuntimeError):
        fused_lncc_loss(x, x, 7)


def test_float64_raises_runtime_error():
    x = torch.zeros(1, 1, 8, 8, 8, dtype=torch.float64)
    with pytest.raises(RuntimeError):
        fused_lncc_loss(x, x, 7)


def test_low_level_checks_pair():
    with pytest.raises(RuntimeError):
        lncc_fused(torch.zeros(2, 4, 4, 4), torch.zeros(2, 4, 4, 4), 3)


def test_custom_ops_registered():
    assert hasattr(torch.ops.fused_lncc, "fwd_grad")
    assert hasattr(torch.ops.fused_lncc, "scale_grad_")


def test_fake_impls_give_fp32_loss_and_pred_dtype_grad():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        p = torch.empty(1, 1, 8, 8, 8, dtype=torch.bfloat16)
        loss, g = torch.ops.fused_lncc.fwd_grad(p, p, 7, 1e-5, True, 0)
        assert loss.dtype == torch.float32 and loss.dim() == 0
        assert g.dtype == torch.bfloat16 and g.shape == p.shape


# ---- compat entry points (the reference extension's names and checks, lncc3d.cu:127-161,253-284,329-344)
def test_compat_ops_registered_with_reference_names():
    assert hasattr(torch.ops.fused_lncc, "forward")
    assert hasattr(torch.ops.fused_lncc, "backward")


def test_compat_fakes_fp32_maps_and_pred_dtype_grad():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        p = torch.empty(2, 8, 8, 8, dtype=torch.bfloat16)
        maps = torch.ops.fused_lncc.forward(p, p, 7, 1e-5)
        assert len(maps) == 4 and all(m.dtype == torch.float32 and m.shape == p.shape for m in maps)
        g = torch.ops.fused_lncc.backward(maps[1], maps[2], maps[3], p, p, 7, 1.0)
        assert g.dtype == torch.bfloat16 and g.shape == p.shape


def test_compat_checks_raise_runtime_error():
    from fused_lncc import compat
    x = torch.zeros(2, 4, 4, 4)
    with pytest.raises(RuntimeError, match="contiguous 4D CUDA"):
        compat.lncc_forward(x, x, 3, 1e-5)
    with pytest.raises(RuntimeError, match="contiguous 4D fp32 CUDA"):
        compat.lncc_backward(x, x, x, x, x, 3, 1.0)
    with pytest.raises(RuntimeError, match="contiguous 4D fp32 CUDA"):
        compat.box3d_sep_forward(x, 3)
    with pytest.raises(RuntimeError):
        compat.lncc_forward(torch.zeros(1, 2, 4, 4, 4), torch.zeros(1, 2, 4, 4, 4), 3, 1e-5)


def test_reduction_ops_registered_with_fakes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    assert hasattr(torch.ops.fused_lncc, "loss_map") and hasattr(torch.ops.fused_lncc, "loss_map_backward")
    with FakeTensorMode():
        p = torch.empty(1, 1, 8, 8, 8, dtype=torch.bfloat16)
        m = torch.ops.fused_lncc.loss_map(p, p, 7, 1e-5)
        assert m.dtype == torch.float32 and m.shape == p.shape
        g = torch.ops.fused_lncc.loss_map_backward(m, p, p, 7, 1e-5)
        assert g.dtype == torch.bfloat16 and g.shape == p.shape
        loss, g2 = torch.ops.fused_lncc.fwd_grad(p, p, 7, 1e-5, True, 1)
        assert loss.dim() == 0 and g2.shape == p.shape


def test_window_argument_checks():
    from fused_lncc.window import window_of
    assert window_of(7) == 7 and window_of((7, 7, 7)) == 7 and window_of([3, 5, 7]) == (3, 5, 7)
    assert window_of((1, 1, 1)) == (1, 1, 1)  # not a reference size: the window path takes it
    for bad in [(3, 4, 3), (3, 3), (3, 3, 3, 3), 6]:
        with pytest.raises(AssertionError):
            window_of(bad)


def test_window_ops_registered_with_fakes():
    import torch
    import fused_lncc  # noqa: F401
    for name in ("aniso_loss", "aniso_grad", "aniso_loss_map", "aniso_loss_map_backward", "grad_times"):
        assert hasattr(torch.ops.fused_lncc, name), name
    p = torch.empty(1, 1, 4, 4, 4, dtype=torch.float16, device="meta")
    assert torch.ops.fused_lncc.aniso_loss(p, p, 3, 5, 7, 1e-5, 0).dtype == torch.float32
    assert torch.ops.fused_lncc.aniso_grad(p, p, 3, 5, 7, 1e-5, 0, p.new_empty((), dtype=torch.float32)).dtype == torch.float16
