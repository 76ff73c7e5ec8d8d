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
        loss, g = torch.ops.fused_lncc.fwd_grad(p, p, 7, 1e-5, True)
        assert loss.dtype == torch.float32 and loss.dim() == 0
        assert g.dtype == torch.bfloat16 and g.shape == p.shape
