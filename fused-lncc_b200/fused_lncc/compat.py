"""The reference extension's entry points, `fused_lncc_cuda.{lncc_forward, lncc_backward,
box3d_sep_forward}` (reference fused_lncc/csrc/lncc3d.cu:346-350), on this library's compat kernels.

Code written against the reference's extension keeps working with

    import fused_lncc.compat as ext          # instead of: import fused_lncc_cuda as ext
    ncc, A, Bc, Cc = ext.lncc_forward(pf, tf, k, 1e-5)
    g = ext.lncc_backward(A, Bc, Cc, pf, tf, k, scale)
    y = ext.box3d_sep_forward(x, k)

with the same argument meaning, output dtypes (fp32 maps, grad in pred's dtype) and RuntimeErrors
for bad arguments. These materialise full fp32 maps. They are for debugging, for the reference's
own checks (ncc map against a torch/MONAI map, the backward against the box-scatter formula), and
for callers of the reference ops `torch.ops.fused_lncc.forward/backward`, which are registered here
with the reference's schemas. The training path, `fused_lncc_loss`, materialises nothing.

Unlike the reference, which launches on the legacy default stream and uses the current device
(lncc3d.cu:118,143), every call runs on the tensor's device and torch's current stream there.
"""
import torch

from . import _lib

__all__ = ["lncc_forward", "lncc_backward", "box3d_sep_forward"]

_DT = {torch.float32: _lib.LNCC_F32, torch.bfloat16: _lib.LNCC_BF16, torch.float16: _lib.LNCC_F16}


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def lncc_forward(P, T, kernel_size, dr):
    """[ncc, A, Bc, Cc]: four fp32 (B, D, H, W) maps of the contiguous 4-D CUDA pair P, T
    (reference lncc_forward, lncc3d.cu:127-161)."""
    _check(P.is_cuda and P.is_contiguous() and P.dim() == 4, "P must be a contiguous 4D CUDA tensor")
    _check(T.is_cuda and T.is_contiguous() and T.shape == P.shape and T.dtype == P.dtype
           and T.device == P.device, "T must match P")
    _check(P.dtype in _DT, f"fused_lncc: float32, bfloat16 or float16 only, got {P.dtype}")
    B, D, H, W = P.shape
    maps = [torch.empty(P.shape, dtype=torch.float32, device=P.device) for _ in range(4)]
    if P.numel() == 0:
        return maps
    with torch.cuda.device(P.device):
        st = _lib.load().lncc_maps_forward(P.data_ptr(), T.data_ptr(), _DT[P.dtype], B, D, H, W,
                                           int(kernel_size), float(dr), *[m.data_ptr() for m in maps],
                                           _stream(P.device))
    _lib.check(st, "fused_lncc lncc_forward")
    return maps


def lncc_backward(A, Bc, Cc, P, T, kernel_size, scale):
    """scale * (box(A) + 2*P*box(Bc) + T*box(Cc)) in P's dtype (reference lncc_backward,
    lncc3d.cu:253-284)."""
    _check(A.is_cuda and A.is_contiguous() and A.dim() == 4 and A.dtype == torch.float32,
           "A must be a contiguous 4D fp32 CUDA tensor")
    _check(Bc.shape == A.shape and Cc.shape == A.shape and Bc.is_contiguous() and Cc.is_contiguous()
           and Bc.dtype == torch.float32 and Cc.dtype == torch.float32
           and Bc.device == A.device and Cc.device == A.device, "B,C must match A")
    _check(P.is_cuda and P.is_contiguous() and P.shape == A.shape and T.is_contiguous()
           and T.shape == A.shape and P.dtype == T.dtype and P.device == A.device
           and T.device == A.device, "P,T must match A shape")
    _check(P.dtype in _DT, f"fused_lncc: float32, bfloat16 or float16 only, got {P.dtype}")
    B, D, H, W = A.shape
    g = torch.empty_like(P)
    if P.numel() == 0:
        return g
    with torch.cuda.device(A.device):
        st = _lib.load().lncc_maps_backward(A.data_ptr(), Bc.data_ptr(), Cc.data_ptr(), P.data_ptr(),
                                            T.data_ptr(), _DT[P.dtype], B, D, H, W, int(kernel_size),
                                            float(scale), g.data_ptr(), _stream(A.device))
    _lib.check(st, "fused_lncc lncc_backward")
    return g


def box3d_sep_forward(x, kernel_size):
    """Zero-padded k^3 box sum of a contiguous 4-D fp32 CUDA tensor (reference box3d_sep_forward,
    lncc3d.cu:329-344)."""
    _check(x.is_cuda and x.is_contiguous() and x.dim() == 4 and x.dtype == torch.float32,
           "x must be a contiguous 4D fp32 CUDA tensor")
    y = torch.empty_like(x)
    if x.numel() == 0:
        return y
    B, D, H, W = x.shape
    with torch.cuda.device(x.device):
        st = _lib.load().lncc_box3d(x.data_ptr(), y.data_ptr(), B, D, H, W, int(kernel_size),
                                    _stream(x.device))
    _lib.check(st, "fused_lncc box3d_sep_forward")
    return y


# The reference's two custom ops, same names and schemas (reference fused_lncc/__init__.py:26-46), so
# code that calls torch.ops.fused_lncc.forward/backward directly, or a compiled graph that holds
# them, runs unchanged.
@torch.library.custom_op("fused_lncc::forward", mutates_args=())
def _forward_op(pf: torch.Tensor, tf: torch.Tensor, kernel_size: int, smooth_dr: float) -> list[torch.Tensor]:
    return lncc_forward(pf, tf, kernel_size, smooth_dr)


@_forward_op.register_fake
def _(pf, tf, kernel_size, smooth_dr):
    return [torch.empty_like(pf, dtype=torch.float32) for _ in range(4)]  # maps are fp32 for bf16 too


@torch.library.custom_op("fused_lncc::backward", mutates_args=())
def _backward_op(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, pf: torch.Tensor, tf: torch.Tensor,
                 kernel_size: int, scale: float) -> torch.Tensor:
    return lncc_backward(A, B, C, pf, tf, kernel_size, scale)


@_backward_op.register_fake
def _(A, B, C, pf, tf, kernel_size, scale):
    return torch.empty_like(pf)
