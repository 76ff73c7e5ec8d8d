"""Non-cubic windows kd x kh x kw for fused_lncc_loss (kernel_size=(kd, kh, kw)).

The reference supports cubic windows only and lists non-cubic ones as open (reference
BENCHMARKS.md:177-178). Here each side is odd in 1 .. 9 and n = kd*kh*kw replaces k^3 in the math;
a cubic tuple takes the fused kernel. The other windows run the materialising C-ABI path
(lncc_aniso_forward, lncc_aniso_loss_map_forward/_backward in include/lncc.h): one pass for the adjoint
maps and the per-block cc sums, a fixed-order reduction for the loss, one pass that boxes the maps into
the gradient. The forward computes the loss only; the backward computes the gradient with grad_out
applied in fp32 before the rounding to pred's dtype.
"""
import torch

from . import _lib

REDUCE_MEAN, REDUCE_SUM = 0, 1


def window_of(kernel_size):
    """An odd int k (cubic) or a (kd, kh, kw) tuple of odd sides -> int k or a 3-tuple.

    AssertionError for an even side or a tuple of the wrong length, as the reference asserts an odd
    kernel_size (reference fused_lncc/__init__.py:81-82)."""
    if isinstance(kernel_size, (tuple, list, torch.Size)):
        assert len(kernel_size) == 3, "kernel_size: an odd int or a (kd, kh, kw) tuple"
        kd, kh, kw = (int(v) for v in kernel_size)
        assert kd % 2 == 1 and kh % 2 == 1 and kw % 2 == 1, "kernel_size must be odd"
        if kd == kh == kw and kd in (3, 5, 7, 9):
            return kd
        return (kd, kh, kw)
    assert kernel_size % 2 == 1, "kernel_size must be odd"
    return int(kernel_size)


def _flat(pred):
    *lead, D, H, W = pred.shape
    B = 1
    for s in lead:
        B *= int(s)
    return B, D, H, W


def _dtype(pred):
    from . import _DTYPES
    return _DTYPES[pred.dtype]


def aniso_fused(pred, target, window, smooth_dr=1e-5, *, grad=False, grad_scale=None, grad_scale_dev=None,
                cc_sum_out=None, loss_count=None):
    """One call of lncc_aniso_forward: returns (loss 0-dim fp32, grad or None).

    grad_scale defaults to -1/M (the gradient of 1 - mean(cc)); grad_scale_dev (a device fp32 scalar)
    multiplies it on the device."""
    from . import _check_pair
    _check_pair(pred, target)
    kd, kh, kw = window
    B, D, H, W = _flat(pred)
    nvox = B * D * H * W
    lib = _lib.load()
    dev = pred.device
    with torch.cuda.device(dev):
        nb = lib.lncc_aniso_scratch_bytes(B, D, H, W, 1 if grad else 0)
        scratch = torch.empty(max(nb, 8), dtype=torch.uint8, device=dev)
        g = torch.empty_like(pred) if grad else None
        loss = torch.empty((), dtype=torch.float32, device=dev)
        st = lib.lncc_aniso_forward(
            pred.data_ptr(), target.data_ptr(), _dtype(pred), B, D, H, W, kd, kh, kw, float(smooth_dr),
            g.data_ptr() if g is not None else None,
            float(-1.0 / max(nvox, 1) if grad_scale is None else grad_scale),
            grad_scale_dev.data_ptr() if grad_scale_dev is not None else None,
            cc_sum_out.data_ptr() if cc_sum_out is not None else None, loss.data_ptr(),
            float(loss_count if loss_count is not None else max(nvox, 1)), scratch.data_ptr(), max(nb, 8),
            torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, "fused_lncc aniso forward")
    return loss, g


# Ops for torch.compile; in eager mode the autograd functions call the implementations directly,
# without the custom-op dispatcher's overhead.
def _aniso_loss_impl(pred: torch.Tensor, target: torch.Tensor, kd: int, kh: int, kw: int, smooth_dr: float,
                     reduction: int) -> torch.Tensor:
    if reduction == REDUCE_SUM:
        cs = torch.empty((), dtype=torch.float64, device=pred.device)
        aniso_fused(pred, target, (kd, kh, kw), smooth_dr, cc_sum_out=cs)
        return (float(pred.numel()) - cs).to(torch.float32)
    loss, _ = aniso_fused(pred, target, (kd, kh, kw), smooth_dr)
    return loss


_aniso_loss_op = torch.library.custom_op("fused_lncc::aniso_loss", mutates_args=())(_aniso_loss_impl)


@_aniso_loss_op.register_fake
def _(pred, target, kd, kh, kw, smooth_dr, reduction):
    return pred.new_empty((), dtype=torch.float32)


def _aniso_grad_impl(pred: torch.Tensor, target: torch.Tensor, kd: int, kh: int, kw: int, smooth_dr: float,
                     reduction: int, grad_out: torch.Tensor) -> torch.Tensor:
    go = grad_out.detach().to(device=pred.device, dtype=torch.float32).contiguous()
    scale = -1.0 if reduction == REDUCE_SUM else None
    _, g = aniso_fused(pred, target, (kd, kh, kw), smooth_dr, grad=True, grad_scale=scale, grad_scale_dev=go)
    return g


_aniso_grad_op = torch.library.custom_op("fused_lncc::aniso_grad", mutates_args=())(_aniso_grad_impl)


@_aniso_grad_op.register_fake
def _(pred, target, kd, kh, kw, smooth_dr, reduction, grad_out):
    return torch.empty_like(pred)


class FusedLNCCWindow(torch.autograd.Function):
    """1 - mean(cc) (or sum(1 - cc)) for a non-cubic window; gradient for pred only."""

    @staticmethod
    def forward(ctx, pred, target, window, smooth_dr, reduction):
        ctx.save_for_backward(pred, target)
        ctx.window = window
        ctx.dr = smooth_dr
        ctx.reduction = reduction
        fn = torch.ops.fused_lncc.aniso_loss if torch.compiler.is_compiling() else _aniso_loss_impl
        return fn(pred, target, *window, smooth_dr, reduction)

    @staticmethod
    def backward(ctx, grad_out):
        pred, target = ctx.saved_tensors
        fn = torch.ops.fused_lncc.aniso_grad if torch.compiler.is_compiling() else _aniso_grad_impl
        g = fn(pred, target, *ctx.window, ctx.dr, ctx.reduction, grad_out)
        return g, None, None, None, None


@torch.library.custom_op("fused_lncc::aniso_loss_map", mutates_args=())
def _aniso_map_op(pred: torch.Tensor, target: torch.Tensor, kd: int, kh: int, kw: int,
                  smooth_dr: float) -> torch.Tensor:
    from . import loss_map
    return loss_map(pred, target, (kd, kh, kw), smooth_dr)


@_aniso_map_op.register_fake
def _(pred, target, kd, kh, kw, smooth_dr):
    return pred.new_empty(pred.shape, dtype=torch.float32)


@torch.library.custom_op("fused_lncc::aniso_loss_map_backward", mutates_args=())
def _aniso_map_bwd_op(grad_map: torch.Tensor, pred: torch.Tensor, target: torch.Tensor, kd: int, kh: int, kw: int,
                      smooth_dr: float) -> torch.Tensor:
    from . import loss_map_backward
    return loss_map_backward(grad_map, pred, target, (kd, kh, kw), smooth_dr)


@_aniso_map_bwd_op.register_fake
def _(grad_map, pred, target, kd, kh, kw, smooth_dr):
    return torch.empty_like(pred)


class FusedLNCCWindowMap(torch.autograd.Function):
    """reduction='none' for a non-cubic window: the per-voxel map 1 - cc and the gradient of
    sum(G * map) for any upstream map G."""

    @staticmethod
    def forward(ctx, pred, target, window, smooth_dr):
        ctx.save_for_backward(pred, target)
        ctx.window = window
        ctx.dr = smooth_dr
        return torch.ops.fused_lncc.aniso_loss_map(pred, target, *window, smooth_dr)

    @staticmethod
    def backward(ctx, grad_map):
        pred, target = ctx.saved_tensors
        g = torch.ops.fused_lncc.aniso_loss_map_backward(grad_map.contiguous(), pred, target, *ctx.window, ctx.dr)
        return g, None, None, None
