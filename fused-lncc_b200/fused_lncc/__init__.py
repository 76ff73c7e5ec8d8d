"""Fused 3-D local (squared) normalized cross-correlation loss for B200 (sm_100a).

Drop-in for the reference package (reference fused_lncc/__init__.py:77-83):

    from fused_lncc import fused_lncc_loss
    loss = fused_lncc_loss(pred, target, kernel_size=7, smooth_dr=1e-5)   # 1 - mean(cc)
    loss.backward()                                                        # grad for pred only

`reduction` ('mean' default, 'sum', 'none') is an addition the reference lists as open
(reference BENCHMARKS.md:177-178): 'sum' gives sum(1 - cc), 'none' the per-voxel map 1 - cc.

Same signature, defaults, assertion errors, RuntimeErrors, fp32 scalar result and pred-dtype
gradient as the reference. Inside, the forward is ONE kernel pass that also produces dL/dpred.
The backward is then one tiny launch that returns immediately when grad_out == 1. The reference
instead materialises four fp32 maps in the forward and box-sums them again in the backward
(reference fused_lncc/__init__.py:50-74).
"""
import contextlib

import torch

from . import _lib

__all__ = ["fused_lncc_loss", "lncc_fused", "loss_map", "FusedLNCC", "FusedLNCCMap", "compat", "window"]

REDUCTIONS = {"mean": 0, "sum": 1}  # the fused kernel's reductions; 'none' has its own path

# fp16 is an addition the reference lists as open (reference BENCHMARKS.md:177-178)
_DTYPES = {torch.float32: _lib.LNCC_F32, torch.bfloat16: _lib.LNCC_BF16, torch.float16: _lib.LNCC_F16}


def _check_pair(pred, target):
    """The TORCH_CHECKs of reference lncc3d.cu:128-129,158 as RuntimeErrors."""
    if not (pred.is_cuda and target.is_cuda):
        raise RuntimeError("fused_lncc: pred and target must be CUDA tensors")
    if pred.device != target.device:
        raise RuntimeError("fused_lncc: pred and target must be on the same device")
    if pred.shape != target.shape or pred.dtype != target.dtype:
        raise RuntimeError("fused_lncc: target must match pred in shape and dtype")
    if pred.dtype not in _DTYPES:
        raise RuntimeError(f"fused_lncc: float32, bfloat16 or float16 only, got {pred.dtype}")
    if not (pred.is_contiguous() and target.is_contiguous()):
        raise RuntimeError("fused_lncc: pred and target must be contiguous")
    if pred.dim() < 3:
        raise RuntimeError("fused_lncc: expect (..., D, H, W) volumes")


# Workspace bytes per call shape, so that a step makes one C call instead of two. The size also
# depends on the process-wide switches (companion launch, kernel choice): a call that finds the cached
# size too small asks the library again once.
_WS_BYTES = {}


def _on_device(dev):
    """torch.cuda.device(dev), or nothing when dev is already current (the common case, and the switch
    costs microseconds that matter for small calls)."""
    return contextlib.nullcontext() if dev.index == torch.cuda.current_device() else torch.cuda.device(dev)


def lncc_fused(pred, target, kernel_size=7, smooth_dr=1e-5, *, grad=True, grad_scale=None,
               loss_count=None, z_range=None, cc_sum_out=None, loss_out=None, grad_scale_dev=None,
               out=None):
    """Run the fused kernel once: returns (loss, grad).

    pred/target: contiguous (..., D, H, W) CUDA tensors, fp32, bf16 or fp16; the leading dims are
    flattened into B volumes (the reference's N*C reshape, fused_lncc/__init__.py:52-55).
    grad: also produce d/dpred, scaled by grad_scale (default -1/M, i.e. of 1 - mean(cc)).
    loss_count: divisor of the loss (default M = number of voxels produced).
    z_range: (z_begin, z_end) output planes of every volume (default the whole volume); planes of
             the array outside the range act as halo. grad then has z_end - z_begin planes.
    cc_sum_out / loss_out: optional preallocated fp64 / fp32 one-element CUDA tensors.
    out: optional preallocated contiguous gradient tensor of the grad's shape and pred's dtype.
    Returns (loss: 0-dim fp32 tensor, grad: tensor or None).
    """
    _check_pair(pred, target)
    *lead, D, H, W = pred.shape
    B = 1
    for s in lead:
        B *= int(s)
    z0, z1 = (0, D) if z_range is None else (int(z_range[0]), int(z_range[1]))
    nout = B * (z1 - z0) * H * W
    lib = _lib.load()
    dt = _DTYPES[pred.dtype]
    dev = pred.device
    with _on_device(dev):
        key = (B, D, H, W, int(kernel_size), dt, z0, z1)
        ws_bytes = _WS_BYTES.get(key)
        if ws_bytes is None:
            ws_bytes = lib.lncc_workspace_bytes(B, D, H, W, int(kernel_size), dt, z0, z1)
            if ws_bytes == 0:
                # invalid size/k/range: let the main call produce the precise status
                ws_bytes = 8
            if len(_WS_BYTES) > 4096:
                _WS_BYTES.clear()
            _WS_BYTES[key] = ws_bytes
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        g = None
        if grad:
            shape = (*lead, z1 - z0, H, W)
            if out is not None:
                if (tuple(out.shape) != shape or out.dtype != pred.dtype or out.device != dev
                        or not out.is_contiguous()):
                    raise RuntimeError(f"fused_lncc: out must be a contiguous {shape} {pred.dtype} tensor")
                g = out
            else:
                g = torch.empty(shape, dtype=pred.dtype, device=dev)
        if loss_out is None:
            loss_out = torch.empty((), dtype=torch.float32, device=dev)
        if grad_scale is None:
            grad_scale = -1.0 / max(nout, 1)
        if loss_count is None:
            loss_count = float(max(nout, 1))
        stream = torch.cuda.current_stream(dev).cuda_stream

        def call():
            return lib.lncc_fused_forward(
                pred.data_ptr(), target.data_ptr(), dt, B, D, H, W, int(kernel_size), float(smooth_dr),
                z0, z1, g.data_ptr() if g is not None else None, float(grad_scale),
                grad_scale_dev.data_ptr() if grad_scale_dev is not None else None,
                cc_sum_out.data_ptr() if cc_sum_out is not None else None, loss_out.data_ptr(),
                float(loss_count), ws.data_ptr(), ws_bytes, stream)
        st = call()
        if st == _lib.LNCC_ERR_WORKSPACE:  # a switch changed the plan since the size was cached
            ws_bytes = max(8, lib.lncc_workspace_bytes(B, D, H, W, int(kernel_size), dt, z0, z1))
            _WS_BYTES[key] = ws_bytes
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            st = call()
    _lib.check(st, "fused_lncc forward")
    return loss_out, g


def scale_grad_(grad, grad_out):
    """In place grad *= grad_out (a 0-dim CUDA tensor); no work when grad_out == 1."""
    lib = _lib.load()
    go = grad_out.detach()
    if go.dtype != torch.float32 or not go.is_contiguous() or go.device != grad.device:
        go = go.to(device=grad.device, dtype=torch.float32).contiguous()
    with _on_device(grad.device):
        st = lib.lncc_scale_grad(grad.data_ptr(), _DTYPES[grad.dtype], grad.numel(), go.data_ptr(),
                                 torch.cuda.current_stream(grad.device).cuda_stream)
    _lib.check(st, "fused_lncc scale_grad")


# torch.library custom ops, so torch.compile traces through without graph breaks (the reference
# registers fused_lncc::forward/backward for the same reason, fused_lncc/__init__.py:22-46). In eager
# mode the autograd glue calls the same Python functions directly: the dispatcher round trip of a
# custom op costs tens of microseconds per call, as much as the kernel of a small call.
def _fwd_grad_impl(pred: torch.Tensor, target: torch.Tensor, kernel_size: int, smooth_dr: float,
                   need_grad: bool, reduction: int) -> tuple[torch.Tensor, torch.Tensor]:
    if reduction == REDUCTIONS["sum"]:
        # sum(1 - cc) = M - sum(cc): the gradient of -sum(cc), the loss from the fp64 cc sum
        cs = torch.empty((), dtype=torch.float64, device=pred.device)
        _, g = lncc_fused(pred, target, kernel_size, smooth_dr, grad=need_grad, grad_scale=-1.0,
                          cc_sum_out=cs)
        loss = (float(pred.numel()) - cs).to(torch.float32)
    else:
        loss, g = lncc_fused(pred, target, kernel_size, smooth_dr, grad=need_grad)
    if g is None:
        g = pred.new_empty((0,))
    return loss, g


_fwd_grad_op = torch.library.custom_op("fused_lncc::fwd_grad", mutates_args=())(_fwd_grad_impl)


@_fwd_grad_op.register_fake
def _(pred, target, kernel_size, smooth_dr, need_grad, reduction):
    loss = pred.new_empty((), dtype=torch.float32)  # the loss is fp32 even for bf16 input
    g = torch.empty_like(pred) if need_grad else pred.new_empty((0,))
    return loss, g


def loss_map(pred, target, kernel_size=7, smooth_dr=1e-5):
    """Per-voxel loss 1 - cc (cc clamped to 1, NaN kept), an fp32 tensor of pred's shape.
    kernel_size: an int k (cubic) or a (kd, kh, kw) tuple (non-cubic window)."""
    _check_pair(pred, target)
    *lead, D, H, W = pred.shape
    B = 1
    for s_ in lead:
        B *= int(s_)
    out = torch.empty(pred.shape, dtype=torch.float32, device=pred.device)
    lib = _lib.load()
    with torch.cuda.device(pred.device):
        stream = torch.cuda.current_stream(pred.device).cuda_stream
        if isinstance(kernel_size, tuple):  # non-cubic window (kd, kh, kw)
            st = lib.lncc_aniso_loss_map_forward(pred.data_ptr(), target.data_ptr(), _DTYPES[pred.dtype], B, D, H,
                                                 W, *kernel_size, float(smooth_dr), out.data_ptr(), stream)
        else:
            st = lib.lncc_loss_map_forward(pred.data_ptr(), target.data_ptr(), _DTYPES[pred.dtype], B, D, H, W,
                                           int(kernel_size), float(smooth_dr), out.data_ptr(), stream)
    _lib.check(st, "fused_lncc loss_map")
    return out


def loss_map_backward(grad_map, pred, target, kernel_size=7, smooth_dr=1e-5):
    """d(sum(grad_map * loss_map(pred, target)))/dpred, in pred's dtype."""
    _check_pair(pred, target)
    if grad_map.shape != pred.shape:
        raise RuntimeError("fused_lncc: grad_map must have pred's shape")
    gm = grad_map.to(device=pred.device, dtype=torch.float32).contiguous()
    *lead, D, H, W = pred.shape
    B = 1
    for s_ in lead:
        B *= int(s_)
    lib = _lib.load()
    g = torch.empty_like(pred)
    with torch.cuda.device(pred.device):
        nb = lib.lncc_loss_map_scratch_bytes(B, D, H, W)
        scratch = torch.empty(max(nb, 4) // 4, dtype=torch.float32, device=pred.device)
        stream = torch.cuda.current_stream(pred.device).cuda_stream
        if isinstance(kernel_size, tuple):  # non-cubic window (kd, kh, kw)
            st = lib.lncc_aniso_loss_map_backward(gm.data_ptr(), pred.data_ptr(), target.data_ptr(),
                                                  _DTYPES[pred.dtype], B, D, H, W, *kernel_size, float(smooth_dr),
                                                  g.data_ptr(), scratch.data_ptr(), nb, stream)
        else:
            st = lib.lncc_loss_map_backward(gm.data_ptr(), pred.data_ptr(), target.data_ptr(), _DTYPES[pred.dtype],
                                            B, D, H, W, int(kernel_size), float(smooth_dr), g.data_ptr(),
                                            scratch.data_ptr(), nb, stream)
    _lib.check(st, "fused_lncc loss_map_backward")
    return g


@torch.library.custom_op("fused_lncc::loss_map", mutates_args=())
def _loss_map_op(pred: torch.Tensor, target: torch.Tensor, kernel_size: int, smooth_dr: float) -> torch.Tensor:
    return loss_map(pred, target, kernel_size, smooth_dr)


@_loss_map_op.register_fake
def _(pred, target, kernel_size, smooth_dr):
    return pred.new_empty(pred.shape, dtype=torch.float32)


@torch.library.custom_op("fused_lncc::loss_map_backward", mutates_args=())
def _loss_map_bwd_op(grad_map: torch.Tensor, pred: torch.Tensor, target: torch.Tensor, kernel_size: int,
                     smooth_dr: float) -> torch.Tensor:
    return loss_map_backward(grad_map, pred, target, kernel_size, smooth_dr)


@_loss_map_bwd_op.register_fake
def _(grad_map, pred, target, kernel_size, smooth_dr):
    return torch.empty_like(pred)


def _grad_times_impl(pred: torch.Tensor, target: torch.Tensor, kernel_size: int, smooth_dr: float, reduction: int,
                     grad_out: torch.Tensor) -> torch.Tensor:
    """grad_out * dL/dpred in one fused pass, grad_out folded into the fp32 scale before the gradient is
    rounded to pred's dtype (fp16: a scaled loss, as with torch.amp.GradScaler, keeps gradients that
    -1/M alone would flush to zero)."""
    go = grad_out.detach().to(device=pred.device, dtype=torch.float32).contiguous()
    scale = -1.0 if reduction == REDUCTIONS["sum"] else None
    _, g = lncc_fused(pred, target, kernel_size, smooth_dr, grad=True, grad_scale=scale, grad_scale_dev=go)
    return g


_grad_times_op = torch.library.custom_op("fused_lncc::grad_times", mutates_args=())(_grad_times_impl)


@_grad_times_op.register_fake
def _(pred, target, kernel_size, smooth_dr, reduction, grad_out):
    return torch.empty_like(pred)


@torch.library.custom_op("fused_lncc::scale_grad_", mutates_args=("grad",))
def _scale_grad_op(grad: torch.Tensor, grad_out: torch.Tensor) -> None:
    scale_grad_(grad, grad_out)


@_scale_grad_op.register_fake
def _(grad, grad_out):
    return None


class FusedLNCC(torch.autograd.Function):
    """Autograd glue (reference _FusedLNCC, fused_lncc/__init__.py:49-74).

    forward: one fused pass -> (loss, dL/dpred for grad_out = 1), the gradient kept for backward.
    backward: scales that gradient by grad_out in place and hands it over (no copy). A second
    backward through the same graph (retain_graph=True) recomputes it from the saved inputs.
    fp16 inputs: the forward computes the loss only and the backward one fused pass with grad_out
    applied in fp32 before the fp16 rounding (the gradient, of order 1/M, is below fp16's normal range
    for large M unless the loss is scaled, as torch.amp.GradScaler does).
    """

    @staticmethod
    def forward(ctx, pred, target, kernel_size, smooth_dr, need_grad=None, reduction=0):
        # Grad mode is off inside forward; the caller passes whether the graph wants d/dpred.
        if need_grad is None:
            need_grad = bool(ctx.needs_input_grad[0])
        ctx.deferred = need_grad and pred.dtype == torch.float16
        fwd = torch.ops.fused_lncc.fwd_grad if torch.compiler.is_compiling() else _fwd_grad_impl
        loss, g = fwd(pred, target, kernel_size, smooth_dr, need_grad and not ctx.deferred, reduction)
        ctx.save_for_backward(pred, target)
        ctx.k = kernel_size
        ctx.dr = smooth_dr
        ctx.reduction = reduction
        ctx.grad = g if need_grad and not ctx.deferred else None
        return loss

    @staticmethod
    def backward(ctx, grad_out):
        compiling = torch.compiler.is_compiling()
        if ctx.deferred:
            pred, target = ctx.saved_tensors
            gt = torch.ops.fused_lncc.grad_times if compiling else _grad_times_impl
            g = gt(pred, target, ctx.k, ctx.dr, ctx.reduction, grad_out)
            return g, None, None, None, None, None
        g = ctx.grad
        ctx.grad = None  # hand the buffer over; a later backward recomputes
        if g is None or g.numel() == 0:
            pred, target = ctx.saved_tensors
            fwd = torch.ops.fused_lncc.fwd_grad if compiling else _fwd_grad_impl
            _, g = fwd(pred, target, ctx.k, ctx.dr, True, ctx.reduction)
        if compiling:
            torch.ops.fused_lncc.scale_grad_(g, grad_out)
        else:
            scale_grad_(g, grad_out)
        return g, None, None, None, None, None


_FusedLNCC = FusedLNCC  # the reference's private name


class FusedLNCCMap(torch.autograd.Function):
    """reduction='none': the per-voxel loss map 1 - cc, with the gradient of sum(G * map) for any
    upstream map G (materialising path: three fp32 adjoint maps weighted by G, then boxed)."""

    @staticmethod
    def forward(ctx, pred, target, kernel_size, smooth_dr):
        ctx.save_for_backward(pred, target)
        ctx.k = kernel_size
        ctx.dr = smooth_dr
        return torch.ops.fused_lncc.loss_map(pred, target, kernel_size, smooth_dr)

    @staticmethod
    def backward(ctx, grad_map):
        pred, target = ctx.saved_tensors
        g = torch.ops.fused_lncc.loss_map_backward(grad_map.contiguous(), pred, target, ctx.k, ctx.dr)
        return g, None, None, None


def fused_lncc_loss(pred, target, kernel_size=7, smooth_dr=1e-5, reduction="mean"):
    """1 - mean(squared local NCC). Gradient flows through `pred` only.

    pred, target: (N, C, D, H, W) fp32, bf16 or fp16 CUDA (fp16 is not in the reference). kernel_size odd (3, 5, 7 or 9),
    or a (kd, kh, kw) tuple of odd sides 1 .. 9 (a non-cubic window, not in the reference).
    Returns a 0-dim fp32 loss in [0, 1] (reference fused_lncc/__init__.py:77-83).
    reduction (not in the reference, which lists it as open): 'mean' (default, the reference's
    loss), 'sum' (sum of 1 - cc, 0-dim fp32) or 'none' (fp32 map 1 - cc of pred's shape)."""
    assert pred.dim() == 5 and pred.shape == target.shape, "expect matching (N,C,D,H,W)"
    kernel_size = window.window_of(kernel_size)
    if reduction == "none":
        if isinstance(kernel_size, tuple):
            return window.FusedLNCCWindowMap.apply(pred.contiguous(), target.contiguous(), kernel_size, smooth_dr)
        return FusedLNCCMap.apply(pred.contiguous(), target.contiguous(), kernel_size, smooth_dr)
    if reduction not in REDUCTIONS:
        raise ValueError(f"fused_lncc: reduction must be 'mean', 'sum' or 'none', got {reduction!r}")
    if isinstance(kernel_size, tuple):
        return window.FusedLNCCWindow.apply(pred.contiguous(), target.contiguous(), kernel_size, smooth_dr,
                                            REDUCTIONS[reduction])
    need_grad = bool(pred.requires_grad and torch.is_grad_enabled())
    return FusedLNCC.apply(pred.contiguous(), target.contiguous(), kernel_size, smooth_dr, need_grad,
                           REDUCTIONS[reduction])


from . import compat  # noqa: E402  (registers the reference's fused_lncc::forward/backward ops)
from . import window  # noqa: E402  (non-cubic windows)
