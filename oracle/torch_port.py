"""TEST INFRASTRUCTURE ONLY: restatement of the reference's PyTorch LNCC (CPU baseline + oracle).

The reference's CPU path is baselines/torch_lncc.py (box sums as grouped conv3d with all-ones
weights, dense `_box_dense` :12-14 or separable `_box_separable` :17-22; loss `_lncc` :25-32).
That file is not available on the GPU box, so this module restates the same algorithm: the same
convolutions, the same formula with no variance clamp, and `clamp(max=1)` through autograd. It is
the `kind: "port"` CPU baseline that bench.py times, and a second parity check beside the C oracle.
"""
import torch
import torch.nn.functional as F


def _sides(k):
    return tuple(int(v) for v in k) if isinstance(k, (tuple, list)) else (int(k),) * 3


def box_dense(x, k):
    """k^3 zero-padded box as one grouped conv3d (reference torch_lncc.py:12-14). k may also be a
    (kd, kh, kw) tuple: the non-cubic window the reference lists as open, same convolution."""
    ch = x.shape[1]
    kd, kh, kw = _sides(k)
    return F.conv3d(x, x.new_ones(ch, 1, kd, kh, kw), padding=(kd // 2, kh // 2, kw // 2), groups=ch)


def box_separable(x, k):
    """Three 1-D grouped convs along D, H, W (reference torch_lncc.py:17-22)."""
    ch = x.shape[1]
    out = x
    for shape in ((ch, 1, k, 1, 1), (ch, 1, 1, k, 1), (ch, 1, 1, 1, k)):
        out = F.conv3d(out, x.new_ones(*shape), padding="same", groups=ch)
    return out


def lncc_loss(pred, target, kernel_size=7, smooth_dr=1e-5, box=box_dense):
    """1 - mean(cc) with autograd (reference torch_lncc.py:25-32)."""
    kd, kh, kw = _sides(kernel_size)
    n = kd * kh * kw
    sp, st = box(pred, kernel_size), box(target, kernel_size)
    cross = box(pred * target, kernel_size) - sp * st / n
    var_p = box(pred * pred, kernel_size) - sp * sp / n + smooth_dr
    var_t = box(target * target, kernel_size) - st * st / n + smooth_dr
    cc = ((cross * cross) / (var_p * var_t)).clamp(max=1.0)
    return 1.0 - cc.mean()


def lncc_dense(pred, target, kernel_size=7, smooth_dr=1e-5):
    return lncc_loss(pred, target, kernel_size, smooth_dr, box_dense)


def lncc_separable(pred, target, kernel_size=7, smooth_dr=1e-5):
    return lncc_loss(pred, target, kernel_size, smooth_dr, box_separable)


def loss_and_grad(pred, target, kernel_size=7, smooth_dr=1e-5, separable=False):
    """(loss float, grad tensor) of the port for one fwd+bwd, on whatever device pred lives."""
    p = pred.detach().clone().requires_grad_(True)
    fn = lncc_separable if separable else lncc_dense
    loss = fn(p, target.detach(), kernel_size, smooth_dr)
    loss.backward()
    return float(loss.item()), p.grad
