"""Multi-GPU LNCC: one process per GPU over torch.distributed (NCCL on B200 / NVLink, gloo on CPU).

The reference has no distributed code; it leaves multi-GPU to user-level DDP (reference README.md:121).
Two partitions of the loss are provided here:

* volume sharding (N*C volumes spread over ranks): the fused kernel runs unchanged on each rank's
  volumes. The gradient needs no collective because its scale, -1/M_global, is static. The loss needs
  ONE all-reduce of one fp64 (the cc sum).
* D-slab sharding of single large volumes: see `slab_plan` / `SlabLNCC` (halo exchange of 2*(k//2)
  planes of pred and target with each neighbour, then the same fused kernel on the padded slab).
"""
import torch
import torch.distributed as dist

from . import lncc_fused, scale_grad_


def volume_range(n_volumes, world, rank):
    """[b0, b1) of the volumes owned by `rank` when n_volumes are split as evenly as possible."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(int(n_volumes), world)
    b0 = rank * base + min(rank, extra)
    return b0, b0 + base + (1 if rank < extra else 0)


def _world(group):
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return 1
    return dist.get_world_size(group)


class ShardedLNCC(torch.autograd.Function):
    """1 - (sum over all ranks of cc) / m_global, with dL/dpred_local (volume sharding)."""

    @staticmethod
    def forward(ctx, pred, target, kernel_size, smooth_dr, m_global, group, need_grad):
        cc_sum = torch.empty(1, dtype=torch.float64, device=pred.device)
        _, g = lncc_fused(pred, target, kernel_size, smooth_dr, grad=need_grad,
                          grad_scale=-1.0 / float(m_global), cc_sum_out=cc_sum)
        if _world(group) > 1:
            dist.all_reduce(cc_sum, op=dist.ReduceOp.SUM, group=group)
        ctx.save_for_backward(pred, target)
        ctx.args = (kernel_size, smooth_dr, m_global)
        ctx.grad = g
        return (1.0 - cc_sum / float(m_global)).to(torch.float32).reshape(())

    @staticmethod
    def backward(ctx, grad_out):
        g = ctx.grad
        ctx.grad = None
        if g is None:
            pred, target = ctx.saved_tensors
            k, dr, m = ctx.args
            _, g = lncc_fused(pred, target, k, dr, grad=True, grad_scale=-1.0 / float(m))
        scale_grad_(g, grad_out)
        return g, None, None, None, None, None, None


def sharded_lncc_loss(pred_local, target_local, kernel_size=7, smooth_dr=1e-5, *, m_global=None,
                      group=None):
    """Loss of the global batch from each rank's shard of volumes.

    pred_local/target_local: this rank's (n, C, D, H, W) slice of the global batch.
    m_global: number of voxels of the global batch (default: all-reduced count of the shards).
    Every rank must call this the same number of times in the same order (one all-reduce each).
    """
    assert pred_local.dim() == 5 and pred_local.shape == target_local.shape, "expect matching (N,C,D,H,W)"
    assert kernel_size % 2 == 1, "kernel_size must be odd"
    if m_global is None:
        m = torch.tensor([float(pred_local.numel())], dtype=torch.float64, device=pred_local.device)
        if _world(group) > 1:
            dist.all_reduce(m, group=group)
        m_global = float(m.item())
    need_grad = bool(pred_local.requires_grad and torch.is_grad_enabled())
    return ShardedLNCC.apply(pred_local.contiguous(), target_local.contiguous(), kernel_size, smooth_dr,
                             float(m_global), group, need_grad)
