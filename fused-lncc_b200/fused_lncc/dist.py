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


# ---- D-slab sharding of single volumes ------------------------------------------------------------
class SlabPlan:
    """Plane ownership of one rank when D planes are split into `world` slabs.

    The rank owns planes [z0, z1) of the volume. Its local slab array holds planes
    [z0 - lo, z1 + hi): `lo` = min(2r, z0) halo planes below and `hi` = min(2r, D - z1) above,
    r = k // 2. Two-level windows (statistics at radius r, their adjoints boxed again at radius r)
    make a plane's gradient depend on planes within 2r. So one exchange of 2r planes of pred and
    target per side is all a slab needs. At the volume ends there is no halo (zero padding).
    """

    def __init__(self, D, world, rank, kernel_size):
        if not (0 <= rank < world) or D < world:
            raise ValueError(f"cannot split D={D} planes over {world} ranks")
        r = kernel_size // 2
        base, extra = divmod(int(D), world)
        self.D, self.world, self.rank, self.r = int(D), world, rank, r
        self.z0 = rank * base + min(rank, extra)
        self.z1 = self.z0 + base + (1 if rank < extra else 0)
        self.own = self.z1 - self.z0
        self.lo = min(2 * r, self.z0)
        self.hi = min(2 * r, self.D - self.z1)
        self.depth = self.lo + self.own + self.hi
        if self.own < 2 * r and world > 1:
            raise ValueError(f"slab of {self.own} planes is thinner than the 2*(k//2)={2 * r} halo")

    @property
    def own_range(self):
        """Plane range of the owned planes inside the local slab array."""
        return self.lo, self.lo + self.own

    def send_recv_specs(self):
        """(peer, slab_send_range, slab_recv_range) for each neighbour; ranges index the slab array."""
        specs = []
        h = 2 * self.r
        if self.rank > 0:      # lower neighbour: send my first h owned planes, receive its last h
            specs.append((self.rank - 1, (self.lo, self.lo + h), (0, self.lo)))
        if self.rank + 1 < self.world:  # upper neighbour: send my last h owned planes, receive its first h
            e = self.lo + self.own
            specs.append((self.rank + 1, (e - h, e), (e, e + self.hi)))
        return specs


def exchange_halos(slabs, plan, group=None):
    """Fill the halo planes of each (1, depth, H, W) slab array from the neighbour ranks.

    Uses one batched isend/irecv round with NCCL (CUDA) or gloo (CPU). Returns the list of works;
    the caller waits on them before using the halo planes, and can overlap interior compute meanwhile.
    """
    ops = []
    for peer, (s0, s1), (r0, r1) in plan.send_recv_specs():
        if s1 <= s0:
            continue
        for x in slabs:
            v = x.detach()
            ops.append(dist.P2POp(dist.isend, v[:, s0:s1], peer, group))
            ops.append(dist.P2POp(dist.irecv, v[:, r0:r1], peer, group))
    if not ops:
        return []
    return dist.batch_isend_irecv(ops)


def _cuda_compute(pred, target, kernel_size, smooth_dr, z_range, grad_scale, grad_out_planes):
    """One fused launch over planes z_range of a (1, depth, H, W) slab; writes those planes of
    grad_out_planes (a (1, depth, H, W) view) and returns the cc sum as a 1-element fp64 tensor."""
    csum = torch.zeros(1, dtype=torch.float64, device=pred.device)
    z0, z1 = z_range
    out = grad_out_planes[:, z0:z1] if grad_out_planes is not None else None  # contiguous: B == 1
    lncc_fused(pred, target, kernel_size, smooth_dr, grad=out is not None, grad_scale=grad_scale,
               z_range=(z0, z1), cc_sum_out=csum, out=out)
    return csum


class SlabLNCC(torch.autograd.Function):
    """Loss of a whole volume from D-slabs held by the ranks (see SlabPlan).

    forward: exchange 2r halo planes of pred and target with the neighbours (in place, into the
    halo planes of the slab arrays). The interior planes, which need no halo, are computed while the
    exchange is in flight, then the boundary planes. One fp64 all-reduce of the cc sum follows.
    The gradient of the halo planes is zero: those voxels belong to the neighbour, which computes
    their gradient.
    """

    @staticmethod
    def forward(ctx, pred_slab, target_slab, kernel_size, smooth_dr, plan, m_global, group, need_grad,
                compute):
        works = exchange_halos([pred_slab, target_slab], plan, group)
        lo, e = plan.own_range
        h = 2 * plan.r
        gscale = -1.0 / float(m_global)
        g = torch.zeros_like(pred_slab) if need_grad else None
        total = torch.zeros(1, dtype=torch.float64, device=pred_slab.device)
        # interior planes need no halo
        i0, i1 = lo + (h if plan.lo else 0), e - (h if plan.hi else 0)
        if i1 > i0:
            total += compute(pred_slab, target_slab, kernel_size, smooth_dr, (i0, i1), gscale, g)
        for w in works:
            w.wait()
        for z0, z1 in ((lo, i0), (max(i1, i0), e)):
            if z1 > z0:
                total += compute(pred_slab, target_slab, kernel_size, smooth_dr, (z0, z1), gscale, g)
        if _world(group) > 1:
            dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
        ctx.grad = g
        return (1.0 - total / float(m_global)).to(torch.float32).reshape(())

    @staticmethod
    def backward(ctx, grad_out):
        g = ctx.grad
        ctx.grad = None
        if g is None:
            raise RuntimeError("slab LNCC: the forward pass ran without gradient")
        if g.is_cuda:
            scale_grad_(g, grad_out)
        else:
            g.mul_(grad_out.to(g.dtype))
        return g, None, None, None, None, None, None, None, None


def slab_lncc_loss(pred_slab, target_slab, plan, kernel_size=7, smooth_dr=1e-5, *, group=None,
                   compute=None):
    """LNCC loss of a volume split in D-slabs across ranks.

    pred_slab/target_slab: (1, plan.depth, H, W) arrays holding this rank's owned planes at
    [plan.lo, plan.lo + plan.own); the halo planes are overwritten by the exchange. Every rank calls
    this collectively. `compute` defaults to the fused CUDA kernel; tests pass a CPU stand-in.
    """
    if pred_slab.dim() != 4 or pred_slab.shape[0] != 1 or pred_slab.shape != target_slab.shape:
        raise ValueError("slab arrays must be (1, depth, H, W) and match")
    if pred_slab.shape[1] != plan.depth:
        raise ValueError(f"slab depth {pred_slab.shape[1]} != plan depth {plan.depth}")
    H, W = pred_slab.shape[2:]
    m_global = float(plan.D) * H * W
    need_grad = bool(pred_slab.requires_grad and torch.is_grad_enabled())
    return SlabLNCC.apply(pred_slab, target_slab, kernel_size, smooth_dr, plan, m_global, group, need_grad,
                          compute or _cuda_compute)
