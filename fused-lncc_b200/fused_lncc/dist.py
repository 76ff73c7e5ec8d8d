"""Multi-GPU LNCC: one process per GPU over torch.distributed (NCCL on B200 / NVLink, gloo on CPU).

The reference has no distributed code; it leaves multi-GPU to user-level DDP (reference README.md:121).
Two partitions of the loss are provided here:

* volume sharding (N*C volumes spread over ranks): the fused kernel runs unchanged on each rank's
  volumes. The gradient needs no collective because its scale, -1/M_global, is static. The loss needs
  the sum of one fp64 per rank (the cc sum): on GPUs of one node through `PeerExchange`, one small
  kernel that writes each rank's sum into every rank's buffer over NVLink peer memory and adds them in
  rank order (no collective library on the step's path); otherwise one all-reduce.
* D-slab sharding of single large volumes: see `slab_plan` / `SlabLNCC` (halo exchange of 2*(k//2)
  planes of pred and target with each neighbour, then the same fused kernel on the padded slab).
"""
import torch
import torch.distributed as dist

from . import _lib, lncc_fused, scale_grad_


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


class PeerExchange:
    """Every rank's exchange buffer mapped into this process (CUDA IPC), for the C-ABI lncc_peer_loss.

    Built once per (process group, device), collectively: each rank allocates its buffer, and the IPC
    handles travel once through the group (all_gather_object). Afterwards a loss needs no collective:
    `loss(local_sum, count)` launches one kernel on the current stream. The epoch counts calls and must
    advance identically on every rank (every rank calls `loss` the same number of times).
    """

    def __init__(self, group=None, device=None):
        from torch.multiprocessing.reductions import reduce_tensor
        self.lib = _lib.load()
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        nbytes = self.lib.lncc_peer_exchange_bytes(self.world)
        if nbytes == 0:
            raise RuntimeError(f"fused_lncc: peer exchange supports 1..32 ranks, not {self.world}")
        self.buf = torch.zeros(nbytes // 8, dtype=torch.int64, device=self.device)
        torch.cuda.synchronize(self.device)
        shared = [None] * self.world
        dist.all_gather_object(shared, reduce_tensor(self.buf), group=group)
        self.peers = []
        for r, (fn, args) in enumerate(shared):
            if r == self.rank:
                self.peers.append(self.buf)
            else:
                args = list(args)
                args[6] = self.device.index  # open the peer's buffer from this process's device
                self.peers.append(fn(*args))
        self.slots = torch.tensor([t.data_ptr() for t in self.peers], dtype=torch.int64, device=self.device)
        self.epoch = 0
        dist.barrier(group=group)

    def loss(self, local_sum, count, cc_sum_out=None):
        """1 - (sum over ranks of local_sum) / count, on the current stream; every rank gets the same
        bits. local_sum: 1-element fp64 device tensor. Returns a 0-dim fp32 tensor."""
        self.epoch += 1
        loss = torch.empty((), dtype=torch.float32, device=self.device)
        st = self.lib.lncc_peer_loss(local_sum.data_ptr(), self.slots.data_ptr(), self.rank, self.world, self.epoch,
                                     float(count), cc_sum_out.data_ptr() if cc_sum_out is not None else None,
                                     loss.data_ptr(), None, torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(st, "fused_lncc peer loss")
        return loss


_PEER = {}
_PEER_ERR = {}  # why a group's exchange could not be built (diagnostics)


def peer_exchange(group=None):
    """The cached PeerExchange of `group` on the current device, or None when the group is not a
    node-local NCCL group or the buffers cannot be mapped (the caller then all-reduces)."""
    key = (id(group), torch.cuda.current_device())
    if key in _PEER:  # every step asks: answer from the cache before querying the group
        return _PEER[key]
    if not (dist.is_available() and dist.is_initialized()) or dist.get_backend(group) != "nccl":
        return None
    if key not in _PEER:
        px, err = None, None
        try:
            px = PeerExchange(group)
        except Exception as e:  # e.g. ranks on several nodes: no peer mapping
            err = e
        # every rank must take the same path: use the exchange only where every rank built it
        ok = torch.tensor([0 if px is None else 1], dtype=torch.int32, device=torch.cuda.current_device())
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        _PEER[key] = px if int(ok.item()) == 1 else None
        _PEER_ERR[key] = err
    return _PEER[key]


class ShardedLNCC(torch.autograd.Function):
    """1 - (sum over all ranks of cc) / m_global, with dL/dpred_local (volume sharding)."""

    @staticmethod
    def forward(ctx, pred, target, kernel_size, smooth_dr, m_global, group, need_grad):
        cc_sum = torch.empty(1, dtype=torch.float64, device=pred.device)
        _, g = lncc_fused(pred, target, kernel_size, smooth_dr, grad=need_grad,
                          grad_scale=-1.0 / float(m_global), cc_sum_out=cc_sum)
        ctx.save_for_backward(pred, target)
        ctx.args = (kernel_size, smooth_dr, m_global)
        ctx.grad = g
        if _world(group) > 1:
            px = peer_exchange(group)
            if px is not None:
                return px.loss(cc_sum, float(m_global))
            dist.all_reduce(cc_sum, op=dist.ReduceOp.SUM, group=group)
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
        ctx.grad = g
        if _world(group) > 1:
            px = peer_exchange(group) if total.is_cuda else None
            if px is not None:
                return px.loss(total, float(m_global))
            dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
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
