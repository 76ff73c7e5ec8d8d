"""CPU, multi-process (gloo): the multi-GPU layer's bookkeeping with the CPU oracle as the kernel.

- volume sharding: per-rank cc sums all-reduced == whole-batch loss; per-rank grads == slices;
- D-slabs: plans, halo exchange and the slab loss/grad == whole-volume oracle, for world 2 and 3;
- failure detection on the host: a rank that raises before the exchange makes the other ranks' next
  collective fail within the process-group timeout (no GPU involved).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fused_lncc.dist import SlabPlan, slab_lncc_loss, volume_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_compute(pred, target, k, dr, z_range, grad_scale, grad_out):
    from oracle import c_oracle
    o = c_oracle.lncc(pred.detach().numpy(), target.detach().numpy(), k, dr, z_range=z_range,
                      grad_scale=grad_scale, grad=grad_out is not None)
    if grad_out is not None:
        grad_out[:, z_range[0]:z_range[1]] = torch.from_numpy(o["grad"])
    return torch.tensor([o["cc_sum"]], dtype=torch.float64)


def _volume(D, H, W, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(1, D, H, W, generator=g), torch.randn(1, D, H, W, generator=g)


def _slab_worker(rank, world, port, D, H, W, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        p, t = _volume(D, H, W, 7)
        plan = SlabPlan(D, world, rank, k)
        ps = torch.zeros(1, plan.depth, H, W)
        ts = torch.zeros(1, plan.depth, H, W)
        lo, e = plan.own_range
        ps[:, lo:e] = p[:, plan.z0:plan.z1]     # each rank starts with its owned planes only
        ts[:, lo:e] = t[:, plan.z0:plan.z1]
        ps.requires_grad_(True)
        loss = slab_lncc_loss(ps, ts, plan, k, compute=_oracle_compute)
        loss.backward()
        # halos must now hold the neighbours' planes
        halo_ok = torch.equal(ps.detach()[:, :lo], p[:, plan.z0 - plan.lo:plan.z0]) and torch.equal(
            ps.detach()[:, e:], p[:, plan.z1:plan.z1 + plan.hi])
        q.put((rank, float(loss.item()), ps.grad[:, lo:e].numpy(), (plan.z0, plan.z1), halo_ok,
               float(ps.grad[:, :lo].abs().sum() + ps.grad[:, e:].abs().sum())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,D,k", [(2, 24, 7), (3, 31, 5), (2, 19, 9), (3, 9, 3)])
def test_slab_loss_and_grad_match_whole_volume(world, D, k):
    from oracle import c_oracle
    H, W = 9, 11
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_slab_worker, args=(r, world, port, D, H, W, k, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    p, t = _volume(D, H, W, 7)
    ref = c_oracle.lncc(p.numpy(), t.numpy(), k)
    for rank, loss, g, (z0, z1), halo_ok, halo_grad in res:
        assert halo_ok, rank
        assert halo_grad == 0.0, rank
        assert abs(loss - ref["loss"]) < 1e-6, (rank, loss, ref["loss"])  # fp32 loss scalar
        np.testing.assert_allclose(g, ref["grad"][:, z0:z1], rtol=1e-5, atol=1e-12)


def test_slab_plan_properties():
    for D in (6, 7, 16, 31, 128, 1024):
        for world in (1, 2, 3, 4, 8):
            for k in (3, 5, 7, 9):
                r = k // 2
                try:
                    plans = [SlabPlan(D, world, i, k) for i in range(world)]
                except ValueError:
                    assert world > 1 and D // world < 2 * r or D < world
                    continue
                assert plans[0].z0 == 0 and plans[-1].z1 == D
                for a, b in zip(plans, plans[1:]):
                    assert a.z1 == b.z0 and a.hi == min(2 * r, D - a.z1) and b.lo == 2 * r
                assert sum(p.own for p in plans) == D


def test_slab_plan_rejects_bad_splits():
    with pytest.raises(ValueError):
        SlabPlan(10, 4, 0, 7)          # 2 or 3 planes per rank < 6-plane halo
    with pytest.raises(ValueError):
        SlabPlan(3, 4, 0, 3)           # fewer planes than ranks
    with pytest.raises(ValueError):
        SlabPlan(16, 2, 2, 3)          # rank out of range


def test_volume_range_partitions():
    for n in (1, 5, 32, 33):
        for world in (1, 2, 3, 8):
            rs = [volume_range(n, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))


def _sharded_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import c_oracle
        g = torch.Generator().manual_seed(3)
        p = torch.randn(5, 1, 8, 9, 10, generator=g)
        t = torch.randn(5, 1, 8, 9, 10, generator=g)
        b0, b1 = volume_range(5, world, rank)
        M = float(p.numel())
        o = c_oracle.lncc(p[b0:b1].numpy(), t[b0:b1].numpy(), 5, grad_scale=-1.0 / M)
        s = torch.tensor([o["cc_sum"]], dtype=torch.float64)
        dist.all_reduce(s)
        q.put((rank, 1.0 - float(s.item()) / M, o["grad"], (b0, b1)))
    finally:
        dist.destroy_process_group()


def test_volume_sharding_bookkeeping():
    """The arithmetic of ShardedLNCC (fixed -1/M_global grad scale + one cc-sum all-reduce)."""
    from oracle import c_oracle
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    g = torch.Generator().manual_seed(3)
    p = torch.randn(5, 1, 8, 9, 10, generator=g)
    t = torch.randn(5, 1, 8, 9, 10, generator=g)
    ref = c_oracle.lncc(p.numpy(), t.numpy(), 5)
    for rank, loss, grad, (b0, b1) in res:
        assert abs(loss - ref["loss"]) < 1e-12
        np.testing.assert_allclose(grad, ref["grad"][b0:b1], rtol=1e-6, atol=1e-14)


def _failing_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            q.put((rank, "raised"))
            raise RuntimeError("injected failure before the halo exchange")
        p, t = _volume(16, 5, 6, 1)
        plan = SlabPlan(16, world, rank, 3)
        ps = torch.zeros(1, plan.depth, 5, 6)
        try:
            slab_lncc_loss(ps, torch.zeros_like(ps), plan, 3, compute=_oracle_compute)
            q.put((rank, "no error"))
        except Exception as e:  # the peer never sends: the exchange must fail, not hang
            q.put((rank, "error: " + type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_failure_surfaces_as_error():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for pr in procs:
        pr.join(timeout=60)
        if pr.is_alive():
            pr.kill()
    assert res[1] == "raised"
    assert res[0].startswith("error"), res[0]
