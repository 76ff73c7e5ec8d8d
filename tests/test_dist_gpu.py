"""GPU, multi-process NCCL (needs >= 2 GPUs; skipped otherwise): the sharded losses equal the
single-GPU loss of the whole batch / volume, and the gradients equal its slices; the loss reduction
over NVLink peer memory equals an NCCL all-reduce and gives every rank the same bits."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from fused_lncc import fused_lncc_loss, synth
        from fused_lncc.dist import SlabPlan, sharded_lncc_loss, slab_lncc_loss, volume_range
        if mode == "peer":
            # the loss reduction over NVLink peer memory (lncc_peer_loss) against an NCCL all-reduce,
            # over several epochs (both buffer parities), equal on every rank
            from fused_lncc.dist import peer_exchange
            px = peer_exchange()
            assert px is not None, "peer exchange not available on this node"
            worst = 0.0
            for it in range(6):
                local = torch.tensor([0.25 * (rank + 1) + it], dtype=torch.float64, device=dev)
                s_out = torch.zeros(1, dtype=torch.float64, device=dev)
                loss = px.loss(local, 10.0, cc_sum_out=s_out)
                ref = local.clone()
                dist.all_reduce(ref)
                worst = max(worst, abs(s_out.item() - ref.item()), abs(loss.item() - (1.0 - ref.item() / 10.0)))
                both = torch.stack([s_out[0], s_out[0]])
                dist.broadcast(both, 0)  # rank 0's bits
                worst = max(worst, abs(both[0].item() - s_out.item()))
            q.put((rank, worst, 0.0))
        elif mode == "volumes":
            p, t = synth.blurred_pair((2, 3, 40, 48, 64), device="cpu")
            p, t = p.to(dev), t.to(dev)
            pf = p.clone().requires_grad_(True)
            lf = fused_lncc_loss(pf, t, 7)
            lf.backward()
            b0, b1 = volume_range(6, world, rank)
            pv = p.reshape(6, 1, 40, 48, 64)[b0:b1].clone().requires_grad_(True)
            tv = t.reshape(6, 1, 40, 48, 64)[b0:b1]
            ls = sharded_lncc_loss(pv, tv, 7, m_global=float(p.numel()))
            ls.backward()
            ref = pf.grad.reshape(6, 1, 40, 48, 64)[b0:b1]
            rel = ((pv.grad - ref).norm() / ref.norm()).item()
            q.put((rank, abs(ls.item() - lf.item()), rel))
        else:
            D, H, W, k = 72, 40, 64, 7
            p, t = synth.blurred_pair((1, 1, D, H, W), device="cpu")
            p, t = p.to(dev), t.to(dev)
            pf = p.clone().requires_grad_(True)
            lf = fused_lncc_loss(pf, t, k)
            lf.backward()
            plan = SlabPlan(D, world, rank, k)
            ps = torch.zeros(1, plan.depth, H, W, device=dev)
            ts = torch.zeros(1, plan.depth, H, W, device=dev)
            lo, e = plan.own_range
            ps[:, lo:e] = p[0, :, plan.z0:plan.z1]
            ts[:, lo:e] = t[0, :, plan.z0:plan.z1]
            ps.requires_grad_(True)
            ls = slab_lncc_loss(ps, ts, plan, k)
            ls.backward()
            ref = pf.grad[0, :, plan.z0:plan.z1]
            rel = ((ps.grad[:, lo:e] - ref).norm() / ref.norm()).item()
            q.put((rank, abs(ls.item() - lf.item()), rel))
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["volumes", "slabs", "peer"])
def test_two_gpu_sharding_matches_single_gpu(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    for rank, dloss, rel in res:
        assert dloss < 1e-6, (rank, dloss)
        assert rel < 1e-4, (rank, rel)
