"""Benchmark of the fused LNCC loss: fwd+bwd Gvoxel/s at (2,16,128^3) fp32 k=7 on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL)

Prints ONE JSON line on rank 0. A step is one forward + backward of the loss through the public API.
Every workload scales strongly: the workload's one batch is split across the ranks. Volume workloads
shard the N*C volumes (rank r owns its share, the loss is the mean over the whole batch through one
fp64 all-reduce); D-slab workloads split one volume into D-slabs. `value` counts the batch's voxels
over the max-over-ranks step time. At N > 1 volume workloads also carry `weak_scaling`: every rank
with a full batch of its own (its own seed), timed the same way.
Timing: W untimed warm-up steps,
then K steps each bracketed by CUDA events on the launching stream, an L2 flush (256 MiB write)
before every step outside the events, barrier + synchronize around the whole timed region, max over
ranks. `roofline` times the dominant kernel alone (one C-ABI launch per timing), `e2e` the same public
call with the inputs copied from pinned host memory and the loss read back every step.
`--impl reference` times the reference algorithm's CPU implementation (the PyTorch port in
oracle/torch_port.py, all host threads) on a bounded sample of the same workload.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "fused-lncc_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

WORKLOADS = {
    # name: (shape, k, dtype, construction); configs of BASELINE.json
    "headline": ((2, 16, 128, 128, 128), 7, "fp32", "blurred"),        # config 2, N*C volumes sharded
    "config1": ((1, 1, 64, 64, 64), 7, "fp32", "blurred"),             # config 1
    "mri": ((8, 1, 160, 192, 224), 9, "bf16", "mri"),                  # config 3, volumes sharded
    "ksweep3": ((1, 1, 256, 256, 256), 3, "fp32", "blurred"),          # config 4, D-slabs
    "ksweep5": ((1, 1, 256, 256, 256), 5, "fp32", "blurred"),
    "ksweep7": ((1, 1, 256, 256, 256), 7, "fp32", "blurred"),
    "ksweep9": ((1, 1, 256, 256, 256), 9, "fp32", "blurred"),
    "gigavoxel": ((1, 1, 1024, 1024, 1024), 7, "fp32", "gigavoxel"),  # config 5, D-slabs
    "small": ((2, 4, 128, 128, 128), 7, "fp32", "blurred"),            # profiling-sized headline case
}
SLAB_WORKLOADS = {"ksweep3", "ksweep5", "ksweep7", "ksweep9", "gigavoxel"}
METRIC = "fwd+bwd Gvoxel/s at (2,16,128^3) fp32 k=7"


def metric_name(workload):
    """The headline metric string for the headline workload, the same unit for the others."""
    if workload == "headline":
        return METRIC
    shape, k, dtype, _ = WORKLOADS[workload]
    return f"fwd+bwd Gvoxel/s at ({','.join(map(str, shape))}) {dtype} k={k}"
BYTES_PER_VOXEL = {"fp32": 12, "bf16": 6}   # read pred + read target + write grad


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peak_gbs():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(kernel, workload):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.json), else None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(f"{kernel}/{workload}")
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock, max clock and throttle reasons through NVML during the timed region."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: report no clock data
            self._nv = None
            self.error = str(e)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self._nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thr is not None:
            self._thr.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def make_inputs(workload, device, seed=0):
    from fused_lncc import synth
    shape, k, dtype, kind = WORKLOADS[workload]
    tdt = torch.float32 if dtype == "fp32" else torch.bfloat16
    if kind == "blurred":
        pred, target = synth.blurred_pair(shape, seed=seed, device=device, dtype=tdt)
    elif kind == "gigavoxel":
        pred, target = synth.gigavoxel_pair(shape, device=device, dtype=tdt)
    else:
        pred, target = synth.mri_pair(shape, device=device, dtype=tdt)
    return pred, target, k, dtype


def cpu_reference_sample(pred, target, k, steps, warmup, sample_volumes):
    """Times the reference algorithm's PyTorch CPU path (oracle/torch_port.py) on `sample_volumes`
    volumes per step; returns (Gvox/s, details)."""
    from oracle import torch_port
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n, c = pred.shape[:2]
    pv = pred.reshape(n * c, 1, *pred.shape[2:])[:sample_volumes].float().cpu().contiguous()
    tv = target.reshape(n * c, 1, *target.shape[2:])[:sample_volumes].float().cpu().contiguous()
    vox = pv.numel()

    def one():
        p = pv.clone().requires_grad_(True)
        loss = torch_port.lncc_separable(p, tv, k)
        loss.backward()
        return loss.item()

    for _ in range(warmup):
        one()
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        one()
        ts.append(time.perf_counter() - t0)
    sec = statistics.median(ts)
    return vox / sec / 1e9, {
        "cores": threads, "kind": "port",
        "sample": f"{sample_volumes} of the workload's volumes ({'x'.join(map(str, pv.shape[2:]))}), "
                  f"lncc_separable fwd+bwd on CPU, median of {steps} after {warmup} warm-up",
        "cpu_model": _cpu_model(), "seconds_per_step": sec,
    }


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


REFERENCE_MAX_STEPS = 40  # bounds the CPU arm at ~1 s per step
REFERENCE_MAX_WARMUP = 3


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    from fused_lncc import synth  # noqa: F401  (inputs only)
    pred, target, k, dtype = make_inputs(args.workload, "cpu")
    steps = max(1, min(args.steps, REFERENCE_MAX_STEPS))
    warmup = max(1, min(args.warmup, REFERENCE_MAX_WARMUP))
    value, info = cpu_reference_sample(pred, target, k, steps, warmup, sample_volumes=args.cpu_sample_volumes)
    shape = WORKLOADS[args.workload][0]
    line = {
        "impl": "reference", "metric": metric_name(args.workload), "value": value, "unit": "Gvoxel/s", "n_gpus": world,
        "steps": steps, "warmup": warmup,
        "ms_per_step": info["seconds_per_step"] * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "shape": list(shape), "kernel_size": k,
                   "input_dtype": dtype, "sample_volumes": args.cpu_sample_volumes},
        "cpu_baseline": {"value": value, "unit": "Gvoxel/s", "cores": info["cores"], "kind": info["kind"],
                         "sample": info["sample"], "sample_volumes": args.cpu_sample_volumes,
                         "cpu_model": info["cpu_model"]},
        "e2e": {"value": value, "unit": "Gvoxel/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        # each step is a per-voxel rate measured on sample_volumes of the workload's volumes; at most
        # REFERENCE_MAX_STEPS steps after at most REFERENCE_MAX_WARMUP warm-up steps are timed
        "steps_requested": args.steps, "warmup_requested": args.warmup,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="headline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-volumes", type=int, default=2)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--kernel-only", action="store_true", help="only the C-ABI launch loop (profiling)")
    args = ap.parse_args()

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    args.warmup = max(3, args.warmup)

    import torch.distributed as dist
    import fused_lncc
    from fused_lncc import _lib
    from fused_lncc.dist import sharded_lncc_loss, volume_range

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    out_fd = 1
    if world > 1:
        # NCCL may print to the process's stdout (its version banner, for one); send all of that to
        # stderr so that stdout carries exactly the one JSON line, written through a saved descriptor
        sys.stdout.flush()
        out_fd = os.dup(1)
        os.dup2(2, 1)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)

    slabs = args.workload in SLAB_WORKLOADS
    # every rank builds the workload's one batch (seed 0) and keeps its share of it
    pred, target, k, dtype = make_inputs(args.workload, dev, seed=0)
    shape = WORKLOADS[args.workload][0]
    n, c = shape[:2]
    nvol = n * c
    input_sha = None
    if rank == 0 and args.workload in ("config1", "headline"):
        input_sha = {"pred": fused_lncc.synth.sha256_of(pred), "target": fused_lncc.synth.sha256_of(target)}
    m_global = float(nvol) * shape[2] * shape[3] * shape[4]
    if slabs:
        # one volume split into D-slabs; each rank keeps its owned planes plus 2r halo planes
        from fused_lncc.dist import SlabPlan, slab_lncc_loss
        plan = SlabPlan(shape[2], world, rank, k)
        lo, e = plan.own_range
        p_loc = torch.zeros((1, plan.depth, shape[3], shape[4]), dtype=pred.dtype, device=dev)
        t_loc = torch.zeros_like(p_loc)
        p_loc[:, lo:e] = pred.reshape(shape[2:])[None, plan.z0:plan.z1]
        t_loc[:, lo:e] = target.reshape(shape[2:])[None, plan.z0:plan.z1]
        p_loc.requires_grad_(True)
        b0, b1 = 0, 1
        z_rng = (lo, e)
        vox_local = plan.own * shape[3] * shape[4]
        parallelism = f"D-slabs/{world} (2r halo planes exchanged per side)"

        def loss_fn(p, t):
            return slab_lncc_loss(p, t, plan, k)
    else:
        b0, b1 = volume_range(nvol, world, rank)  # this rank's share of the batch's volumes
        vshape = (nvol, 1, *shape[2:])
        p_loc = pred.reshape(vshape)[b0:b1].contiguous().requires_grad_(True)
        t_loc = target.reshape(vshape)[b0:b1].contiguous()
        z_rng = (0, shape[2])
        vox_local = p_loc.numel()
        parallelism = f"volume-sharded/{world} ({b1 - b0} of {nvol} volumes per rank)"
        if world > 1:
            def loss_fn(p, t):
                return sharded_lncc_loss(p, t, k, m_global=m_global)
        else:
            def loss_fn(p, t):
                return fused_lncc.fused_lncc_loss(p, t, k)
    del pred, target
    torch.cuda.empty_cache()

    def step():
        p_loc.grad = None
        loss = loss_fn(p_loc, t_loc)
        loss.backward()
        return loss

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x):
        if world == 1:
            return x
        tt = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(local_rank)
    lib = _lib.load()
    esz = 4 if dtype == "fp32" else 2
    dtc = 0 if dtype == "fp32" else 1
    if slabs:
        nb, D, H, W = 1, p_loc.shape[1], shape[3], shape[4]
    else:
        nb, D, H, W = p_loc.shape[0], shape[2], shape[3], shape[4]
    ws_bytes = lib.lncc_workspace_bytes(nb, D, H, W, k, dtc, z_rng[0], z_rng[1])
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    gbuf = torch.empty((nb, z_rng[1] - z_rng[0], H, W), dtype=p_loc.dtype, device=dev)

    def kernel_launch():
        st = lib.lncc_fused_forward(p_loc.data_ptr(), t_loc.data_ptr(), dtc, nb, D, H, W, k, 1e-5,
                                    z_rng[0], z_rng[1], gbuf.data_ptr(), -1.0 / m_global, None,
                                    None, None, 1.0, ws.data_ptr(), ws_bytes, stream.cuda_stream)
        _lib.check(st, "bench launch")

    result = {}
    with sampler:
        if not args.kernel_only:
            # ---- value: the public fwd+bwd step, inputs resident in HBM ---------------------------------
            for _ in range(args.warmup):
                step()
            torch.cuda.synchronize(dev)
            barrier()
            torch.cuda.synchronize(dev)
            evs = []
            torch.cuda.nvtx.range_push("timed_steps")
            for _ in range(args.steps):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                step()
                e.record(stream)
                evs.append((s, e))
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize(dev)
            barrier()
            torch.cuda.synchronize(dev)
            ms_step = sum(s.elapsed_time(e) for s, e in evs) / len(evs)
            result["ms_step"] = max_over_ranks(ms_step)
            if world > 1 and not slabs:
                # weak scaling as well: every rank with a full batch of its own (its own seed), the
                # loss over all ranks' volumes
                pw, tw, _, _ = make_inputs(args.workload, dev, seed=1000 * (rank + 1))
                p_s = pw.reshape(vshape).contiguous().requires_grad_(True)
                t_s = tw.reshape(vshape).contiguous()
                del pw, tw
                m_weak = float(world * nvol) * shape[2] * shape[3] * shape[4]

                def step_weak():
                    p_s.grad = None
                    sharded_lncc_loss(p_s, t_s, k, m_global=m_weak).backward()

                for _ in range(args.warmup):
                    step_weak()
                torch.cuda.synchronize(dev)
                barrier()
                torch.cuda.synchronize(dev)
                sev = []
                for _ in range(args.steps):
                    flush.zero_()
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record(stream)
                    step_weak()
                    e.record(stream)
                    sev.append((s, e))
                torch.cuda.synchronize(dev)
                barrier()
                torch.cuda.synchronize(dev)
                ms_s = max_over_ranks(sum(s.elapsed_time(e) for s, e in sev) / len(sev))
                result["weak"] = {"value": m_weak / (ms_s * 1e-3) / 1e9, "unit": "Gvoxel/s",
                                  "ms_per_step": ms_s, "volumes_per_rank": nvol,
                                  "global_batch": world * nvol}
                del p_s, t_s
        # ---- roofline: the dominant kernel alone -----------------------------------------------------
        for _ in range(args.warmup):
            kernel_launch()
        torch.cuda.synchronize(dev)
        kev = []
        nk = max(args.steps, 20)
        torch.cuda.nvtx.range_push("timed_kernel")
        for _ in range(nk):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            kernel_launch()
            e.record(stream)
            kev.append((s, e))
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
        ms_kernel = sum(s.elapsed_time(e) for s, e in kev) / len(kev)
        result["ms_kernel"] = max_over_ranks(ms_kernel)
    clocks = sampler.summary()
    if args.kernel_only:
        if rank == 0:
            sys.stdout.flush()
            os.write(out_fd, (json.dumps({"kernel_only": True, "ms_kernel": result["ms_kernel"],
                                          "clocks": clocks}) + "\n").encode())
        if world > 1:
            dist.destroy_process_group()
        return 0

    # ---- e2e: public call with host buffers ---------------------------------------------------------
    # host copies of this rank's own voxels only (slab halos arrive over NCCL inside the step)
    own = (slice(None), slice(z_rng[0], z_rng[1])) if slabs else (slice(None),)
    p_host = p_loc.detach()[own].cpu().pin_memory()
    t_host = t_loc[own].cpu().pin_memory()
    p_dev = torch.zeros_like(p_loc).requires_grad_(True)
    t_dev = torch.zeros_like(t_loc)
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e_step():
        with torch.no_grad():
            p_dev[own].copy_(p_host, non_blocking=True)
            t_dev[own].copy_(t_host, non_blocking=True)
        p_dev.grad = None
        loss = loss_fn(p_dev, t_dev)
        loss.backward()
        loss_host.copy_(loss.detach(), non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    eev = []
    for _ in range(args.e2e_steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        e2e_step()
        e.record(stream)
        e.synchronize()
        eev.append(s.elapsed_time(e))
    barrier()
    ms_e2e = max_over_ranks(sum(eev) / len(eev))
    loss_val = float(loss_host.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, info = cpu_reference_sample(p_loc.detach(), t_loc, k, steps=3, warmup=1,
                                       sample_volumes=args.cpu_sample_volumes)
        cpu = {"value": v, "unit": "Gvoxel/s", "cores": info["cores"], "kind": info["kind"],
               "sample": info["sample"], "sample_volumes": args.cpu_sample_volumes,
               "cpu_model": info["cpu_model"]}

    if rank == 0:
        vox_global = m_global
        value = vox_global / (result["ms_step"] * 1e-3) / 1e9
        peak, peak_src = measured_peak_gbs()
        bpv = BYTES_PER_VOXEL[dtype]
        achieved = vox_local * bpv / (result["ms_kernel"] * 1e-3) / 1e9   # GB/s, rank 0's launch
        # which kernel the library picks for this shape (automatic choice, include/lncc.h): the
        # warp-specialised cluster kernel whenever W % 4 == 0 (torch allocations are aligned)
        kname = "lncc_ws_kernel" if W % 4 == 0 else "lncc_sweep_kernel"
        launches_per_call = max(1, lib.lncc_launch_count(nb, D, H, W, k, dtc, z_rng[0], z_rng[1], 1))
        traffic = profile_traffic(kname, args.workload) if world == 1 else None
        # the loss of a sharded step: one peer-memory reduction kernel of ours (else NCCL's all-reduce)
        from fused_lncc import dist as fdist
        peer_kernels = 1 if world > 1 and any(v is not None for v in fdist._PEER.values()) else 0
        line = {
            "metric": metric_name(args.workload), "value": value, "unit": "Gvoxel/s", "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": result["ms_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": args.workload, "shape": list(shape), "kernel_size": k,
                       "input_dtype": dtype, "volumes_per_rank": b1 - b0,
                       "global_batch": nvol,
                       "parallelism": parallelism, "l2": "flushed (256 MiB write) before every step",
                       "input_sha256": input_sha},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_src,
                         "traffic": traffic, "kernel": kname,
                         "algorithmic_bytes_per_voxel": bpv, "ms_per_launch": result["ms_kernel"],
                         "launches_per_call": launches_per_call},
            "e2e": {"value": vox_global / (ms_e2e * 1e-3) / 1e9, "unit": "Gvoxel/s",
                    "h2d_bytes_per_step": 2 * p_host.numel() * esz, "d2h_bytes_per_step": 4,
                    "ms_per_step": ms_e2e},
            # per compute call the fused kernel (plus its companion launch on idle SMs when the
            # library plans one) and the loss reduction, 3 calls per slab step when halos are
            # exchanged (to overlap the interior); plus the grad_out scale kernel and, at N > 1, the
            # peer-memory loss kernel
            "gpu_launches": ((launches_per_call + 1) * (3 if slabs and world > 1 else 1) + 1 + peer_kernels) * args.steps,
            "clocks": clocks,
            "loss": loss_val,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if "weak" in result:
            line["weak_scaling"] = result["weak"]
        sys.stdout.flush()
        os.write(out_fd, (json.dumps(line) + "\n").encode())
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
