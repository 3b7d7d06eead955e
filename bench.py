#!/usr/bin/env python
"""Benchmark of the submanifold sparse conv3d engine (one JSON line on rank 0).

Workload: one 3x3x3 submanifold conv at 256^3,
batch 1, a seeded union of 6 ellipsoid shells (~406k voxels), bf16 features
Ci = Co = 128, f32 accumulation.  One step = kernel-map build (hash probe,
neighbour-mask tile sort) + the fused tcgen05 conv, on inputs resident in HBM;
L2 is flushed (256 MB write) between steps outside the timed events.

Metric: active voxels per second (whole job; every rank runs its own replica
of the workload, data-parallel, so scaling is weak).  Extra keys report the conv
kernel's useful TFLOP/s (2*Ci*Co*M, M = valid (output, offset) pairs) against
the measured bf16 peak, the map-build time, the end-to-end number through the
public Python API with host buffers, a CPU baseline, and sampled clocks.

``--impl reference`` times the CPU restatement of the reference path
(flat-key sort + searchsorted map, 27 x gather-matmul-scatter conv on torch
CPU with all host threads) on the same workload: the reference's own
conv_none.py / hashmap_fallback.py are not in the reference tree, and its
WGSL path needs WebGPU, which these machines do not have.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "sparse conv3d active-voxels/sec and effective TFLOP/s; % of bf16 tensor peak"
UNIT = "voxels/s"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-steps", type=int, default=3, help="timed CPU-baseline steps (rank 0, N=1)")
    ap.add_argument("--c5-reserve-sms", type=int, default=-1,
                    help="c5 on >1 GPU: SMs left to NCCL while the interior conv runs beside the halo exchange; "
                         "-1 (default): exchange first, then one conv over all owned outputs (faster at 2 GPUs, "
                         "where the exchange is 0.04 ms)")
    ap.add_argument("--c5-exchange", choices=["nccl", "peer", "peer-conv-wait", "peer-interior-first"],
                    default="peer",
                    help="c5 on >1 GPU: halo exchange by the library's peer-memory push and wait kernels over NVLink, "
                         "then the conv (peer, default); the same push, then the conv waiting for the peers inside "
                         "its kernel before its first tile (peer-conv-wait) or, on the interior+boundary map, before "
                         "its first boundary tile (peer-interior-first); or NCCL all_to_all_single (nccl)")
    ap.add_argument("--workload", choices=["c2", "c5", "table"], default="c2",
                    help="c2: BASELINE configs[1] (default, data-parallel across ranks); "
                         "c5: configs[4] 1024^3 Morton-sharded across ranks with NCCL halo exchange (strong scaling)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_traffic():
    """DRAM bytes per conv launch from the committed ncu summary, if any."""
    try:
        with open(os.path.join(ROOT, "profiles", "conv_c2_traffic.json")) as f:
            return json.load(f)
    except OSError:
        return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "20",
                 "-i", str(self.dev), "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        # the timed region starts only once the sampler is producing rows
        t_end = time.time() + 10.0
        while time.time() < t_end and self.proc.poll() is None:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for ln in f:
                parts = [x.strip() for x in ln.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def make_inputs(rank):
    """configs[1] on every rank: N data-parallel replicas of the same seeded shape."""
    import numpy as np
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    w = pkg.workloads.make_workload(2)
    return w, np.ascontiguousarray(w.coords)


def cpu_reference_steps(w, steps, warmup):
    """Times the CPU restatement of the reference path on the full workload."""
    import torch
    from oracle import sparse_conv_ref as R
    torch.set_num_threads(os.cpu_count() or 1)
    coords = torch.from_numpy(w.coords)
    feats = torch.from_numpy(w.feats).to(torch.bfloat16).float()
    weight = torch.from_numpy(w.weight).to(torch.bfloat16).float()
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        km = R.torch_cpu_kmap(coords, w.spatial_shape)
        R.torch_cpu_conv(feats, km, weight)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    return times, torch.get_num_threads()


def run_reference(args):
    rank, _, _ = dist_env()
    if rank != 0:
        return 0
    w, _ = make_inputs(0)
    steps = max(1, min(args.steps, 5))
    warm = max(1, min(args.warmup, 1))
    times, cores = cpu_reference_steps(w, steps, warm)
    t = sum(times)
    value = w.n * len(times) / t
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": len(times), "warmup": warm, "ms_per_step": 1e3 * t / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded union of 6 ellipsoid shells at 256^3 (BASELINE configs[1])",
        "config": {"workload": w.name, "voxels": w.n, "ci": w.ci, "co": w.co, "step": "kernel map + conv",
                   "implementation": "CPU restatement (torch CPU: flat-key sort + searchsorted, "
                                     "27 x index_select/matmul/index_add_)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"full workload ({w.n} voxels), {len(times)} timed steps"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    rank, local_rank, world = dist_env()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    peaks, peak_src = measured_peaks()

    w, coords_np = make_inputs(rank)
    eng = pkg.get_engine(dev)
    coords = torch.from_numpy(coords_np).to(dev)
    feats = torch.from_numpy(w.feats).to(dev, torch.bfloat16)
    weight = torch.from_numpy(w.weight).to(dev, torch.bfloat16)
    out = torch.empty((w.n, w.co), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step():
        km = pkg.build_kmap(coords, engine=eng, check=False)
        pkg.conv3d(km, feats, weight, out=out)
        return km

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    km_check = step()
    km_check.check()
    info = km_check.info()
    eng.synchronize()
    del km_check

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        # ranks leave the barrier together, after their samplers are running
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = eng.launch_count()
        for k in range(args.steps):
            flush.zero_()
            ev[k][0].record()
            km = pkg.build_kmap(coords, engine=eng, check=False)
            ev[k][1].record()
            pkg.conv3d(km, feats, weight, out=out)
            ev[k][2].record()
            if k + 1 < args.steps:
                km.free()  # stream-ordered; the next step reuses the pooled memory
        torch.cuda.synchronize()
    launches = eng.launch_count() - launches0
    km.check()  # device status of the last build (all steps build the same coords)
    eng.synchronize()  # device status of the conv kernels
    del km
    t_total = sum(e[0].elapsed_time(e[2]) for e in ev) / 1e3
    t_map = sum(e[0].elapsed_time(e[1]) for e in ev) / 1e3
    t_conv = sum(e[1].elapsed_time(e[2]) for e in ev) / 1e3
    if dist is not None:
        tt = torch.tensor([t_total, t_map, t_conv], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_total, t_map, t_conv = tt.tolist()
        nv = torch.tensor([w.n], device=dev, dtype=torch.float64)
        dist.all_reduce(nv)
        n_all = float(nv.item())
    else:
        n_all = float(w.n)
    value = n_all * args.steps / t_total

    # conv kernel roofline (useful flops only: padded tile rows earn nothing)
    flops = 2.0 * w.ci * w.co * info["num_pairs"]
    conv_s = t_conv / args.steps
    achieved = flops / conv_s / 1e12
    peak = float(peaks["bf16_tflops"])
    traffic = load_traffic()

    # end to end through the public API with host buffers: HostConvPipeline runs
    # every step's H2D copy, map build + conv and D2H copy, overlapping the
    # transfers of consecutive steps on separate streams
    coords_h = torch.from_numpy(coords_np).pin_memory()
    feats_h = torch.from_numpy(w.feats).to(torch.bfloat16).pin_memory()
    out_h = torch.empty((w.n, w.co), dtype=torch.bfloat16).pin_memory()
    pipe = pkg.HostConvPipeline(weight, depth=3)  # model parameters stay resident
    for _ in range(3):
        pipe.submit(coords_h, feats_h, out_h)
    pipe.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, args.steps // 2)
    e0.record(pipe.s_in)
    for _ in range(e2e_steps):
        pipe.submit(coords_h, feats_h, out_h)
    e1.record(pipe.s_out)
    pipe.synchronize()
    t_e2e = e0.elapsed_time(e1) / 1e3
    if dist is not None:
        tt = torch.tensor([t_e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_e2e = float(tt.item())
    e2e_value = n_all * e2e_steps / t_e2e
    h2d = coords_h.numel() * 4 + feats_h.numel() * 2
    d2h = out_h.numel() * 2
    ref_out = out_h.clone()
    o_chk = pkg.conv3d(pkg.build_kmap(coords, engine=eng), feats, weight)
    e2e_matches = bool(torch.equal(o_chk.cpu(), ref_out))

    # CPU baseline (rank 0, single GPU only)
    cpu = None
    if rank == 0 and world == 1 and args.cpu_steps > 0:
        times, cores = cpu_reference_steps(w, args.cpu_steps, 1)
        cpu = {"value": w.n * len(times) / sum(times), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"full workload ({w.n} voxels), {len(times)} timed steps after 1 warm-up, "
                         f"torch CPU restatement with {cores} threads"}

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded union of 6 ellipsoid shells at 256^3 (BASELINE configs[1]); the same shape on every rank",
        "config": {"workload": w.name, "voxels_per_rank": w.n, "ci": w.ci, "co": w.co, "kernel": "3x3x3 submanifold",
                   "pairs": info["num_pairs"], "tile_pairs": info["tile_pairs"],
                   "step": "kernel-map build (hash probe + mask-sorted tiles) + fused tcgen05 conv",
                   "l2": "flushed between steps by a 256 MB write outside the timed events",
                   "parallelism": f"data-parallel x{world} (one replica of the workload per rank)"},
        "map_build_ms": 1e3 * t_map / args.steps, "conv_ms": 1e3 * conv_s,
        "conv_tflops": achieved, "conv_pct_of_bf16_peak": 100.0 * achieved / peak,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": f"{peak_src} bf16_tflops (burst)",
                     "kernel": "conv_tc_kernel", "units": "2*Ci*Co*M useful flops per launch",
                     "traffic": (traffic or {}).get("dram_bytes_per_launch")},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "matches_device_api": e2e_matches,
                "api": "HostConvPipeline.submit: per step H2D of coords+feats from pinned memory, map build + conv, "
                       "D2H of the output; consecutive steps overlap on 3 streams (depth 3)"},
        "clocks": clk.summary(),
        "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_c5(args):
    """one 1024^3 shape (6.1M voxels, Ci=Co=32) Morton-sharded over the ranks.

    Every rank generates the same seeded shape, keeps its Morton range, builds
    its halo plan and owned-output map once (cached per coord set, as the
    reference caches neighbour maps), then each timed step is one conv layer:
    halo exchange (NCCL all_to_all_single) + conv on owned outputs.
    """
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from sparseconv_b200 import sharding as S
    rank, local_rank, world = dist_env()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    peaks, peak_src = measured_peaks()
    w = pkg.workloads.make_workload(5)
    eng = pkg.get_engine(dev)
    coords = torch.from_numpy(w.coords).to(dev)
    feats = torch.from_numpy(w.feats).to(dev, torch.bfloat16)
    weight = torch.from_numpy(w.weight).to(dev, torch.bfloat16)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for _ in range(2):  # the first pass warms the stream-ordered memory pool
      t0.record()
      if world > 1:
        part = S.MortonPartition.balanced(coords, world)
        own = part.owned_rows(coords, rank)
        own_c = coords.index_select(0, own).contiguous()
        plan = S.build_halo_plan(own_c, part, rank, world)
        loc_c = S.local_coords(plan, own_c)
        own_f = feats.index_select(0, S.owned_local(plan, own)).contiguous()
        buf = torch.empty((plan.n_own + plan.n_halo, w.ci), dtype=torch.bfloat16, device=dev)
        buf[:plan.n_own].copy_(own_f)
        n_own, n_halo, n_int = plan.n_own, plan.n_halo, plan.n_interior
        km_i = pkg.build_kmap(loc_c, n_out=n_int, engine=eng)
        km_b = pkg.build_kmap(loc_c, out_begin=n_int, n_out=n_own - n_int, engine=eng)
        kms = [km_i, km_b]
      else:
        plan, loc_c, buf, n_own, n_halo, n_int = None, coords, feats, w.n, 0, w.n
        kms = [pkg.build_kmap(loc_c, engine=eng)]
      t1.record()
      torch.cuda.synchronize()
      setup_ms = t0.elapsed_time(t1)
    infos = [km.info() for km in kms]
    out = torch.empty((n_own, w.co), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    reserve = args.c5_reserve_sms  # SMs left to the NCCL kernels while the interior conv runs
    peer = None
    in_kernel_wait = plan is not None and args.c5_exchange in ("peer-conv-wait", "peer-interior-first")
    if plan is not None and args.c5_exchange == "peer-interior-first":
        kms = [pkg.concat_kmaps(km_i, km_b)]  # interior tiles, then boundary tiles
    elif plan is not None and (reserve < 0 or args.c5_exchange.startswith("peer")):
        kms = [pkg.build_kmap(loc_c, n_out=n_own, engine=eng)]
    if plan is not None and args.c5_exchange.startswith("peer"):
        peer = S.PeerHaloExchange(plan, own_f, eng)

    def layer(ev=None):
        """Halo exchange beside the interior conv, then the boundary conv."""
        if in_kernel_wait:
            loc, hw = peer.push()
            if ev: ev[1].record()
            pkg.conv3d(kms[0], loc, weight, out=out, halo_wait=hw)
            return
        if peer is not None:
            loc = peer.exchange()
            if ev: ev[1].record()
            pkg.conv3d(kms[0], loc, weight, out=out)
            return
        if plan is None or reserve < 0:
            if plan is not None:
                S.exchange_halo(plan, buf[:n_own], out=buf)
            if ev: ev[1].record()
            pkg.conv3d(kms[0], buf, weight, out=out)
            return
        _, work = S.exchange_halo(plan, buf[:n_own], out=buf, async_op=True)
        eng.set_conv_ctas(n_sms - reserve)
        pkg.conv3d(kms[0], buf, weight, out=out[:n_int])
        eng.set_conv_ctas(0)
        work.wait()
        if ev: ev[1].record()
        pkg.conv3d(kms[1], buf, weight, out=out[n_int:])

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        layer()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        # ranks leave the barrier together, after their samplers are running
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = eng.launch_count()
        for k in range(args.steps):
            flush.zero_()
            ev[k][0].record()
            layer(ev[k])
            ev[k][2].record()
        torch.cuda.synchronize()
    launches = eng.launch_count() - launches0
    eng.synchronize()
    if peer is not None:
        peer.close()
    t_total = sum(e[0].elapsed_time(e[2]) for e in ev) / 1e3
    t_first = sum(e[0].elapsed_time(e[1]) for e in ev) / 1e3  # exchange (+ interior conv when overlapped)
    t_last = sum(e[1].elapsed_time(e[2]) for e in ev) / 1e3   # boundary conv
    per_rank = [t_total]
    if dist is not None:
        allt = [torch.zeros(1, device=dev, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(allt, torch.tensor([t_total], device=dev, dtype=torch.float64))
        per_rank = [float(x.item()) for x in allt]
        tt = torch.tensor([t_total, t_first, t_last, setup_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_total, t_first, t_last, setup_ms = tt.tolist()
        hh = torch.tensor([n_halo, sum(i["num_pairs"] for i in infos), n_int], device=dev, dtype=torch.float64)
        dist.all_reduce(hh)
        halo_total, pairs, int_total = int(hh[0]), int(hh[1]), int(hh[2])
        dist.barrier()
        dist.destroy_process_group()
    else:
        halo_total, pairs, int_total = 0, infos[0]["num_pairs"], w.n
    if rank != 0:
        return 0
    value = w.n * args.steps / t_total
    flops = 2.0 * w.ci * w.co * pairs
    achieved_gbs = (w.n * (w.ci + w.co) * 2) / (t_total / args.steps) / 1e9  # all ranks together
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded union of 4 ellipsoid shells + 5% interior fill at 1024^3 (BASELINE configs[4])",
        "config": {"workload": w.name, "voxels": w.n, "ci": w.ci, "co": w.co, "pairs": pairs,
                   "halo_voxels_total": halo_total, "interior_voxels_total": int_total,
                   "step": ("halo push kernel over NVLink (peer memory), then one conv of all owned outputs that "
                            "runs its interior tiles first and waits for the peers' pushes inside the kernel before "
                            "its boundary tiles" if args.c5_exchange == "peer-interior-first" and world > 1 else
                            "halo push kernel over NVLink (peer memory), then one conv of all owned outputs that "
                            "waits for the peers' pushes inside the kernel before its first tile" if in_kernel_wait else
                            "halo exchange by peer-memory push/wait kernels over NVLink, then the conv of all "
                            "owned outputs" if peer is not None else
                            "halo exchange (NCCL all_to_all_single), then the conv of all owned outputs"
                            if reserve < 0 or world == 1 else
                            "halo exchange (NCCL all_to_all_single) beside the conv of interior outputs "
                            f"(on {n_sms - reserve} of {n_sms} SMs), then the conv of boundary outputs") +
                           "; plan and maps built once per coord set",
                   "l2": "flushed between steps by a 256 MB write outside the timed events",
                   "parallelism": f"Morton-range sharding x{world}"},
        "setup_ms": setup_ms,
        "phases": ("exchange_and_interior_ms = the push kernel, boundary_ms = the conv with its in-kernel wait"
                   if in_kernel_wait else "exchange_and_interior_ms = exchange (+ interior conv when overlapped), "
                   "boundary_ms = the conv after it"),
        "exchange_and_interior_ms": 1e3 * t_first / args.steps,
        "boundary_ms": 1e3 * t_last / args.steps, "ms_per_step_by_rank": [1e3 * t / args.steps for t in per_rank],
        "conv_tflops_total": flops / (t_total / args.steps) / 1e12,
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": float(peaks["hbm_gbs"]) * world,
                     "unit": "GB/s", "frac": achieved_gbs / (float(peaks["hbm_gbs"]) * world),
                     "peak_source": f"{peak_src} hbm_gbs x n_gpus",
                     "units": "feature bytes in + out (N*(Ci+Co)*2) per layer step, summed over ranks"},
        "clocks": clk.summary(), "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def _cpu_chain(idx, w, sample_rows):
    """One CPU step of config `idx` (torch CPU restatement) on the first `sample_rows`
    Morton-ordered voxels; returns (seconds, pairs-in-sample)."""
    import numpy as np
    import torch
    from oracle import sparse_conv_ref as R
    n = min(w.n, sample_rows)
    c_np = np.ascontiguousarray(w.coords[:n])
    coords = torch.from_numpy(c_np)
    f = torch.from_numpy(w.feats[:n]).float()
    wt = lambda a: torch.from_numpy(np.asarray(a)).to(torch.bfloat16).float()
    t0 = time.perf_counter()
    if idx == 4:
        parents, dmap = R.down2_map(c_np)
        h = R.torch_cpu_conv(f, torch.from_numpy(dmap), wt(w.weight))
        km = R.torch_cpu_kmap(torch.from_numpy(parents), tuple(s // 2 for s in w.spatial_shape))
        h = R.torch_cpu_conv(h, km, wt(w.extra["w_sub"]))
        umap = R.up2_map(c_np, parents)
        R.torch_cpu_conv(h, torch.from_numpy(umap), wt(w.extra["w_up"]))
        pairs = int((dmap >= 0).sum() + (km >= 0).sum() + (umap >= 0).sum())
    else:
        km = R.torch_cpu_kmap(coords, w.spatial_shape)
        W = torch.from_numpy(w.weight) if idx == 1 else wt(w.weight)
        h = R.torch_cpu_conv(f, km, W)
        if idx == 3:
            h = torch.nn.functional.layer_norm(h, (h.shape[1],), eps=1e-6)
            h = torch.nn.functional.silu(h)
            h = R.torch_cpu_conv(h, km, wt(w.extra["weight2"])) + f
        pairs = int((km >= 0).sum())
    return time.perf_counter() - t0, pairs, n


def run_table(args):
    """Every BASELINE config on one GPU: map build and conv chain (median of CUDA-event
    times, L2 flushed before each step), next to the CPU restatement on a bounded
    Morton-prefix sample.  One JSON line per config; not the driver's headline line."""
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.set_num_threads(os.cpu_count() or 1)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, peak_src = measured_peaks()
    eng = pkg.get_engine(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    steps = max(args.steps, 5)
    for idx in (1, 2, 3, 4, 5):
        w = pkg.workloads.make_workload(idx)
        dt = torch.float32 if w.dtype == "f32" else torch.bfloat16
        coords = torch.from_numpy(w.coords).to(dev)
        feats = torch.from_numpy(w.feats).to(dev, dt)
        dW = lambda a: torch.from_numpy(np.asarray(a)).to(dev, dt)
        W1 = dW(w.weight)

        def build():
            if idx == 4:
                d = pkg.build_down2(coords, engine=eng)
                s = pkg.build_kmap(d.out_coords(), engine=eng, check=False)
                return (d, s, pkg.build_up2(d))
            return (pkg.build_kmap(coords, engine=eng, check=False),)

        if idx == 3:
            W2 = dW(w.extra["weight2"])
            conv = lambda m: pkg.conv3d(m[0], pkg.conv3d(m[0], feats, W1, silu=True, layernorm=True), W2,
                                        residual=feats)
        elif idx == 4:
            Ws, Wu = dW(w.extra["w_sub"]), dW(w.extra["w_up"])
            conv = lambda m: pkg.conv3d(m[2], pkg.conv3d(m[1], pkg.conv3d(m[0], feats, W1), Ws), Wu)
        else:
            conv = lambda m: pkg.conv3d(m[0], feats, W1)
        t_map, t_conv = [], []
        for k in range(3 + steps):
            flush.zero_()
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record()
            maps = build()
            e[1].record()
            conv(maps)
            e[2].record()
            torch.cuda.synchronize()
            if k >= 3:
                t_map.append(e[0].elapsed_time(e[1]))
                t_conv.append(e[1].elapsed_time(e[2]))
            if k < 2 + steps:
                del maps
        eng.synchronize()
        infos = [m.info() for m in maps]
        chans = {1: [(64, 64)], 2: [(128, 128)], 3: [(256, 256), (256, 256)], 5: [(32, 32)],
                 4: [(64, 128), (128, 128), (128, 64)]}[idx]
        if idx == 3:
            infos = infos * 2
        flops = sum(2.0 * ci * co * inf["num_pairs"] for (ci, co), inf in zip(chans, infos))
        gm, gc = statistics.median(t_map), statistics.median(t_conv)
        del maps
        cpu_runs = [_cpu_chain(idx, w, 400_000) for _ in range(2 + 5)][2:]  # 2 warm-ups, median of 5
        cpu_s, cpu_n = statistics.median(r[0] for r in cpu_runs), cpu_runs[0][2]
        cpu_full_ms = 1e3 * cpu_s * (w.n / cpu_n)
        line = {
            "table": w.name, "voxels": w.n, "pairs": [inf["num_pairs"] for inf in infos],
            "dtype": w.dtype, "gpu_map_ms": gm, "gpu_conv_ms": gc, "gpu_total_ms": gm + gc,
            "conv_tflops": flops / (gc * 1e-3) / 1e12,
            "conv_pct_of_bf16_peak": 100.0 * flops / (gc * 1e-3) / 1e12 / float(peaks["bf16_tflops"]),
            "peak_source": f"{peak_src} bf16_tflops (burst)",
            "gpu_voxels_per_s": w.n / ((gm + gc) * 1e-3),
            "cpu_ms": cpu_full_ms, "cpu_threads": torch.get_num_threads(), "cpu_runs": "median of 5 after 2 warm-ups",
            "cpu_sample": ("full workload" if cpu_n == w.n else
                           f"first {cpu_n} Morton-ordered voxels, time scaled by {w.n / cpu_n:.2f}"),
            "speedup_vs_cpu": cpu_full_ms / (gm + gc), "steps": steps,
            "chain": {1: "map + conv (f32 SIMT path)", 2: "map + conv", 3: "map + conv(LN,SiLU) + conv(+skip)",
                      4: "down map + subm map + up map; down 64->128, subm 128, up 128->64",
                      5: "map + conv"}[idx],
        }
        print(json.dumps(line), flush=True)
        del coords, feats
        torch.cuda.empty_cache()
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "c5":
        return run_c5(args)
    if args.workload == "table":
        return run_table(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
