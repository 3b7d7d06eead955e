#!/usr/bin/env python
"""Benchmark of the submanifold sparse conv3d engine (one JSON line on rank 0).

Workload: one 3x3x3 submanifold conv at 256^3,
batch 1, a seeded union of 6 ellipsoid shells (~406k voxels), bf16 features
Ci = Co = 128, f32 accumulation.  One step = kernel-map build (hash probe,
neighbour-mask tile sort) + the fused tcgen05 conv, on inputs resident in HBM;
L2 is flushed (256 MB write) between steps outside the timed events.

* N = 1: the whole workload on one GPU.
* N > 1 (default): the same workload strong-scaled over the ranks: Morton-range
  partition and halo plan once per coord set (outside the timed steps, like
  the reference's cached neighbour map), then per step every rank builds the
  map of its owned outputs, exchanges the one-voxel halo of input features
  over NVLink (peer-memory push/wait kernels) and runs the conv of its owned
  outputs.  Outside the timed region every rank checks its owned outputs
  against a one-GPU conv of the whole workload, bit for bit
  (``sharded_parity``).  ``--replicas`` instead runs one independent replica
  of the workload per rank (weak scaling, no exchange).
* Every N also reports a ``c5`` block: BASELINE.json configs[4] (1024^3,
  6.1M voxels, Ci = Co = 32) Morton-sharded the same way, one conv layer per
  step with the map built once per coord set.

Metric: active voxels per second over the whole job.  Extra keys report the
conv kernel's useful TFLOP/s (2*Ci*Co*M, M = valid (output, offset) pairs)
against the measured bf16 peak, the map-build time, the end-to-end number
through the public Python API with host buffers, a CPU baseline, and sampled
clocks.

``--impl reference`` times the CPU restatement of the reference path
(flat-key sort + searchsorted map, 27 x gather-matmul-scatter conv on torch
CPU with all host threads) on the same workload and config: the reference's
own conv_none.py / hashmap_fallback.py are not in the reference tree, and its
WGSL path needs WebGPU, which these machines do not have.

Other workloads: ``--workload c3`` (configs[2]: 4 ResBlock shapes split
data-parallel over the ranks by greedy LPT on voxel count), ``--workload c4``
(configs[3]: 512^3 down -> subm -> up, Morton-sharded, halo exchange only for
the coarse submanifold conv), ``--workload c5`` (configs[4] alone),
``--workload table`` (every config on one GPU next to its CPU sample).
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
    ap.add_argument("--replicas", action="store_true",
                    help="N>1: one independent replica of the workload per rank (weak scaling, no exchange) "
                         "instead of the Morton-sharded strong-scaling run")
    ap.add_argument("--no-c5", action="store_true", help="skip the c5 (1024^3) block of the default run")
    ap.add_argument("--c5-steps", type=int, default=20, help="timed layer steps of the c5 block")
    ap.add_argument("--c5-reserve-sms", type=int, default=-1,
                    help="c5 with --c5-exchange nccl on >1 GPU: SMs left to NCCL while the interior conv runs "
                         "beside the halo exchange; -1 (default): exchange first, then one conv over all owned "
                         "outputs")
    ap.add_argument("--c5-exchange", choices=["nccl", "peer", "peer-conv-wait", "peer-interior-first"],
                    default="peer",
                    help="sharded convs on >1 GPU: halo exchange by the library's peer-memory push and wait kernels "
                         "over NVLink, then the conv (peer, default); the same push, then the conv waiting for the "
                         "peers inside its kernel before its first tile (peer-conv-wait) or, on the "
                         "interior+boundary map, before its first boundary tile (peer-interior-first); or NCCL "
                         "all_to_all_single (nccl)")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5", "table", "dec", "attn"], default="c2",
                    help="c2: BASELINE configs[1] (default); c3: configs[2] ResBlock batch, data-parallel; "
                         "c4: configs[3] down/subm/up, Morton-sharded; c5: configs[4] 1024^3, Morton-sharded; "
                         "table: every config on one GPU; dec: the decoder rows (ConvNeXt block with a depthwise "
                         "conv, 2x2x2 subdivision) on configs[1]'s voxels, one GPU; attn: varlen attention of the "
                         "SLat flow model (16 heads of 64, two sequences of 10,000 and 6,384 tokens), one GPU")
    ap.add_argument("--map-mode", choices=["hash", "sort"], default="hash",
                    help="c2 on one GPU / replicas: kernel-map construction by hash probe (default) or radix sort")
    ap.add_argument("--halo-map", action="store_true",
                    help="c2 on one GPU / replicas: build the map with SC_BUILD_HALO (row-order tiles, halo-staged "
                         "conv)")
    ap.add_argument("--configs", default="1,2,3,4,5", help="table: which BASELINE configs (1-based, comma list)")
    ap.add_argument("--dec-channels", type=int, default=64, help="dec: channels of the ConvNeXt block")
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


L2_NOTE = "flushed between steps by a 256 MB write outside the timed events"


def c2_config(w, world, pairs, replicas=False):
    """The ``config`` object of the default workload; both arms print the same one."""
    if world == 1:
        par, step = "single GPU", "kernel-map build + conv"
    elif replicas:
        par, step = f"data-parallel x{world} (one replica of the workload per rank)", "kernel-map build + conv"
    else:
        par = f"Morton-range sharding x{world} (strong scaling)"
        step = "owned-output kernel-map build + halo exchange + conv (partition and halo plan once per coord set)"
    return {"workload": w.name, "voxels": w.n, "ci": w.ci, "co": w.co, "kernel": "3x3x3 submanifold",
            "pairs": int(pairs), "step": step, "l2": L2_NOTE, "parallelism": par}


def make_inputs(rank):
    """configs[1], the same seeded shape on every rank."""
    import numpy as np
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    w = pkg.workloads.make_workload(2)
    return w, np.ascontiguousarray(w.coords)


def cpu_reference_steps(w, steps, warmup):
    """Times the CPU restatement of the reference path on the full workload;
    returns (seconds per timed step, threads, valid pairs of the map)."""
    import torch
    from oracle import sparse_conv_ref as R
    torch.set_num_threads(os.cpu_count() or 1)
    coords = torch.from_numpy(w.coords)
    feats = torch.from_numpy(w.feats).to(torch.bfloat16).float()
    weight = torch.from_numpy(w.weight).to(torch.bfloat16).float()
    times, pairs = [], 0
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        km = R.torch_cpu_kmap(coords, w.spatial_shape)
        R.torch_cpu_conv(feats, km, weight)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
        pairs = int((km >= 0).sum())
    return times, torch.get_num_threads(), pairs


def run_reference(args):
    """The reference arm: the CPU restatement of the reference path (the
    reference's own conv_none.py / hashmap_fallback.py are absent), honouring
    --steps / --warmup, with the same metric, unit and config as our arm."""
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    w, _ = make_inputs(0)
    steps, warm = max(1, args.steps), max(0, args.warmup)
    times, cores, pairs = cpu_reference_steps(w, steps, warm)
    t = sum(times)
    value = w.n * len(times) / t
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": len(times), "warmup": warm, "ms_per_step": 1e3 * t / len(times), "higher_is_better": True,
        "scaling": "weak" if world == 1 or args.replicas else "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded union of 6 ellipsoid shells at 256^3 (BASELINE configs[1])",
        "config": c2_config(w, world, pairs, args.replicas),
        "implementation": "CPU restatement of conv_none.py + hashmap_fallback.py (torch CPU: flat-key sort + "
                          "searchsorted map, 27 x index_select/matmul/index_add_ conv), all host threads; "
                          "inputs rounded to bf16, computed in f32",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"full workload ({w.n} voxels) per step, {len(times)} timed steps after "
                                   f"{warm} warm-up"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def init_dist(dev, world, seconds=300):
    if world == 1:
        return None
    import torch.distributed as dist
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=seconds), device_id=dev)
    return dist


def max_over_ranks(dist, dev, values):
    import torch
    if dist is None:
        return list(values)
    tt = torch.tensor(list(values), device=dev, dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    return tt.tolist()


def sum_over_ranks(dist, dev, values):
    import torch
    if dist is None:
        return list(values)
    tt = torch.tensor(list(values), device=dev, dtype=torch.float64)
    dist.all_reduce(tt)
    return tt.tolist()


def roofline_conv(ci, co, pairs, conv_s, peaks, peak_src):
    flops = 2.0 * ci * co * pairs
    achieved = flops / conv_s / 1e12
    peak = float(peaks["bf16_tflops"])
    traffic = load_traffic()
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{peak_src} bf16_tflops (burst)", "kernel": "conv_tc_kernel",
            "units": "2*Ci*Co*M useful flops per launch",
            "traffic": (traffic or {}).get("dram_bytes_per_launch"),
            "traffic_source": ((traffic or {}).get("source") or "no committed ncu capture")}


def run_ours(args):
    """Default workload.  N=1 or --replicas: the whole workload per rank; N>1:
    strong scaling through the Morton-sharded path (run_sharded_c2)."""
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    rank, local_rank, world = dist_env()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = init_dist(dev, world, 180)
    if world > 1 and not args.replicas:
        return run_sharded_c2(args, pkg, dist, rank, world, dev)
    peaks, peak_src = measured_peaks()

    w, coords_np = make_inputs(rank)
    eng = pkg.get_engine(dev, map_mode=args.map_mode)
    coords = torch.from_numpy(coords_np).to(dev)
    feats = torch.from_numpy(w.feats).to(dev, torch.bfloat16)
    weight = torch.from_numpy(w.weight).to(dev, torch.bfloat16)
    out = torch.empty((w.n, w.co), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step():
        km = pkg.build_kmap(coords, engine=eng, check=False, halo=args.halo_map)
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
            km = pkg.build_kmap(coords, engine=eng, check=False, halo=args.halo_map)
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
    t_total, t_map, t_conv = max_over_ranks(dist, dev, [t_total, t_map, t_conv])
    n_all = sum_over_ranks(dist, dev, [float(w.n)])[0]
    value = n_all * args.steps / t_total
    conv_s = t_conv / args.steps
    roof = roofline_conv(w.ci, w.co, info["num_pairs"], conv_s, peaks, peak_src)

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
    t_e2e = max_over_ranks(dist, dev, [e0.elapsed_time(e1) / 1e3])[0]
    e2e_value = n_all * e2e_steps / t_e2e
    h2d = coords_h.numel() * 4 + feats_h.numel() * 2
    d2h = out_h.numel() * 2
    ref_out = out_h.clone()
    o_chk = pkg.conv3d(pkg.build_kmap(coords, engine=eng, halo=args.halo_map), feats, weight)
    e2e_matches = bool(torch.equal(o_chk.cpu(), ref_out))

    c5 = None if args.no_c5 else c5_block(args, pkg, dist, rank, world, dev, eng, peaks, peak_src)

    # CPU baseline (rank 0, single GPU only)
    cpu = None
    if rank == 0 and world == 1 and args.cpu_steps > 0:
        times, cores, _ = cpu_reference_steps(w, args.cpu_steps, 1)
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
        "data": "synthetic: seeded union of 6 ellipsoid shells at 256^3 (BASELINE configs[1]); the same shape "
                "on every rank",
        "config": dict(c2_config(w, world, info["num_pairs"], args.replicas),
                       **({"map_mode": args.map_mode} if args.map_mode != "hash" else {}),
                       **({"map_layout": "SC_BUILD_HALO"} if args.halo_map else {})),
        "tile_pairs": info["tile_pairs"],
        "map_build_ms": 1e3 * t_map / args.steps, "conv_ms": 1e3 * conv_s,
        "conv_tflops": roof["achieved"], "conv_pct_of_bf16_peak": 100.0 * roof["frac"],
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "matches_device_api": e2e_matches,
                "api": "HostConvPipeline.submit: per step H2D of coords+feats from pinned memory, map build + conv, "
                       "D2H of the output; consecutive steps overlap on 3 streams (depth 3)"},
        "c5": c5,
        "clocks": clk.summary(),
        "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def shard_setup(pkg, S, coords, feats, world, rank, eng, exchange="peer"):
    """Morton partition, halo plan and (peer) exchange of one coord set: the
    per-coord-set work, done once like the reference's cached neighbour map."""
    part = S.MortonPartition.balanced(coords, world)
    own = part.owned_rows(coords, rank)
    own_c = coords.index_select(0, own).contiguous()
    plan = S.build_halo_plan(own_c, part, rank, world)
    loc_c = S.local_coords(plan, own_c)
    own_f = feats.index_select(0, S.owned_local(plan, own)).contiguous()
    peer = S.PeerHaloExchange(plan, own_f, eng) if exchange.startswith("peer") else None
    return part, own, plan, loc_c, own_f, peer


def run_sharded_c2(args, pkg, dist, rank, world, dev):
    """configs[1] strong-scaled over the ranks (Morton ranges, one-voxel halo over NVLink)."""
    import torch
    from sparseconv_b200 import sharding as S
    peaks, peak_src = measured_peaks()
    w, coords_np = make_inputs(rank)
    eng = pkg.get_engine(dev, map_mode=args.map_mode)
    coords = torch.from_numpy(coords_np).to(dev)
    feats = torch.from_numpy(w.feats).to(dev, torch.bfloat16)
    weight = torch.from_numpy(w.weight).to(dev, torch.bfloat16)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    part, own, plan, loc_c, own_f, peer = shard_setup(pkg, S, coords, feats, world, rank, eng)
    t1.record()
    torch.cuda.synchronize()
    setup_ms = t0.elapsed_time(t1)
    out = torch.empty((plan.n_own, w.co), dtype=torch.bfloat16, device=dev)

    def step(ev=None):
        if ev:
            ev[0].record()
        km = pkg.build_kmap(loc_c, n_out=plan.n_own, engine=eng, check=False)
        if ev:
            ev[1].record()
        loc = peer.exchange()
        if ev:
            ev[2].record()
        pkg.conv3d(km, loc, weight, out=out)
        if ev:
            ev[3].record()
        return km

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step().free()
    torch.cuda.synchronize()
    km = step()
    km.check()
    info = km.info()
    eng.synchronize()
    km.free()

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        dist.barrier()
        torch.cuda.synchronize()
        launches0 = eng.launch_count()
        for k in range(args.steps):
            flush.zero_()
            km = step(ev[k])
            if k + 1 < args.steps:
                km.free()
        torch.cuda.synchronize()
    launches = eng.launch_count() - launches0
    km.check()
    eng.synchronize()
    km.free()
    seg = [sum(e[i].elapsed_time(e[i + 1]) for e in ev) / 1e3 for i in range(3)]
    t_total = sum(e[0].elapsed_time(e[3]) for e in ev) / 1e3
    per_rank = [torch.zeros(1, device=dev, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(per_rank, torch.tensor([t_total], device=dev, dtype=torch.float64))
    per_rank = [1e3 * float(x.item()) / args.steps for x in per_rank]
    conv_rank0_s = seg[2] / args.steps
    pairs_rank0 = info["num_pairs"]
    t_total, t_map, t_exch, t_conv, setup_ms = max_over_ranks(dist, dev, [t_total] + seg + [setup_ms])
    pairs_all, halo_all = sum_over_ranks(dist, dev, [float(info["num_pairs"]), float(plan.n_halo)])
    value = w.n * args.steps / t_total

    # bit-exact check of every rank's owned outputs against a one-GPU conv of the whole workload
    full = pkg.conv3d(pkg.build_kmap(coords, engine=eng), feats, weight)
    ok = torch.equal(out, full.index_select(0, own.index_select(0, plan.order)))
    okt = torch.tensor([1 if ok else 0], device=dev, dtype=torch.int32)
    dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    parity = bool(okt.item())
    del full

    # end to end through the public API: per step H2D of this rank's owned
    # coords and features from pinned memory, owned-output map build, halo
    # exchange, conv, D2H of the owned outputs (the plan is per coord set)
    own_c_h = loc_c[:plan.n_own].cpu().pin_memory()
    own_f_h = own_f.cpu().pin_memory()
    out_h = torch.empty((plan.n_own, w.co), dtype=torch.bfloat16).pin_memory()
    loc_d = loc_c.clone()

    def e2e_step():
        loc_d[:plan.n_own].copy_(own_c_h, non_blocking=True)
        peer.next_owned_rows().copy_(own_f_h, non_blocking=True)
        k = pkg.build_kmap(loc_d, n_out=plan.n_own, engine=eng, check=False)
        loc = peer.exchange()
        pkg.conv3d(k, loc, weight, out=out)
        out_h.copy_(out, non_blocking=True)
        return k

    for _ in range(3):
        e2e_step().free()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, args.steps // 2)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step().free()
    e1.record()
    torch.cuda.synchronize()
    t_e2e = max_over_ranks(dist, dev, [e0.elapsed_time(e1) / 1e3])[0]
    e2e_ok = torch.equal(out_h, out.cpu())
    h2d = own_c_h.numel() * 4 + own_f_h.numel() * 2
    d2h = out_h.numel() * 2
    h2d, d2h = sum_over_ranks(dist, dev, [float(h2d), float(d2h)])

    c5 = None if args.no_c5 else c5_block(args, pkg, dist, rank, world, dev, eng, peaks, peak_src)
    peer.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return 0
    roof = roofline_conv(w.ci, w.co, pairs_rank0, conv_rank0_s, peaks, peak_src)
    roof["kernel"] = "conv_tc_kernel (rank 0's shard)"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded union of 6 ellipsoid shells at 256^3 (BASELINE configs[1]), one shape "
                "partitioned over the ranks",
        "config": c2_config(w, world, int(pairs_all)),
        "sharded_parity": parity,
        "halo_voxels_total": int(halo_all), "setup_ms": setup_ms,
        "map_build_ms": 1e3 * t_map / args.steps, "exchange_ms": 1e3 * t_exch / args.steps,
        "conv_ms": 1e3 * t_conv / args.steps, "ms_per_step_by_rank": per_rank,
        "phases": "map_build_ms / exchange_ms / conv_ms: max over ranks of each phase (peer push + wait kernels "
                  "for the exchange)",
        "roofline": roof,
        "cpu_baseline": None,
        "e2e": {"value": w.n * e2e_steps / t_e2e, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "steps": e2e_steps, "matches_device_api": bool(e2e_ok),
                "api": "per rank and step: H2D of owned coords + features (pinned), build_kmap of owned outputs, "
                       "PeerHaloExchange.exchange, conv3d, D2H of owned outputs; steps not overlapped"},
        "c5": c5,
        "clocks": clk.summary(),
        "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def c5_block(args, pkg, dist, rank, world, dev, eng, peaks, peak_src):
    """configs[4] (1024^3, 6.1M voxels, Ci = Co = 32) Morton-sharded over the
    ranks: per coord set the partition, halo plan and owned-output map; per
    layer step the halo exchange and the conv.  Returns a dict (every rank)."""
    import torch
    from sparseconv_b200 import sharding as S
    w = pkg.workloads.make_workload(5)
    coords = torch.from_numpy(w.coords).to(dev)
    feats = torch.from_numpy(w.feats).to(dev, torch.bfloat16)
    weight = torch.from_numpy(w.weight).to(dev, torch.bfloat16)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    mode = args.c5_exchange
    reserve = args.c5_reserve_sms
    n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(2):  # the first pass warms the stream-ordered memory pool
        torch.cuda.synchronize()
        t0.record()
        if world > 1:
            part, own, plan, loc_c, own_f, peer = shard_setup(pkg, S, coords, feats, world, rank, eng, mode)
            n_own, n_int = plan.n_own, plan.n_interior
            buf = torch.empty((plan.n_own + plan.n_halo, w.ci), dtype=torch.bfloat16, device=dev)
            buf[:n_own].copy_(own_f)
            if mode == "peer-interior-first":
                kms = [pkg.concat_kmaps(pkg.build_kmap(loc_c, n_out=n_int, engine=eng),
                                        pkg.build_kmap(loc_c, out_begin=n_int, n_out=n_own - n_int, engine=eng))]
            elif mode == "nccl" and reserve >= 0:
                kms = [pkg.build_kmap(loc_c, n_out=n_int, engine=eng),
                       pkg.build_kmap(loc_c, out_begin=n_int, n_out=n_own - n_int, engine=eng)]
            else:
                kms = [pkg.build_kmap(loc_c, n_out=n_own, engine=eng)]
        else:
            plan, peer, buf, n_own, n_int = None, None, feats, w.n, w.n
            kms = [pkg.build_kmap(coords, engine=eng)]
        t1.record()
        torch.cuda.synchronize()
        setup_ms = t0.elapsed_time(t1)
        if _ == 0 and world > 1:
            if peer is not None:
                peer.close()
            del kms
    infos = [km.info() for km in kms]
    out = torch.empty((n_own, w.co), dtype=torch.bfloat16, device=dev)
    in_kernel_wait = plan is not None and mode in ("peer-conv-wait", "peer-interior-first")

    def layer(ev=None):
        if plan is None:
            if ev: ev[1].record()
            pkg.conv3d(kms[0], buf, weight, out=out)
            return
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
        if reserve < 0:
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
    steps = max(1, args.c5_steps)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    for k in range(steps):
        flush.zero_()
        ev[k][0].record()
        layer(ev[k])
        ev[k][2].record()
    torch.cuda.synchronize()
    eng.synchronize()
    t_total = sum(e[0].elapsed_time(e[2]) for e in ev) / 1e3
    t_first = sum(e[0].elapsed_time(e[1]) for e in ev) / 1e3
    t_last = sum(e[1].elapsed_time(e[2]) for e in ev) / 1e3
    per_rank = [t_total]
    if dist is not None:
        allt = [torch.zeros(1, device=dev, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(allt, torch.tensor([t_total], device=dev, dtype=torch.float64))
        per_rank = [float(x.item()) for x in allt]
    t_total, t_first, t_last, setup_ms = max_over_ranks(dist, dev, [t_total, t_first, t_last, setup_ms])
    halo_total, pairs, int_total = sum_over_ranks(
        dist, dev, [float(plan.n_halo if plan is not None else 0), float(sum(i["num_pairs"] for i in infos)),
                    float(n_int)])
    if peer is not None:
        peer.close()
    ms = 1e3 * t_total / steps
    feat_bytes = w.n * (w.ci + w.co) * 2
    return {
        "workload": w.name, "voxels": w.n, "ci": w.ci, "co": w.co, "pairs": int(pairs), "n_gpus": world,
        "steps": steps, "value": w.n * steps / t_total, "unit": UNIT, "ms_per_step": ms,
        "exchange_ms": 1e3 * t_first / steps, "conv_ms": 1e3 * t_last / steps,
        "ms_per_step_by_rank": [1e3 * t / steps for t in per_rank], "setup_ms": setup_ms,
        "halo_voxels_total": int(halo_total), "interior_voxels_total": int(int_total),
        "exchange": "single GPU: none" if world == 1 else mode,
        "step": "one conv layer (map built once per coord set)" + ("" if world == 1 else
                                                                   " after the halo exchange of that layer"),
        "phases": "exchange_ms = from step start to the conv launch (push + wait, or push only with an in-kernel "
                  "wait); conv_ms = the conv",
        "conv_tflops_total": 2.0 * w.ci * w.co * pairs / (t_total / steps) / 1e12,
        "feature_gbs_total": feat_bytes / (t_total / steps) / 1e9,
        "feature_frac_of_hbm": feat_bytes / (t_total / steps) / 1e9 / (float(peaks["hbm_gbs"]) * world),
        "hbm_peak_source": f"{peak_src} hbm_gbs x n_gpus",
    }


def run_c5(args):
    """configs[4] alone: one 1024^3 shape Morton-sharded over the ranks."""
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    rank, local_rank, world = dist_env()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = init_dist(dev, world, 300)
    peaks, peak_src = measured_peaks()
    eng = pkg.get_engine(dev)
    args.c5_steps = args.steps
    with ClockSampler(dev.index) as clk:
        blk = c5_block(args, pkg, dist, rank, world, dev, eng, peaks, peak_src)
    launches = eng.launch_count()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": blk["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": blk["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded union of 4 ellipsoid shells + 5% interior fill at 1024^3 (BASELINE configs[4])",
        "config": {"workload": blk["workload"], "voxels": blk["voxels"], "ci": blk["ci"], "co": blk["co"],
                   "pairs": blk["pairs"], "step": blk["step"], "l2": L2_NOTE,
                   "parallelism": f"Morton-range sharding x{world}"},
        "c5": blk,
        "roofline": {"bound": "hbm", "achieved": blk["feature_gbs_total"],
                     "peak": float(peaks["hbm_gbs"]) * world, "unit": "GB/s", "frac": blk["feature_frac_of_hbm"],
                     "peak_source": blk["hbm_peak_source"],
                     "units": "feature bytes in + out (N*(Ci+Co)*2) per layer step, summed over ranks"},
        "clocks": clk.summary(), "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_c3(args):
    """a batch of 4 ResBlock shapes (conv -> LN -> SiLU -> conv + skip,
    256 channels) split data-parallel over the ranks by greedy LPT on voxel count;
    weights replicated, no collective on the forward."""
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from sparseconv_b200 import sharding as S
    rank, local_rank, world = dist_env()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = init_dist(dev, world, 180)
    peaks, peak_src = measured_peaks()
    eng = pkg.get_engine(dev)
    w = pkg.workloads.make_workload(3)
    sizes = [int(np.sum(w.coords[:, 0] == b)) for b in range(w.batch_size)]
    assign = S.lpt_assign(sizes, world)
    mine = assign[rank]
    coords_all = torch.from_numpy(w.coords).to(dev)
    rows = S.batch_rows(coords_all, mine)
    coords = coords_all.index_select(0, rows).contiguous()
    feats_all = torch.from_numpy(w.feats).to(dev, torch.bfloat16)
    feats = feats_all.index_select(0, rows).contiguous()
    w1 = torch.from_numpy(w.weight).to(dev, torch.bfloat16)
    w2 = torch.from_numpy(w.extra["weight2"]).to(dev, torch.bfloat16)
    n = int(coords.shape[0])
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    h = torch.empty((max(n, 1), w.co), dtype=torch.bfloat16, device=dev)
    out = torch.empty((max(n, 1), w.co), dtype=torch.bfloat16, device=dev)

    def step(ev=None):
        if ev: ev[0].record()
        if n == 0:
            if ev: ev[1].record(); ev[2].record()
            return None
        km = pkg.build_kmap(coords, engine=eng, check=False)
        if ev: ev[1].record()
        pkg.conv3d(km, feats, w1, silu=True, layernorm=True, out=h[:n])
        pkg.conv3d(km, h[:n], w2, residual=feats, out=out[:n])
        if ev: ev[2].record()
        return km

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    km = step()
    pairs = km.info()["num_pairs"] if km is not None else 0
    eng.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = eng.launch_count()
        for k in range(args.steps):
            flush.zero_()
            step(ev[k])
        torch.cuda.synchronize()
    launches = eng.launch_count() - launches0
    eng.synchronize()
    t_total = sum(e[0].elapsed_time(e[2]) for e in ev) / 1e3
    t_map = sum(e[0].elapsed_time(e[1]) for e in ev) / 1e3
    t_conv = sum(e[1].elapsed_time(e[2]) for e in ev) / 1e3
    conv_rank_s = t_conv / args.steps
    # bit-exact check against one GPU running the whole batch
    ok = True
    if n:
        kf = pkg.build_kmap(coords_all, engine=eng)
        hf = pkg.conv3d(kf, feats_all, w1, silu=True, layernorm=True)
        of = pkg.conv3d(kf, hf, w2, residual=feats_all)
        ok = torch.equal(out[:n], of.index_select(0, rows))
    okt = torch.tensor([1 if ok else 0], device=dev, dtype=torch.int32)
    if dist is not None:
        dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    per_rank = [1e3 * t_total / args.steps]
    if dist is not None:
        allt = [torch.zeros(1, device=dev, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(allt, torch.tensor([1e3 * t_total / args.steps], device=dev, dtype=torch.float64))
        per_rank = [float(x.item()) for x in allt]
    t_total, t_map, t_conv = max_over_ranks(dist, dev, [t_total, t_map, t_conv])
    pairs_all = sum_over_ranks(dist, dev, [float(pairs)])[0]
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    roof = roofline_conv(w.ci, w.co, 2 * pairs, conv_rank_s, peaks, peak_src)
    roof["kernel"] = "conv_tc_kernel (two convs of rank 0's batch elements)"
    line = {
        "metric": METRIC, "value": w.n * args.steps / t_total, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: 4 seeded ellipsoid shells at 128^3, one per batch element (BASELINE configs[2])",
        "config": {"workload": w.name, "voxels": w.n, "batch": w.batch_size, "channels": w.ci,
                   "pairs_per_conv": int(pairs_all),
                   "step": "kernel-map build + conv(LN, SiLU) + conv(+skip)", "l2": L2_NOTE,
                   "parallelism": f"data-parallel x{world}: batch elements by greedy LPT on voxel count",
                   "assignment": assign, "voxels_per_batch_element": sizes},
        "dp_parity": bool(okt.item()),
        "map_build_ms": 1e3 * t_map / args.steps, "convs_ms": 1e3 * t_conv / args.steps,
        "ms_per_step_by_rank": per_rank, "roofline": roof,
        "clocks": clk.summary(), "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_c4(args):
    """512^3 down (64->128) -> subm (128) -> up (128->64) Morton-sharded
    over the ranks.  Boundaries are multiples of 8, so every 2x2x2 sibling group
    (and so every parent) lives on one rank: down and up need no exchange; the
    coarse submanifold conv exchanges a one-voxel coarse halo over NVLink.  The
    maps and plans are built once per coord set (setup_ms); a step is the three
    convs and the exchange."""
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from sparseconv_b200 import sharding as S
    rank, local_rank, world = dist_env()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = init_dist(dev, world, 300)
    peaks, peak_src = measured_peaks()
    eng = pkg.get_engine(dev)
    w = pkg.workloads.make_workload(4)
    coords_all = torch.from_numpy(w.coords).to(dev)
    feats_all = torch.from_numpy(w.feats).to(dev, torch.bfloat16)
    wd = torch.from_numpy(w.weight).to(dev, torch.bfloat16)
    ws = torch.from_numpy(w.extra["w_sub"]).to(dev, torch.bfloat16)
    wu = torch.from_numpy(w.extra["w_up"]).to(dev, torch.bfloat16)
    cmid = int(ws.shape[0])
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    if world > 1:
        part = S.MortonPartition.balanced(coords_all, world)
        own = part.owned_rows(coords_all, rank)
    else:
        part, own = None, torch.arange(w.n, device=dev)
    fine = coords_all.index_select(0, own).contiguous()
    f_own = feats_all.index_select(0, own).contiguous()
    kd = pkg.build_down2(fine, engine=eng)
    coarse = kd.out_coords()
    ku = pkg.build_up2(kd)
    peer = None
    if world > 1:
        plan = S.build_halo_plan(coarse, part.coarsen(), rank, world, interior_first=False)
        loc_c = S.local_coords(plan, coarse)
        peer = S.PeerHaloExchange(plan, torch.zeros((plan.n_own, cmid), dtype=torch.bfloat16, device=dev), eng)
        ks = pkg.build_kmap(loc_c, n_out=plan.n_own, engine=eng)
        halo = plan.n_halo
    else:
        ks = pkg.build_kmap(coarse, engine=eng)
        halo = 0
    t1.record()
    torch.cuda.synchronize()
    setup_ms = t0.elapsed_time(t1)
    n_coarse = int(coarse.shape[0])
    hd = torch.empty((n_coarse, cmid), dtype=torch.bfloat16, device=dev)
    hs = torch.empty((n_coarse, cmid), dtype=torch.bfloat16, device=dev)
    out = torch.empty((fine.shape[0], int(wu.shape[0])), dtype=torch.bfloat16, device=dev)

    def chain(ev=None):
        if ev: ev[0].record()
        if peer is None:
            pkg.conv3d(kd, f_own, wd, out=hd)
            if ev: ev[1].record(); ev[2].record()
            pkg.conv3d(ks, hd, ws, out=hs)
        else:
            pkg.conv3d(kd, f_own, wd, out=peer.next_owned_rows())
            if ev: ev[1].record()
            loc = peer.exchange()
            if ev: ev[2].record()
            pkg.conv3d(ks, loc, ws, out=hs)
        pkg.conv3d(ku, hs, wu, out=out)
        if ev: ev[3].record()

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        chain()
    torch.cuda.synchronize()
    eng.synchronize()
    infos = [k.info() for k in (kd, ks, ku)]
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = eng.launch_count()
        for k in range(args.steps):
            flush.zero_()
            chain(ev[k])
        torch.cuda.synchronize()
    launches = eng.launch_count() - launches0
    eng.synchronize()
    seg = [sum(e[i].elapsed_time(e[i + 1]) for e in ev) / 1e3 for i in range(3)]
    t_total = sum(e[0].elapsed_time(e[3]) for e in ev) / 1e3
    per_rank = [1e3 * t_total / args.steps]
    if dist is not None:
        allt = [torch.zeros(1, device=dev, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(allt, torch.tensor([1e3 * t_total / args.steps], device=dev, dtype=torch.float64))
        per_rank = [float(x.item()) for x in allt]
    # bit-exact check against one GPU running the whole chain
    kdf = pkg.build_down2(coords_all, engine=eng)
    ksf = pkg.build_kmap(kdf.out_coords(), engine=eng)
    kuf = pkg.build_up2(kdf)
    of = pkg.conv3d(kuf, pkg.conv3d(ksf, pkg.conv3d(kdf, feats_all, wd), ws), wu)
    ok = torch.equal(out, of.index_select(0, own))
    okt = torch.tensor([1 if ok else 0], device=dev, dtype=torch.int32)
    if dist is not None:
        dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    del of, kdf, ksf, kuf
    t_total, t_down, t_exch, t_rest, setup_ms = max_over_ranks(dist, dev, [t_total] + seg + [setup_ms])
    pairs = sum_over_ranks(dist, dev, [float(i["num_pairs"]) for i in infos] + [float(halo), float(n_coarse)])
    flops = 2.0 * (64 * 128 * pairs[0] + 128 * 128 * pairs[1] + 128 * 64 * pairs[2])
    if peer is not None:
        peer.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": w.n * args.steps / t_total, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded union of 6 ellipsoid shells at 512^3 (BASELINE configs[3])",
        "config": {"workload": w.name, "voxels": w.n, "coarse_voxels": int(pairs[4]),
                   "pairs": {"down": int(pairs[0]), "subm": int(pairs[1]), "up": int(pairs[2])},
                   "step": "down conv 64->128, coarse halo exchange, subm conv 128, up conv 128->64 "
                           "(maps and plans once per coord set)",
                   "l2": L2_NOTE, "parallelism": f"Morton-range sharding x{world}" if world > 1 else "single GPU"},
        "sharded_parity": bool(okt.item()),
        "halo_voxels_total": int(pairs[3]), "setup_ms": setup_ms,
        "down_ms": 1e3 * t_down / args.steps, "exchange_ms": 1e3 * t_exch / args.steps,
        "subm_up_ms": 1e3 * t_rest / args.steps, "ms_per_step_by_rank": per_rank,
        "conv_tflops_total": flops / (t_total / args.steps) / 1e12,
        "conv_pct_of_bf16_peak_total": 100.0 * flops / (t_total / args.steps) / 1e12 /
                                        (float(peaks["bf16_tflops"]) * world),
        "clocks": clk.summary(), "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_dec(args):
    """The decoder rows on one GPU, on configs[1]'s 406k voxels: one step is a
    ConvNeXt block (depthwise 3x3x3 conv -> LayerNorm -> Linear C->4C ->
    LayerNorm + SiLU -> Linear 4C->C + skip, the map cached per coord set as
    the decoder does) followed by a 2x2x2 subdivision of its output under a
    seeded child mask (half the children kept).  Device-timed with the L2
    flushed between steps; the depthwise conv and the subdivision are also
    timed alone for their rooflines.  Not the driver's headline line."""
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    rank, local_rank, world = dist_env()
    if world > 1:
        if rank == 0:
            print(json.dumps({"workload": "dec", "unavailable": "the decoder rows are measured on one GPU"}))
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, peak_src = measured_peaks()
    eng = pkg.get_engine(dev)
    w = pkg.workloads.make_workload(2)
    C = int(args.dec_channels)
    rng = np.random.default_rng(2024)

    def dW(shape, scale):
        return torch.from_numpy((scale * rng.standard_normal(shape)).astype(np.float32)).to(dev, torch.bfloat16)

    ws = (dW((C, 3, 3, 3, 1), 1 / np.sqrt(27)), dW(C, 0.1), dW((4 * C, C), 1 / np.sqrt(C)), dW(4 * C, 0.1),
          dW((C, 4 * C), 1 / np.sqrt(4 * C)), dW(C, 0.1))
    coords_np = np.ascontiguousarray(w.coords)
    feats_np = rng.standard_normal((w.n, C)).astype(np.float32)
    mask_np = (rng.random((w.n, 8)) < 0.5)
    bits_np = (mask_np * (1 << np.arange(8))).sum(1).astype(np.uint8)
    coords = torch.from_numpy(coords_np).to(dev)
    feats = torch.from_numpy(feats_np).to(dev, torch.bfloat16)
    bits = torch.from_numpy(bits_np).to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    x = pkg.SparseTensor(feats, coords)
    km = pkg.SparseConv3d(ws[0]).neighbour_map(x)   # cached on x, as the decoder's blocks share it
    info = km.info()

    def step():
        y = pkg.sparse_convnext_block(x, *ws)
        return pkg.subdivide2(y, bits)

    def timed(fn, n):
        ts = []
        for _ in range(n):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / 1e3)
        return ts

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    fine, _ = step()
    n_child = int(fine.coords.shape[0])
    with ClockSampler(dev.index) as clk:
        launches0 = eng.launch_count()
        t_step = timed(step, args.steps)
        launches = eng.launch_count() - launches0
    dw_out = torch.empty_like(feats)
    t_dw = timed(lambda: pkg.conv3d_depthwise(km, feats, ws[0], ws[1], out=dw_out), max(args.steps, 5))
    t_sub = timed(lambda: pkg.subdivide2(x, bits), max(args.steps, 5))
    eng.synchronize()
    dw_s, sub_s = statistics.median(t_dw), statistics.median(t_sub)
    # algorithmic bytes of one depthwise launch: every input row read once,
    # every output row written once, the tile-padded gather indices, the tile
    # row list and the weights
    dw_bytes = 2 * w.n * C * 2 + 4 * info["tile_pairs"] + 4 * 128 * info["num_tiles"] + 27 * C * 2
    # subdivision: coords, mask and feature rows read once; child coords,
    # parents and feature rows written once
    sub_bytes = w.n * (16 + 1 + 2 * C) + n_child * (16 + 4 + 2 * C)
    hbm = float(peaks["hbm_gbs"])
    roof = {"bound": "hbm", "kernel": "k_conv_dw<bf16>", "achieved": dw_bytes / dw_s / 1e9, "peak": hbm,
            "unit": "GB/s", "frac": dw_bytes / dw_s / 1e9 / hbm,
            "algorithmic_bytes_per_launch": dw_bytes, "traffic": None,
            "peak_source": f"{peak_src} hbm_gbs (burst: the kernel is timed alone)"}
    sub_roof = {"bound": "hbm", "kernels": "k_subdiv_count/scan/write + k_gather_rows",
                "achieved": sub_bytes / sub_s / 1e9, "peak": hbm, "unit": "GB/s",
                "frac": sub_bytes / sub_s / 1e9 / hbm, "algorithmic_bytes_per_call": sub_bytes,
                "note": "includes the host read of the child count (one stream synchronize per masked call)"}

    # end to end through the public API: H2D of coords + feats + mask from
    # pinned memory, map build, block, subdivision, D2H of the child features
    coords_h = torch.from_numpy(coords_np).pin_memory()
    feats_h = torch.from_numpy(feats_np).to(torch.bfloat16).pin_memory()
    bits_h = torch.from_numpy(bits_np).pin_memory()
    out_h = torch.empty((n_child, C), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        c_d = coords_h.to(dev, non_blocking=True)
        f_d = feats_h.to(dev, non_blocking=True)
        b_d = bits_h.to(dev, non_blocking=True)
        xx = pkg.SparseTensor(f_d, c_d)
        fine_d, _ = pkg.subdivide2(pkg.sparse_convnext_block(xx, *ws), b_d)
        out_h.copy_(fine_d.feats, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    t_e2e = timed(e2e_step, max(3, args.steps // 2))
    e2e_matches = bool(torch.equal(out_h, fine.feats.cpu()))

    # CPU baseline: the oracle's block and subdivision on a bounded sample of
    # rows (their neighbour lookups still search every voxel), one BLAS thread
    cpu = None
    if args.cpu_steps > 0:
        from threadpoolctl import threadpool_limits
        from oracle import sparse_conv_ref as R
        sample = 20000
        rows = np.arange(sample)
        f64 = feats.float().cpu().numpy().astype(np.float64)
        w64 = [t.float().cpu().numpy().astype(np.float64) for t in ws]
        times = []
        with threadpool_limits(1):
            for k in range(1 + args.cpu_steps):
                t0 = time.perf_counter()
                kmr = R.kmap_sorted(coords_np, w.spatial_shape, rows=rows)
                h = R.conv_depthwise(f64, kmr, w64[0], w64[1])
                h = R.layer_norm(h)
                h = R.silu(R.layer_norm(h @ w64[2].T + w64[3]))
                y = h @ w64[4].T + w64[5] + f64[rows]
                R.subdivide2(coords_np[rows], y, mask_np[rows])
                if k:
                    times.append(time.perf_counter() - t0)
        cpu = {"value": sample * len(times) / sum(times), "unit": "voxels/s", "cores": 1, "kind": "port",
               "sample": f"first {sample} of {w.n} voxels (ConvNeXt block + subdivision), "
                         f"{len(times)} timed runs after 1 warm-up, numpy float64, 1 thread"}

    step_s = statistics.median(t_step)
    line = {
        "metric": "sparse ConvNeXt decoder block + 2x2x2 subdivision, active voxels/s", "workload": "dec",
        "value": w.n / step_s, "unit": "voxels/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": 1e3 * step_s, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": f"synthetic: BASELINE configs[1] voxels, seeded features and weights, C={C}",
        "config": {"workload": f"convnext_block_c{C}_subdivide_{w.name}", "voxels": w.n, "channels": C,
                   "hidden": 4 * C, "children": n_child, "pairs": info["num_pairs"], "l2": L2_NOTE,
                   "map": "built once per coord set (cached on the tensor), not in the step"},
        "depthwise_ms": 1e3 * dw_s, "subdivide_ms": 1e3 * sub_s,
        "roofline": roof, "subdivide_roofline": sub_roof,
        "cpu_baseline": cpu,
        "e2e": {"value": w.n / statistics.median(t_e2e), "unit": "voxels/s",
                "h2d_bytes_per_step": coords_h.numel() * 4 + feats_h.numel() * 2 + bits_h.numel(),
                "d2h_bytes_per_step": out_h.numel() * 2, "matches_device_api": e2e_matches,
                "api": "per step: H2D of coords, feats and child mask, map build, sparse_convnext_block, "
                       "subdivide2, D2H of the child features"},
        "clocks": clk.summary(),
        "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


ATTN_LENS = (10000, 6384)
ATTN_HEADS = 16


def run_attn(args):
    """Varlen self-attention on one GPU: the SLat flow model's sparse
    attention (``src/sparse/ops/attention.ts``) over two sequences of 10,000
    and 6,384 tokens, 16 heads of 64, bf16.  A step is one attention call;
    device-timed with inputs resident (K/V of one head fit L2, as in the
    model), `e2e` with the H2D copy of q, k, v and the D2H copy of the output.
    Not the driver's headline line."""
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    rank, local_rank, world = dist_env()
    if world > 1:
        if rank == 0:
            print(json.dumps({"workload": "attn", "unavailable": "the attention row is measured on one GPU"}))
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, peak_src = measured_peaks()
    eng = pkg.get_engine(dev)
    lens = list(ATTN_LENS)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    n_tok, H = cu[-1], ATTN_HEADS
    rng = np.random.default_rng(7)
    host = [torch.from_numpy(rng.standard_normal((n_tok, H, 64)).astype(np.float32)).to(torch.bfloat16)
            for _ in range(3)]
    q, k, v = (t.to(dev) for t in host)
    out = torch.empty_like(q)
    flops = 4.0 * sum(n * n for n in lens) * H * 64

    def timed(fn, n):
        ts = []
        for _ in range(n):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / 1e3)
        return ts

    step = lambda: pkg.sparse_attention(q, k, v, cu, out=out)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        launches0 = eng.launch_count()
        t_step = timed(step, args.steps)
        launches = eng.launch_count() - launches0
    eng.synchronize()
    step_s = statistics.median(t_step)
    bf16_peak = float(peaks["bf16_tflops"])
    roof = {"bound": "tensor", "kernel": "k_attn_fwd<bf16>", "achieved": flops / step_s / 1e12, "peak": bf16_peak,
            "unit": "TFLOP/s", "frac": flops / step_s / 1e12 / bf16_peak,
            "flops_per_call": flops, "units": "4 * sum(len^2) * heads * 64 (QK^T and PV), the whole call timed",
            "traffic": None, "peak_source": f"{peak_src} bf16_tflops (burst)"}
    # end to end: H2D of q, k, v from pinned memory, attention, D2H of the output
    pin = [t.pin_memory() for t in host]
    out_h = torch.empty_like(host[0]).pin_memory()

    def e2e_step():
        qd, kd, vd = (t.to(dev, non_blocking=True) for t in pin)
        out_h.copy_(pkg.sparse_attention(qd, kd, vd, cu), non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    t_e2e = statistics.median(timed(e2e_step, max(3, args.steps // 2)))
    e2e_matches = bool(torch.equal(out_h, out.cpu()))
    cpu = None
    if args.cpu_steps > 0:
        # the reference's multi-sequence path runs dense attention per sequence
        # (src/sparse/ops/attention.ts:40-73); here torch's CPU attention in
        # float32 with all host threads, on a bounded sample of query rows
        torch.set_num_threads(os.cpu_count() or 1)
        sample = 1024  # query rows of the 10,000-token sequence against all its keys
        qs, ks, vs = (t[:lens[0]].float().transpose(0, 1).contiguous() for t in host)
        times = []
        for i in range(1 + args.cpu_steps):
            t0 = time.perf_counter()
            torch.nn.functional.scaled_dot_product_attention(qs[:, :sample], ks, vs)
            if i:
                times.append(time.perf_counter() - t0)
        per_q = statistics.median(times) / sample          # seconds per query row against 10,000 keys
        cpu_s = per_q * sum(n * n for n in lens) / lens[0]  # all rows, scaled by key count
        cpu = {"value": n_tok / cpu_s, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{sample} query rows of the 10,000-token sequence against its keys, torch CPU "
                         f"scaled_dot_product_attention in float32, scaled by query rows x key rows to the call"}
    line = {
        "metric": "varlen sparse attention tokens/s and TFLOP/s", "workload": "attn",
        "value": n_tok / step_s, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": 1e3 * step_s, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic: seeded normal q, k, v",
        "config": {"workload": f"attn_varlen_{'+'.join(map(str, lens))}x{H}h64d", "sequences": lens, "heads": H,
                   "head_dim": 64, "l2": "inputs resident; K and V of a head (2.6 MB) stay in L2 by design"},
        "attention_tflops": roof["achieved"], "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": n_tok / t_e2e, "unit": "tokens/s", "h2d_bytes_per_step": 3 * host[0].numel() * 2,
                "d2h_bytes_per_step": out_h.numel() * 2, "matches_device_api": e2e_matches},
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
    for idx in sorted({int(x) for x in args.configs.split(",") if x.strip()}):
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
        if args.cpu_steps > 0:
            cpu_runs = [_cpu_chain(idx, w, 400_000) for _ in range(2 + 5)][2:]  # 2 warm-ups, median of 5
            cpu_s, cpu_n = statistics.median(r[0] for r in cpu_runs), cpu_runs[0][2]
            cpu_full_ms = 1e3 * cpu_s * (w.n / cpu_n)
        else:
            cpu_n, cpu_full_ms = 0, None
        line = {
            "table": w.name, "voxels": w.n, "pairs": [inf["num_pairs"] for inf in infos],
            "dtype": w.dtype, "gpu_map_ms": gm, "gpu_conv_ms": gc, "gpu_total_ms": gm + gc,
            "conv_tflops": flops / (gc * 1e-3) / 1e12,
            "conv_pct_of_bf16_peak": 100.0 * flops / (gc * 1e-3) / 1e12 / float(peaks["bf16_tflops"]),
            "peak_source": f"{peak_src} bf16_tflops (burst)",
            "gpu_voxels_per_s": w.n / ((gm + gc) * 1e-3),
            "cpu_ms": cpu_full_ms, "cpu_threads": torch.get_num_threads(), "cpu_runs": "median of 5 after 2 warm-ups",
            "cpu_sample": ("not run (--cpu-steps 0)" if cpu_full_ms is None else "full workload" if cpu_n == w.n else
                           f"first {cpu_n} Morton-ordered voxels, time scaled by {w.n / cpu_n:.2f}"),
            "speedup_vs_cpu": None if cpu_full_ms is None else cpu_full_ms / (gm + gc), "steps": steps,
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
    if args.workload == "c3":
        return run_c3(args)
    if args.workload == "c4":
        return run_c4(args)
    if args.workload == "table":
        return run_table(args)
    if args.workload == "dec":
        return run_dec(args)
    if args.workload == "attn":
        return run_attn(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
