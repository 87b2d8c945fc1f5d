"""
Benchmark of Image-GS's rasterization training step on B200: forward + L1 backward steps/s and Gaussian-pixel evaluations/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg3_1080p] [--impl ours|reference]

A step (default workload: 1920x1080 RGB target, 20,000 Gaussians, 16x16 tiles, top-10) is projection -> prefix sum -> tile binning ->
top-K forward with the L1 loss and its gradient fused -> top-K backward -> projection backward, replayed from one CUDA graph with inputs
resident in HBM (`value`). With N GPUs (torchrun, one process per GPU, NCCL for the barrier and the max over ranks) every rank renders its
own independent image (weak scaling, no data-path communication); `--workload cfg4_2160p` splits one image into tile-row bands (strong
scaling, one NCCL all-reduce per step). `e2e` runs the same step through the C ABI with host buffers: the Gaussian parameters copied
host->device from pinned memory and the loss read back every step; `e2e_autograd` does the same through the drop-in gsplat API with
autograd and F.l1_loss (what Image-GS's model.py calls). The L2 cache is flushed (a 256 MB write) between timed steps, outside the
per-step CUDA-event intervals.

`--impl reference` times the CPU restatement of the reference's path (the reference has no CPU implementation of its own) on the host's
cores, on rank 0 only.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "image-gs_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from igs_b200 import workloads  # noqa: E402

METRIC = "fwd+bwd raster steps/s at 1080p/20k (also Gaussian-pixel evals/s, % of HBM roofline)"
L2_FLUSH_BYTES = 256 << 20


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons of one GPU sampled through NVML every ~0.5 ms while running (the timed region can be a few ms)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.samples = []
        self.stop = threading.Event()
        self.ok = False

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[self.gpu_index]) if visible else self.gpu_index
            self.nvml, self.handle = pynvml, pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:  # no NVML: report no samples
            self.ok = False
        return self

    def _run(self):
        while not self.stop.is_set():
            try:
                mhz = self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
                reasons = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(0.0005)

    def __exit__(self, *exc):
        self.stop.set()
        if self.ok:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = sorted({name for _, r in self.samples for name, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "NVML, polled every 0.5 ms during the timed steps"}


def dist_setup(gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus and world > 1:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        # NCCL prints its version banner on the process's stdout when it creates the communicator: send file descriptor 1 to stderr
        # meanwhile, so that rank 0's stdout holds only the JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            os.dup2(saved, 1)
            os.close(saved)
    return world, rank, local


def cpu_step_rate(wl, inp, min_seconds=10.0, max_steps=1000):
    """Steps/s of the CPU oracle (all host threads) over whole steps of the workload: (rate, threads, steps)."""
    sys.path.insert(0, ROOT)
    from oracle import cpu

    threads = len(os.sched_getaffinity(0))
    cpu.set_threads(threads)
    args = [inp[k].numpy() for k in ("means", "scales", "rotations", "features", "target")]
    cpu.train_step(*args, wl.height, wl.width)  # warm-up
    t0 = time.perf_counter()
    steps = 0
    while steps < max_steps and (steps == 0 or time.perf_counter() - t0 < min_seconds):
        cpu.train_step(*args, wl.height, wl.width)
        steps += 1
    return steps / (time.perf_counter() - t0), threads, steps


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


L2_NOTE = ("GPU arm: L2 flushed between timed steps (256 MB write outside the event intervals); the CPU arm (--impl reference) times "
           "whole steps on the host")


def workload_config(wl, num_isect, world):
    """The workload as both arms describe it (one independent image per GPU; the CPU arm's rank 0 times its share)."""
    return {"workload": wl.name, "height": wl.height, "width": wl.width, "gaussians": wl.num_gaussians, "channels": wl.channels,
            "tile": 16, "top_k": 10, "intersections": num_isect, "parallelism": f"dp{world} (independent images)", "l2": L2_NOTE}


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    inp = workloads.make_inputs(wl)
    sys.path.insert(0, ROOT)
    from oracle import cpu

    threads = len(os.sched_getaffinity(0))
    cpu.set_threads(threads)
    a = [inp[k].numpy() for k in ("means", "scales", "rotations", "features", "target")]
    _, _, _, hits = cpu.project_fwd(a[0], a[1], a[2], wl.height, wl.width)
    num_isect = int(np.asarray(hits, dtype=np.int64).sum())
    for _ in range(args.warmup):
        cpu.train_step(*a, wl.height, wl.width)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu.train_step(*a, wl.height, wl.width)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = args.steps / total
    sample = f"{args.steps} whole {wl.width}x{wl.height} steps (N={wl.num_gaussians}) of the C restatement, {threads} threads, {cpu_model()}"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded sinusoid target, random Gaussians)",
        "config": workload_config(wl, num_isect, args.gpus),
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU implementation of this path; this is the oracle's C restatement of its kernels",
    }))


def time_graph(graph, reps, flush):
    """Mean ms of `reps` replays, each bracketed by CUDA events, with an L2 flush between replays."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    for i in range(reps):
        flush.zero_()
        starts[i].record()
        graph.replay()
        ends[i].record()
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / reps


RATE_MODEL = os.path.join(ROOT, "tests", "golden", "py_cfg2_480p_yuv.npz")

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the step's raster kernels, from ncu captures of this workload
# (`ncu --set full --clock-control none -k regex:raster_step -s 2 -c 1 python bench.py --steps 2 --warmup 3 --no-cpu --no-e2e
# --no-stages`, and the same with `-k regex:"raster_(fwd|bwd_pairs)" -c 2 ... --split`; caches flushed before each pass, writes still
# in L2 when a kernel ended not counted); None where no capture was taken
NCU_TRAFFIC = {("cfg3_1080p", "raster_step"): 26.994e6 + 0.238e6,
               ("cfg3_1080p", "raster_forward"): 26.447e6 + 36.868e6,
               ("cfg3_1080p", "raster_backward"): 68.466e6 + 1.702e6}
# the same captures' smsp__issue_active.avg.pct_of_peak_sustained_active: what bounds these kernels (instruction issue, not HBM)
NCU_ISSUE_ACTIVE = {("cfg3_1080p", "raster_step"): 0.841, ("cfg3_1080p", "raster_forward"): 0.711,
                    ("cfg3_1080p", "raster_backward"): 0.765}


def raster_roofline(stage_ms, p, c, n, k, num_isect, num_tiles, hbm_peak, peak_kind, workload=None, label=""):
    """The roofline entry of the step's dominant raster kernel from the single-stage times. algorithmic_bytes is the per-step figure of
    the operator surface (the reference's dataflow: the image and the [H, W, 10] lists written by the forward and read back by the
    backward, the image gradient, the Gaussians' parameters and gradients, the list IDs) for the work the kernel does:
      forward with the L1 loss: P (4C + 4K) + I 4 + N 4 (5 + C) + 12 C P (the loss reads the image and the target, writes the gradient);
      backward: P (4C + 4K) + N 4 ((5 + C) + (2 + 3 + C));
      the fused step kernel (stage "raster"): both.
    moved_bytes is what the kernel itself must move: the fused kernel only reads the target and the lists' Gaussians and writes the image
    and the gradients (8 C P + I 4 + 2 N 4 (5 + C) + 8 T), since it keeps the lists and the image gradient on chip."""
    fwd_bytes = p * (4 * c + 4 * k) + num_isect * 4 + n * 4 * (5 + c) + 12 * c * p
    bwd_bytes = p * (4 * c + 4 * k) + n * 4 * ((5 + c) + (2 + 3 + c))
    if "raster" in stage_ms:
        name, ms = "raster_step", stage_ms["raster"]
        nbytes = fwd_bytes + bwd_bytes
        moved = p * 8 * c + num_isect * 4 + n * 4 * (5 + c) * 2 + num_tiles * 8
    else:
        dominant = max(("forward", "backward"), key=lambda s: stage_ms.get(s, 0.0))
        name, ms = f"raster_{dominant}", stage_ms[dominant]
        nbytes = fwd_bytes if dominant == "forward" else bwd_bytes
        moved = nbytes
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "kernel": name + label, "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "peak_kind": peak_kind, "traffic": NCU_TRAFFIC.get((workload, name)), "algorithmic_bytes": nbytes, "moved_bytes": moved,
            "kernel_ms": ms, "issue_active": NCU_ISSUE_ACTIVE.get((workload, name))}


def step_options(wl, device):
    """Extra stages of the workload's step: for the 480p YUV configuration the straight-through quantizer, the luma-weighted loss
    transform and the rate term, whose fixed inputs (neighbours, slopes, Laplace scales) are the ones the reference's
    compress.rate.rate_model computed for this seeded workload (tests/golden/py_cfg2_480p_yuv.npz)."""
    if not wl.rate_term:
        return {}
    z = np.load(RATE_MODEL)
    return dict(quant=workloads.quant_settings(wl, device), loss_transform=workloads.loss_transform_yuv().to(device),
                rate=dict(model=workloads.RateModelTensors(z, device), inv_rot_step=float(z["inv_rot_step"]), factor=float(z["factor"])))


def run_ours(args, wl):
    from igs_b200 import pipeline

    world, rank, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    inp = workloads.make_inputs(wl, image_index=rank if not wl.rate_term else 0)
    d = {k: v.to(device) for k, v in inp.items()}
    target = d["loss_target"] if "loss_target" in d else d["target"]
    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], target, fused=not args.split,
                               **step_options(wl, device))
    graph = step.capture()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    num_isect = int(step.num_intersects.item())
    if num_isect > step.capacity:
        raise SystemExit(f"intersections {num_isect} exceed the capacity {step.capacity}")
    evals = step.gaussian_pixel_evals()

    barrier = (lambda: torch.distributed.barrier()) if world > 1 else (lambda: None)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            graph.replay()
            ends[i].record()
        torch.cuda.synchronize()
    barrier()
    ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = torch.tensor([sum(ms)], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(total_ms, op=torch.distributed.ReduceOp.MAX)
    total_ms = float(total_ms.item())
    ms_per_step = total_ms / args.steps
    value = world * args.steps / (total_ms / 1e3)

    # per-stage breakdown and the dominant kernel's roofline (graphs of single stages, same flush discipline)
    stage_ms = {}
    for s in step.BREAKDOWN_STAGES if not args.no_stages else ():
        g = step.capture([s])
        stage_ms[s.strip("_")] = time_graph(g, max(5, min(50, args.steps)), flush)
        del g
    if not stage_ms:
        stage_ms = {"raster": ms_per_step}  # no per-stage times: the whole step stands in for the raster kernel
    hbm_peak, peak_kind = peaks()
    p, c, n, k = wl.num_pixels, wl.channels, wl.num_gaussians, pipeline.TOP_K
    roofline = raster_roofline(stage_ms, p, c, n, k, num_isect, wl.num_tiles, hbm_peak, peak_kind, wl.name)
    kernels_per_step, capacity = step.kernels_per_step, step.capacity
    step_bytes = (p * (8 * c + 8 * k) + n * 4 * (5 + 7 + 2 * (5 + c) + (5 + c) + 5 + 5) + num_isect * 4 * 5 + wl.num_tiles * 16)
    loss_bytes = 12 * c * p

    # end to end with host buffers: through the C ABI (the step as above, parameters copied in and the loss read back every step), and
    # through the drop-in gsplat API with autograd (what model.py calls)
    e2e = e2e_autograd = e2e_autograd_graph = e2e_autograd_graph_l1 = None
    if not args.no_e2e:
        e2e = run_step_e2e(args, step, step.raw, inp, device, world, "step")
        e2e_autograd = run_e2e(args, wl, inp, device, step.capacity, world)
        e2e_autograd_graph = run_e2e(args, wl, inp, device, step.capacity, world, graph=True)
        e2e_autograd_graph_l1 = run_e2e(args, wl, inp, device, step.capacity, world, graph=True, routed_l1=True)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, threads, steps = cpu_step_rate(wl, inp)
        cpu = {"value": rate, "unit": "steps/s", "cores": threads, "kind": "port",
               "sample": f"{steps} whole {wl.width}x{wl.height} steps of the C restatement on {threads} threads ({cpu_model()})"}

    # the 2160p image split into tile-row bands over the same ranks (strong scaling; at N=1 the whole image on one GPU, the reference
    # point of the scaling), reported beside the independent-image line
    bands_leg = bands_leg_other = None
    if not args.no_bands and wl.name == "cfg3_1080p":
        del graph, step
        torch.cuda.empty_cache()
        # with several GPUs both exchanges are measured: the peer-memory exchange (the default) and NCCL's all-reduce
        exchanges = [args.exchange] + ([x for x in ("peer", "nccl") if x != args.exchange] if world > 1 else [])
        for ex in exchanges:
            try:
                b = measure_bands(args, workloads.get_workload("cfg4_2160p"), world, rank, local, exchange=ex, steps=min(args.steps, 50),
                                  e2e=False, cpu=False, stages=False)
                leg = None
                if rank == 0:
                    leg = {k: b[k] for k in ("value", "unit", "n_gpus", "ms_per_step", "scaling", "exchange", "exchange_ms",
                                             "band_ms_per_rank", "band_intersections", "gaussian_pixel_evals_per_s", "clocks")}
                    leg["config"] = b["config"]
            except Exception as err:  # the band leg is reported beside the main line; its failure must not lose the main measurement
                leg = {"error": f"{type(err).__name__}: {err}"[:500]}
            if ex == args.exchange:
                bands_leg = leg
            else:
                bands_leg_other = leg

    if rank == 0:
        clk = clocks.summary()
        out = {
            "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded sinusoid target, random Gaussians; one independent image per GPU)",
            "config": workload_config(wl, num_isect, world),
            "capacity": capacity, "graph": "one CUDA graph per step",
            "gaussian_pixel_evals_per_step": evals, "gaussian_pixel_evals_per_s": evals * value,
            "stages_ms": stage_ms,
            "roofline": roofline,
            "step_roofline": {"algorithmic_bytes": step_bytes, "loss_bytes": loss_bytes,
                              "frac_raster": step_bytes / (ms_per_step * 1e-3) / 1e9 / hbm_peak,
                              "frac_with_loss": (step_bytes + loss_bytes) / (ms_per_step * 1e-3) / 1e9 / hbm_peak},
            "e2e": e2e, "e2e_autograd": e2e_autograd, "e2e_autograd_graph": e2e_autograd_graph,
            "e2e_autograd_graph_l1": e2e_autograd_graph_l1, "cpu_baseline": cpu,
            "gpu_launches": kernels_per_step * args.steps, "clocks": clk, "bands_2160p": bands_leg,
            "bands_2160p_other_exchange": bands_leg_other,
        }
        print(json.dumps(out))
    if world > 1:
        torch.distributed.destroy_process_group()


def measure_bands(args, wl, world, rank, local, exchange="peer", steps=None, e2e=True, cpu=True, stages=True):
    """One image in tile-row bands, one band per GPU (strong scaling), on an initialised process group: every rank projects all
    Gaussians, bins, renders and back-propagates its rows; the partials are combined by the peer-memory exchange (igs_band_reduce: each
    rank reduces one share of the Gaussians and runs its projection backward, the whole step one CUDA graph) or by an NCCL all-reduce
    followed by the projection backward on every rank. value = whole-image steps/s; per-step time is the max over ranks. Returns rank
    0's JSON dict (None on the other ranks)."""
    from igs_b200 import bands

    steps = steps or args.steps
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    inp = workloads.make_inputs(wl)  # the same image on every rank
    d = {k: v.to(device) for k, v in inp.items()}
    tiles_x, tiles_y, _ = wl.tile_bounds
    per_row = bands.row_intersections(d["means"], d["scales"], d["rotations"], wl.height, wl.width)
    r0, r1 = bands.band_rows(tiles_y, world, rank, [r + 32.0 * tiles_x for r in per_row])
    group = torch.distributed.group.WORLD if world > 1 else None
    step = bands.BandStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], wl.height, wl.width, r0, r1, group=group,
                          fused=not args.split, exchange=exchange)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    for _ in range(args.warmup):
        step.replay()
    torch.cuda.synchronize()
    step.check()
    band_isect = int(step.num_intersects.item())
    if band_isect > step.capacity:
        raise SystemExit(f"intersections {band_isect} exceed the capacity {step.capacity}")
    evals = torch.tensor([step.gaussian_pixel_evals()], device=device, dtype=torch.float64)

    barrier = (lambda: torch.distributed.barrier()) if world > 1 else (lambda: None)
    # the ranks' steps are coupled by the exchange, so each L2 flush is followed by a one-float all-reduce that lines up the ranks'
    # start events: otherwise a rank's timed step would include waiting for the other ranks' flushes
    token = torch.zeros(1, device=device)
    align = (lambda: torch.distributed.all_reduce(token)) if world > 1 else (lambda: None)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(steps):
            flush.zero_()
            align()
            starts[i].record()
            step.replay()
            ends[i].record()
        torch.cuda.synchronize()
    barrier()
    step.check()
    total_ms = torch.tensor([sum(s.elapsed_time(e) for s, e in zip(starts, ends))], device=device, dtype=torch.float64)

    # the band's own work (one graph, no communication) and the exchange alone, per rank
    local_graph = step._capture(step.LOCAL)
    local_ms = time_graph(local_graph, max(5, min(50, steps)), flush)
    del local_graph
    stage_ms = {}
    for s_ in ((("_forward",), ("_backward",)) if args.split else (("_raster",),)) if stages else ():
        g = step._capture(s_)
        stage_ms[s_[0].strip("_")] = time_graph(g, max(5, min(50, steps)), flush)
        del g
    xchg_ms = 0.0
    if world > 1:
        # the exchange alone: with the peer exchange, its two kernels as a CUDA graph (captured on every rank) replayed back to back;
        # with NCCL, the all-reduce and the projection backward's graph
        xgraph = step._capture(step.FINAL)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        a.record()
        for _ in range(20):
            step.all_reduce()
            xgraph.replay()
        b.record()
        torch.cuda.synchronize()
        step.check()
        xchg_ms = a.elapsed_time(b) / 20
        del xgraph
    per_rank = torch.tensor([local_ms, float(r0), float(r1), float(band_isect)], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(total_ms, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(evals)
        gathered = [torch.empty_like(per_rank) for _ in range(world)]
        torch.distributed.all_gather(gathered, per_rank)
    else:
        gathered = [per_rank]
    total_ms = float(total_ms.item())
    ms_per_step = total_ms / steps
    value = steps / (total_ms / 1e3)

    e2e_out = None
    if e2e and not args.no_e2e:
        e2e_out = run_step_e2e(args, step, (step.means, step.scales, step.rotations, step.features), inp, device, world, "bands")

    cpu_out = None
    if cpu and rank == 0 and world == 1 and not args.no_cpu:
        rate, threads, nsteps = cpu_step_rate(wl, inp)
        cpu_out = {"value": rate, "unit": "steps/s", "cores": threads, "kind": "port",
                   "sample": f"{nsteps} whole {wl.width}x{wl.height} steps of the C restatement on {threads} threads ({cpu_model()})"}

    out = None
    if rank == 0:
        hbm_peak, peak_kind = peaks()
        c, n, k = wl.channels, wl.num_gaussians, 10
        p = step.band_h * wl.width
        roofline = None
        if stage_ms:
            roofline = raster_roofline(stage_ms, p, c, n, k, band_isect, step.num_tiles, hbm_peak, peak_kind, None, " (rank 0's band)")
        total_evals = float(evals.item())
        how = ("peer-memory exchange (igs_band_reduce: each rank sums one share of the Gaussians from every rank's partials over NVLink "
               "and runs its projection backward)" if step.exchange == "peer" else
               f"NCCL all-reduce of {step.reduced.numel()} floats, projection backward on every rank") if world > 1 else "one band"
        out = {
            "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded sinusoid target, random Gaussians; one image split into tile-row bands)",
            "config": {"workload": wl.name, "height": wl.height, "width": wl.width, "gaussians": wl.num_gaussians, "channels": wl.channels,
                       "tile": 16, "top_k": 10, "parallelism": f"{world} tile-row bands + {how}",
                       "bands": [[int(g[1].item()), int(g[2].item())] for g in gathered],
                       "l2": "flushed between timed steps (256 MB write outside the event intervals)",
                       "graph": ("the whole step as one CUDA graph" if step.exchange == "peer" or world == 1 else
                                 "band work as one CUDA graph, NCCL all-reduce, projection backward as a second graph")},
            "exchange": step.exchange if world > 1 else None,
            "gaussian_pixel_evals_per_step": total_evals, "gaussian_pixel_evals_per_s": total_evals * value,
            "band_ms_per_rank": [float(g[0].item()) for g in gathered],
            "band_intersections": [int(g[3].item()) for g in gathered], "exchange_ms": xchg_ms, "stages_ms": stage_ms,
            "roofline": roofline, "e2e": e2e_out, "cpu_baseline": cpu_out, "gpu_launches": step.kernels_per_step * steps,
            "clocks": clocks.summary(),
        }
    step.release()
    return out


def run_bands(args, wl):
    """`--workload cfg4_2160p`: the band split as the JSON line's own measurement."""
    world, rank, local = dist_setup(args.gpus)
    out = measure_bands(args, wl, world, rank, local, exchange=args.exchange)
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        torch.distributed.destroy_process_group()


def run_step_e2e(args, step, dev_params, inp, device, world, api):
    """The step through the C ABI with host buffers: the Gaussian parameters copied host -> device from pinned memory into the step's
    input tensors and the loss read back to the host every step. For the one-image step the copies are nodes of the step's CUDA graph
    (one graph launch per step); the bands' step copies around its graphs and its all-reduce."""
    keys = ("means", "scales", "rotations", "features")
    host = [inp[k].pin_memory() for k in keys]
    dev = list(dev_params)
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    if api == "step":
        # the parameters as the caller keeps them for this API: one pinned host buffer in the step's packed layout, one transfer per step
        from igs_b200 import pipeline

        offsets, length = pipeline.RasterStep.packed_layout(step.n, step.c)
        flat_host = torch.zeros(length, dtype=torch.float32).pin_memory()
        for t, at in zip(host, offsets):
            flat_host[at:at + t.numel()] = t.reshape(-1)
        dev, host = [step.pack_inputs()], [flat_host]

    def copy_in():
        for d, h in zip(dev, host):
            d.copy_(h, non_blocking=True)

    def copy_out():
        loss_host.copy_(step.loss, non_blocking=True)

    if api == "step":
        graph = step.capture(before=copy_in, after=copy_out)

        def one():
            graph.replay()
    else:
        def one():
            copy_in()
            step.replay()
            copy_out()

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        one()
        torch.cuda.current_stream().synchronize()
        float(loss_host)
    end.record()
    torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end)], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    h2d = sum(v.numel() * v.element_size() for v in host)
    return {"value": world * args.steps / (float(t.item()) / 1e3) if api != "bands" else args.steps / (float(t.item()) / 1e3),
            "unit": "steps/s", "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": 4 * world,
            "api": ("igs_b200.bands.BandStep" if api == "bands" else "igs_b200.pipeline.RasterStep") +
                   " over the C ABI (host parameters copied in and the loss read back every step" +
                   (", the parameters as one packed pinned buffer: one copy in and one out per step, both captured in the step's CUDA "
                    "graph)" if api == "step" else ")")}


def run_e2e(args, wl, inp, device, capacity, world, graph=False, routed_l1=False):
    """The step through the drop-in gsplat API with autograd and F.l1_loss, as model.py calls it, with the parameters copied in from
    pinned host memory and the loss read back every step: eagerly (graph=False), or captured in one CUDA graph with the copies, the
    forward, the loss and the backward pass as model.py's CUDA-graph step does (model.py:1160-1209; the optimizer is outside the metric).
    routed_l1: F.l1_loss as igs_b200.autograd.install_l1() routes model.py's call (the library's one-pass loss keeping the signs)."""
    import torch.nn.functional as F

    import gsplat

    from igs_b200 import autograd as ag

    l1_loss = ag._routed_l1_loss if routed_l1 else F.l1_loss

    from igs_b200 import pipeline

    keys = ("means", "scales", "rotations", "features")
    target = (inp["loss_target"] if "loss_target" in inp else inp["target"]).to(device)
    # the parameters packed as for the C-ABI leg (one pinned host buffer, one copy per step); the leaf tensors autograd sees are
    # detached views of the device buffer
    n, c = inp["features"].shape
    offsets, length = pipeline.RasterStep.packed_layout(n, c)
    flat_host = torch.zeros(length, dtype=torch.float32).pin_memory()
    flat_dev = torch.empty(length, dtype=torch.float32, device=device)
    dev = {}
    for k, at in zip(keys, offsets):
        t = inp[k]
        flat_host[at:at + t.numel()] = t.reshape(-1)
        dev[k] = flat_dev[at:at + t.numel()].view(t.shape).detach().requires_grad_(True)
    host = {"packed": flat_host}
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    tb = wl.tile_bounds
    opts = step_options(wl, device)

    def body():
        with torch.no_grad():
            flat_dev.copy_(flat_host, non_blocking=True)
        means, scales, rots, feats = [dev[k] for k in ("means", "scales", "rotations", "features")]
        raw_feats, raw_rots = feats, rots
        if "quant" in opts:  # model._get_params (model.py:993-1006) and the loss-space features (model.py:963-964)
            q = opts["quant"]
            means, scales, rots, feats = ag.quantize_ste(means, scales, rots, feats, q["pos_steps"], q["scale_step"], q["rot_step"],
                                                         q["feat_steps"])
            feats = feats @ opts["loss_transform"].T
        xys, radii, conics, hits = gsplat.project_gaussians_2d_scale_rot(means, scales, rots, wl.height, wl.width, tb)
        img = gsplat.rasterize_gaussians_sum(xys, radii, conics, hits, feats, wl.height, wl.width, topk_norm=True, capacity=capacity)
        img = img.permute(2, 0, 1).contiguous()
        loss = l1_loss(img, target)
        if "rate" in opts:  # model._get_total_loss (model.py:1235-1240)
            r = opts["rate"]
            loss = loss + ag.rate_loss(raw_feats, raw_rots, loss, r["model"], r["inv_rot_step"], 1.0, r["factor"])
        loss.backward()
        loss_host.copy_(loss.detach(), non_blocking=True)

    def clear_grads():
        for v in dev.values():
            v.grad = None

    if graph:
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(max(3, args.warmup)):  # eager warm-up on a side stream, as before any capture
                clear_grads()
                body()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize()
        clear_grads()  # backward() then allocates the gradients from the graph's memory pool
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            body()
        one = g.replay
    else:
        def one():
            clear_grads()
            body()

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        one()
        torch.cuda.current_stream().synchronize()  # the loss is read on the host every step
        float(loss_host)
    end.record()
    torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end)], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    value = world * args.steps / (float(t.item()) / 1e3)
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    return {"value": value, "unit": "steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
            "api": ("igs_b200.autograd.quantize_ste + feat @ T.T + " if "quant" in opts else "") +
                   "gsplat.project_gaussians_2d_scale_rot + gsplat.rasterize_gaussians_sum(topk_norm=True, capacity) + " +
                   ("F.l1_loss routed by igs_b200.autograd.install_l1()" if routed_l1 else "F.l1_loss") +
                   (" + igs_b200.autograd.rate_loss" if "rate" in opts else "") + " + backward" +
                   (", copies, forward, loss and backward replayed as one CUDA graph (model.py's graph-captured step)" if graph else
                    ", eager") + "; the parameters as one packed pinned buffer, one copy in per step"}


def run_aux(args):
    """The rows around the step, each timed on the GPU and beside the reference's CPU code where it has one: the neighbour search of the
    rate model's preparation at 80,000 Gaussians (vs the reference's C++ causal_neighbors, built from source into oracle/_ref, on all host
    threads) and the whole rate model of those Gaussians, the per-Gaussian feature weights and the leave-one-out loss increase at
    1080p/20k. One JSON line."""
    from igs_b200 import neighbors as nb
    from igs_b200 import ops

    device = torch.device("cuda", 0)
    out = {"aux": True, "unit": "ms"}

    def gpu_ms(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    # neighbour search: the 2160p/80k workload's positions quantized with the default 1/8-pixel step, in bitstream order
    wl4 = workloads.get_workload("cfg4_2160p")
    inp4 = workloads.make_inputs(wl4)
    q = torch.round(inp4["means"].double() * torch.tensor([wl4.width, wl4.height], dtype=torch.float64) / 0.125).long().numpy()
    order = nb.bitstream_order(q, 3)
    sq = torch.from_numpy(np.ascontiguousarray(q[order])).to(device)
    ms = gpu_ms(lambda: nb.causal_neighbors(sq))
    entry = {"gaussians": len(q), "gpu_ms": ms}
    sys.path.insert(0, ROOT)
    try:
        from oracle import build_ref

        ref = build_ref.load_prediction()
        host = np.ascontiguousarray(q[order])
        ref.causal_neighbors(host)
        t0 = time.perf_counter()
        reps = 5
        for _ in range(reps):
            ref_out = ref.causal_neighbors(host)
        entry["reference_cpu_ms"] = 1e3 * (time.perf_counter() - t0) / reps
        entry["reference_cpu_threads"] = len(os.sched_getaffinity(0))
        entry["identical"] = bool(np.array_equal(nb.causal_neighbors(sq).cpu().numpy(), ref_out))
    except ImportError as e:
        entry["reference_cpu_ms"] = None
        entry["reference_note"] = str(e)
    out["causal_neighbors"] = entry

    # the whole rate model (compress.rate.rate_model) of the same 80,000 Gaussians, YUV prediction references: bitstream order,
    # neighbour search and igs_rate_model on the GPU; wall time per call (it reads the positions' range and the list length back)
    from igs_b200 import rate_model as rm

    steps = torch.full((wl4.channels,), 1.0 / 64, device=device)
    feat = torch.round(inp4["features"].to(device) / steps) * steps
    log2_scale = torch.round(torch.log2(inp4["scales"].abs().to(device)) / 0.03125) * 0.03125
    q_rot = torch.round(inp4["rotations"].to(device)[:, 0] / (np.pi / 256))
    weights = torch.tensor([1.0, 0.25, 0.25], device=device)

    def prepare():
        return rm.rate_model(q, feat, log2_scale, q_rot, [-1, -1, -1], [-1, 0, 1], steps, weights, refine_bits=3)

    prepare()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(5):
        prepare()
    torch.cuda.synchronize()
    out["rate_model_80k"] = {"wall_ms": 1e3 * (time.perf_counter() - t0) / 5,
                             "note": "bitstream order (igs_bitstream_order), neighbour search and igs_rate_model on the GPU; two small "
                                     "read-backs"}

    # feature weights and leave-one-out at 1080p/20k from the step's top-K lists
    wl = workloads.get_workload("cfg3_1080p")
    inp = workloads.make_inputs(wl)
    d = {k: v.to(device) for k, v in inp.items()}
    h, w, n = wl.height, wl.width, wl.num_gaussians
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(n, d["means"], d["scales"], d["rotations"], h, w, tb)
    cum, total = ops.cumulative_intersects(hits)
    ids, bins = ops.sort_intersects_by_tile(n, int(total.item()), xys, radii, cum, tb)
    _, topk = ops.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, d["features"])
    out["feature_weights_1080p"] = {"gpu_ms": gpu_ms(lambda: ops.topk_feature_weights_fixed(h, w, xys, conics, topk))}
    out["loo_1080p"] = {"gpu_ms": gpu_ms(lambda: ops.topk_norm_loo_loss_increase(h, w, xys, conics, d["features"], topk, d["target"],
                                                                                  False, 1e-4))}

    # the bitstream of those 80,000 Gaussians (positions, scales, rotations, features in bitstream order): the rANS coder's encode
    # (model search on host threads + one rANS pass) and decode against the reference's C++ coder built from source (oracle/_ref), on
    # the same streams; and the size estimate of the rate decisions (histograms on the GPU) against the reference's
    out["bitstream_80k"] = codec_aux(q, inp4, order)
    print(json.dumps(out))


def codec_aux(q, inp, order):
    """Encode / decode / estimate timings of the bitstream's streams of the 2160p/80k workload, ours against the reference's coder."""
    from igs_b200 import bitstream, codec

    rot = np.round(inp["rotations"].numpy()[:, :1] / (np.pi / 256)).astype(np.int64)
    scale = np.round(np.log2(np.abs(inp["scales"].numpy())) / 0.03125).astype(np.int64)
    feat = np.round(inp["features"].numpy() * 64).astype(np.int64)
    _, _, codes = bitstream.bitstream_order(q, 3)
    streams = [np.diff(codes, prepend=np.uint64(0)).astype(np.int64)] + [a[order][:, c].copy() for a in (scale, rot, feat)
                                                                          for c in range(a.shape[1])]

    def wall_ms(fn, reps=5):
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            result = fn()
        return 1e3 * (time.perf_counter() - t0) / reps, result

    class Sink:  # a writer that only counts (the headers are written in Python by both sides)
        num_bits = 0

        def write(self, *a):
            pass

        def write_se(self, *a):
            pass

        def write_ue(self, *a):
            pass

    entry = {"gaussians": len(q), "streams": len(streams), "threads": len(os.sched_getaffinity(0))}
    entry["encode_ms"], (payload, _) = wall_ms(lambda: codec.encode_streams([streams], Sink()))
    entry["estimate_ms_gpu"], est = wall_ms(lambda: codec.estimate_stream_bits(streams))
    sys.path.insert(0, ROOT)
    try:
        from oracle import build_ref

        rans = build_ref.load_cpp_module(build_ref.RANS)
        entry["reference_encode_ms"], (ref_payload, ref_models) = wall_ms(lambda: rans.encode_streams(streams))
        entry["identical_payload"] = bytes(ref_payload) == payload
        models = [(m[3], m[4], m[5], np.asarray(m[6], dtype=np.int64)) for m in ref_models]
        entry["reference_decode_ms"], _ = wall_ms(lambda: rans.decode_streams(ref_payload, models, len(q)))
        table = np.zeros((len(streams), codec.MAX_TOKENS), dtype=np.int64)
        rows = np.zeros((len(streams), codec.MODEL_FIELDS), dtype=np.int64)
        for k, (sp, msb, mb, cds) in enumerate(models):
            rows[k, 3:7] = (sp, msb, mb, len(cds))
            table[k, :len(cds)] = cds
        buf = np.frombuffer(bytes(ref_payload), dtype=np.uint8).copy()
        vals = np.zeros((len(streams), len(q)), dtype=np.int64)
        lib = codec._lib.load()
        p = lambda a: codec.ctypes.c_void_p(a.ctypes.data)  # noqa: E731
        entry["decode_ms"], _ = wall_ms(lambda: lib.igs_rans_decode(len(streams), len(q), p(rows), p(table), p(buf), buf.size, p(vals)))
        entry["reference_estimate_ms"], ref_est = wall_ms(lambda: [rans.estimate_stream_bits(x) for x in streams])
        entry["identical_estimates"] = bool(np.array_equal(np.array(est), np.array(ref_est)))
    except ImportError as e:
        entry["reference_note"] = str(e)
    return entry


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="cfg3_1080p")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end API leg")
    ap.add_argument("--no-stages", action="store_true", help="skip the per-stage timing")
    ap.add_argument("--split", action="store_true", help="run the step with the separate top-K forward and backward kernels instead of "
                    "the fused step kernel (for comparison)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"], help="how the tile-row bands combine their gradients")
    ap.add_argument("--no-bands", action="store_true", help="skip the 2160p tile-row band leg of the default workload")
    ap.add_argument("--aux", action="store_true", help="time the rows around the step (neighbour search, feature weights, LOO) instead")
    args = ap.parse_args()
    wl = workloads.get_workload(args.workload)
    if args.aux:
        run_aux(args)
    elif args.impl == "reference":
        run_reference(args, wl)
    elif wl.sharding == "bands":
        run_bands(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
