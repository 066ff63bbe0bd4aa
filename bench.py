"""Benchmark of the nerf_b200 training hot path (train samples/s) on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (bounded training): a seeded procedural scene of 12
spheres/boxes with value-noise albedo in [-1.5,1.5]^3, 100 training views at
800x800 rendered exactly on the host (stands in for the Blender dataset);
hash grid L16 F2 T=2^19 N_max=2048; <= 1024 steps per ray; 2^18 target
compacted samples per step per GPU; 128^3 occupancy refreshed every 16 steps;
random background; Adam lr 1e-2, betas 0.9/0.99, eps 1e-15.  One "step" is
one nerf_train_step.  The timed steps run after an untimed pretrain of 2000
steps: past the occupancy warm-up and the ~1440 steps the decayed warm-up
densities need to fall below the threshold, so empty space is pruned and the
steps measure steady-state training.

value: compacted samples trained per second over all ranks (device time, CUDA
events on each context's stream, max over ranks).  e2e: the same metric for
a whole job through the C ABI from pinned host memory: create (uploads the
images), configure, then every step nerf_train_step + nerf_read_train_stats
(20-byte device-to-host read).  Extra keys: roofline of the dominant kernel
from event-timed kernel-by-kernel steps, per-kernel times with their own
bounds, held-out PSNR after the configuration's step count (training goes on
after the timed steps: config 2 20k steps, config 4 10k), render MRays/s
(config 3: the 200 orbit views), cpu_baseline (the CPU oracle on a bounded
sample of the same step shape).

--impl reference times the reference algorithm's CPU implementation (the
oracle port; the reference backend has no CPU path) on the host cores, rank 0
only; its line also carries "reference_cuda": the reference's own CUDA
backend (built from its sources for sm_100a) timed through its nerf.h on
this GPU (training samples/s, held-out PSNR, render MRays/s).
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# ---------------------------------------------------------------- workload
CFG2 = dict(kind=1, seed=2, n_primitives=12, density=100.0, extent=1.0, size_min=0.1, size_max=0.6, n_views=100,
            width=800, height=800, fov=0.69, radius=4.0, camera_mode=1)
AABB2 = ((-1.5, -1.5, -1.5), (1.5, 1.5, 1.5))
TARGET_SAMPLES = 1 << 18
MAX_STEPS_PER_RAY = 1024
GRID_RES = 128
# BASELINE config 4 (large unbounded-style scene; `--config 4`): 40 spheres/boxes on a ground slab inside a sky shell
# at radius 12, cameras on a radius-3 ring at height 0.3 looking outward and inward, 1920x1080 (300 views in the
# configuration; --views sets the count, default 60); five 128^3 occupancy cascades over the AABB [-1,1]^3 scaled by
# up to 16; hash grid L16 F2 T2^22 N_max 8192.  The field of view is not given by the configuration: 1.2 rad.
CFG4 = dict(kind=2, seed=4, n_primitives=40, density=100.0, extent=6.0, size_min=0.1, size_max=0.6, n_views=60,
            width=1920, height=1080, fov=1.2, radius=3.0, camera_mode=3, orbit_elevation=0.3, orbit_views=300)
AABB4 = ((-1.0, -1.0, -1.0), (1.0, 1.0, 1.0))
CASCADES4 = 5
CONFIG = 2  # the workload bench.py runs (main() sets it from --config)
WORKLOAD = ("config2 bounded training: 12 spheres/boxes, 100 views 800x800, hash L16 F2 T2^19 Nmax2048, "
            "2^18 target samples/step/GPU, <=1024 steps/ray, 128^3 occupancy every 16 steps, random bg")


WORKLOAD4 = ("config4 unbounded-style training: 40 spheres/boxes on a ground slab, sky shell r=12, 1920x1080 ring views, "
             "hash L16 F2 T2^22 Nmax8192, 5 occupancy cascades of 128^3 (scale 16), 2^18 target samples/step/GPU, "
             "<=1024 steps/ray, one cascade's worth of cells refreshed every 16 steps, random bg")


def workload_name():
    return WORKLOAD4 if CONFIG == 4 else WORKLOAD


def metric_name():
    return f"train samples/s (config {CONFIG}, steady state)"


def config_dict(args):
    """The workload both arms run (the same dict in the reference arm's line)."""
    return {"workload": workload_name(), "pretrain_steps": args.pretrain,
            "l2": "inputs larger than L2: each step streams the 171 MB fp32 master/m/v through Adam and reads a 256 MB "
                  "image set; the 24 MB hash table is meant to stay L2-resident"}


def options(nb, **kw):
    if CONFIG == 4:
        return nb.default_options(log2_hashmap_size=22, max_resolution=8192, background=1, stop_transmittance=1e-4,
                                  target_samples_per_step=TARGET_SAMPLES, max_samples_per_step=2 * TARGET_SAMPLES,
                                  n_cascades=CASCADES4, **kw)
    return nb.default_options(log2_hashmap_size=19, max_resolution=2048, background=1, stop_transmittance=1e-4,
                              target_samples_per_step=TARGET_SAMPLES, max_samples_per_step=2 * TARGET_SAMPLES, **kw)


def train_config(nb):
    # config 4: 5 x 128^3 cells; each refresh queries 128^3 of them (round robin), so every cell is refreshed every
    # 80 steps
    return nb.training_config(aabb=AABB4 if CONFIG == 4 else AABB2, rays=4096, steps=MAX_STEPS_PER_RAY, lr=1e-2,
                              beta1=0.9, beta2=0.99, eps=1e-15, clip=1e9, guard=1e12, loss_scale=128.0,
                              lr_decay_ksteps=0, decay=0.95, threshold=0.01, cells_per_update=GRID_RES ** 3,
                              update_interval=16, warmup=256)


def scene_cfg():
    return CFG4 if CONFIG == 4 else CFG2


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []  # (arrival time, csv line)
        self.window = (0.0, float("inf"))

    def start(self):
        """Starts sampling (nvidia-smi needs a moment to start: call before the warm-up steps)."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, t0, t1):
        """The timed region, as host times; samples that arrive within it (plus one interval) count."""
        self.window = (t0, t1 + 0.06)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, l in self.lines:
            if not (self.window[0] <= ts <= self.window[1]):
                continue
            parts = [x.strip() for x in l.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_dataset(nb, views=None, renderer=None):
    """The training views of the workload.  renderer: the scene function (default nb.make_scene, the product
    library's copy of the scene renderer; the reference arm passes oracle_scene, the oracle library's copy of the
    same source, so that it never loads libnerf_b200.so)."""
    cfg = dict(scene_cfg())
    if views is not None:
        cfg["n_views"] = views
    if CONFIG == 4:  # the ring is shared out over the views actually rendered
        cfg["orbit_views"] = cfg["n_views"]
    t0 = time.time()
    ds = (renderer or nb.make_scene)(**cfg)
    return ds, time.time() - t0


def cached_dataset(nb, args, rank, world):
    """make_dataset, or with --scene-cache DIR the same views from DIR (rank 0 renders and writes them once; the
    other ranks, and later runs of the same configuration, load them), so that a multi-GPU or multi-run measurement
    of a large scene does not render it once per rank and per run.  The file holds exactly what the renderer
    produced."""
    if not args.scene_cache:
        return make_dataset(nb, args.views)
    import torch.distributed as dist
    views = args.views or scene_cfg()["n_views"]
    path = pathlib.Path(args.scene_cache) / f"scene_config{CONFIG}_views{views}.npz"
    t0 = time.time()
    if rank == 0 and not path.exists():
        ds, _ = make_dataset(nb, args.views)
        try:
            path.parent.mkdir(parents=True, exist_ok=True)
            tmp = path.with_suffix(".tmp.npz")
            np.savez(tmp, images=ds.images, cameras=ds.cameras, intrinsics=np.array(ds.intrinsics, np.float64))
            tmp.rename(path)
        except OSError as e:  # no room for the cache: every rank renders its own copy
            print(f"scene cache not written ({e})", file=sys.stderr)
    if world > 1:
        dist.barrier()
    if not path.exists():
        return make_dataset(nb, args.views)
    z = np.load(path)
    ds = nb.Dataset(np.ascontiguousarray(z["images"]), np.ascontiguousarray(z["cameras"]),
                    tuple(float(x) for x in z["intrinsics"]))
    return ds, time.time() - t0


def oracle_scene(**cfg):
    """nb.make_scene through the oracle library (oracle_scene_render: the same scene.cpp, built into liboracle.so)."""
    import nerf_b200 as nb  # the Dataset container only; this loads no native library
    from oracle import oracle
    imgs, cams, intr = oracle.make_scene(**cfg)
    return nb.Dataset(imgs, cams, intr)


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import ctypes as C

    import torch
    import torch.distributed as dist

    import nerf_b200 as nb
    from nerf_b200 import abi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=__import__("datetime").timedelta(seconds=300))

    lib = abi.load()
    ds, gen_s = cached_dataset(nb, args, rank, world)
    ds_pinned = None
    if not args.skip_e2e:  # host buffer of the e2e job, pinned up front (as a caller would keep its images)
        pinned_imgs = torch.from_numpy(ds.images).pin_memory()
        ds_pinned = nb.Dataset(pinned_imgs.numpy(), ds.cameras, ds.intrinsics)

    ctx = nb.Context(ds, grid_res=GRID_RES, max_sample_steps=2 * TARGET_SAMPLES, max_batch_rays=1 << 16,
                     options=options(nb))
    if world > 1:
        dp_setup(nb, ctx, rank, world)
    ctx.configure(train_config(nb))
    sp = C.c_void_p()
    abi.check("stream", lib.nerf_b200_context_stream(ctx.handle, C.byref(sp)))
    stream = torch.cuda.ExternalStream(sp.value)

    def step():
        if args.eager:  # the same kernels launched one by one (nerf_b200_train_step_profiled): no graph launches
            abi.check("eager step", lib.nerf_b200_train_step_profiled(ctx.handle, C.byref(abi.NerfB200StepProfile())))
        else:
            ctx.train_step()

    clocks = ClockSampler(local)
    clocks.start()  # running well before the timed region
    state_in = args.state_in and pathlib.Path(args.state_in).exists() and world == 1
    if state_in:  # the pretrained training state of an earlier run (exact resume), instead of the pretrain steps
        ctx.load_state(args.state_in)
    else:
        for _ in range(args.pretrain):
            step()
        if args.state_out and world == 1:
            ctx.save_state(args.state_out)
    for _ in range(args.warmup):
        step()
    c0 = ctx.counters()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    h0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(h0, time.time())
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    c1 = ctx.counters()
    kernels_per_step = int(c1.kernels_per_step)  # this library's launches per step, as the library counts them
    samples = c1.total_samples - c0.total_samples
    rays = c1.total_rays - c0.total_rays
    t = torch.tensor([ms, float(samples), float(rays)], dtype=torch.float64, device="cuda")
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        ms_max, samples_all, rays_all = float(tmax[0]), float(tsum[1]), float(tsum[2])
    else:
        ms_max, samples_all, rays_all = ms, float(samples), float(rays)
    value = samples_all / (ms_max / 1e3)
    stats = ctx.stats()

    # Kernel-by-kernel timing of the same step (events between launches).
    prof = np.zeros(len(abi.STEP_KERNELS))
    n_prof = args.profile_steps
    prof_samples = 0
    for _ in range(n_prof):
        cb = ctx.counters()
        p = abi.NerfB200StepProfile()
        abi.check("profiled step", lib.nerf_b200_train_step_profiled(ctx.handle, C.byref(p)))
        prof += np.array(p.milliseconds[:])
        prof_samples += ctx.counters().total_samples - cb.total_samples
    prof /= max(1, n_prof)
    mean_samples = prof_samples / max(1, n_prof)
    l2 = l2_peaks(stream)
    kernels = kernel_table(ctx, prof, mean_samples, l2, world)

    # Train on to the configuration's step count (config 2: 20k steps, config 4: 10k) before the held-out PSNR;
    # every rank steps (the data-parallel step is collective), rank 0 measures.
    psnr = None
    if args.psnr_views > 0:
        while ctx.counters().frame_index < args.psnr_steps:
            ctx.train_step()
        psnr = psnr_heldout(nb, ctx, args) if rank == 0 else None
    render = None
    if not args.skip_render:
        render = run_render(nb, ctx, rank, world, args)

    e2e = None
    if not args.skip_e2e:
        ctx.close()
        torch.cuda.synchronize()
        e2e = run_e2e(nb, lib, ds_pinned, rank, world, args)

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:  # the CPU baseline: rank 0 at N = 1 only
        cpu = cpu_baseline(ds, args)
    dio = None
    if rank == 0 and not args.skip_dataset_io:
        dio = dataset_io(lib, ds)

    if rank == 0:
        line = {
            "metric": metric_name(),
            "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 (fp32 accumulate, fp32 Adam masters)", "data": "synthetic",
            "config": config_dict(args),
            "parallelism": f"dp{world}",
            "run": {"samples_per_step": samples_all / args.steps, "rays_per_step": rays_all / args.steps,
                    "final_loss": stats.loss, "dataset_gen_s": gen_s},
            "e2e": e2e,
            "gpu_launches": kernels_per_step * args.steps,
            "roofline": roofline(kernels),
            "l2": l2,
            "kernels": kernels,
            "render": render,
            "psnr": psnr,
            "cpu_baseline": cpu,
            "dataset_io": dio,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# Per training sample, from one ncu capture of this build's step kernels on config 2 (steady state, the eager
# step resumed from a saved training state): L1 sectors the forward's gathers request (the hash-table lookups after
# coalescing and pairing; about half hit in L1), and L2 f16x2 reduction operations the scatter issues (after run
# merging and 16-byte pairing).  Counts over the captured launch / the samples of that step.
NCU_PER_SAMPLE = {"field_forward_l1_sectors": 48.1, "field_forward_l2_sectors": 26.6, "grid_scatter_l2_red_ops": 38.0}
# DRAM bytes (read + write) per launch from the same capture (cold-cache replay, so the hash table and its gradient
# count as DRAM traffic although a live step keeps them in L2).
NCU_TRAFFIC = {"mlp_backward": 36.41e6, "grid_scatter": 71.09e6, "field_forward": 30.58e6, "adam": 311.31e6}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops_sustained": float(d["bf16_tflops_sustained"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def kernel_table(ctx, prof_ms, samples, l2, world):
    """Each step kernel against the roofline that bounds it.  Algorithmic work per launch (per-unit figures in the
    comments) / the kernel's mean CUDA-event time in the kernel-by-kernel step, over the measured peak of its bound:
    HBM copy bandwidth (MEASURED_PEAKS.json), the sustained bf16 tensor rate (same file; these kernels run inside a
    long step), or the live L2 probes (gathers and f16x2 reductions at hashed addresses, 16-byte reads)."""
    from nerf_b200 import abi
    pk = measured_peaks()
    n_params, n_grid = ctx.n_params, ctx.n_grid
    cells = GRID_RES ** 3 * (CASCADES4 if CONFIG == 4 else 1)
    # (bound, unit, algorithmic amount per launch, note)
    per = {
        # one thread per 32-cell word: density read + write 8 B per cell, bitfield word 1/8 B per cell
        "occupancy_update": ("hbm", cells * 8 + cells // 8),
        # t of every kept step written to the ray's kept list
        "sample_bits": ("latency", samples * 4),
        # kept t read, pos/dt 16 + ray id 4 written
        "sample_write": ("hbm", samples * (4 + 16 + 4)),
        # L1 sectors the corner lookups request per sample (ncu), against the sector rate of the hashed 4-byte
        # gather probe (one sector per load); algorithmic bytes: pos/dt 16 + ray id 4 + 512 corner bytes + 112
        # training row + 16 raw out, against the 16-byte L2 read probe
        "field_forward": ("l2_gather", samples * NCU_PER_SAMPLE["field_forward_l1_sectors"]),
        # raw 16 + pos/dt 16 read twice, dout 16 written, transmittance 8
        "composite": ("hbm", samples * (2 * 32 + 16 + 8)),
        # forward recompute 20,480 + input-gradient 20,480 + weight-gradient 20,480 FLOP per sample
        "mlp_backward": ("tensor", samples * 61440),
        # L2 reduction operations issued per sample (ncu), against the .v4 f16x2 reduction probe
        "grid_scatter": ("l2_red", samples * NCU_PER_SAMPLE["grid_scatter_l2_red_ops"]),
        # partials: one row of 10240 fp32 per backward CTA read, 10240 sums written
        "wgrad_reduce": ("hbm", (ctx_partials(ctx) + 1) * 10240 * 4),
        # fp16 hash gradients 2 B and fp32 MLP gradients 4 B read
        "grad_stats": ("hbm", n_grid * 2 + (n_params - n_grid) * 4),
        # fp32 master, m, v read + written (24), fp16 gradient read + cleared (4), fp16 parameter written (2)
        "adam": ("hbm", n_params * 30),
        # peer mode: this rank's 1/N of every rank's fp16 hash gradients read over NVLink
        "allreduce": ("nvlink", n_grid * 2 * (world - 1) / max(world, 1)),
        "occupancy_query": ("latency", 0),
        "sample_scan": ("latency", 0),
        "march": ("latency", 0),
    }
    out = []
    for name, ms in zip(abi.STEP_KERNELS, prof_ms):
        bound, amount = per.get(name, ("latency", 0))
        rec = {"kernel": name, "ms": float(ms), "bound": bound}
        t = ms / 1e3
        if ms > 0 and amount:
            if bound == "hbm":
                rec.update(achieved=amount / t / 1e9, peak=pk["hbm_gbs"], unit="GB/s")
            elif bound == "tensor":
                rec.update(achieved=amount / t / 1e12, peak=pk["bf16_tflops_sustained"], unit="TFLOP/s")
            elif bound == "l2_gather":
                rec.update(achieved=amount / t / 1e9, peak=l2["gather_4b_gops"], unit="G L1 sectors/s",
                           corner_lookups_g_per_s=samples * 128 / t / 1e9,
                           l2_sectors_g_per_s=samples * NCU_PER_SAMPLE["field_forward_l2_sectors"] / t / 1e9,
                           l2_read_gbs=samples * 660 / t / 1e9, l2_read_frac=samples * 660 / t / 1e9 / l2["read_gbs"])
            elif bound == "l2_red":
                rec.update(achieved=amount / t / 1e9, peak=l2["red_v4_f16x2_gops"], unit="G red ops/s",
                           corner_updates_g_per_s=samples * 128 / t / 1e9)
            elif bound == "nvlink":
                rec.update(achieved=amount / t / 1e9, peak=770.0, unit="GB/s")
            else:
                rec.update(bytes=int(amount), gbs=amount / t / 1e9)
            if "peak" in rec:
                rec["frac"] = rec["achieved"] / rec["peak"]
        out.append(rec)
    return out


def probe_lib():
    """libnerf_b200_l2probe.so: the benchmark's L2 microbenchmarks (a library of their own, not part of the
    product library)."""
    import ctypes as C
    path = ROOT / "nerf_b200" / "libnerf_b200_l2probe.so"
    if not path.exists():
        raise RuntimeError(f"{path} is not built (make -C nerf_b200/csrc)")
    lib = C.CDLL(str(path))
    P, U32 = C.c_void_p, C.c_uint32
    lib.nerf_b200_probe_l2_read.argtypes = [P, C.c_uint64, U32, P, P]
    lib.nerf_b200_probe_l2_red.argtypes = [P, U32, U32, U32, C.POINTER(C.c_uint64), P]
    lib.nerf_b200_probe_l2_gather.argtypes = [P, U32, U32, U32, P, C.POINTER(C.c_uint64), P]
    for f in (lib.nerf_b200_probe_l2_read, lib.nerf_b200_probe_l2_red, lib.nerf_b200_probe_l2_gather):
        f.restype = C.c_int
    return lib


def l2_peaks(stream):
    """L2 peaks of this GPU from the benchmark's probes: 16-byte read bandwidth of an L2-resident 64 MB buffer,
    4- and 8-byte gathers at hashed addresses of a 32 MB buffer (the shape of the hash-table lookups), and f16x2 /
    v2 / v4 reduction rates at hashed addresses of the same buffer (the shape of the hash-table scatter)."""
    import ctypes as C

    import torch
    lib = probe_lib()
    h = C.c_void_p(stream.cuda_stream)
    sink = torch.zeros(1024, dtype=torch.int32, device="cuda")
    res = {}

    def timed(fn, reps=5):
        fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    buf = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    passes = 16
    t = timed(lambda: lib.nerf_b200_probe_l2_read(buf.data_ptr(), buf.numel(), passes, sink.data_ptr(), h))
    res["read_gbs"] = buf.numel() * passes / t / 1e9
    del buf
    words = 1 << 23
    rb = torch.zeros(words, dtype=torch.int32, device="cuda")
    ops = C.c_uint64()
    for vec, key in ((0, "red_f16x2_gops"), (1, "red_v2_f16x2_gops"), (2, "red_v4_f16x2_gops")):
        t = timed(lambda: lib.nerf_b200_probe_l2_red(rb.data_ptr(), words, 64, vec, C.byref(ops), h))
        res[key] = ops.value / t / 1e9
    for vec, key in ((0, "gather_4b_gops"), (1, "gather_8b_gops")):
        t = timed(lambda: lib.nerf_b200_probe_l2_gather(rb.data_ptr(), words, 64, vec, sink.data_ptr(), C.byref(ops), h))
        res[key] = ops.value / t / 1e9
    res["note"] = ("probes: 64 MB L2-resident buffer, 16 sweeps of 16-byte loads; 4- / 8-byte loads and f16x2 "
                   "reductions (v2 / v4: 8- / 16-byte forms) at hashed word addresses of a 32 MB buffer, 64 per thread "
                   "over 8 blocks x 256 threads per SM")
    return res


def ctx_partials(ctx):
    from nerf_b200 import abi
    return int(abi.load().nerf_b200_field_backward_partial_floats()) // 10240


def roofline(kernels):
    """The dominant kernel (longest mean time in the kernel-by-kernel step) against its own bound."""
    pk = measured_peaks()
    timed = [k for k in kernels if "frac" in k]
    if not timed:  # no kernel-by-kernel steps were run (--profile-steps 0)
        return None
    dom = max(timed, key=lambda k: k["ms"])
    src = {"hbm": f"MEASURED_PEAKS.json hbm_gbs ({pk['source']})",
           "tensor": f"MEASURED_PEAKS.json bf16_tflops_sustained ({pk['source']})",
           "l2_gather": "live probe: 4-byte loads at hashed addresses of an L2-resident 32 MB buffer (one sector each)",
           "l2_red": "live probe: 16-byte f16x2 reductions at hashed addresses of an L2-resident 32 MB buffer",
           "nvlink": "measured peer copy, 770 GB/s per direction"}[dom["bound"]]
    return {"kernel": dom["kernel"], "bound": dom["bound"], "achieved": dom["achieved"], "peak": dom["peak"],
            "unit": dom["unit"], "frac": dom["frac"], "peak_source": src,
            "traffic": NCU_TRAFFIC.get(dom["kernel"]),
            "note": "achieved = algorithmic work per launch / mean CUDA-event launch time (kernel-by-kernel step, "
                    "same kernels as the graph); traffic = ncu DRAM bytes per launch (cold-cache replay); every "
                    "step kernel's own bound and fraction is in the kernels list"}


def psnr_heldout(nb, ctx, args):
    """PSNR of the trained model on held-out views (config 2: cameras after the 100 training views; config 4: ring
    positions between the training views), ground truth composited on white, the render's background."""
    n = args.psnr_views
    if n <= 0:
        return None
    sc = scene_cfg()
    if CONFIG == 4:  # ring positions halfway between training views, and training positions looking the other way
        n_train = args.views or sc["n_views"]
        held = nb.make_scene(**{**sc, "n_views": n, "view_offset": 1, "orbit_views": 2 * n_train})
    else:
        held = nb.make_scene(**{**sc, "n_views": n, "view_offset": sc["n_views"], "orbit_views": sc["n_views"] + n})
    W, H = sc["width"], sc["height"]
    errs = []
    img = np.zeros((H, W, 4), np.uint8)
    for v in range(n):
        ctx.render(held.cameras[v], W, H, held.intrinsics, max_steps=MAX_STEPS_PER_RAY, stop=1e-4, dst=img)
        gt = held.images[v].astype(np.float64) / 255.0
        ref = gt[..., :3] * gt[..., 3:4] + (1.0 - gt[..., 3:4])
        out = img[..., :3].astype(np.float64) / 255.0
        errs.append(float(np.mean((out - ref) ** 2)))
    psnr = [10.0 * np.log10(1.0 / max(e, 1e-12)) for e in errs]
    return {"value": float(np.mean(psnr)), "unit": "dB", "views": n, "resolution": f"{W}x{H}",
            "train_steps": int(ctx.counters().frame_index),
            "note": "mean over held-out views (config 2: the cameras after the training views; config 4: ring "
                    "positions between the training views) of PSNR against the exact render composited on white; "
                    "rendered with the training occupancy grid, T < 1e-4 termination"}


def run_render(nb, ctx, rank, world, args):
    """Config 3: config-2 architecture, seeded random-init weights, fixed 30% Bernoulli(seed 1) occupancy,
    orbit views at radius 4 (800x800), T < 1e-4 termination, 64x64 tiles round-robin over the ranks."""
    import torch
    import torch.distributed as dist
    ds = ctx.ds
    views = nb.make_scene(**{**CFG2, "n_views": args.render_views, "camera_mode": 2, "orbit_elevation": 0.35,
                             "orbit_views": 200, "view_offset": 0}, with_images=False)
    rctx = nb.Context(nb.Dataset(ds.images[:1], ds.cameras[:1], ds.intrinsics), grid_res=GRID_RES,
                      max_sample_steps=1 << 16, max_batch_rays=4096, options=options(nb))
    rctx.configure(train_config(nb))
    rng = np.random.default_rng(1)
    bits = np.packbits(rng.random(GRID_RES ** 3) < 0.3, bitorder="little").view(np.uint32)
    rctx.set_occupancy(bitfield=bits)
    W, H = 800, 800
    for v in range(min(2, args.render_views)):  # warm-up
        rctx.render(views.cameras[v], W, H, views.intrinsics, max_steps=MAX_STEPS_PER_RAY, stop=1e-4, tile=64, rank=rank,
                    world=world)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    ms = 0.0
    rays = samples = 0
    for v in range(args.render_views):
        info = rctx.render(views.cameras[v], W, H, views.intrinsics, max_steps=MAX_STEPS_PER_RAY, stop=1e-4, tile=64,
                           rank=rank, world=world)
        ms += info.milliseconds
        rays += info.rays
        samples += info.samples
    wall = time.time() - t0
    t = torch.tensor([ms, float(rays), float(samples)], dtype=torch.float64, device="cuda")
    if world > 1:
        tm = t.clone()
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ts = t.clone()
        dist.all_reduce(ts, op=dist.ReduceOp.SUM)
        ms, rays, samples = float(tm[0]), float(ts[1]), float(ts[2])
    rctx.close()
    return {"metric": "render MRays/s (config 3)", "value": rays / (ms / 1e3) / 1e6, "unit": "MRays/s",
            "views": args.render_views, "resolution": "800x800", "samples_per_ray": samples / max(rays, 1),
            "device_ms": ms, "wall_s": wall, "tiles": "64x64 round-robin over ranks"}


def dp_setup(nb, ctx, rank, world):
    """Data-parallel set-up of a context.  Peer mode (default): the ranks' peer handles are all-gathered over the
    job's own process group and mapped (nerf_b200_dp_init_peers; no NCCL communicator of the library's own).
    NERF_B200_DP_PEER=0: the NCCL all-reduce path (nerf_b200_dp_init with a fresh NCCL id)."""
    import torch.distributed as dist
    if os.environ.get("NERF_B200_DP_PEER", "1") == "0":
        obj = [nb.dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.dp_init(rank, world, obj[0])
        return
    handles = [None] * world
    dist.all_gather_object(handles, ctx.dp_peer_handle())
    ctx.dp_init_peers(rank, world, handles)


def run_e2e(nb, lib, ds_pinned, rank, world, args):
    """Whole job through the C ABI with host buffers: create (uploads the pinned images), data-parallel set-up,
    configure, and each step nerf_train_step + nerf_read_train_stats.  Samples come from the additive counters
    export."""
    import torch
    import torch.distributed as dist
    steps = args.e2e_steps
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ctx = nb.Context(ds_pinned, grid_res=GRID_RES, max_sample_steps=2 * TARGET_SAMPLES, max_batch_rays=1 << 16,
                     options=options(nb))
    t_upload = time.perf_counter()
    if world > 1:
        dp_setup(nb, ctx, rank, world)
    t_create = time.perf_counter()
    ctx.configure(train_config(nb))
    t_configure = time.perf_counter()
    for _ in range(steps):
        ctx.train_step()
        ctx.stats()
    t1 = time.perf_counter()
    c = ctx.counters()
    ctx.close()
    t = torch.tensor([t1 - t0, float(c.total_samples)], dtype=torch.float64, device="cuda")
    if world > 1:
        tm = t.clone()
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ts = t.clone()
        dist.all_reduce(ts, op=dist.ReduceOp.SUM)
        secs, samples = float(tm[0]), float(ts[1])
    else:
        secs, samples = float(t[0]), float(t[1])
    h2d = ds_pinned.images.nbytes + ds_pinned.cameras.nbytes
    return {"value": samples / secs, "unit": "samples/s", "steps": steps, "seconds": secs,
            "create_upload_s": t_upload - t0, "dp_setup_s": t_create - t_upload, "configure_s": t_configure - t_create,
            "steps_s": t1 - t_configure,
            "h2d_bytes_per_step": h2d / steps, "d2h_bytes_per_step": 20,
            "note": "create+upload, data-parallel set-up (peer handles all-gathered and mapped), configure and every "
                    "step train_step + read_train_stats, wall clock on each rank (the phases: rank 0's), max over "
                    "ranks; includes the occupancy warm-up phase of a fresh job"}


def dataset_io(lib, ds):
    """The config-2 dataset through the reference's file format (Blender transforms JSON + RGBA8 PNG): written once,
    then loaded into pinned host memory with all host threads and with one (the reference driver decodes its PNGs one
    after another with stb_image, benchmark.cpp:188-205)."""
    import ctypes as C
    import shutil
    import tempfile

    import torch
    from nerf_b200 import abi
    n, h, w = ds.images.shape[:3]
    d = tempfile.mkdtemp(prefix="nerf_b200_ds_")
    try:
        imgs = np.ascontiguousarray(ds.images)
        cams = np.ascontiguousarray(ds.cameras)
        t0 = time.perf_counter()
        abi.check("blender write", lib.nerf_b200_blender_write(d.encode(), imgs.ctypes.data, cams.ctypes.data, n, w, h,
                                                              CFG2["fov"], 0))
        t_write = time.perf_counter() - t0
        dst = torch.empty(imgs.nbytes, dtype=torch.uint8)
        if torch.cuda.is_available():
            dst = dst.pin_memory()
        cam_out = np.zeros((n, 4, 4), np.float32)
        intr = np.zeros(4, np.float32)
        res = {"images": n, "resolution": f"{w}x{h}", "bytes_rgba8": int(imgs.nbytes), "write_s": t_write}
        for threads, key in ((0, "load_all_threads"), (1, "load_one_thread")):
            t0 = time.perf_counter()
            abi.check("blender load", lib.nerf_b200_blender_load(d.encode(), 0, threads, dst.data_ptr(), imgs.nbytes,
                                                                cam_out.ctypes.data, intr.ctypes.data))
            dt = time.perf_counter() - t0
            res[key] = {"s": dt, "images_per_s": n / dt, "MB_per_s": imgs.nbytes / dt / 1e6}
        res["bit_exact"] = bool(np.array_equal(dst.numpy().reshape(imgs.shape), imgs))
        res["threads"] = os.cpu_count()
        res["note"] = ("PNG stored-deflate files written by nerf_b200_blender_write, decoded by nerf_b200_blender_load "
                       "(inflate, CRC-32 / Adler-32 checks, unfilter) into pinned memory; host wall clock")
        return res
    finally:
        shutil.rmtree(d, ignore_errors=True)


def cpu_baseline(ds, args, threads=None, seconds=20.0, max_steps=None):
    """The CPU oracle (the scalar C++ restatement of the same algorithm) on the workload's own step shape: 4096
    initial rays, 2^18 target samples per step, 2^19 capacity, <= 1024 steps per ray, on all host threads.  The
    sample is bounded by wall time, not by shrinking the batch: one untimed step (the fresh job's first step, cut at
    the 2^19 capacity), then whole steps until `seconds` have passed (at least two).  Returns the samples/s of the
    timed steps."""
    from oracle import oracle
    from nerf_b200.abi import NerfCreateDesc
    import nerf_b200 as nb  # ctypes structures and the training-config builder only; no native library is loaded
    threads = threads or os.cpu_count() or 1
    images = np.ascontiguousarray(ds.images)
    cams = np.ascontiguousarray(ds.cameras)
    fx, fy, cx, cy = ds.intrinsics
    d = NerfCreateDesc(GRID_RES, 2 * TARGET_SAMPLES, 1 << 16, 256, images.ctypes.data, images.nbytes, cams.ctypes.data,
                       cams.nbytes, ds.n, ds.width, ds.height, fx, fy, cx, cy)
    big = CONFIG == 4
    oc = oracle.Context(d, oracle.options(log2_hashmap_size=22 if big else 19, max_resolution=8192 if big else 2048,
                                          background=1, stop_transmittance=1e-4, target_samples_per_step=TARGET_SAMPLES,
                                          max_samples_per_step=2 * TARGET_SAMPLES, n_threads=threads,
                                          n_cascades=CASCADES4 if big else 1), images, cams)
    oc.configure(train_config(nb))
    oc.step()  # untimed: the first step of a fresh job (all cells occupied, cut at the capacity)
    first = oc.info().samples
    t0 = time.perf_counter()
    samples = n = 0
    while True:
        oc.step()
        samples += oc.info().samples
        n += 1
        el = time.perf_counter() - t0
        if n >= 2 and (el > seconds or (max_steps and n >= max_steps)):
            break
    dt = time.perf_counter() - t0
    oc.close()
    return {"value": samples / dt, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{n} whole oracle training steps of config {CONFIG} after one untimed step ({first} samples): "
                      f"{samples} samples in {dt:.1f} s, 4096 initial rays, 2^18 target samples per step, "
                      f"occupancy warm-up phase of a fresh job"}


# ------------------------------------------------------------ microbench
def run_micro(args):
    """the kernel-level entry points on seeded synthetic inputs, each point against its roofline.

    encode fwd / bwd (nerf_b200_grid_forward / _backward): n points U[0,1]^3, L16 F2 fp16, N_max 2048,
      T = 2^14..2^24; bwd upstream gradients N(0,1).  Algorithmic bytes per point: fwd 12 in + 128 x 4 gathers +
      64 out = 588; bwd 12 + 64 in + 128 x 8 read-modify-write = 1100.  Tables that fit L2 are compared with the
      live L2 probes (fwd: 16-byte L2 read GB/s; bwd: corner reductions / s against the f16x2 reduction rate),
      larger tables with the measured HBM copy peak.
    MLP fwd / bwd (nerf_b200_mlp_forward / _backward, the fused field's MLPs on given features): rows of 32 fp16
      features N(0,1) and unit directions; 20,480 FLOP per row forward, 61,440 backward (forward recompute,
      input-gradient and weight-gradient products), against the measured dense bf16 peak.
    composite fwd+bwd (nerf_b200_composite, one fused kernel): 2^16 rays x S samples, sigma ~ Exp(1) (raw =
      log sigma), rgb U[0,1] (raw = logit), dt = 1/S, no early termination; 88 bytes per sample for this two-pass
      layout (raw 16 + pos_dt 16 read in each pass, transmittance 8, d raw 16 written), against HBM.
    Each point: 2 untimed launches, then the mean of `reps` launches between CUDA events on one stream.
    """
    import ctypes as C

    import torch

    import nerf_b200 as nb
    from nerf_b200 import abi

    torch.cuda.set_device(0)
    lib = abi.load()
    stream = torch.cuda.current_stream()
    h = C.c_void_p(stream.cuda_stream)
    hbm, src = peaks()
    tf_peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"]) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    l2 = l2_peaks(stream)
    gen = torch.Generator(device="cuda").manual_seed(5)
    reps = args.micro_reps

    def timed(fn):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    def st(name, rc):
        abi.check(name, rc)

    out = {"encode": [], "mlp": [], "composite": []}
    L = 16
    for log2n in args.micro_points:
        n = 1 << log2n
        pos = torch.rand((n, 3), generator=gen, device="cuda", dtype=torch.float32)
        feat = torch.empty((n, 2 * L), device="cuda", dtype=torch.float16)
        dfeat = torch.randn((n, 2 * L), generator=gen, device="cuda", dtype=torch.float32).half()
        for log2T in args.micro_tables:
            g = nb.grid_layout(L, log2T, 16, 2048)
            entries = int(g.offset[L])
            table_mb = entries * 4 / 1e6
            params = (torch.rand(2 * entries, generator=gen, device="cuda") * 2e-4 - 1e-4).half()
            grad = torch.zeros(2 * entries, device="cuda", dtype=torch.float16)
            tf = timed(lambda: st("grid_forward", lib.nerf_b200_grid_forward(
                C.byref(g), pos.data_ptr(), n, params.data_ptr(), feat.data_ptr(), h)))
            tb = timed(lambda: st("grid_backward", lib.nerf_b200_grid_backward(
                C.byref(g), pos.data_ptr(), n, dfeat.data_ptr(), grad.data_ptr(), h)))
            in_l2 = table_mb < 100.0
            fwd_gbs, bwd_gbs = n * 588 / tf / 1e9, n * 1100 / tb / 1e9
            red_gops = n * 128 / tb / 1e9
            rec = {"points": n, "log2_T": log2T, "table_MB": table_mb, "fwd_ms": tf * 1e3, "bwd_ms": tb * 1e3,
                   "fwd_gbs": fwd_gbs, "bwd_gbs": bwd_gbs, "bwd_corner_updates_g_per_s": red_gops,
                   "bound": "L2" if in_l2 else "HBM",
                   "fwd_frac": fwd_gbs / (l2["read_gbs"] if in_l2 else hbm),
                   "bwd_frac": (red_gops / l2["red_f16x2_gops"]) if in_l2 else bwd_gbs / hbm}
            if in_l2:
                # Random points: per level and (y, z) corner pair, the x-pair is one 8-byte load when its entries
                # form an aligned pair (1 case in 2) else two loads -> 96 sector reads per point; one 16-byte
                # reduction when both entries share an aligned 4-entry block (3 in 4) else two -> 80 ops per point.
                rec["fwd_l2_sector_frac"] = n * 96 * 32 / tf / 1e9 / l2["read_gbs"]
                rec["bwd_l2_op_frac"] = n * 80 / tb / 1e9 / l2["red_v4_f16x2_gops"]
            out["encode"].append(rec)
            del params, grad
        del pos, feat, dfeat
    torch.cuda.empty_cache()

    mlp = (torch.rand(10240, generator=gen, device="cuda") * 0.3 - 0.15).half()
    parts = torch.zeros(int(lib.nerf_b200_field_backward_partial_floats()), device="cuda", dtype=torch.float32)
    mg = torch.zeros(10240, device="cuda", dtype=torch.float32)
    for log2n in args.micro_rows:
        n = 1 << log2n
        x = torch.randn((n, 32), generator=gen, device="cuda").half()
        d = torch.randn((n, 3), generator=gen, device="cuda")
        d = (d / d.norm(dim=1, keepdim=True)).contiguous()
        raw = torch.empty((n, 4), device="cuda", dtype=torch.float32)
        dout = torch.randn((n, 4), generator=gen, device="cuda") * 0.5
        dx = torch.empty((n, 32), device="cuda", dtype=torch.float16)
        tf = timed(lambda: st("mlp_forward", lib.nerf_b200_mlp_forward(
            mlp.data_ptr(), x.data_ptr(), d.data_ptr(), n, raw.data_ptr(), h)))
        err = torch.zeros(1, device="cuda", dtype=torch.int32)
        ttc = timed(lambda: st("mlp_forward_tc", lib.nerf_b200_mlp_forward_tc(
            mlp.data_ptr(), x.data_ptr(), d.data_ptr(), n, raw.data_ptr(), err.data_ptr(), h)))
        tb = timed(lambda: st("mlp_backward", lib.nerf_b200_mlp_backward(
            mlp.data_ptr(), x.data_ptr(), d.data_ptr(), n, dout.data_ptr(), dx.data_ptr(), parts.data_ptr(),
            mg.data_ptr(), h)))
        tbc = timed(lambda: st("mlp_backward_tc", lib.nerf_b200_mlp_backward_tc(
            mlp.data_ptr(), x.data_ptr(), d.data_ptr(), n, dout.data_ptr(), dx.data_ptr(), parts.data_ptr(),
            mg.data_ptr(), err.data_ptr(), h)))
        ff, fb, ftc = n * 20480 / tf / 1e12, n * 61440 / tb / 1e12, n * 20480 / ttc / 1e12
        fbc = n * 61440 / tbc / 1e12
        out["mlp"].append({"rows": n, "fwd_ms": tf * 1e3, "bwd_ms": tb * 1e3, "fwd_tflops": ff, "bwd_tflops": fb,
                           "fwd_frac": ff / tf_peak, "bwd_frac": fb / tf_peak, "fwd_tc_ms": ttc * 1e3,
                           "fwd_tc_tflops": ftc, "fwd_tc_frac": ftc / tf_peak, "bwd_tc_ms": tbc * 1e3,
                           "bwd_tc_tflops": fbc, "bwd_tc_frac": fbc / tf_peak, "tc_error_word": int(err.item()),
                           "bound": "tensor"})
        del x, d, raw, dout, dx
    torch.cuda.empty_cache()

    rays = 1 << 16
    for S in args.micro_samples:
        m = rays * S
        rec = np.zeros((rays, 12), np.float32)
        rec[:, 0] = 1.0
        rec.view(np.uint32)[:, 3] = np.arange(rays, dtype=np.uint32) * S
        rec[:, 4:8] = 0.5
        rec[:, 8:11] = 1.0
        rec.view(np.uint32)[:, 11] = S
        rec_d = torch.from_numpy(rec).cuda()
        sig = torch.empty(m, device="cuda").exponential_(1.0, generator=gen).clamp_min(1e-12)
        col = torch.rand((m, 3), generator=gen, device="cuda").clamp(1e-6, 1 - 1e-6)
        raw = torch.cat([sig.log()[:, None], torch.log(col / (1 - col))], dim=1).contiguous()
        del sig, col
        pos = torch.zeros((m, 4), device="cuda")
        pos[:, 3] = 1.0 / S
        dout = torch.empty((m, 4), device="cuda")
        loss = torch.zeros(1, device="cuda")
        t = timed(lambda: st("composite", lib.nerf_b200_composite(
            rec_d.data_ptr(), rays, raw.data_ptr(), pos.data_ptr(), 1.0 / rays, 128.0, 0.0, dout.data_ptr(), None, None,
            loss.data_ptr(), h)))
        gbs = m * 88 / t / 1e9
        out["composite"].append({"rays": rays, "samples_per_ray": S, "ms": t * 1e3, "gbs": gbs, "frac": gbs / hbm,
                                 "bound": "HBM"})
        del raw, pos, dout, rec_d
    torch.cuda.empty_cache()
    info = (C.c_uint32 * 4)()
    lib.nerf_b200_mlp_tc_info(info)
    out["mlp_tc_launch"] = {"fwd_grid": info[0], "bwd_grid": info[1], "runtime_occupancy_fwd": info[2],
                            "runtime_occupancy_bwd": info[3]}
    line = {"metric": "kernel microbench (config 5)", "unit": "see points", "n_gpus": 1, "reps": reps,
            "peaks": {"hbm_gbs": hbm, "hbm_source": src, "bf16_tflops": tf_peak, "l2": l2},
            "dtype": "f16 (fp32 accumulate)", "data": "synthetic", **out}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ reference arm
def run_reference(args):
    """The reference arm: the CPU oracle (kind "port": the reference backend has no CPU implementation of the path)
    on this arm's own workload and config, rank 0 only, with all host threads.  It loads no product library: the
    dataset comes from the oracle library's copy of the scene renderer.  Its line also carries "reference_cuda", the
    reference's own CUDA backend (oracle/_ref/libref_stock.so) run in a child process."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ds, _ = make_dataset(None, args.views, renderer=oracle_scene)
    res = cpu_baseline(ds, args, seconds=args.reference_seconds)
    ref_cuda = None if args.skip_reference_cuda else reference_cuda(args)
    line = {"metric": metric_name(), "value": res["value"], "unit": "samples/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (fp16-rounded operands)", "data": "synthetic", "impl": "reference",
            "config": config_dict(args), "parallelism": "cpu",
            "cpu_baseline": res,
            "e2e": {"value": res["value"], "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_cuda": ref_cuda}
    print(json.dumps(line), flush=True)


def reference_cuda(args):
    """The reference's own CUDA backend (oracle/_ref/libref_stock.so: backend-cuda.cu built for sm_100a) through its
    nerf.h on this GPU: config-2 training throughput, held-out PSNR and the config-3 render.  Runs in a child
    process (the library exports the same nerf_* names as libnerf_b200.so) with a time limit."""
    lib = ROOT / "oracle" / "_ref" / "libref_stock.so"
    if not lib.exists():
        return {"unavailable": "oracle/_ref/libref_stock.so is not built (the reference checkout was absent at build)"}
    cmd = [sys.executable, "-m", "oracle.ref_backend", "--pretrain", str(args.pretrain), "--steps",
           str(args.reference_cuda_steps), "--render-views", "4", "--psnr-views", "5", "--psnr-steps",
           str(args.psnr_steps)]  # the steps after which the own arm measures PSNR
    try:
        r = subprocess.run(cmd, cwd=str(ROOT), capture_output=True, text=True, timeout=900)
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference backend run exceeded 900 s"}
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not lines:
        tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
        return {"unavailable": f"reference backend run failed (exit {r.returncode}): {tail[0][:300]}"}
    return json.loads(lines[-1])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--pretrain", type=int, default=2000)
    ap.add_argument("--profile-steps", type=int, default=20)
    ap.add_argument("--render-views", type=int, default=200, help="config-3 views rendered (the configuration's 200)")
    ap.add_argument("--psnr-views", type=int, default=20)
    ap.add_argument("--psnr-steps", type=int, default=None,
                    help="training steps before the held-out PSNR (default: the configuration's, 20k / 10k)")
    ap.add_argument("--e2e-steps", type=int, default=1000)
    ap.add_argument("--views", type=int, default=None)
    ap.add_argument("--state-out", default=None,
                    help="one GPU: save the training state after the pretrain steps (for --state-in)")
    ap.add_argument("--state-in", default=None,
                    help="one GPU: start from this saved training state instead of running the pretrain steps "
                         "(profilers: a few launches before the captured ones); ignored when the file is absent")
    ap.add_argument("--scene-cache", default=None,
                    help="directory for the rendered training views (rendered once by rank 0, then loaded)")
    ap.add_argument("--skip-render", action="store_true")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-reference-cuda", action="store_true")
    ap.add_argument("--skip-dataset-io", action="store_true")
    ap.add_argument("--config", type=int, default=2, choices=[2, 4],
                    help="2: bounded training (the headline); 4: the large unbounded-style scene with cascades")
    ap.add_argument("--micro", action="store_true", help="kernel microbench sweep (config 5) instead of the step")
    ap.add_argument("--eager", action="store_true",
                    help="launch every step kernel by kernel instead of as the captured graph (for profilers, which "
                         "are slow on graph launches; the same kernels in the same order)")
    ap.add_argument("--micro-reps", type=int, default=10)
    ap.add_argument("--micro-points", type=int, nargs="*", default=[20, 22, 24])
    ap.add_argument("--micro-tables", type=int, nargs="*", default=[14, 19, 22, 24])
    ap.add_argument("--micro-rows", type=int, nargs="*", default=[16, 18, 20, 22])
    ap.add_argument("--micro-samples", type=int, nargs="*", default=[1, 16, 64, 256, 1024])
    ap.add_argument("--reference-cuda-steps", type=int, default=200)
    ap.add_argument("--reference-seconds", type=float, default=30.0,
                    help="wall time of the reference arm's timed CPU-oracle steps")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    global CONFIG
    CONFIG = args.config
    if CONFIG == 4:  # config-2-only legs: the render (config 3), the e2e job, the CPU oracle, the dataset files
        args.skip_render = args.skip_e2e = args.skip_cpu = args.skip_dataset_io = True
        if args.psnr_views == 20:
            args.psnr_views = 4
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 4 needs occupancy cascades and an AABB of "
                              "scale 16, which the reference backend does not have (one [0,1]^3 grid)"}), flush=True)
            return
    if args.psnr_steps is None:
        args.psnr_steps = 10000 if CONFIG == 4 else 20000
    if args.micro:
        run_micro(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
