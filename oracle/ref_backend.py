"""The reference backend's own training step and render, timed on a GPU.

Test and baseline infrastructure only (bench.py's reference arm runs it in a
child process).  It loads oracle/_ref/libref_stock.so -- the reference's
backend-cuda.cu compiled unchanged for sm_100a by oracle/ref/Makefile -- and
drives it through the reference's public nerf.h entry points
(nerf_create_context, nerf_configure_training, nerf_train_step,
nerf_read_train_stats, nerf_inference, nerf_save/load_network_weights;
backend-cuda.cu:2067-2592).  Two launchers of the harness add what the
reference does not export: ref_train_timed (CUDA-event timing of K
nerf_train_step calls plus a per-step read of the reference's compacted sample
count) and ref_inference_timed (CUDA-event timing of one nerf_inference).

The reference's model is its own (frequency encoding, 128-wide MLPs,
softplus density, backend-cuda.cu:252-292, 664-909); it caps marching at 256
steps per ray (:2138; its graph build fails above 128 here, see REF_MAX_STEPS)
and renders with uniform samples along the AABB chord,
without occupancy skipping or early termination (:534-635).

    python -m oracle.ref_backend [--pretrain N] [--steps K] [--render-views V]

prints one JSON object.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import pathlib
import sys
import tempfile
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

LIB = ROOT / "oracle" / "_ref" / "libref_stock.so"
U32, F32, P = C.c_uint32, C.c_float, C.c_void_p

# The largest per-ray step count whose training graph the reference builds here: with CUDA 12.9 its
# nerf_configure_training returns NERF_STATUS_CUDA_ERROR at 4096 rays x 256 steps (2049 captured buckets) and
# succeeds at 4096 x 128 (1025 buckets).
REF_MAX_STEPS = 128


def load(path=LIB):
    from nerf_b200 import abi
    # RTLD_LOCAL (ctypes' default) and the harness's -Bsymbolic keep these
    # nerf_* definitions apart from libnerf_b200.so's identically named ones.
    global _LIB
    lib = C.CDLL(str(path))
    _LIB = lib
    lib.nerf_create_context.argtypes = [C.POINTER(abi.NerfCreateDesc), C.POINTER(P)]
    lib.nerf_destroy_context.argtypes = [P]
    lib.nerf_configure_training.argtypes = [P, C.POINTER(abi.NerfTrainingConfig)]
    lib.nerf_train_step.argtypes = [P]
    lib.nerf_read_train_stats.argtypes = [P, C.POINTER(abi.NerfTrainStats)]
    lib.nerf_inference.argtypes = [P, C.POINTER(abi.NerfInferenceRequest), C.POINTER(abi.NerfInferenceInfo)]
    lib.nerf_save_network_weights.argtypes = [P, C.POINTER(abi.NerfCheckpointFileDesc)]
    lib.nerf_load_network_weights.argtypes = [P, C.POINTER(abi.NerfCheckpointFileDesc)]
    lib.ref_train_timed.argtypes = [P, U32, C.POINTER(F32), C.POINTER(C.c_uint64)]
    lib.ref_inference_timed.argtypes = [P, U32, U32, C.POINTER(F32)]
    lib.ref_last_cuda_error.argtypes = [C.c_char_p, U32]
    for n in ("nerf_create_context", "nerf_destroy_context", "nerf_configure_training", "nerf_train_step",
              "nerf_read_train_stats", "nerf_inference", "nerf_save_network_weights", "nerf_load_network_weights",
              "ref_train_timed", "ref_inference_timed", "ref_last_cuda_error"):
        getattr(lib, n).restype = C.c_int
    return lib


_LIB = None


def _check(where, rc):
    if rc != 0:
        detail = ""
        if _LIB is not None:
            buf = C.create_string_buffer(64)
            code = _LIB.ref_last_cuda_error(buf, 64)
            detail = f" (last CUDA error {code} {buf.value.decode()})"
        raise RuntimeError(f"reference {where} failed: status {rc}{detail}")


class RefContext:
    """A reference-backend context over a dataset (images and cameras are copied at create, as nerf.h states)."""

    def __init__(self, lib, ds, grid_res, max_sample_steps, max_batch_rays):
        from nerf_b200 import abi
        self.lib = lib
        self.images = np.ascontiguousarray(ds.images)
        self.cams = np.ascontiguousarray(ds.cameras, dtype=np.float32)
        fx, fy, cx, cy = ds.intrinsics
        n, h, w = self.images.shape[:3]
        self.desc = abi.NerfCreateDesc(grid_res, max_sample_steps, max_batch_rays, 256, self.images.ctypes.data,
                                       self.images.nbytes, self.cams.ctypes.data, self.cams.nbytes, n, w, h, fx, fy,
                                       cx, cy)
        self.h = P()
        _check("nerf_create_context", lib.nerf_create_context(C.byref(self.desc), C.byref(self.h)))

    def configure(self, cfg):
        _check("nerf_configure_training", self.lib.nerf_configure_training(self.h, C.byref(cfg)))

    def steps(self, k):
        for _ in range(k):
            _check("nerf_train_step", self.lib.nerf_train_step(self.h))

    def stats(self):
        from nerf_b200 import abi
        s = abi.NerfTrainStats()
        _check("nerf_read_train_stats", self.lib.nerf_read_train_stats(self.h, C.byref(s)))
        return s

    def timed(self, k):
        ms = F32()
        out = (C.c_uint64 * 2)()
        _check("ref_train_timed", self.lib.ref_train_timed(self.h, k, C.byref(ms), out))
        return float(ms.value), int(out[0]), int(out[1])

    def render(self, camera_idx, spp, dst=None):
        from nerf_b200 import abi
        req = abi.NerfInferenceRequest(camera_idx, spp, abi.NERF_MEMORY_HOST, dst.ctypes.data if dst is not None else None,
                                       dst.nbytes if dst is not None else 0)
        info = abi.NerfInferenceInfo()
        _check("nerf_inference", self.lib.nerf_inference(self.h, C.byref(req), C.byref(info)))

    def render_timed(self, camera_idx, spp):
        ms = F32()
        _check("ref_inference_timed", self.lib.ref_inference_timed(self.h, camera_idx, spp, C.byref(ms)))
        return float(ms.value)

    def save(self, path):
        from nerf_b200 import abi
        d = abi.NerfCheckpointFileDesc(str(path).encode())
        _check("nerf_save_network_weights", self.lib.nerf_save_network_weights(self.h, C.byref(d)))

    def load_weights(self, path):
        from nerf_b200 import abi
        d = abi.NerfCheckpointFileDesc(str(path).encode())
        _check("nerf_load_network_weights", self.lib.nerf_load_network_weights(self.h, C.byref(d)))

    def close(self):
        if self.h:
            self.lib.nerf_destroy_context(self.h)
            self.h = P()


def reference_train_config(nb, bench, max_steps_per_ray=REF_MAX_STEPS):
    """Config 2's scene, batch (4096 rays), AABB and occupancy schedule, at the reference's step limit, with the
    optimiser settings of the reference's own driver for its network (benchmark.cpp:423-430: lr 5e-4, clip 1,
    update guard 100, decay over 250 k steps; Adam betas 0.9 / 0.99, loss scale 128)."""
    cfg = bench.train_config(nb)
    cfg.max_sample_steps_per_ray = max_steps_per_ray
    hp = cfg.hyper_params
    hp.learning_rate, hp.grad_clip_norm, hp.update_guard_grad_norm, hp.lr_decay_ksteps = 5e-4, 1.0, 100.0, 250
    hp.adam_eps = 1e-15
    return cfg


def run(pretrain=2000, steps=200, render_views=4, render_spp=256, psnr_views=5, max_steps_per_ray=REF_MAX_STEPS,
        psnr_steps=3010):
    """Config-2 training (the reference's limits: 128 steps per ray here, white background) and the config-3 render,
    both through the reference backend's nerf.h."""
    import bench  # the config-2 workload definition (dataset, training configuration)
    import nerf_b200 as nb  # ctypes structures and the Dataset container; the product library is never loaded

    lib = load()
    out = {"library": "oracle/_ref/libref_stock.so (reference backend-cuda.cu, unchanged kernels, sm_100a)"}
    ds, _ = bench.make_dataset(nb, renderer=bench.oracle_scene)
    cfg = reference_train_config(nb, bench, max_steps_per_ray)
    rays = cfg.rays_per_batch
    t0 = time.perf_counter()
    ctx = RefContext(lib, ds, bench.GRID_RES, rays * max_steps_per_ray, 1 << 16)
    ctx.configure(cfg)
    configure_s = time.perf_counter() - t0
    ctx.steps(pretrain)
    ctx.stats()
    ms, samples, active = ctx.timed(steps)
    st = ctx.stats()
    out["train"] = {
        "metric": "train samples/s (config 2, steady state)", "value": samples / (ms / 1e3), "unit": "samples/s",
        "steps_per_s": steps / (ms / 1e3), "ms_per_step": ms / steps, "steps": steps, "pretrain_steps": pretrain,
        "samples_per_step": samples / steps, "active_rays_per_step": active / steps, "rays_per_batch": rays,
        "max_steps_per_ray": max_steps_per_ray, "final_loss": float(st.loss), "configure_s": configure_s,
        "note": "config-2 dataset, batch and occupancy schedule at the reference's limits (128 steps per ray, "
                "white background), the reference driver's optimiser settings; device time of the timed nerf_train_step calls with CUDA events on the context's "
                "stream; samples = the reference's compacted sample count of each timed step"}
    if psnr_views > 0:
        # PSNR after as many steps as bench.py's own arm has trained when it measures PSNR (pretrain, warm-up,
        # timed and profiled steps: 3010 with the defaults).
        extra = max(0, psnr_steps - pretrain - steps)
        ctx.steps(extra)
        out["psnr"] = heldout_psnr(lib, ctx, nb, bench, psnr_views, render_spp)
        out["psnr"]["train_steps"] = pretrain + steps + extra
    ctx.close()
    if render_views > 0:
        out["render"] = render_config3(lib, nb, bench, render_views, render_spp)
    return out


def heldout_psnr(lib, ctx, nb, bench, n, spp):
    """PSNR of the trained reference model on held-out views (the same cameras and ground truth as bench.py's
    psnr_heldout): weights saved, loaded into a context whose dataset cameras are the held-out views."""
    held = bench.oracle_scene(**{**bench.CFG2, "n_views": n, "view_offset": bench.CFG2["n_views"],
                            "orbit_views": bench.CFG2["n_views"] + n})
    with tempfile.TemporaryDirectory() as d:
        path = pathlib.Path(d) / "ref.ckpt"
        ctx.save(path)
        hc = RefContext(lib, nb.Dataset(np.zeros_like(held.images), held.cameras, held.intrinsics), bench.GRID_RES,
                        RENDER_ROWS, 1 << 16)
        hc.configure(render_config(nb, bench))  # the AABB and the row capacity the render uses
        hc.load_weights(path)
        W, H = bench.CFG2["width"], bench.CFG2["height"]
        img = np.zeros((H, W, 4), np.uint8)
        psnr = []
        for v in range(n):
            hc.render(v, spp, img)
            gt = held.images[v].astype(np.float64) / 255.0
            ref = gt[..., :3] * gt[..., 3:4] + (1.0 - gt[..., 3:4])
            mse = float(np.mean((img[..., :3].astype(np.float64) / 255.0 - ref) ** 2))
            psnr.append(10.0 * np.log10(1.0 / max(mse, 1e-12)))
        hc.close()
    return {"value": float(np.mean(psnr)), "unit": "dB", "views": n, "samples_per_ray": spp,
            "note": "reference render (uniform samples, white background) of the held-out views after the same "
                    "number of training steps"}


# Render contexts are configured like the training one: the reference renders in chunks of (workspace rows /
# samples per ray) rays, and its workspace holds max(rays x steps, occupancy cells) rows.
RENDER_ROWS = 4096 * REF_MAX_STEPS


def render_config(nb, bench):
    return reference_train_config(nb, bench, REF_MAX_STEPS)


def render_config3(lib, nb, bench, views, spp):
    """Config 3 through the reference: orbit poses passed as the dataset cameras (dummy images), the reference's
    seeded initial weights, uniform samples (the reference renders without the occupancy grid)."""
    orbit = bench.oracle_scene(**{**bench.CFG2, "n_views": views, "camera_mode": 2, "orbit_elevation": 0.35,
                             "orbit_views": 200, "view_offset": 0}, with_images=False)
    rc = RefContext(lib, orbit, bench.GRID_RES, RENDER_ROWS, 1 << 16)
    rc.configure(render_config(nb, bench))
    rc.render_timed(0, spp)  # warm-up
    ms = sum(rc.render_timed(v, spp) for v in range(views))
    rc.close()
    rays = views * orbit.width * orbit.height
    return {"metric": "render MRays/s (config 3)", "value": rays / (ms / 1e3) / 1e6, "unit": "MRays/s",
            "views": views, "samples_per_ray": spp, "device_ms": ms,
            "note": "nerf_inference of orbit views at 800x800, uniform samples along the AABB chord, no occupancy "
                    "skipping, no early termination (the reference's render path)"}


def probe_configs():
    """Configures the reference on the config-2 dataset at several batch shapes and reports each outcome."""
    import bench
    import nerf_b200 as nb
    lib = load()
    ds, _ = bench.make_dataset(nb, renderer=bench.oracle_scene)
    res = []
    shapes = [tuple(int(x) for x in s.split(",")) for s in os.environ.get(
        "REF_PROBE_SHAPES", "4096,64,65536,1,32;4096,128,65536,1,32;4096,64,2097152,16,256;4096,128,2097152,16,256").split(";")]
    for rays, steps, cells, interval, warmup in shapes:
        cfg = reference_train_config(nb, bench, steps)
        cfg.rays_per_batch = rays
        op = cfg.occupancy_params
        op.cells_per_update, op.update_interval, op.warmup_steps = cells, interval, warmup
        t0 = time.perf_counter()
        ctx = None
        try:
            ctx = RefContext(lib, ds, bench.GRID_RES, rays * steps, 1 << 16)
            ctx.configure(cfg)
            ms, samples, _ = ctx.timed(20)
            out = f"ok: 20 steps {ms:.2f} ms, {samples} samples"
        except RuntimeError as e:
            out = str(e)
        finally:
            if ctx is not None:
                ctx.close()
        res.append({"rays": rays, "steps": steps, "cells": cells, "s": time.perf_counter() - t0, "result": out})
        print(json.dumps(res[-1]), flush=True)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--probe", action="store_true")
    ap.add_argument("--pretrain", type=int, default=2000)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--render-views", type=int, default=4)
    ap.add_argument("--render-spp", type=int, default=256)
    ap.add_argument("--psnr-views", type=int, default=5)
    ap.add_argument("--psnr-steps", type=int, default=3010)
    a = ap.parse_args()
    import torch
    torch.cuda.init()
    if a.probe:
        probe_configs()
        return
    print(json.dumps(run(a.pretrain, a.steps, a.render_views, a.render_spp, a.psnr_views, psnr_steps=a.psnr_steps)),
          flush=True)


if __name__ == "__main__":
    main()
