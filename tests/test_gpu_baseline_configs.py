"""BASELINE configurations as parity gates on the GPU, through the nerf.h C ABI.

Config 1 (the smoke scene, tests/config1.py): 200 training steps from a fresh
context.  At five synced steps (the oracle given the GPU's parameters,
occupancy and frame; none of them an occupancy-refresh frame) the step's
sample stream -- per-ray counts, kept rays, compaction offsets, positions and
steps -- is bit-exact against the oracle's, and the loss within 1e-4
relative.  After the 200 steps the held-out PSNR of the GPU's render is within
0.1 dB of the oracle trained independently on the CPU for the same 200 steps
(tests/golden/config1_oracle.json).  The first step is also compared with
that fixture directly (both start from the same seeded state).

Config 2 shapes: the sampler and the ordered compaction at 128^3 occupancy,
1024 steps per ray, 4096 rays, a 2^18 sample target and the 2^19 capacity
cut, over a seeded sparse bitfield: bit-exact against the oracle on the step
that hits the capacity and on the next step, whose ray count both adapted
from the first.
"""
import json
import os
import pathlib

import numpy as np
import pytest

import config1
import nerf_b200
from oracle import oracle
from test_gpu_train import compare_batch, sync_oracle

pytestmark = pytest.mark.gpu

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "config1_oracle.json"
SYNC_STEPS = (0, 1, 41, 101, 199)  # no refresh frame (32, 48, ...) among them


def test_config1_training_parity_and_heldout_psnr(cuda):
    golden = json.loads(GOLDEN.read_text())
    ds = nerf_b200.make_scene(**config1.SCENE)
    opts = nerf_b200.default_options(log2_hashmap_size=config1.LOG2T, max_resolution=config1.MAX_RES,
                                     stop_transmittance=config1.STOP_T, background=0)
    ctx = nerf_b200.Context(ds, grid_res=config1.GRID_RES, max_sample_steps=config1.RAYS * config1.STEPS_PER_RAY,
                            max_batch_rays=config1.RAYS, options=opts)
    oc = None
    try:
        ctx.configure(config1.training_config(nerf_b200))
        oc = config1.oracle_context(oracle, ds.images, ds.cameras, ds.intrinsics, os.cpu_count() or 1)
        for step in range(config1.TRAIN_STEPS):
            if step in SYNC_STEPS:
                if step:
                    sync_oracle(ctx, oc)
                ctx.train_step()
                oc.step()
                g = compare_batch(ctx, oc)
                s, os_ = ctx.stats(), oc.stats()
                assert abs(s.loss - os_.loss) <= 1e-4 * abs(os_.loss), (step, s.loss, os_.loss)
                if step == 0:
                    assert len(g["pos_dt"]) == golden["log"][0]["samples"]
                    assert abs(s.loss - golden["log"][0]["loss"]) <= 1e-4 * golden["log"][0]["loss"]
            else:
                ctx.train_step()
        s = ctx.stats()
        assert s.completed_steps == config1.TRAIN_STEPS and not s.has_nonfinite
        held = nerf_b200.make_scene(**config1.HELD)
        W, H = config1.HELD["width"], config1.HELD["height"]
        img = np.zeros((H, W, 4), np.uint8)
        psnr = []
        for v in range(held.n):
            ctx.render(held.cameras[v], W, H, held.intrinsics, max_steps=config1.STEPS_PER_RAY, stop=config1.STOP_T,
                       dst=img)
            psnr.append(config1.psnr_on_white(img, held.images[v]))
        gpu, ref = float(np.mean(psnr)), golden["heldout_psnr_mean"]
        assert ref > 20.0  # the configuration trains: the fixture is not a degenerate model
        assert abs(gpu - ref) <= 0.1, (gpu, ref, psnr, golden["heldout_psnr"])
    finally:
        if oc is not None:
            oc.close()
        ctx.close()


def test_config2_shape_sampler_and_capacity_cut(cuda):
    rays, steps, res, target, cap = 4096, 1024, 128, 1 << 18, 1 << 19
    ds = nerf_b200.make_scene(kind=1, seed=2, n_primitives=12, density=100.0, extent=1.0, size_min=0.1, size_max=0.6,
                              n_views=4, width=800, height=800, fov=0.69, radius=4.0, camera_mode=1)
    aabb = ((-1.5, -1.5, -1.5), (1.5, 1.5, 1.5))
    opts = nerf_b200.default_options(log2_hashmap_size=19, max_resolution=2048, stop_transmittance=1e-4, background=1,
                                     target_samples_per_step=target, max_samples_per_step=cap)
    ctx = nerf_b200.Context(ds, grid_res=res, max_sample_steps=cap, max_batch_rays=1 << 16, options=opts)
    cfg = nerf_b200.training_config(aabb=aabb, rays=rays, steps=steps, warmup=1, update_interval=100000,
                                    cells_per_update=res ** 3)
    oc = None
    try:
        ctx.configure(cfg)
        oc = oracle.Context(ctx.desc, oracle.options(log2_hashmap_size=19, max_resolution=2048, stop_transmittance=1e-4,
                                                     background=1, target_samples_per_step=target,
                                                     max_samples_per_step=cap, n_threads=os.cpu_count() or 1),
                            ctx._images, ctx._cams)
        oc.configure(cfg)
        rng = np.random.default_rng(31)
        words = res ** 3 // 32
        # ~19% of the cells occupied: enough samples per ray that 4096 rays overflow the 2^19 capacity
        bits = (rng.integers(0, 2 ** 32, words, dtype=np.uint64) & rng.integers(0, 2 ** 32, words, dtype=np.uint64)
                & (rng.integers(0, 2 ** 32, words, dtype=np.uint64) | rng.integers(0, 2 ** 32, words, dtype=np.uint64))
                ).astype(np.uint32)
        for k in range(2):
            ctx.set_occupancy(bitfield=bits)
            oc.set_occupancy(bits=bits)
            ctx.set_frame(7 + k)
            oc.set_frame(7 + k)
            oc.set_params(ctx.params()[0])
            ctx.train_step()
            oc.step()
            g = compare_batch(ctx, oc)
            c = ctx.counters()
            assert c.rays == oc.info().rays
            if k == 0:
                assert c.rays == rays
                assert g["counts"].max() > 256  # more than the reference's 256-step cap would allow
                assert int(g["counts"].sum()) > cap  # the marched samples overflow the capacity ...
                assert len(g["pos_dt"]) <= cap and c.active_rays < c.marched_active_rays  # ... and rays are cut
            else:
                assert c.rays < rays  # adapted toward the target from the first step's count
    finally:
        if oc is not None:
            oc.close()
        ctx.close()
