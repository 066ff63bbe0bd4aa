"""Failure detection without a GPU fault: the bounded waits of the data-parallel barrier.

In data-parallel peer mode each training step passes three barriers over
peer flags.  A rank whose peer stops stepping must not hang its GPU: every
wait is bounded, and when it runs out the barrier records an error, the step
finishes, and nerf_read_train_stats reports NERF_STATUS_CUDA_ERROR.  This
test makes one wait run out on one GPU -- the barrier kernel as rank 0 of two,
against a second rank whose flag nothing ever writes, with a 10 ms limit --
and checks that the kernel returns, the error reaches nerf_read_train_stats,
and the context stays usable.  (The reference has no multi-GPU path; its
failure report is the non-finite flag of its step statistics,
backend-cuda.cu:1495-1508.)
"""
import ctypes as C
import time

import numpy as np
import pytest

import nerf_b200
from nerf_b200 import abi

pytestmark = pytest.mark.gpu


def test_dp_barrier_wait_runs_out_and_is_reported(cuda):
    lib = abi.load()
    ds = nerf_b200.make_scene(kind=0, seed=0, n_views=4, width=32, height=32)
    opts = nerf_b200.default_options(log2_hashmap_size=14, max_resolution=256, stop_transmittance=0.0)
    ctx = nerf_b200.Context(ds, grid_res=32, max_sample_steps=256 * 64, max_batch_rays=256, options=opts)
    try:
        ctx.configure(nerf_b200.training_config(rays=256, steps=64, warmup=4))
        ctx.train_step()
        st = abi.NerfTrainStats()
        assert lib.nerf_read_train_stats(ctx.handle, C.byref(st)) == abi.NERF_STATUS_OK
        cuda.cuda.synchronize()
        t0 = time.perf_counter()
        abi.check("dp_barrier_test", lib.nerf_b200_dp_barrier_test(ctx.handle, 10000))  # 10 ms limit
        rc = lib.nerf_read_train_stats(ctx.handle, C.byref(st))  # synchronises the context's stream
        waited = time.perf_counter() - t0
        assert rc == abi.NERF_STATUS_CUDA_ERROR
        assert 0.009 <= waited < 2.0, waited  # the wait ran its limit, then the kernel returned
        assert st.completed_steps == 1
        # the context is still usable after the expired wait
        img = ctx.inference(camera_idx=0, samples_per_ray=32)
        assert img.shape == (32, 32, 4) and np.isfinite(img).all()
        assert lib.nerf_b200_dp_barrier_test(ctx.handle, 0) == abi.NERF_STATUS_INVALID_USAGE
    finally:
        ctx.close()


def test_dp_barrier_test_needs_a_configured_context(cuda):
    lib = abi.load()
    ds = nerf_b200.make_scene(kind=0, seed=0, n_views=2, width=16, height=16)
    ctx = nerf_b200.Context(ds, grid_res=16, max_sample_steps=1 << 12, max_batch_rays=64,
                            options=nerf_b200.default_options(log2_hashmap_size=12, max_resolution=128))
    try:
        assert lib.nerf_b200_dp_barrier_test(ctx.handle, 1000) == abi.NERF_STATUS_STATE_ERROR
    finally:
        ctx.close()
