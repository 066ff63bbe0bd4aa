"""The reference's own benchmark driver, unchanged, on this library (the nerf.h drop-in).

oracle/_ref/benchmark_b200 is the reference's benchmark.cpp compiled from the
reference checkout against the reference's nerf.h and linked against
libnerf_b200.so (oracle/ref/Makefile; stb and `import std` are provided by
oracle/ref/driver/).  The test writes the smoke scene in
the driver's Blender format, runs the driver's training loop with periodic
statistics and evaluation, saves and reloads the network weights through
nerf_save_network_weights / nerf_load_network_weights, and checks what the
driver prints and writes (reference benchmark.cpp:305-546).  The driver's own
hyper-parameters apply (lr 5e-4, its occupancy schedule, AABB [0,1]^3 after
its camera remap); the hash-grid size comes from the NERF_B200_* environment.
"""
import math
import os
import pathlib
import re
import subprocess

import numpy as np
import pytest

import config1
import nerf_b200
from nerf_b200 import abi

pytestmark = pytest.mark.gpu

DRIVER = pathlib.Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "benchmark_b200"


@pytest.mark.skipif(not DRIVER.exists(), reason="the driver is built only where the reference checkout is present")
def test_reference_driver_trains_evaluates_and_saves(cuda, tmp_path):
    lib = abi.load()
    ds = nerf_b200.make_scene(**config1.SCENE)
    imgs, cams = np.ascontiguousarray(ds.images), np.ascontiguousarray(ds.cameras)
    abi.check("blender write", lib.nerf_b200_blender_write(str(tmp_path).encode(), imgs.ctypes.data, cams.ctypes.data,
                                                          ds.n, ds.width, ds.height, config1.SCENE["fov"], 0))
    env = dict(os.environ, NERF_B200_LOG2_HASHMAP_SIZE=str(config1.LOG2T), NERF_B200_MAX_RESOLUTION=str(config1.MAX_RES))
    out_png, ckpt = tmp_path / "render.png", tmp_path / "weights.ckpt"
    args = [str(DRIVER), "--dataset", str(tmp_path), "--steps", "60", "--rays", "4096", "--max-sample-steps", "128",
            "--log-interval", "20", "--inference-interval", "30", "--inference-samples", "128",
            "--inference-out", str(out_png), "--save-weights", str(ckpt)]
    r = subprocess.run(args, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    train = [dict(kv.split("=") for kv in l.split()[1:]) for l in r.stdout.splitlines() if l.startswith("[train]")]
    evals = [l for l in r.stdout.splitlines() if l.startswith("[eval]") and "psnr=" in l]
    assert [int(t["step"]) for t in train] == [20, 40, 60]
    losses = [float(t["loss"]) for t in train]
    assert all(math.isfinite(x) for x in losses) and losses[-1] < losses[0], losses
    assert all(t["nonfinite"] == "0" for t in train)
    psnr = [float(re.search(r"psnr=(\S+)", l).group(1)) for l in evals]
    assert len(psnr) == 2 and all(math.isfinite(p) and p > 10.0 for p in psnr), psnr
    w, h = abi.C.c_uint32(), abi.C.c_uint32()
    abi.check("png", lib.nerf_b200_png_read(str(out_png).encode(), None, 0, abi.C.byref(w), abi.C.byref(h)))
    assert (w.value, h.value) == (config1.SCENE["width"], config1.SCENE["height"])
    assert ckpt.stat().st_size > 0
    # the saved weights load back through the driver's --load-weights path
    args2 = [str(DRIVER), "--dataset", str(tmp_path), "--steps", "1", "--max-sample-steps", "128",
             "--load-weights", str(ckpt), "--inference-out", str(tmp_path / "again.png")]
    r2 = subprocess.run(args2, capture_output=True, text=True, timeout=600, env=env)
    assert r2.returncode == 0, r2.stdout[-2000:] + r2.stderr[-2000:]
    assert "[train] step=1 " in r2.stdout
