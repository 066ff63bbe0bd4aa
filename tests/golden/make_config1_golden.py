"""Writes tests/golden/config1_oracle.json: the CPU oracle trained on the smoke configuration (
defined in tests/config1.py) for its 200 steps from a fresh context, independently of any GPU run.  Records the
loss, kept-ray and sample counts of every step and the held-out PSNR of the oracle's own render of the trained
model (4 views, 128 marching steps, early termination at 1e-4, on white).  The GPU test trains the same
configuration through the C ABI and must land within 0.1 dB of this PSNR; a CPU test re-runs the first steps to
check that the fixture still matches the oracle.

    python tests/golden/make_config1_golden.py [threads]
"""
import json
import os
import pathlib
import sys
import time

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parents[1]))

import numpy as np  # noqa: E402

import config1  # noqa: E402
from oracle import oracle  # noqa: E402


def main():
    threads = int(sys.argv[1]) if len(sys.argv) > 1 else (os.cpu_count() or 1)
    imgs, cams, intr = oracle.make_scene(**config1.SCENE)
    held_imgs, held_cams, held_intr = oracle.make_scene(**config1.HELD)
    oc = config1.oracle_context(oracle, imgs, cams, intr, threads)
    log = []
    t0 = time.time()
    for step in range(config1.TRAIN_STEPS):
        oc.step()
        st, info = oc.stats(), oc.info()
        log.append({"loss": float(st.loss), "grad_norm": float(st.grad_norm), "active_rays": int(info.active_rays),
                    "samples": int(info.samples), "camera": int(info.camera)})
        if step % 20 == 0:
            print(f"step {step} loss {st.loss:.6f} samples {info.samples} {time.time() - t0:.0f}s", flush=True)
    W, H = config1.HELD["width"], config1.HELD["height"]
    psnr = []
    for v in range(held_imgs.shape[0]):
        rgba, _ = oc.render(held_cams[v], W, H, held_intr, config1.STEPS_PER_RAY, config1.STOP_T)
        psnr.append(config1.psnr_on_white(rgba.view(np.uint8).reshape(H, W, 4), held_imgs[v]))
    oc.close()
    out = {"config": "BASELINE config 1 (tests/config1.py)", "steps": config1.TRAIN_STEPS, "threads": threads,
           "log": log, "heldout_psnr": psnr, "heldout_psnr_mean": float(sum(psnr) / len(psnr)),
           "seconds": time.time() - t0}
    (HERE / "config1_oracle.json").write_text(json.dumps(out, indent=0) + "\n")
    print(f"wrote config1_oracle.json: held-out PSNR {out['heldout_psnr_mean']:.3f} dB in {out['seconds']:.0f} s")


if __name__ == "__main__":
    main()
