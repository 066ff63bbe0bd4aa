"""The config-1 fixture (tests/golden/config1_oracle.json) still describes the current oracle.

The fixture holds the CPU oracle's independent 200-step training run of BASELINE
config 1; the GPU test lands its held-out PSNR against it.  Re-running the first
two oracle steps here must give the fixture's sample and kept-ray counts exactly
and its losses within 1e-6 relative (the loss sum's order may follow the thread
count), so an oracle change that would invalidate the fixture fails on the CPU.
Regenerate with tests/golden/make_config1_golden.py.
"""
import json
import os
import pathlib

import config1
from oracle import oracle

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "config1_oracle.json"


def test_config1_fixture_matches_oracle():
    golden = json.loads(GOLDEN.read_text())
    assert golden["steps"] == config1.TRAIN_STEPS == len(golden["log"])
    imgs, cams, intr = oracle.make_scene(**config1.SCENE)
    oc = config1.oracle_context(oracle, imgs, cams, intr, os.cpu_count() or 1)
    try:
        for step in range(2):
            oc.step()
            st, info, want = oc.stats(), oc.info(), golden["log"][step]
            assert info.samples == want["samples"] and info.active_rays == want["active_rays"], step
            assert info.camera == want["camera"], step
            assert abs(st.loss - want["loss"]) <= 1e-6 * abs(want["loss"]), (step, st.loss, want["loss"])
    finally:
        oc.close()
