"""Data-parallel GPU training (needs two GPUs; skipped otherwise).

Two processes, one per GPU, train through nerf_b200_dp_init (or
nerf_b200_dp_init_peers) + nerf_train_step, in both exchange modes: peer mode (each rank sums its owned range of every
rank's hash gradients over NVLink, runs Adam on it and writes the fp16
parameters into every rank's mirror) and the NCCL all-reduce path
(NERF_B200_DP_PEER=0).  Both replicas must be bitwise identical after every
step; each rank's sample stream must equal the oracle's for that rank bit for
bit; the first Adam moment (the clipped, summed gradient) must match the
two-rank oracle emulation within the tolerances of the single-GPU test.
"""
import os

import numpy as np
import pytest
import torch

import dp_worker
from test_dp_gloo import _run

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("peer,steps,target,setup", [
    ("1", 1, 0, "nccl"), ("1", 3, 0, "nccl"), ("0", 1, 0, "nccl"), ("0", 3, 0, "nccl"),
    ("1", 3, dp_worker.TARGET, "nccl"), ("0", 3, dp_worker.TARGET, "nccl"),
    ("1", 3, 0, "handles"), ("1", 3, dp_worker.TARGET, "handles")])
def test_two_gpu_training_matches_oracle(peer, steps, target, setup):
    """target > 0: both ranks size every batch from the samples of both (the same ray count on both ranks).
    setup "handles": peer mode set up from all-gathered peer handles without NCCL (nerf_b200_dp_init_peers)."""
    old = os.environ.get("NERF_B200_DP_PEER")
    os.environ["NERF_B200_DP_PEER"] = peer
    try:
        res = _run(dp_worker.gpu_rank, 2, steps, target, setup)
    finally:
        if old is None:
            del os.environ["NERF_B200_DP_PEER"]
        else:
            os.environ["NERF_B200_DP_PEER"] = old
    (g0, m0, c0, l0, r0), (g1, m1, c1, l1, r1) = res[0], res[1]
    assert np.array_equal(g0, g1) and np.array_equal(m0, m1), "replicas diverged"
    assert l0 == l1
    assert r0 == r1
    _, batches, params = dp_worker.serial_emulation(2, steps, target)
    assert np.array_equal(batches[0]["counts"], c0)
    assert np.array_equal(batches[1]["counts"], c1)
    om = params[0][2]
    n_grid = len(om) - 10240
    mlp_err = np.linalg.norm(m0[n_grid:] - om[n_grid:]) / np.linalg.norm(om[n_grid:])
    grid_err = np.linalg.norm(m0[:n_grid] - om[:n_grid]) / np.linalg.norm(om[:n_grid])
    assert mlp_err < 2e-2, mlp_err
    # The hash-table gradients are summed in fp16 (f16x2 reductions) on the GPU and in float64 by the oracle.  With a
    # sample target the second and third steps train on ~150 rays per rank instead of 512, and the fp16 sums of these
    # smaller batches land further from the float64 ones: 4.2% relative L2 measured on two B200s in every exchange
    # mode and set-up (2-3% at 512 rays), with bit-exact sample streams.
    assert grid_err < (5e-2 if target else 3e-2), grid_err
