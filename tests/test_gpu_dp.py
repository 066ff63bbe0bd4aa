"""Data-parallel GPU training over NCCL (needs two GPUs; skipped otherwise).

Two processes, one per GPU, train through nerf_b200_dp_init + nerf_train_step.
Both replicas must be bitwise identical after every step (same summed
gradients, same Adam); each rank's sample stream must equal the oracle's for
that rank bit for bit; the first Adam moment (the clipped, summed gradient)
must match the two-rank oracle emulation within the tolerances of the
single-GPU test.
"""
import numpy as np
import pytest
import torch

import dp_worker
from test_dp_gloo import _run

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_training_matches_oracle():
    res = _run(dp_worker.gpu_rank, 2, 1)
    (g0, m0, c0, l0), (g1, m1, c1, l1) = res[0], res[1]
    assert np.array_equal(g0, g1) and np.array_equal(m0, m1), "replicas diverged"
    assert l0 == l1
    _, batches, params = dp_worker.serial_emulation(2, 1)
    assert np.array_equal(batches[0]["counts"], c0)
    assert np.array_equal(batches[1]["counts"], c1)
    om = params[0][2]
    n_grid = len(om) - 10240
    mlp_err = np.linalg.norm(m0[n_grid:] - om[n_grid:]) / np.linalg.norm(om[n_grid:])
    grid_err = np.linalg.norm(m0[:n_grid] - om[:n_grid]) / np.linalg.norm(om[:n_grid])
    assert mlp_err < 2e-2, mlp_err
    assert grid_err < 3e-2, grid_err
