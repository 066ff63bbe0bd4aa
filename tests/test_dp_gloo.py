"""Data-parallel training semantics on the CPU: two gloo ranks of the oracle.

Every rank samples its own rays, the gradients and the loss are summed with an
all-reduce and every rank applies the same update (the exchange the GPU step
performs with NCCL).  The replicas must stay identical, the ranks' ray batches
must differ, and the result must equal the same two ranks emulated in one
process.
"""
import multiprocessing as mp
import socket

import numpy as np
import pytest

import dp_worker


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, world, steps, *extra):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, steps, q, *extra)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = [q.get(timeout=600) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in out:
        assert not isinstance(r[1], str), f"rank {r[0]} failed: {r[1]}"
    return {r[0]: r[1:] for r in out}


@pytest.mark.parametrize("target", [0, dp_worker.TARGET])
def test_two_rank_oracle_training_matches_serial_emulation(target):
    """target > 0: the ray count adapts to a per-step sample target from the samples of both ranks, so both ranks
    march the same number of rays every step (and it moves away from the configured count)."""
    steps = 3
    res = _run(dp_worker.oracle_rank, 2, steps, target)
    (m0, c0, l0, r0), (m1, c1, l1, r1) = res[0], res[1]
    assert np.array_equal(m0, m1), "replicas diverged"
    assert l0 == l1 and np.isfinite(l0)
    assert len(c0) == len(c1) and not np.array_equal(c0, c1), "ranks must sample different rays"
    assert r0 == r1
    if target:
        assert len(set(r0)) > 1
    serial_master, serial_batches, _ = dp_worker.serial_emulation(2, steps, target)
    assert np.array_equal(serial_master[0], m0)
    assert np.array_equal(serial_batches[0]["counts"], c0)
    assert np.array_equal(serial_batches[1]["counts"], c1)
