"""Rank bodies of the data-parallel tests (run in spawned processes).

The data-parallel step (reference training step backend-cuda.cu:2216-2401,
sharded by ray batch): every rank samples its own rays (global ray index
rank * rays_per_batch + r), normalises its loss by its kept rays times the
world size, the gradients and the loss are summed over ranks, and every rank
applies the same Adam update to its replica.
"""
import datetime
import os

import numpy as np

RAYS, STEPS, RES, LOG2T, MAXRES = 512, 96, 32, 15, 512
# With a per-step sample target (target > 0) every rank sizes its next batch from the samples of all ranks.
TARGET = 6000


def small_problem():
    import nerf_b200
    ds = nerf_b200.make_scene(kind=0, seed=0, n_views=8, width=48, height=48, fov=0.69, radius=3.0)
    cfg = nerf_b200.training_config(rays=RAYS, steps=STEPS, warmup=4, update_interval=2, cells_per_update=RES ** 3 // 2)
    return ds, cfg


def oracle_context(ds, cfg, rank, world, target=0):
    import nerf_b200
    from oracle import oracle
    desc, imgs, cams = nerf_b200.create_desc(ds, grid_res=RES, max_sample_steps=RAYS * STEPS, max_batch_rays=4 * RAYS)
    oc = oracle.Context(desc, oracle.options(log2_hashmap_size=LOG2T, max_resolution=MAXRES, dp_rank=rank,
                                             dp_world=world, n_threads=4, target_samples_per_step=target), imgs, cams)
    oc._desc_keep = (desc, imgs, cams)
    oc.configure(cfg)
    return oc


def _init(rank, world, port):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    return dist


def oracle_rank(rank, world, port, steps, q, target=0):
    """One rank of oracle data-parallel training with a gloo all-reduce."""
    try:
        import torch
        dist = _init(rank, world, port)
        ds, cfg = small_problem()
        oc = oracle_context(ds, cfg, rank, world, target)
        rays = []
        for _ in range(steps):
            oc.step_grads()
            rays.append(oc.info().rays)
            grad = torch.from_numpy(oc.params()[4].copy())
            loss_sum, active = oc.loss()
            loss = torch.tensor([loss_sum], dtype=torch.float32)
            samples = torch.tensor([oc.info().samples], dtype=torch.int64)
            dist.all_reduce(grad)
            dist.all_reduce(loss)
            dist.all_reduce(samples)
            oc.set_grads(grad.numpy(), float(loss[0]), active)
            oc.set_global_samples(int(samples[0]))
            oc.step_apply()
        q.put((rank, oc.params()[0], oc.batch()["counts"], oc.stats().loss, rays))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent instead of hanging it
        q.put((rank, repr(e), None, None, None))


def serial_emulation(world, steps, target=0):
    """The same data-parallel training with all ranks in this process."""
    ds, cfg = small_problem()
    ocs = [oracle_context(ds, cfg, r, world, target) for r in range(world)]
    for _ in range(steps):
        for oc in ocs:
            oc.step_grads()
        grad = ocs[0].params()[4].copy()
        loss = np.float32(ocs[0].loss()[0])
        for oc in ocs[1:]:
            grad += oc.params()[4]
            loss += np.float32(oc.loss()[0])
        samples = sum(oc.info().samples for oc in ocs)
        for oc in ocs:
            oc.set_grads(grad, float(loss), oc.loss()[1])
            oc.set_global_samples(samples)
            oc.step_apply()
    return [oc.params()[0] for oc in ocs], [oc.batch() for oc in ocs], [oc.params() for oc in ocs]


def gpu_rank(rank, world, port, steps, q, target=0, setup="nccl"):
    """One rank of GPU data-parallel training.  setup "nccl": nerf_b200_dp_init (an NCCL communicator; peer mode
    unless NERF_B200_DP_PEER=0); "handles": the ranks' peer handles all-gathered over gloo and mapped with
    nerf_b200_dp_init_peers (peer mode, no NCCL)."""
    try:
        import torch
        import nerf_b200
        dist = _init(rank, world, port)
        torch.cuda.set_device(rank)
        ds, cfg = small_problem()
        ctx = nerf_b200.Context(ds, grid_res=RES, max_sample_steps=RAYS * STEPS, max_batch_rays=4 * RAYS,
                                options=nerf_b200.default_options(log2_hashmap_size=LOG2T, max_resolution=MAXRES,
                                                                  target_samples_per_step=target))
        if setup == "handles":
            handles = [None] * world
            dist.all_gather_object(handles, ctx.dp_peer_handle())
            ctx.dp_init_peers(rank, world, handles)
        else:
            uid = [nerf_b200.dp_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            ctx.dp_init(rank, world, uid[0])
        ctx.configure(cfg)
        assert ctx.counters().dp_peer == (0 if os.environ.get("NERF_B200_DP_PEER") == "0" and setup == "nccl" else 1)
        rays = []
        for _ in range(steps):
            ctx.train_step()
            rays.append(ctx.counters().rays)
        master, _, m, v = ctx.params()
        b = ctx.batch()
        q.put((rank, master, m, b["counts"], ctx.stats().loss, rays))
        ctx.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e), None, None, None, None))
