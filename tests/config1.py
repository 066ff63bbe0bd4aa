"""The smoke configuration shared by its golden-fixture script and its tests.

Scene: 3 analytic spheres, centres U[-0.5,0.5]^3, radii U[0.15,0.35], density
50, RGB U[0,1], seed 0, in the AABB [-1,1]^3; 16 training views at 128x128 on
a radius-3 sphere looking at the origin, fov 0.69 rad, white background.
Hash grid L16 F2 T=2^15, N_min 16, N_max 512, fp16 parameters drawn
U(-1e-4, 1e-4); the north-star MLPs.  Training: 4096 rays per batch, 200
Adam steps at lr 1e-2 (betas 0.9/0.99, eps 1e-15, loss scale 128), 64^3
occupancy grid.  Choices the configuration leaves open: at most 128 marching
steps per ray (the largest count the reference backend trains with here),
occupancy warm-up 32 steps then a full-grid refresh every 16 steps (decay
0.95, threshold 0.01), early termination at transmittance 1e-4.  Held-out
views: 4 more cameras of the same seeded sphere sequence (views 16-19).
"""
import numpy as np

SCENE = dict(kind=0, seed=0, n_primitives=3, density=50.0, extent=0.5, size_min=0.15, size_max=0.35, n_views=16,
             width=128, height=128, fov=0.69, radius=3.0, camera_mode=0)
HELD = dict(SCENE, n_views=4, view_offset=16)
RAYS, STEPS_PER_RAY, GRID_RES, TRAIN_STEPS = 4096, 128, 64, 200
LOG2T, MAX_RES, STOP_T = 15, 512, 1e-4


def training_config(nb):
    return nb.training_config(aabb=((-1, -1, -1), (1, 1, 1)), rays=RAYS, steps=STEPS_PER_RAY, lr=1e-2, beta1=0.9,
                              beta2=0.99, eps=1e-15, clip=1e9, guard=1e12, loss_scale=128.0, lr_decay_ksteps=0,
                              decay=0.95, threshold=0.01, cells_per_update=GRID_RES ** 3, update_interval=16,
                              warmup=32)


def create_desc(images, cams, intrinsics):
    from nerf_b200.abi import NerfCreateDesc
    fx, fy, cx, cy = intrinsics
    return NerfCreateDesc(GRID_RES, RAYS * STEPS_PER_RAY, RAYS, 256, images.ctypes.data, images.nbytes,
                          cams.ctypes.data, cams.nbytes, images.shape[0], images.shape[2], images.shape[1], fx, fy, cx,
                          cy)


def oracle_context(oracle, images, cams, intrinsics, threads):
    import nerf_b200 as nb  # ctypes structures only
    images, cams = np.ascontiguousarray(images), np.ascontiguousarray(cams)
    oc = oracle.Context(create_desc(images, cams, intrinsics),
                        oracle.options(log2_hashmap_size=LOG2T, max_resolution=MAX_RES, stop_transmittance=STOP_T,
                                       background=0, n_threads=threads), images, cams)
    oc.configure(training_config(nb))
    return oc


def psnr_on_white(rgba, gt_rgba):
    gt = gt_rgba.astype(np.float64) / 255.0
    ref = gt[..., :3] * gt[..., 3:4] + (1.0 - gt[..., 3:4])
    mse = float(np.mean((rgba[..., :3].astype(np.float64) / 255.0 - ref) ** 2))
    return 10.0 * np.log10(1.0 / max(mse, 1e-12))
