"""nerf_b200 -- B200-native instant-ngp-style NeRF train/render backend.

The product is libnerf_b200.so: the nerf.h C ABI of Xayah-Graphics/NeRF
implemented with hand-written sm_100a kernels.  This package is the host
mirror of that interface for Python callers: ctypes bindings (abi.py), a thin
Context wrapper with the same call sequence as the reference driver
(create -> configure -> train_step* -> read_train_stats / inference ->
save/load), and the synthetic-scene presets that stand in for the reference's
datasets.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import abi
from .abi import (NERF_MEMORY_CUDA_DEVICE, NERF_MEMORY_HOST, NerfB200Counters, NerfB200GridLayout, NerfB200Options,
                  NerfB200RenderInfo, NerfB200RenderRequest, NerfB200SceneDesc, NerfCheckpointFileDesc, NerfCreateDesc,
                  NerfError, NerfHyperParams, NerfInferenceInfo, NerfInferenceRequest, NerfOccupancyParams,
                  NerfTrainingConfig, NerfTrainStats, check)

__all__ = ["abi", "Context", "Dataset", "make_scene", "default_options", "grid_layout", "training_config", "NerfError"]


def lib():
    return abi.load()


def default_options(**overrides) -> NerfB200Options:
    o = NerfB200Options()
    lib().nerf_b200_default_options(C.byref(o))
    for k, v in overrides.items():
        setattr(o, k, v)
    return o


def grid_layout(n_levels=16, log2_hashmap_size=19, base_resolution=16, max_resolution=2048) -> NerfB200GridLayout:
    g = NerfB200GridLayout()
    check("nerf_b200_grid_layout", lib().nerf_b200_grid_layout(n_levels, log2_hashmap_size, base_resolution, max_resolution, C.byref(g)))
    return g


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


@dataclass
class Dataset:
    images: np.ndarray      # [n, H, W, 4] uint8
    cameras: np.ndarray     # [n, 4, 4] float32 (row-major camera-to-world)
    intrinsics: tuple       # fx, fy, cx, cy

    @property
    def n(self):
        return self.images.shape[0]

    @property
    def width(self):
        return self.images.shape[2]

    @property
    def height(self):
        return self.images.shape[1]


def make_scene(kind=0, seed=0, n_primitives=3, density=50.0, extent=0.5, size_min=0.15, size_max=0.35, n_views=16,
               width=128, height=128, fov=0.69, radius=3.0, camera_mode=0, orbit_elevation=0.5, orbit_views=0,
               view_offset=0, n_threads=0, with_images=True) -> Dataset:
    """Seeded procedural scene and its exact ground-truth renders (nerf_b200_scene_render)."""
    d = NerfB200SceneDesc(kind, seed, n_primitives, density, extent, size_min, size_max, n_views, width, height, fov,
                          radius, camera_mode, orbit_elevation, orbit_views or n_views, view_offset, n_threads)
    imgs = np.zeros((n_views, height, width, 4), np.uint8) if with_images else None
    cams = np.zeros((n_views, 4, 4), np.float32)
    intr = np.zeros(4, np.float32)
    check("nerf_b200_scene_render", lib().nerf_b200_scene_render(C.byref(d), _ptr(imgs), _ptr(cams), _ptr(intr)))
    if imgs is None:
        imgs = np.zeros((n_views, height, width, 4), np.uint8)
    return Dataset(imgs, cams, tuple(float(x) for x in intr))


def training_config(aabb=((-1, -1, -1), (1, 1, 1)), rays=4096, steps=200, lr=1e-2, beta1=0.9, beta2=0.99, eps=1e-15,
                    clip=1e9, guard=1e12, loss_scale=128.0, lr_decay_ksteps=0, decay=0.95, threshold=0.01,
                    cells_per_update=1 << 21, update_interval=16, warmup=256) -> NerfTrainingConfig:
    hp = NerfHyperParams(lr, beta1, beta2, eps, clip, guard, loss_scale, lr_decay_ksteps)
    oc = NerfOccupancyParams(decay, threshold, cells_per_update, update_interval, warmup)
    (x0, y0, z0), (x1, y1, z1) = aabb
    return NerfTrainingConfig(x0, y0, z0, x1, y1, z1, hp, oc, rays, steps)


def create_desc(ds: Dataset, grid_res=128, max_sample_steps=1 << 22, max_batch_rays=1 << 16, alignment=256):
    """NerfCreateDesc for a dataset, with the host arrays it points to (keep
    them alive while the descriptor is used)."""
    images = np.ascontiguousarray(ds.images)
    cams = np.ascontiguousarray(ds.cameras, dtype=np.float32)
    fx, fy, cx, cy = ds.intrinsics
    desc = NerfCreateDesc(grid_res, max_sample_steps, max_batch_rays, alignment, images.ctypes.data, images.nbytes,
                          cams.ctypes.data, cams.nbytes, ds.n, ds.width, ds.height, fx, fy, cx, cy)
    return desc, images, cams


class Context:
    """One nerf.h context (device = the current CUDA device at creation)."""

    def __init__(self, ds: Dataset, grid_res=128, max_sample_steps=1 << 22, max_batch_rays=1 << 16, options=None,
                 alignment=256):
        self.lib = lib()
        self.ds = ds
        self.desc, self._images, self._cams = create_desc(ds, grid_res, max_sample_steps, max_batch_rays, alignment)
        self.grid_res = grid_res
        self.handle = C.c_void_p()
        opts = options if options is not None else default_options()
        self.cascades = max(1, int(opts.n_cascades))
        check("nerf_b200_create_context",
              self.lib.nerf_b200_create_context(C.byref(self.desc), C.byref(opts), C.byref(self.handle)))
        n_grid, n_mlp = C.c_uint64(), C.c_uint64()
        check("nerf_b200_param_counts", self.lib.nerf_b200_param_counts(self.handle, C.byref(n_grid), C.byref(n_mlp)))
        self.n_grid, self.n_mlp = n_grid.value, n_mlp.value
        self.n_params = self.n_grid + self.n_mlp

    def close(self):
        if self.handle:
            check("nerf_destroy_context", self.lib.nerf_destroy_context(self.handle))
            self.handle = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- nerf.h
    def configure(self, cfg: NerfTrainingConfig):
        self.cfg = cfg
        check("nerf_configure_training", self.lib.nerf_configure_training(self.handle, C.byref(cfg)))

    def train_step(self):
        check("nerf_train_step", self.lib.nerf_train_step(self.handle))

    def stats(self) -> NerfTrainStats:
        s = NerfTrainStats()
        check("nerf_read_train_stats", self.lib.nerf_read_train_stats(self.handle, C.byref(s)))
        return s

    def inference(self, camera_idx=0, samples_per_ray=128) -> np.ndarray:
        out = np.zeros((self.ds.height, self.ds.width, 4), np.uint8)
        req = NerfInferenceRequest(camera_idx, samples_per_ray, NERF_MEMORY_HOST, out.ctypes.data, out.nbytes)
        info = NerfInferenceInfo()
        check("nerf_inference", self.lib.nerf_inference(self.handle, C.byref(req), C.byref(info)))
        return out

    def save(self, path: str):
        d = NerfCheckpointFileDesc(str(path).encode())
        check("nerf_save_network_weights", self.lib.nerf_save_network_weights(self.handle, C.byref(d)))

    def load(self, path: str):
        d = NerfCheckpointFileDesc(str(path).encode())
        check("nerf_load_network_weights", self.lib.nerf_load_network_weights(self.handle, C.byref(d)))

    # ---- nerf_b200.h
    def save_state(self, path: str):
        """Training-state checkpoint (masters, Adam moments, occupancy, step state) for an exact resume."""
        check("nerf_b200_save_training_state", lib().nerf_b200_save_training_state(self.handle, str(path).encode()))

    def load_state(self, path: str):
        check("nerf_b200_load_training_state", lib().nerf_b200_load_training_state(self.handle, str(path).encode()))

    def counters(self) -> NerfB200Counters:
        c = NerfB200Counters()
        check("nerf_b200_read_counters", self.lib.nerf_b200_read_counters(self.handle, C.byref(c)))
        return c

    def layout(self) -> NerfB200GridLayout:
        g = NerfB200GridLayout()
        check("nerf_b200_context_grid_layout", self.lib.nerf_b200_context_grid_layout(self.handle, C.byref(g)))
        return g

    def params(self):
        master = np.zeros(self.n_params, np.float32)
        p16 = np.zeros(self.n_params, np.uint16)
        m = np.zeros(self.n_params, np.float32)
        v = np.zeros(self.n_params, np.float32)
        check("nerf_b200_read_params", self.lib.nerf_b200_read_params(self.handle, _ptr(master), _ptr(p16), _ptr(m), _ptr(v)))
        return master, p16, m, v

    def set_params(self, master: np.ndarray):
        master = np.ascontiguousarray(master, np.float32)
        check("nerf_b200_write_params", self.lib.nerf_b200_write_params(self.handle, _ptr(master)))

    def occupancy(self):
        cells = self.grid_res ** 3 * self.cascades
        dens = np.zeros(cells, np.float32)
        bits = np.zeros((cells + 31) // 32, np.uint32)
        check("nerf_b200_read_occupancy", self.lib.nerf_b200_read_occupancy(self.handle, _ptr(dens), _ptr(bits)))
        return dens, bits

    def set_occupancy(self, density=None, bitfield=None):
        d = None if density is None else np.ascontiguousarray(density, np.float32)
        b = None if bitfield is None else np.ascontiguousarray(bitfield, np.uint32)
        check("nerf_b200_write_occupancy", self.lib.nerf_b200_write_occupancy(self.handle, _ptr(d), _ptr(b)))

    def set_frame(self, frame: int):
        check("nerf_b200_set_frame_index", self.lib.nerf_b200_set_frame_index(self.handle, frame))

    def batch(self):
        c = self.counters()
        counts = np.zeros(c.rays, np.uint32)
        index = np.zeros(c.active_rays, np.uint32)
        recs = (abi.NerfB200RayRecord * max(1, c.active_rays))()
        pos = np.zeros((c.samples, 4), np.float32)
        sray = np.zeros(c.samples, np.uint32)
        check("nerf_b200_read_batch", self.lib.nerf_b200_read_batch(self.handle, _ptr(counts), _ptr(index),
                                                                    C.cast(recs, C.c_void_p), _ptr(pos), _ptr(sray)))
        rec = np.frombuffer(recs, dtype=np.uint8).reshape(-1, 48)[: c.active_rays]
        f = rec.view(np.float32).reshape(-1, 12)
        u = rec.view(np.uint32).reshape(-1, 12)
        return dict(counts=counts, index=index, dir=f[:, 0:3].copy(), begin=u[:, 3].copy(), gt=f[:, 4:8].copy(),
                    bg=f[:, 8:11].copy(), count=u[:, 11].copy(), pos_dt=pos, sample_ray=sray)

    def dp_peer_handle(self) -> bytes:
        """This rank's peer handle (nerf_b200_dp_peer_handle) for a host-side all-gather."""
        buf = (C.c_uint8 * 128)()
        check("nerf_b200_dp_peer_handle", self.lib.nerf_b200_dp_peer_handle(self.handle, buf))
        return bytes(buf)

    def dp_init_peers(self, rank: int, world: int, handles: list):
        """Peer-mode data parallelism from the world's handles in rank order (nerf_b200_dp_init_peers): no NCCL."""
        blob = b"".join(handles)
        assert len(blob) == 128 * world
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check("nerf_b200_dp_init_peers", self.lib.nerf_b200_dp_init_peers(self.handle, rank, world, buf))

    def dp_init(self, rank: int, world: int, uid: bytes):
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        check("nerf_b200_dp_init", self.lib.nerf_b200_dp_init(self.handle, rank, world, buf))

    def render(self, c2w: np.ndarray, width: int, height: int, intrinsics, max_steps=1024, stop=-1.0, tile=0, rank=0,
               world=1, dst: np.ndarray | None = None, device_ptr: int | None = None):
        c2w = np.ascontiguousarray(np.asarray(c2w, np.float32).reshape(-1)[:12])
        fx, fy, cx, cy = intrinsics
        if device_ptr is not None:
            kind, ptr, nbytes = NERF_MEMORY_CUDA_DEVICE, device_ptr, width * height * 4
        elif dst is not None:
            kind, ptr, nbytes = NERF_MEMORY_HOST, dst.ctypes.data, dst.nbytes
        else:
            kind, ptr, nbytes = NERF_MEMORY_HOST, None, 0
        req = NerfB200RenderRequest(c2w.ctypes.data, width, height, fx, fy, cx, cy, max_steps, stop, tile, rank, world,
                                    kind, ptr, nbytes)
        info = NerfB200RenderInfo()
        check("nerf_b200_render", self.lib.nerf_b200_render(self.handle, C.byref(req), C.byref(info)))
        return info


def dp_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    check("nerf_b200_dp_unique_id", lib().nerf_b200_dp_unique_id(buf))
    return bytes(buf)
