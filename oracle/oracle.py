"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU oracle (oracle/liboracle.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
this module, as the checker or the timed CPU baseline.  The product
(libnerf_b200.so) never links or calls it.
"""
from __future__ import annotations

import ctypes as C
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

P = C.c_void_p
U32, U64, F32 = C.c_uint32, C.c_uint64, C.c_float

MAX_LEVELS = 32


class GridLayout(C.Structure):
    _fields_ = [
        ("n_levels", U32), ("log2_hashmap_size", U32), ("base_resolution", U32), ("max_resolution", U32),
        ("scale", F32 * MAX_LEVELS), ("resolution", U32 * MAX_LEVELS), ("dense", U32 * MAX_LEVELS),
        ("offset", U32 * (MAX_LEVELS + 1)),
    ]


class AdamScalars(C.Structure):
    _fields_ = [("learning_rate", F32), ("grad_scale", F32), ("inv_bias_correction1", F32),
                ("inv_bias_correction2", F32), ("inv_loss_scale", F32), ("skip_update", U32)]


class Options(C.Structure):
    _fields_ = [("n_levels", U32), ("log2_hashmap_size", U32), ("base_resolution", U32), ("max_resolution", U32),
                ("hash_init_scale", F32), ("background", U32), ("stop_transmittance", F32),
                ("target_samples_per_step", U32), ("max_samples_per_step", U32), ("dp_rank", U32), ("dp_world", U32),
                ("n_threads", U32), ("n_cascades", U32)]


class BatchInfo(C.Structure):
    _fields_ = [("rays", U32), ("active_rays", U32), ("samples", U32), ("camera", U32)]


class SceneDesc(C.Structure):
    """Mirror of NerfB200SceneDesc (include/nerf_b200.h): the synthetic-scene renderer's description."""
    _fields_ = [("kind", U32), ("seed", U32), ("n_primitives", U32), ("density", F32), ("extent", F32),
                ("size_min", F32), ("size_max", F32), ("n_views", U32), ("width", U32), ("height", U32), ("fov", F32),
                ("radius", F32), ("camera_mode", U32), ("orbit_elevation", F32), ("orbit_views", U32),
                ("view_offset", U32), ("n_threads", U32)]


_PROTOS = {
    "oracle_scene_render": (C.c_int, [C.POINTER(SceneDesc), P, P, P]),
    "oracle_hash_u32": (U32, [U32]),
    "oracle_rand01": (F32, [U32]),
    "oracle_train_camera": (U32, [U32, U32]),
    "oracle_occupancy_mode": (U32, [U32, U32, U32]),
    "oracle_splitmix_xavier": (None, [U64, U64, P, P, U32, P]),
    "oracle_splitmix_uniform": (None, [U64, U64, U64, F32, P]),
    "oracle_grid_layout": (C.c_int, [U32, U32, U32, U32, C.POINTER(GridLayout)]),
    "oracle_grid_corners": (None, [C.POINTER(GridLayout), P, U32, P, P]),
    "oracle_grid_forward": (None, [C.POINTER(GridLayout), P, P, U32, P]),
    "oracle_grid_backward": (None, [C.POINTER(GridLayout), P, P, U32, P]),
    "oracle_sh4": (None, [P, U32, P]),
    "oracle_mlp_forward": (None, [P, P, P, U32, P]),
    "oracle_mlp_backward": (None, [P, P, P, P, U32, P, P]),
    "oracle_composite": (None, [P, P, P, P, U32, P, P, F32, F32, F32, P, P, P, P]),
    "oracle_adam_scalars": (None, [F32, U32, U32, P, C.POINTER(AdamScalars)]),
    "oracle_adam": (None, [P, P, P, P, P, U64, F32, F32, F32, C.POINTER(AdamScalars)]),
    "oracle_occupancy_update": (None, [P, P, P, U32, U32, U32, U32, F32, F32]),
    "oracle_ctx_create": (P, [P, C.POINTER(Options)]),
    "oracle_ctx_destroy": (None, [P]),
    "oracle_ctx_configure": (C.c_int, [P, P]),
    "oracle_ctx_step": (C.c_int, [P]),
    "oracle_ctx_step_grads": (C.c_int, [P]),
    "oracle_ctx_step_apply": (C.c_int, [P]),
    "oracle_ctx_stats": (C.c_int, [P, P]),
    "oracle_ctx_batch_info": (C.c_int, [P, C.POINTER(BatchInfo)]),
    "oracle_ctx_param_count": (U64, [P, C.POINTER(U64), C.POINTER(U64)]),
    "oracle_ctx_get_params": (C.c_int, [P, P, P, P, P, P]),
    "oracle_ctx_set_params": (C.c_int, [P, P]),
    "oracle_ctx_set_grads": (C.c_int, [P, P, F32, U32]),
    "oracle_ctx_set_global_samples": (C.c_int, [P, U64]),
    "oracle_ctx_get_loss": (C.c_int, [P, P, P]),
    "oracle_occupancy_cells": (None, [U32, U32, U32, U32, P, P, P]),
    "oracle_ctx_get_occupancy": (C.c_int, [P, P, P]),
    "oracle_ctx_set_occupancy": (C.c_int, [P, P, P]),
    "oracle_ctx_set_frame": (C.c_int, [P, U32]),
    "oracle_ctx_get_batch": (C.c_int, [P, P, P, P, P, P, P, P, P]),
    "oracle_ctx_render": (C.c_int, [P, P, U32, U32, F32, F32, F32, F32, U32, F32, P, P, U32, U32]),
}

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        l = C.CDLL(str(LIB))
        for name, (res, args) in _PROTOS.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def ptr(a):
    return None if a is None else a.ctypes.data


def make_scene(kind=0, seed=0, n_primitives=3, density=50.0, extent=0.5, size_min=0.15, size_max=0.35, n_views=16,
               width=128, height=128, fov=0.69, radius=3.0, camera_mode=0, orbit_elevation=0.5, orbit_views=0,
               view_offset=0, n_threads=0, with_images=True):
    """The seeded synthetic scenes and their exact renders, from this library's copy of the scene renderer (the same
    source as nerf_b200_scene_render).  Returns (images [n,H,W,4] uint8, cameras [n,4,4] float32, (fx, fy, cx, cy))."""
    d = SceneDesc(kind, seed, n_primitives, density, extent, size_min, size_max, n_views, width, height, fov, radius,
                  camera_mode, orbit_elevation, orbit_views or n_views, view_offset, n_threads)
    imgs = np.zeros((n_views, height, width, 4), np.uint8)
    cams = np.zeros((n_views, 4, 4), np.float32)
    intr = np.zeros(4, np.float32)
    rc = lib().oracle_scene_render(C.byref(d), ptr(imgs) if with_images else None, ptr(cams), ptr(intr))
    if rc != 0:
        raise ValueError(f"oracle_scene_render failed with status {rc}")
    return imgs, cams, tuple(float(x) for x in intr)


def grid_layout(n_levels=16, log2_hashmap_size=19, base_resolution=16, max_resolution=2048) -> GridLayout:
    g = GridLayout()
    if lib().oracle_grid_layout(n_levels, log2_hashmap_size, base_resolution, max_resolution, C.byref(g)) != 0:
        raise ValueError("invalid grid layout")
    return g


def grid_forward(g: GridLayout, params16: np.ndarray, pos: np.ndarray) -> np.ndarray:
    pos = np.ascontiguousarray(pos, np.float32)
    n = pos.shape[0]
    feat = np.zeros((n, 2 * g.n_levels), np.uint16)
    lib().oracle_grid_forward(C.byref(g), ptr(np.ascontiguousarray(params16, np.uint16)), ptr(pos), n, ptr(feat))
    return feat


def grid_corners(g: GridLayout, pos: np.ndarray):
    pos = np.ascontiguousarray(pos, np.float32)
    n = pos.shape[0]
    idx = np.zeros((n, g.n_levels, 8), np.uint32)
    w = np.zeros((n, g.n_levels, 8), np.float32)
    lib().oracle_grid_corners(C.byref(g), ptr(pos), n, ptr(idx), ptr(w))
    return idx, w


def grid_backward(g: GridLayout, pos: np.ndarray, dfeat: np.ndarray) -> np.ndarray:
    pos = np.ascontiguousarray(pos, np.float32)
    dfeat = np.ascontiguousarray(dfeat, np.float32)
    grad = np.zeros(2 * g.offset[g.n_levels], np.float64)
    lib().oracle_grid_backward(C.byref(g), ptr(pos), ptr(dfeat), pos.shape[0], ptr(grad))
    return grad


def sh4(dirs: np.ndarray) -> np.ndarray:
    dirs = np.ascontiguousarray(dirs, np.float32)
    out = np.zeros((dirs.shape[0], 16), np.float32)
    lib().oracle_sh4(ptr(dirs), dirs.shape[0], ptr(out))
    return out


def mlp_forward(mlp16: np.ndarray, feat16: np.ndarray, dirs: np.ndarray) -> np.ndarray:
    feat16 = np.ascontiguousarray(feat16, np.uint16)
    dirs = np.ascontiguousarray(dirs, np.float32)
    out = np.zeros((feat16.shape[0], 4), np.float32)
    lib().oracle_mlp_forward(ptr(np.ascontiguousarray(mlp16, np.uint16)), ptr(feat16), ptr(dirs), feat16.shape[0], ptr(out))
    return out


def mlp_backward(mlp16, feat16, dirs, dout):
    feat16 = np.ascontiguousarray(feat16, np.uint16)
    dirs = np.ascontiguousarray(dirs, np.float32)
    dout = np.ascontiguousarray(dout, np.float32)
    n = feat16.shape[0]
    dfeat = np.zeros((n, 32), np.float32)
    wg = np.zeros(10240, np.float64)
    lib().oracle_mlp_backward(ptr(np.ascontiguousarray(mlp16, np.uint16)), ptr(feat16), ptr(dirs), ptr(dout), n,
                              ptr(dfeat), ptr(wg))
    return dfeat, wg


def composite(raw, dt, begin, count, gt, bg, inv_norm, loss_scale, stop):
    raw = np.ascontiguousarray(raw, np.float32)
    dt = np.ascontiguousarray(dt, np.float32)
    begin = np.ascontiguousarray(begin, np.uint32)
    count = np.ascontiguousarray(count, np.uint32)
    gt = np.ascontiguousarray(gt, np.float32)
    bg = np.ascontiguousarray(bg, np.float32)
    n = begin.shape[0]
    dout = np.zeros_like(raw)
    loss = np.zeros(n, np.float32)
    used = np.zeros(n, np.uint32)
    rgb = np.zeros((n, 3), np.float32)
    lib().oracle_composite(ptr(raw), ptr(dt), ptr(begin), ptr(count), n, ptr(gt), ptr(bg), inv_norm, loss_scale, stop,
                           ptr(dout), ptr(loss), ptr(used), ptr(rgb))
    return dout, loss, used, rgb


def adam_scalars(grad_norm, nonfinite, step, hp) -> AdamScalars:
    s = AdamScalars()
    lib().oracle_adam_scalars(grad_norm, nonfinite, step, C.cast(C.pointer(hp), C.c_void_p), C.byref(s))
    return s


def adam(master, p16, grad, m, v, b1, b2, eps, s: AdamScalars):
    lib().oracle_adam(ptr(master), ptr(p16), ptr(grad), ptr(m), ptr(v), master.shape[0], b1, b2, eps, C.byref(s))


def occupancy_update(density, bits, sigma, cell_count, update_count, frame, mode, decay, threshold):
    lib().oracle_occupancy_update(ptr(density), ptr(bits), ptr(sigma), cell_count, update_count, frame, mode, decay,
                                  threshold)


def occupancy_cells(frame, update_count, cell_count, grid_res, aabb_min, aabb_max):
    """World positions of the cells an occupancy refresh queries at this frame."""
    out = np.zeros((update_count, 3), np.float32)
    mn, mx = np.asarray(aabb_min, np.float32), np.asarray(aabb_max, np.float32)
    lib().oracle_occupancy_cells(frame, update_count, cell_count, grid_res, ptr(mn), ptr(mx), ptr(out))
    return out


def options(n_levels=16, log2_hashmap_size=19, base_resolution=16, max_resolution=2048, hash_init_scale=1e-4,
            background=0, stop_transmittance=1e-4, target_samples_per_step=0, max_samples_per_step=0, dp_rank=0,
            dp_world=1, n_threads=1, n_cascades=1) -> Options:
    return Options(n_levels, log2_hashmap_size, base_resolution, max_resolution, hash_init_scale, background,
                   stop_transmittance, target_samples_per_step, max_samples_per_step, dp_rank, dp_world, n_threads,
                   n_cascades)


class Context:
    """CPU emulation of one nerf.h context (same create/configure/step semantics)."""

    def __init__(self, desc, opts: Options, images=None, cams=None):
        self.lib = lib()
        self._keep = (images, cams)
        self.h = self.lib.oracle_ctx_create(C.cast(C.pointer(desc), C.c_void_p), C.byref(opts))
        if not self.h:
            raise RuntimeError("oracle_ctx_create failed")
        ng, nm = U64(), U64()
        self.n_params = self.lib.oracle_ctx_param_count(self.h, C.byref(ng), C.byref(nm))
        self.n_grid, self.n_mlp = ng.value, nm.value
        self.grid_res = desc.occupancy_grid_res
        self.cascades = max(1, int(opts.n_cascades))

    def close(self):
        if self.h:
            self.lib.oracle_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def configure(self, cfg):
        self.cfg = cfg
        st = self.lib.oracle_ctx_configure(self.h, C.cast(C.pointer(cfg), C.c_void_p))
        if st != 0:
            raise RuntimeError(f"oracle configure status {st}")

    def step(self):
        assert self.lib.oracle_ctx_step(self.h) == 0

    def step_grads(self):
        assert self.lib.oracle_ctx_step_grads(self.h) == 0

    def step_apply(self):
        assert self.lib.oracle_ctx_step_apply(self.h) == 0

    def stats(self):
        from nerf_b200.abi import NerfTrainStats
        s = NerfTrainStats()
        self.lib.oracle_ctx_stats(self.h, C.cast(C.pointer(s), C.c_void_p))
        return s

    def info(self) -> BatchInfo:
        b = BatchInfo()
        self.lib.oracle_ctx_batch_info(self.h, C.byref(b))
        return b

    def params(self):
        n = self.n_params
        master, p16 = np.zeros(n, np.float32), np.zeros(n, np.uint16)
        m, v, g = np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.float32)
        self.lib.oracle_ctx_get_params(self.h, ptr(master), ptr(p16), ptr(m), ptr(v), ptr(g))
        return master, p16, m, v, g

    def set_params(self, master):
        master = np.ascontiguousarray(master, np.float32)
        self.lib.oracle_ctx_set_params(self.h, ptr(master))

    def set_grads(self, grad, loss_sum, active):
        grad = np.ascontiguousarray(grad, np.float32)
        self.lib.oracle_ctx_set_grads(self.h, ptr(grad), loss_sum, active)

    def set_global_samples(self, samples):
        """Data parallel: the pending step's compacted samples summed over all ranks."""
        self.lib.oracle_ctx_set_global_samples(self.h, int(samples))

    def loss(self):
        """(normalised loss sum, kept rays) of the pending step."""
        ls, act = F32(), U32()
        self.lib.oracle_ctx_get_loss(self.h, C.byref(ls), C.byref(act))
        return ls.value, act.value

    def occupancy(self):
        cells = self.grid_res ** 3 * self.cascades
        d = np.zeros(cells, np.float32)
        b = np.zeros((cells + 31) // 32, np.uint32)
        self.lib.oracle_ctx_get_occupancy(self.h, ptr(d), ptr(b))
        return d, b

    def set_occupancy(self, density=None, bits=None):
        d = None if density is None else np.ascontiguousarray(density, np.float32)
        b = None if bits is None else np.ascontiguousarray(bits, np.uint32)
        self.lib.oracle_ctx_set_occupancy(self.h, ptr(d), ptr(b))

    def set_frame(self, f):
        self.lib.oracle_ctx_set_frame(self.h, f)

    def batch(self):
        inf = self.info()
        counts = np.zeros(inf.rays, np.uint32)
        index = np.zeros(inf.active_rays, np.uint32)
        begin = np.zeros(inf.active_rays, np.uint32)
        count = np.zeros(inf.active_rays, np.uint32)
        gt = np.zeros((inf.active_rays, 4), np.float32)
        bg = np.zeros((inf.active_rays, 3), np.float32)
        dirs = np.zeros((inf.active_rays, 3), np.float32)
        pos = np.zeros((inf.samples, 4), np.float32)
        self.lib.oracle_ctx_get_batch(self.h, ptr(counts), ptr(index), ptr(begin), ptr(count), ptr(gt), ptr(bg),
                                      ptr(dirs), ptr(pos))
        return dict(counts=counts, index=index, begin=begin, count=count, gt=gt, bg=bg, dir=dirs, pos_dt=pos)

    def render(self, c2w, width, height, intrinsics, max_steps, stop, pixel_begin=0, pixel_end=None):
        c2w = np.ascontiguousarray(np.asarray(c2w, np.float32).reshape(-1)[:12])
        rgba = np.zeros(width * height, np.uint32)
        spp = np.zeros(width * height, np.uint32)
        fx, fy, cx, cy = intrinsics
        end = width * height if pixel_end is None else pixel_end
        self.lib.oracle_ctx_render(self.h, ptr(c2w), width, height, fx, fy, cx, cy, max_steps, stop, ptr(rgba),
                                   ptr(spp), pixel_begin, end)
        return rgba, spp
