"""ctypes binding of libnerf_b200.so: the nerf.h ABI and the nerf_b200.h extensions.

This is the Python side of the drop-in boundary.  Structure layouts mirror
include/nerf.h (byte-identical to the reference's nerf.h) and
include/nerf_b200.h.  Loading fails loudly when the shared library is absent:
there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libnerf_b200.so"

# ---------------------------------------------------------------- nerf.h
NERF_STATUS_OK = 0
NERF_STATUS_INVALID_USAGE = 1
NERF_STATUS_STATE_ERROR = 2
NERF_STATUS_IO_ERROR = 3
NERF_STATUS_CUDA_ERROR = 4
NERF_STATUS_FAILURE = 5
STATUS_NAMES = {0: "OK", 1: "INVALID_USAGE", 2: "STATE_ERROR", 3: "IO_ERROR", 4: "CUDA_ERROR", 5: "FAILURE"}
NERF_MEMORY_HOST = 1
NERF_MEMORY_CUDA_DEVICE = 2


class NerfError(RuntimeError):
    def __init__(self, where: str, status: int):
        super().__init__(f"{where} failed: NERF_STATUS_{STATUS_NAMES.get(status, status)}")
        self.status = status


class NerfCreateDesc(C.Structure):
    _fields_ = [
        ("occupancy_grid_res", C.c_uint32),
        ("max_sample_steps", C.c_uint32),
        ("max_batch_rays", C.c_uint32),
        ("arena_alignment_bytes", C.c_uint64),
        ("images_rgba8", C.c_void_p),
        ("images_bytes", C.c_uint64),
        ("cameras_4x4_packed", C.c_void_p),
        ("cameras_bytes", C.c_uint64),
        ("image_count", C.c_uint32),
        ("image_width", C.c_uint32),
        ("image_height", C.c_uint32),
        ("fx", C.c_float),
        ("fy", C.c_float),
        ("cx", C.c_float),
        ("cy", C.c_float),
    ]


class NerfHyperParams(C.Structure):
    _fields_ = [
        ("learning_rate", C.c_float),
        ("adam_beta1", C.c_float),
        ("adam_beta2", C.c_float),
        ("adam_eps", C.c_float),
        ("grad_clip_norm", C.c_float),
        ("update_guard_grad_norm", C.c_float),
        ("loss_scale", C.c_float),
        ("lr_decay_ksteps", C.c_uint32),
    ]


class NerfOccupancyParams(C.Structure):
    _fields_ = [
        ("decay", C.c_float),
        ("threshold", C.c_float),
        ("cells_per_update", C.c_uint32),
        ("update_interval", C.c_uint32),
        ("warmup_steps", C.c_uint32),
    ]


class NerfTrainingConfig(C.Structure):
    _fields_ = [
        ("aabb_min_x", C.c_float),
        ("aabb_min_y", C.c_float),
        ("aabb_min_z", C.c_float),
        ("aabb_max_x", C.c_float),
        ("aabb_max_y", C.c_float),
        ("aabb_max_z", C.c_float),
        ("hyper_params", NerfHyperParams),
        ("occupancy_params", NerfOccupancyParams),
        ("rays_per_batch", C.c_uint32),
        ("max_sample_steps_per_ray", C.c_uint32),
    ]


class NerfTrainStats(C.Structure):
    _fields_ = [
        ("loss", C.c_float),
        ("grad_norm", C.c_float),
        ("has_nonfinite", C.c_uint32),
        ("completed_steps", C.c_uint32),
        ("last_train_camera", C.c_uint32),
    ]


class NerfInferenceRequest(C.Structure):
    _fields_ = [
        ("camera_idx", C.c_uint32),
        ("samples_per_ray", C.c_uint32),
        ("memory_kind", C.c_uint32),
        ("dst_rgba8", C.c_void_p),
        ("dst_bytes", C.c_uint64),
    ]


class NerfInferenceInfo(C.Structure):
    _fields_ = [
        ("capacity_bytes", C.c_uint64),
        ("valid_bytes", C.c_uint64),
        ("row_stride_bytes", C.c_uint32),
        ("width", C.c_uint32),
        ("height", C.c_uint32),
        ("generation", C.c_uint32),
    ]


class NerfCheckpointFileDesc(C.Structure):
    _fields_ = [("path_utf8", C.c_char_p)]


# ----------------------------------------------------------- nerf_b200.h
class NerfB200Options(C.Structure):
    _fields_ = [
        ("n_levels", C.c_uint32),
        ("log2_hashmap_size", C.c_uint32),
        ("base_resolution", C.c_uint32),
        ("max_resolution", C.c_uint32),
        ("hash_init_scale", C.c_float),
        ("background", C.c_uint32),
        ("stop_transmittance", C.c_float),
        ("render_stop_transmittance", C.c_float),
        ("target_samples_per_step", C.c_uint32),
        ("max_samples_per_step", C.c_uint32),
        ("n_cascades", C.c_uint32),
    ]


class NerfB200Counters(C.Structure):
    _fields_ = [
        ("frame_index", C.c_uint32),
        ("rays", C.c_uint32),
        ("active_rays", C.c_uint32),
        ("samples", C.c_uint32),
        ("marched_active_rays", C.c_uint32),
        ("next_rays", C.c_uint32),
        ("total_samples", C.c_uint64),
        ("total_rays", C.c_uint64),
        ("kernels_per_step", C.c_uint32),
        ("dp_peer", C.c_uint32),
    ]


MAX_LEVELS = 32


class NerfB200GridLayout(C.Structure):
    _fields_ = [
        ("n_levels", C.c_uint32),
        ("log2_hashmap_size", C.c_uint32),
        ("base_resolution", C.c_uint32),
        ("max_resolution", C.c_uint32),
        ("scale", C.c_float * MAX_LEVELS),
        ("resolution", C.c_uint32 * MAX_LEVELS),
        ("dense", C.c_uint32 * MAX_LEVELS),
        ("offset", C.c_uint32 * (MAX_LEVELS + 1)),
    ]


class NerfB200RayRecord(C.Structure):
    _fields_ = [
        ("dir", C.c_float * 3),
        ("begin", C.c_uint32),
        ("gt", C.c_float * 4),
        ("bg", C.c_float * 3),
        ("count", C.c_uint32),
    ]


class NerfB200RenderRequest(C.Structure):
    _fields_ = [
        ("c2w_3x4", C.c_void_p),
        ("width", C.c_uint32),
        ("height", C.c_uint32),
        ("fx", C.c_float),
        ("fy", C.c_float),
        ("cx", C.c_float),
        ("cy", C.c_float),
        ("max_steps", C.c_uint32),
        ("stop_transmittance", C.c_float),
        ("tile_size", C.c_uint32),
        ("tile_rank", C.c_uint32),
        ("tile_world", C.c_uint32),
        ("memory_kind", C.c_uint32),
        ("dst_rgba8", C.c_void_p),
        ("dst_bytes", C.c_uint64),
    ]


class NerfB200RenderInfo(C.Structure):
    _fields_ = [("rays", C.c_uint64), ("samples", C.c_uint64), ("milliseconds", C.c_float)]


STEP_KERNELS = ["occupancy_query", "occupancy_update", "sample_bits", "sample_scan", "sample_write", "field_forward",
                "composite", "mlp_backward", "grid_scatter", "wgrad_reduce", "allreduce", "grad_stats", "march", "adam"]


class NerfB200StepProfile(C.Structure):
    _fields_ = [("milliseconds", C.c_float * len(STEP_KERNELS)), ("total_milliseconds", C.c_float)]


class NerfB200SceneDesc(C.Structure):
    _fields_ = [
        ("kind", C.c_uint32),
        ("seed", C.c_uint32),
        ("n_primitives", C.c_uint32),
        ("density", C.c_float),
        ("extent", C.c_float),
        ("size_min", C.c_float),
        ("size_max", C.c_float),
        ("n_views", C.c_uint32),
        ("width", C.c_uint32),
        ("height", C.c_uint32),
        ("fov", C.c_float),
        ("radius", C.c_float),
        ("camera_mode", C.c_uint32),
        ("orbit_elevation", C.c_float),
        ("orbit_views", C.c_uint32),
        ("view_offset", C.c_uint32),
        ("n_threads", C.c_uint32),
    ]


P = C.c_void_p
U32 = C.c_uint32
U64 = C.c_uint64
F32 = C.c_float
S = C.c_int  # NerfStatus


class NerfB200BlenderInfo(C.Structure):
    _fields_ = [("image_count", C.c_uint32), ("width", C.c_uint32), ("height", C.c_uint32), ("camera_angle_x", C.c_float)]


# name -> (restype, argtypes); the ABI surface, in header order.
NERF_H_EXPORTS = {
    "nerf_create_context": (S, [C.POINTER(NerfCreateDesc), C.POINTER(P)]),
    "nerf_destroy_context": (S, [P]),
    "nerf_configure_training": (S, [P, C.POINTER(NerfTrainingConfig)]),
    "nerf_train_step": (S, [P]),
    "nerf_read_train_stats": (S, [P, C.POINTER(NerfTrainStats)]),
    "nerf_inference": (S, [P, C.POINTER(NerfInferenceRequest), C.POINTER(NerfInferenceInfo)]),
    "nerf_save_network_weights": (S, [P, C.POINTER(NerfCheckpointFileDesc)]),
    "nerf_load_network_weights": (S, [P, C.POINTER(NerfCheckpointFileDesc)]),
}
B200_EXPORTS = {
    "nerf_b200_default_options": (None, [C.POINTER(NerfB200Options)]),
    "nerf_b200_create_context": (S, [C.POINTER(NerfCreateDesc), C.POINTER(NerfB200Options), C.POINTER(P)]),
    "nerf_b200_read_counters": (S, [P, C.POINTER(NerfB200Counters)]),
    "nerf_b200_context_stream": (S, [P, C.POINTER(P)]),
    "nerf_b200_train_step_profiled": (S, [P, C.POINTER(NerfB200StepProfile)]),
    "nerf_b200_grid_layout": (S, [U32, U32, U32, U32, C.POINTER(NerfB200GridLayout)]),
    "nerf_b200_context_grid_layout": (S, [P, C.POINTER(NerfB200GridLayout)]),
    "nerf_b200_param_counts": (S, [P, C.POINTER(U64), C.POINTER(U64)]),
    "nerf_b200_read_params": (S, [P, P, P, P, P]),
    "nerf_b200_write_params": (S, [P, P]),
    "nerf_b200_read_occupancy": (S, [P, P, P]),
    "nerf_b200_write_occupancy": (S, [P, P, P]),
    "nerf_b200_set_frame_index": (S, [P, U32]),
    "nerf_b200_read_batch": (S, [P, P, P, P, P, P]),
    "nerf_b200_dp_unique_id": (S, [P]),
    "nerf_b200_dp_init": (S, [P, U32, U32, P]),
    "nerf_b200_dp_barrier_test": (S, [P, U32]),
    "nerf_b200_dp_peer_handle": (S, [P, P]),
    "nerf_b200_dp_init_peers": (S, [P, U32, U32, P]),
    "nerf_b200_render": (S, [P, C.POINTER(NerfB200RenderRequest), C.POINTER(NerfB200RenderInfo)]),
    "nerf_b200_render_output": (S, [P, C.POINTER(P)]),
    "nerf_b200_scene_render": (S, [C.POINTER(NerfB200SceneDesc), P, P, P]),
    "nerf_b200_grid_forward": (S, [C.POINTER(NerfB200GridLayout), P, U32, P, P, P]),
    "nerf_b200_grid_backward": (S, [C.POINTER(NerfB200GridLayout), P, U32, P, P, P]),
    "nerf_b200_field_forward": (S, [C.POINTER(NerfB200GridLayout), P, P, P, U32, P, P, P]),
    "nerf_b200_field_backward_partial_floats": (U64, []),
    "nerf_b200_field_backward": (S, [C.POINTER(NerfB200GridLayout), P, P, P, U32, P, P, P, P, P, P]),
    "nerf_b200_mlp_forward": (S, [P, P, P, U32, P, P]),
    "nerf_b200_mlp_backward": (S, [P, P, P, U32, P, P, P, P, P]),
    "nerf_b200_mlp_forward_tc": (S, [P, P, P, U32, P, P, P]),
    "nerf_b200_mlp_backward_tc": (S, [P, P, P, U32, P, P, P, P, P, P]),
    "nerf_b200_mlp_tc_info": (S, [P]),
    "nerf_b200_save_training_state": (S, [P, C.c_char_p]),
    "nerf_b200_blender_probe": (S, [C.c_char_p, P]),
    "nerf_b200_blender_load": (S, [C.c_char_p, U32, U32, P, U64, P, P]),
    "nerf_b200_blender_write": (S, [C.c_char_p, P, P, U32, U32, U32, F32, U32]),
    "nerf_b200_png_read": (S, [C.c_char_p, P, U64, P, P]),
    "nerf_b200_png_write": (S, [C.c_char_p, P, U32, U32]),
    "nerf_b200_load_training_state": (S, [P, C.c_char_p]),
    "nerf_b200_field_backward_noalloc_max_rows": (U32, []),
    "nerf_b200_field_backward_noalloc": (S, [C.POINTER(NerfB200GridLayout), P, P, P, U32, P, P, P, P, P]),
    "nerf_b200_composite": (S, [P, U32, P, P, F32, F32, F32, P, P, P, P, P]),
    "nerf_b200_adam": (S, [P, P, P, P, P, P, U64, U64, P, U32, F32, F32, F32, P]),
    "nerf_b200_occupancy_update": (S, [P, P, P, U32, U32, U32, U32, F32, F32, P]),
}
ALL_EXPORTS = {**NERF_H_EXPORTS, **B200_EXPORTS}

_lib = None


def load(path: os.PathLike | str | None = None) -> C.CDLL:
    """Loads libnerf_b200.so and declares every prototype.  Raises when the
    library or any declared symbol is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = pathlib.Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is not built; run __graft_entry__.build() or `make -C nerf_b200/csrc`")
    lib = C.CDLL(str(p))
    for name, (res, args) in ALL_EXPORTS.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is absent
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(where: str, status: int) -> None:
    if status != NERF_STATUS_OK:
        raise NerfError(where, status)
