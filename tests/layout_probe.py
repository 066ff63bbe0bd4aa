"""Compiles a probe against a nerf.h and reports sizeof/offsetof of every ABI struct field.

Used by tests/test_abi.py (our include/nerf.h) and tests/golden/make_layout_golden.py
(the reference's nerf.h, to produce tests/golden/nerf_h_layout.json).
"""
import json
import pathlib
import subprocess
import tempfile

FIELDS = {
    "NerfCreateDesc": ["occupancy_grid_res", "max_sample_steps", "max_batch_rays", "arena_alignment_bytes", "images_rgba8",
                       "images_bytes", "cameras_4x4_packed", "cameras_bytes", "image_count", "image_width",
                       "image_height", "fx", "fy", "cx", "cy"],
    "NerfHyperParams": ["learning_rate", "adam_beta1", "adam_beta2", "adam_eps", "grad_clip_norm",
                        "update_guard_grad_norm", "loss_scale", "lr_decay_ksteps"],
    "NerfOccupancyParams": ["decay", "threshold", "cells_per_update", "update_interval", "warmup_steps"],
    "NerfTrainingConfig": ["aabb_min_x", "aabb_min_y", "aabb_min_z", "aabb_max_x", "aabb_max_y", "aabb_max_z",
                           "hyper_params", "occupancy_params", "rays_per_batch", "max_sample_steps_per_ray"],
    "NerfTrainStats": ["loss", "grad_norm", "has_nonfinite", "completed_steps", "last_train_camera"],
    "NerfInferenceRequest": ["camera_idx", "samples_per_ray", "memory_kind", "dst_rgba8", "dst_bytes"],
    "NerfInferenceInfo": ["capacity_bytes", "valid_bytes", "row_stride_bytes", "width", "height", "generation"],
    "NerfCheckpointFileDesc": ["path_utf8"],
}
ENUMS = ["NERF_STATUS_OK", "NERF_STATUS_INVALID_USAGE", "NERF_STATUS_STATE_ERROR", "NERF_STATUS_IO_ERROR",
         "NERF_STATUS_CUDA_ERROR", "NERF_STATUS_FAILURE", "NERF_MEMORY_HOST", "NERF_MEMORY_CUDA_DEVICE"]


def probe(header_dir: str) -> dict:
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "nerf.h"', "int main(void) {", 'printf("{");']
    first = True
    for s, fields in FIELDS.items():
        for f in [None] + fields:
            key = f"{s}.{f}" if f else f"{s}.__size__"
            expr = f"offsetof({s}, {f})" if f else f"sizeof({s})"
            sep = "" if first else ","
            lines.append(f'printf("{sep}\\"{key}\\": %zu", (size_t)({expr}));')
            first = False
    for e in ENUMS:
        lines.append(f'printf(",\\"{e}\\": %d", (int){e});')
    lines += ['printf("}\\n");', "return 0; }"]
    with tempfile.TemporaryDirectory() as td:
        src = pathlib.Path(td) / "probe.c"
        exe = pathlib.Path(td) / "probe"
        src.write_text("\n".join(lines))
        subprocess.run(["gcc", "-std=c11", "-I", header_dir, str(src), "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return json.loads(out)
