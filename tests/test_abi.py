"""CPU tests of the drop-in boundary: exports, struct layouts, host-side logic.

No CUDA device is needed: only host entry points of libnerf_b200.so are
called (grid layout, options, scene generator).
"""
import ctypes as C
import json
import pathlib
import re
import subprocess

import numpy as np
import pytest

import nerf_b200
from nerf_b200 import abi
from layout_probe import probe
from oracle import oracle

ROOT = pathlib.Path(__file__).resolve().parents[1]


def declared_exports():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"NERF_API\s+[\w\s\*]+?\b(nerf_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = abi.load()
    declared = declared_exports()
    assert declared, "no NERF_API declarations found"
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    out = subprocess.run(["nm", "-D", "--defined-only", str(abi.LIB_PATH)], capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert declared <= exported
    # every exported nerf_* symbol is declared in a header
    assert {n for n in exported if n.startswith("nerf_")} <= declared
    # the python binding covers the whole surface
    assert set(abi.ALL_EXPORTS) == declared


def test_nerf_h_has_the_reference_entry_points():
    ref_entry_points = {"nerf_create_context", "nerf_destroy_context", "nerf_configure_training", "nerf_train_step",
                        "nerf_read_train_stats", "nerf_inference", "nerf_save_network_weights",
                        "nerf_load_network_weights"}
    text = (ROOT / "include" / "nerf.h").read_text()
    assert set(re.findall(r"NERF_API\s+NerfStatus\s+(nerf_\w+)", text)) == ref_entry_points


def test_struct_layouts_match_reference_golden():
    golden = json.loads((ROOT / "tests" / "golden" / "nerf_h_layout.json").read_text())
    assert probe(str(ROOT / "include")) == golden


def test_ctypes_mirror_matches_c_layout():
    lay = probe(str(ROOT / "include"))
    for name in ["NerfCreateDesc", "NerfHyperParams", "NerfOccupancyParams", "NerfTrainingConfig", "NerfTrainStats",
                 "NerfInferenceRequest", "NerfInferenceInfo", "NerfCheckpointFileDesc"]:
        cls = getattr(abi, name)
        assert C.sizeof(cls) == lay[f"{name}.__size__"], name
        for fname, _ in cls._fields_:
            assert getattr(cls, fname).offset == lay[f"{name}.{fname}"], (name, fname)


@pytest.mark.parametrize("cfg", [(16, 15, 16, 512), (16, 19, 16, 2048), (16, 22, 16, 8192), (8, 14, 16, 256),
                                 (16, 24, 16, 4096), (1, 12, 32, 32)])
def test_grid_layout_library_equals_oracle(cfg):
    g = nerf_b200.grid_layout(*cfg)
    o = oracle.grid_layout(*cfg)
    assert bytes(g) == bytes(o)
    L = cfg[0]
    T = 1 << cfg[1]
    for l in range(L):
        R = g.resolution[l]
        size = g.offset[l + 1] - g.offset[l]
        assert g.dense[l] == (R ** 3 <= T)
        assert size == ((R ** 3 + 7) // 8 * 8 if g.dense[l] else T)
        assert g.offset[l] % 8 == 0
    # top level reaches the requested resolution
    assert abs(g.scale[L - 1] - (cfg[3] - 1)) < 1e-3 * cfg[3] or L == 1


def test_grid_layout_rejects_bad_input():
    g = abi.NerfB200GridLayout()
    lib = abi.load()
    assert lib.nerf_b200_grid_layout(0, 19, 16, 2048, C.byref(g)) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_b200_grid_layout(40, 19, 16, 2048, C.byref(g)) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_b200_grid_layout(16, 19, 64, 32, C.byref(g)) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_b200_grid_layout(16, 19, 16, 2048, None) == abi.NERF_STATUS_INVALID_USAGE


def test_default_options_and_env(monkeypatch):
    o = nerf_b200.default_options()
    assert (o.n_levels, o.log2_hashmap_size, o.base_resolution, o.max_resolution) == (16, 19, 16, 2048)
    assert o.background == 0 and o.target_samples_per_step == 0
    monkeypatch.setenv("NERF_B200_LOG2_HASHMAP_SIZE", "15")
    monkeypatch.setenv("NERF_B200_BACKGROUND", "1")
    monkeypatch.setenv("NERF_B200_STOP_T", "0")
    o = nerf_b200.default_options()
    assert o.log2_hashmap_size == 15 and o.background == 1 and o.stop_transmittance == 0.0


def test_null_arguments_are_invalid_usage_without_a_device():
    lib = abi.load()
    out = C.c_void_p()
    assert lib.nerf_create_context(None, C.byref(out)) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_destroy_context(None) == abi.NERF_STATUS_OK  # destroy(NULL) is allowed (reference :2099)
    assert lib.nerf_configure_training(None, None) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_train_step(None) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_read_train_stats(None, None) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_inference(None, None, None) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_save_network_weights(None, None) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_load_network_weights(None, None) == abi.NERF_STATUS_INVALID_USAGE
    desc = abi.NerfCreateDesc()
    desc.occupancy_grid_res = 0
    assert lib.nerf_create_context(C.byref(desc), C.byref(out)) == abi.NERF_STATUS_INVALID_USAGE


def test_misaligned_tables_are_invalid_usage_without_a_device():
    """Kernel-level entry points refuse parameter / gradient tables that do not
    start on a 16-byte boundary before any device work (the pointers here are
    never dereferenced)."""
    lib = abi.load()
    g = abi.NerfB200GridLayout()
    assert lib.nerf_b200_grid_layout(16, 15, 16, 2048, C.byref(g)) == abi.NERF_STATUS_OK
    ok, bad = C.c_void_p(0x10000), C.c_void_p(0x10008)
    pos = C.cast(ok, C.POINTER(C.c_float))
    fl = C.cast(ok, C.POINTER(C.c_float))
    inv = abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_b200_grid_forward(C.byref(g), pos, 1, bad, ok, None) == inv
    assert lib.nerf_b200_grid_backward(C.byref(g), pos, 1, ok, bad, None) == inv
    assert lib.nerf_b200_field_forward(C.byref(g), bad, pos, pos, 1, ok, fl, None) == inv
    assert lib.nerf_b200_field_backward(C.byref(g), bad, pos, pos, 1, ok, fl, ok, fl, fl, None) == inv
    assert lib.nerf_b200_field_backward(C.byref(g), ok, pos, pos, 1, ok, fl, bad, fl, fl, None) == inv
    assert lib.nerf_b200_field_backward_noalloc(C.byref(g), ok, pos, pos, 1, ok, fl, bad, fl, None) == inv
    assert lib.nerf_b200_mlp_forward(bad, ok, pos, 1, fl, None) == inv
    assert lib.nerf_b200_mlp_backward(bad, ok, pos, 1, fl, ok, fl, fl, None) == inv


def test_scene_generator_is_deterministic_and_sane():
    a = nerf_b200.make_scene(kind=0, seed=0, n_views=4, width=32, height=32, n_threads=2)
    b = nerf_b200.make_scene(kind=0, seed=0, n_views=4, width=32, height=32, n_threads=3)
    assert np.array_equal(a.images, b.images) and np.array_equal(a.cameras, b.cameras)
    assert a.images[..., 3].max() == 255 and a.images[..., 3].min() == 0  # objects and background both visible
    R = a.cameras[:, :3, :3]
    assert np.allclose(np.einsum("nij,nkj->nik", R, R), np.eye(3), atol=1e-5)
    assert np.allclose(np.linalg.norm(a.cameras[:, :3, 3], axis=1), 3.0, atol=1e-5)
    c = nerf_b200.make_scene(kind=1, seed=3, n_primitives=12, density=100.0, extent=1.0, size_min=0.1, size_max=0.6,
                             n_views=2, width=24, height=24, radius=4.0, camera_mode=1, n_threads=2)
    assert (c.cameras[:, 2, 3] > 0).all()  # upper hemisphere


def test_extension_struct_mirrors_match_c_layout(tmp_path):
    """Every NerfB200* ctypes mirror in nerf_b200.abi has the size and field offsets of its C struct in
    include/nerf_b200.h (compiled probe), and the step profile has one slot per named segment."""
    import inspect
    structs = {n: c for n, c in inspect.getmembers(abi, inspect.isclass)
               if n.startswith("NerfB200") and issubclass(c, C.Structure)}
    assert "NerfB200StepProfile" in structs and "NerfB200Options" in structs
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "nerf_b200.h"', "int main(void) {"]
    for n, c in structs.items():
        lines.append(f'printf("{n}.__size__ %zu\\n", sizeof({n}));')
        for fname, _ in c._fields_:
            lines.append(f'printf("{n}.{fname} %zu\\n", offsetof({n}, {fname}));')
    lines.append('printf("NERF_B200_STEP_KERNELS %d\\n", NERF_B200_STEP_KERNELS);')
    lines.append("return 0; }")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                          check=True).stdout.splitlines())
    for n, c in structs.items():
        assert C.sizeof(c) == int(got[f"{n}.__size__"]), n
        for fname, _ in c._fields_:
            assert getattr(c, fname).offset == int(got[f"{n}.{fname}"]), (n, fname)
    assert int(got["NERF_B200_STEP_KERNELS"]) == len(abi.STEP_KERNELS)


def test_oracle_scene_renderer_matches_the_library():
    """The oracle library carries the same scene renderer (oracle_scene_render, compiled from the package's
    scene.cpp) so that the benchmark's reference arm can build its datasets without loading libnerf_b200.so: its
    images, cameras and intrinsics equal the library's bit for bit."""
    from oracle import oracle
    for kw in (dict(kind=0, seed=0, n_views=3, width=40, height=32),
               dict(kind=1, seed=2, n_primitives=12, density=100.0, extent=1.0, size_min=0.1, size_max=0.6, n_views=2,
                    width=48, height=48, radius=4.0, camera_mode=1),
               dict(kind=2, seed=4, n_primitives=10, density=100.0, extent=6.0, size_min=0.1, size_max=0.6, n_views=2,
                    width=40, height=24, fov=1.2, radius=3.0, camera_mode=3, orbit_elevation=0.3, orbit_views=6)):
        a = nerf_b200.make_scene(n_threads=2, **kw)
        imgs, cams, intr = oracle.make_scene(n_threads=3, **kw)
        assert np.array_equal(a.images, imgs) and np.array_equal(a.cameras, cams) and a.intrinsics == intr
