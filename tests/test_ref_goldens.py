"""The CPU oracle against the reference backend's own kernels.

tests/golden/ref_{stock,parity}.npz hold outputs of the reference's CUDA
kernels (backend-cuda.cu, compiled by oracle/ref/ and run on a GPU by
tests/golden/make_ref_goldens.py).  "parity" is the reference with its
approximate rsqrtf replaced by a correctly rounded 1/sqrt (the only
approximate operation on the sampler's path); "stock" is the reference as
shipped.

Bit-exact: hashing, the camera / occupancy-mode sequence, the occupancy
bitfield and query cells, Adam (step scalars, masters, moments, fp16
weights), and -- against the parity build -- the whole sampler (kept rays,
per-ray counts, ray directions, sample positions and steps, ground truth).
Against the stock build the sampler is compared statistically, since rsqrtf
moves ray directions by an ulp or two.  Floating point with tolerances:
compositing loss and gradients (the reference's sigma is softplus of its raw
input, the north star's is exp; both are compared as derivatives with respect
to sigma) and the occupancy densities (the reference's softplus goes through
__expf / log1pf).
"""
import pathlib

import numpy as np
import pytest

import nerf_b200
from oracle import oracle

GOLDEN = pathlib.Path(__file__).parent / "golden"
SCENE = dict(kind=0, seed=0, n_views=8, width=64, height=64, fov=0.69, radius=3.0)
AABB = ((-1, -1, -1), (1, 1, 1))
GRID, RAYS, MAX_STEPS = 32, 512, 128
OCC_GRID = 16


def _load(variant):
    return np.load(GOLDEN / f"ref_{variant}.npz")


@pytest.fixture(scope="module", params=["stock", "parity"])
def ref(request):
    return request.param, _load(request.param)


def test_struct_sizes(ref):
    _, d = ref
    assert list(d["struct_sizes"][:3]) == [68, 28, 8]


def test_hash_and_rand01_bit_exact(ref):
    _, d = ref
    lib = oracle.lib()
    x = d["hash_in"]
    ours = np.array([lib.oracle_hash_u32(int(v)) for v in x], np.uint32)
    assert np.array_equal(ours, d["hash_sampler"])
    assert np.array_equal(ours, d["hash_runtime"])
    r = np.array([lib.oracle_rand01(int(v)) for v in x], np.float32)
    assert np.array_equal(r.view(np.uint32), d["rand01"].view(np.uint32))


def test_camera_and_occupancy_mode_sequence(ref):
    _, d = ref
    lib = oracle.lib()
    for warmup, interval, frame, camera, mode in d["step"]:
        assert lib.oracle_train_camera(int(frame), 100) == camera
        assert lib.oracle_occupancy_mode(int(frame), int(warmup), int(interval)) == mode


def _oracle_sampler(bits, frame):
    ds = nerf_b200.make_scene(**SCENE)
    cfg = nerf_b200.training_config(aabb=AABB, rays=RAYS, steps=MAX_STEPS, warmup=1 << 20, update_interval=1,
                                     cells_per_update=1)
    desc, imgs, cams = nerf_b200.create_desc(ds, grid_res=GRID, max_sample_steps=RAYS * MAX_STEPS, max_batch_rays=RAYS)
    oc = oracle.Context(desc, oracle.options(log2_hashmap_size=15, max_resolution=512, n_threads=4), imgs, cams)
    oc.configure(cfg)
    oc.set_occupancy(bits=bits)
    oc.set_frame(frame)
    oc.step_grads()
    return ds, oc.batch()


@pytest.mark.parametrize("frame", [3, 7])
def test_sampler_against_reference(ref, frame):
    variant, d = ref
    ds, b = _oracle_sampler(d["sampler_bits"], frame)
    assert int(ds.images.astype(np.uint64).sum()) == int(d["sampler_images_sum"][0]), "scene generator changed"
    idx, cnt = d[f"sampler_f{frame}_index"], d[f"sampler_f{frame}_count"]
    ray, smp = d[f"sampler_f{frame}_ray"], d[f"sampler_f{frame}_samples"]
    if variant == "parity":
        assert np.array_equal(b["index"], idx), "kept rays"
        assert np.array_equal(b["count"], cnt), "per-ray sample counts"
        assert np.array_equal(b["counts"][idx], cnt)
        assert np.array_equal(b["pos_dt"].view(np.uint32), smp.view(np.uint32)), "sample positions and steps"
        assert np.array_equal(b["dir"].view(np.uint32), ray[:, 3:6].view(np.uint32)), "ray directions"
        # ground truth: the reference composites on white, as does background mode 0
        assert np.array_equal(b["gt"].view(np.uint32), ray[:, 11:15].view(np.uint32))
        assert np.array_equal(np.cumsum(np.concatenate([[0], cnt[:-1]])).astype(np.uint32), b["begin"]), "offsets"
    else:
        # rsqrtf: directions within a few ulps, nearly every ray keeps the same samples
        common, ia, ib = np.intersect1d(b["index"], idx, return_indices=True)
        assert len(common) >= 0.995 * len(idx)
        assert np.max(np.abs(b["dir"][ia] - ray[ib, 3:6])) < 1e-6
        same = b["count"][ia] == cnt[ib]
        assert same.mean() >= 0.99, same.mean()
        assert abs(int(b["count"].sum()) - int(cnt.sum())) <= 0.002 * cnt.sum()


def test_composite_loss_and_gradients(ref):
    _, d = ref
    count, begin, sigma = d["loss_count"], d["loss_begin"], d["loss_sigma"]
    S, n = len(sigma), len(count)
    raw = np.zeros((S, 4), np.float32)
    raw[:, 0] = np.log(sigma.astype(np.float64)).astype(np.float32)  # exp(raw) = sigma
    raw[:, 1:] = d["loss_raw_rgb"]
    bg = np.ones((n, 3), np.float32)
    dout, loss, _, _ = oracle.composite(raw, d["loss_dt"], begin, count, d["loss_gt"], bg, 1.0 / n, 1.0, 0.0)
    ref_loss = float(d["loss_sum"][0])
    assert abs(float(loss.astype(np.float64).sum()) - ref_loss) <= 2e-5 * abs(ref_loss), (loss.sum(), ref_loss)
    # dL/dsigma: ours dL/draw / sigma (exp), reference dL/draw_ref / sigmoid(raw_ref) (softplus)
    raw_ref = d["loss_raw_sigma_ref"].astype(np.float64)
    ref_dsig = d["loss_d_sigma_ref"].astype(np.float64) * (1.0 + np.exp(-raw_ref))
    our_dsig = dout[:, 0].astype(np.float64) / np.exp(raw[:, 0].astype(np.float64))
    err = np.linalg.norm(our_dsig - ref_dsig) / np.linalg.norm(ref_dsig)
    assert err < 2e-4, err
    err_rgb = np.linalg.norm(dout[:, 1:] - d["loss_d_rgb"]) / np.linalg.norm(d["loss_d_rgb"])
    assert err_rgb < 2e-5, err_rgb


def test_adam_against_reference(ref):
    _, d = ref
    from nerf_b200.abi import NerfHyperParams
    for i, (step, gn, nf, lr, dk, clip, guard) in enumerate(d["adam_cases"]):
        hp = NerfHyperParams(np.float32(lr), 0.9, 0.999, 1e-8, np.float32(clip), np.float32(guard), 128.0, int(dk))
        s = oracle.adam_scalars(np.float32(gn), int(nf), int(step), hp)
        rs = d["adam_scalars"][i]
        ours = np.array([s.learning_rate, s.grad_scale, s.inv_bias_correction1, s.inv_bias_correction2, s.inv_loss_scale,
                         s.skip_update], np.float64)
        assert np.array_equal(ours.astype(np.float32), rs), (i, ours, rs)
        p32, g, m, v = [a.copy() for a in d[f"adam{i}_in"]]
        p16 = np.zeros(len(p32), np.uint16)
        oracle.adam(p32, p16, g.astype(np.float32), m, v, 0.9, 0.999, 1e-8, s)
        rp, rp16, rm, rv = d[f"adam{i}_out"]
        if s.skip_update:
            assert np.array_equal(p32, d[f"adam{i}_in"][0]) and np.array_equal(rp, d[f"adam{i}_in"][0])
            continue
        # bit-exact: same contraction of b*m + (1-b)*g as the reference's compiler
        for ours_a, ref_a in ((m, rm), (v, rv), (p32, rp), (p16.view(np.float16).astype(np.float32), rp16)):
            assert np.array_equal(ours_a.view(np.uint32), ref_a.view(np.uint32))


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_occupancy_update_against_reference(ref, mode):
    _, d = ref
    frame = int(d[f"occ_m{mode}_frame"][0])
    density = d[f"occ_m{mode}_density_in"].copy()
    bits = d[f"occ_m{mode}_bits_in"].copy()
    sigma = d[f"occ_m{mode}_sigma"]
    cells, update = OCC_GRID ** 3, len(sigma)
    oracle.occupancy_update(density, bits, sigma, cells, update, frame, mode, 0.97, 0.01)
    assert np.array_equal(bits, d[f"occ_m{mode}_bits_out"]), "occupancy bitfield"
    # the reference's sigma is softplus(raw) through __expf / log1pf: a few ulps from the exact values
    assert np.allclose(density, d[f"occ_m{mode}_density_out"], rtol=1e-5, atol=0.0)
    if mode == 2:
        pos = oracle.occupancy_cells(frame, update, cells, OCC_GRID, AABB[0], AABB[1])
        assert np.array_equal(pos.view(np.uint32), d[f"occ_m{mode}_inputs"][:, :3].view(np.uint32)), "query cells"


def test_reference_harness_exports_timing_loops():
    """The reference-backend timing loops (bench.py's reference arm) are exported by the harness build."""
    lib = GOLDEN.parents[1] / "oracle" / "_ref" / "libref_stock.so"
    if not lib.exists():
        pytest.skip("reference harness not built (reference checkout absent at build time)")
    from oracle import ref_backend
    ref_backend.load()  # declares every entry point; AttributeError if one is missing
