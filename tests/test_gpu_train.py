"""End-to-end parity of the nerf.h ABI on the GPU against the CPU oracle.

Integer outputs are compared bit for bit: per-ray sample counts, the ordered
compaction (kept ray indices, sample offsets), sample positions and steps,
the occupancy bitfield given the density grid.  Floating-point outputs use
the tolerances written at each assert.
"""
import os
import tempfile

import numpy as np
import pytest

import nerf_b200
from nerf_b200 import abi
from oracle import oracle

pytestmark = pytest.mark.gpu

RAYS, STEPS, RES = 512, 96, 32


def make_pair(stop=0.0, background=0, warmup=4, interval=2, log2T=15, n_views=8, size=48, rays=RAYS, steps=STEPS,
              res=RES, cells=None, target=0, max_samples=0, cascades=1):
    ds = nerf_b200.make_scene(kind=0, seed=0, n_views=n_views, width=size, height=size, fov=0.69, radius=3.0)
    opts = nerf_b200.default_options(log2_hashmap_size=log2T, max_resolution=512, stop_transmittance=stop,
                                     background=background, target_samples_per_step=target,
                                     max_samples_per_step=max_samples, n_cascades=cascades)
    ctx = nerf_b200.Context(ds, grid_res=res, max_sample_steps=max(rays * steps, max_samples), max_batch_rays=4 * rays,
                            options=opts)
    cfg = nerf_b200.training_config(rays=rays, steps=steps, warmup=warmup, update_interval=interval,
                                    cells_per_update=cells or res ** 3 // 2)
    ctx.configure(cfg)
    oc = oracle.Context(ctx.desc, oracle.options(log2_hashmap_size=log2T, max_resolution=512, stop_transmittance=stop,
                                                 background=background, target_samples_per_step=target,
                                                 max_samples_per_step=max_samples, n_threads=8, n_cascades=cascades),
                        ctx._images, ctx._cams)
    oc.configure(cfg)
    return ds, ctx, oc, cfg


def sync_oracle(ctx, oc):
    master = ctx.params()[0]
    oc.set_params(master)
    d, b = ctx.occupancy()
    oc.set_occupancy(d, b)
    oc.set_frame(ctx.counters().frame_index)


def compare_batch(ctx, oc):
    g, o = ctx.batch(), oc.batch()
    assert np.array_equal(g["counts"], o["counts"]), "per-ray sample counts"
    assert np.array_equal(g["index"], o["index"]), "kept rays"
    assert np.array_equal(g["begin"], o["begin"]), "compaction offsets"
    assert np.array_equal(g["count"], o["count"])
    assert np.array_equal(g["pos_dt"].view(np.uint32), o["pos_dt"].view(np.uint32)), "sample positions / steps"
    assert np.array_equal(g["dir"].view(np.uint32), o["dir"].view(np.uint32))
    assert np.allclose(g["gt"], o["gt"], atol=1e-6)
    assert np.array_equal(g["bg"], o["bg"])
    # the sample stream is laid out ray after ray
    assert np.array_equal(g["sample_ray"], np.repeat(np.arange(len(g["count"]), dtype=np.uint32), g["count"]))
    return g


def test_initial_parameters_equal_oracle(cuda):
    _, ctx, oc, _ = make_pair()
    master, p16, m, v = ctx.params()
    om, op, _, _, _ = oc.params()
    assert np.array_equal(master, om) and np.array_equal(p16, op)
    assert not m.any() and not v.any()
    ctx.close()


@pytest.mark.parametrize("stop,background,mlp_tc", [(0.0, 0, "0"), (1e-4, 1, "0"), (0.0, 0, "1"), (1e-4, 1, "1")])
def test_first_step_matches_oracle(cuda, monkeypatch, stop, background, mlp_tc):
    """mlp_tc "1": the training step's MLPs on tcgen05 (encode kernel + tensor-core MLP kernels)."""
    monkeypatch.setenv("NERF_B200_MLP_TC", mlp_tc)
    _, ctx, oc, cfg = make_pair(stop=stop, background=background)
    ctx.train_step()
    oc.step()
    g = compare_batch(ctx, oc)
    assert len(g["count"]) > 100 and g["count"].max() > 20
    s, os_ = ctx.stats(), oc.stats()
    assert s.completed_steps == os_.completed_steps == 1
    assert s.last_train_camera == os_.last_train_camera
    assert s.has_nonfinite == 0
    assert abs(s.loss - os_.loss) <= 1e-4 * abs(os_.loss), (s.loss, os_.loss)
    assert abs(s.grad_norm - os_.grad_norm) <= 2e-2 * os_.grad_norm, (s.grad_norm, os_.grad_norm)
    _, _, m, v = ctx.params()
    _, _, om, ov, _ = oc.params()
    n_grid = ctx.n_grid
    # first Adam moment = (1 - beta1) * clipped gradient: compare gradients through it
    mlp_err = np.linalg.norm(m[n_grid:] - om[n_grid:]) / np.linalg.norm(om[n_grid:])
    grid_err = np.linalg.norm(m[:n_grid] - om[:n_grid]) / np.linalg.norm(om[:n_grid])
    assert mlp_err < 2e-2, mlp_err
    assert grid_err < 3e-2, grid_err
    ctx.close()


@pytest.mark.parametrize("mlp_tc", ["0", "1"])
def test_warmup_steps_sampler_bit_exact(cuda, monkeypatch, mlp_tc):
    monkeypatch.setenv("NERF_B200_MLP_TC", mlp_tc)
    _, ctx, oc, _ = make_pair(warmup=6, interval=2)
    losses = []
    for step in range(5):
        sync_oracle(ctx, oc)
        ctx.train_step()
        oc.step()
        compare_batch(ctx, oc)
        losses.append(ctx.stats().loss)
        assert ctx.counters().frame_index == step + 1
    assert losses[-1] < losses[0]  # training makes progress
    ctx.close()


def test_occupancy_refresh_and_later_sampler(cuda):
    _, ctx, oc, _ = make_pair(warmup=3, interval=2, cells=RES ** 3 // 3)
    for _ in range(3):
        ctx.train_step()
    for step in range(4):  # frames 3..6: refresh on 4 and 6
        sync_oracle(ctx, oc)
        ctx.train_step()
        oc.step()
        gd, gb = ctx.occupancy()
        od, ob = oc.occupancy()
        # density grid: same rule, densities from fp16-operand MLPs -> relative tolerance
        assert np.allclose(gd, od, rtol=2e-2, atol=1e-4)
        # bitfield bit-exact except cells whose density sits at the threshold
        mismatch = np.unpackbits((gb ^ ob).view(np.uint8), bitorder="little")[: RES ** 3]
        near = np.abs(od - 0.01) < 2e-2 * 0.01 + 1e-4
        assert not (mismatch.astype(bool) & ~near).any()
    ctx.close()


def test_sampler_bit_exact_with_given_bitfield(cuda):
    """A sparse random bitfield exercises skipping, ragged counts and empty rays."""
    _, ctx, oc, _ = make_pair(warmup=1, interval=1000)
    rng = np.random.default_rng(21)
    words = (RES ** 3 + 31) // 32
    bits = (rng.integers(0, 2 ** 32, words, dtype=np.uint64) & rng.integers(0, 2 ** 32, words, dtype=np.uint64)).astype(np.uint32)
    ctx.set_occupancy(bitfield=bits)
    ctx.set_frame(5)
    oc.set_occupancy(bits=bits)
    oc.set_frame(5)
    oc.set_params(ctx.params()[0])
    ctx.train_step()
    oc.step()
    g = compare_batch(ctx, oc)
    assert (g["counts"] == 0).any()
    ctx.close()


def test_cascades_sampler_bit_exact_with_given_bitfield(cuda):
    """Three occupancy cascades (the configured box [-1,1]^3 scaled by 1, 2, 4; cameras at radius 3 start inside the
    outermost): per-ray counts, compaction and sample positions bit-exact against the oracle over a sparse random
    bitfield of all three cascades, with samples in every cascade."""
    _, ctx, oc, _ = make_pair(warmup=1, interval=1000, cascades=3)
    rng = np.random.default_rng(22)
    words = (3 * RES ** 3 + 31) // 32
    bits = (rng.integers(0, 2 ** 32, words, dtype=np.uint64) & rng.integers(0, 2 ** 32, words, dtype=np.uint64)).astype(np.uint32)
    ctx.set_occupancy(bitfield=bits)
    ctx.set_frame(5)
    oc.set_occupancy(bits=bits)
    oc.set_frame(5)
    oc.set_params(ctx.params()[0])
    ctx.train_step()
    oc.step()
    g = compare_batch(ctx, oc)
    m = np.abs(g["pos_dt"][:, :3]).max(axis=1)
    assert (m <= 1).any() and ((m > 1) & (m <= 2)).any() and (m > 2).any()
    ctx.close()


def test_cascades_occupancy_refresh(cuda):
    """Occupancy refreshes over three cascades (cell centres cascade after cascade): densities as in the single-grid
    test, bitfield bit-exact except at the threshold, and the next steps' samples bit-exact."""
    _, ctx, oc, _ = make_pair(warmup=2, interval=2, cascades=3, cells=3 * RES ** 3 // 2)
    for _ in range(2):
        ctx.train_step()
    for step in range(3):  # frames 2..4: refresh on 2 and 4
        sync_oracle(ctx, oc)
        ctx.train_step()
        oc.step()
        compare_batch(ctx, oc)
        gd, gb = ctx.occupancy()
        od, ob = oc.occupancy()
        assert gd.shape == (3 * RES ** 3,)
        assert np.allclose(gd, od, rtol=2e-2, atol=1e-4)
        mismatch = np.unpackbits((gb ^ ob).view(np.uint8), bitorder="little")[: 3 * RES ** 3]
        near = np.abs(od - 0.01) < 2e-2 * 0.01 + 1e-4
        assert not (mismatch.astype(bool) & ~near).any()
    ctx.close()


def test_cascades_render_matches_oracle(cuda):
    ds, ctx, oc, _ = make_pair(warmup=2, interval=1, cascades=2)
    for _ in range(5):
        ctx.train_step()
    sync_oracle(ctx, oc)
    W = H = 32
    fx, fy, cx, cy = ds.intrinsics
    s = W / ds.width
    intr = (fx * s, fy * s, (W - 1) / 2, (H - 1) / 2)
    img = np.zeros((H, W, 4), np.uint8)
    ctx.render(ds.cameras[2], W, H, intr, max_steps=STEPS, stop=1e-4, dst=img)
    rgba, _ = oc.render(ds.cameras[2], W, H, intr, STEPS, 1e-4)
    diff = np.abs(img.astype(int) - rgba.view(np.uint8).reshape(H, W, 4).astype(int))
    assert diff.max() <= 2 and diff.mean() < 0.1
    ctx.close()


def test_capacity_cut_and_adaptive_rays(cuda):
    cap = 6000
    _, ctx, oc, _ = make_pair(max_samples=cap, target=cap // 2, warmup=50)
    for _ in range(3):
        sync_oracle(ctx, oc)
        ctx.train_step()
        oc.step()
        g = compare_batch(ctx, oc)
        c = ctx.counters()
        assert c.samples <= cap and c.samples == int(g["count"].sum())
        assert c.rays == oc.info().rays
    c = ctx.counters()
    assert c.next_rays != RAYS  # the ray count adapts toward the sample target
    ctx.close()


def test_render_matches_oracle(cuda):
    ds, ctx, oc, _ = make_pair(warmup=2, interval=1)
    for _ in range(6):
        ctx.train_step()
    sync_oracle(ctx, oc)
    W = H = 40
    cam = ds.cameras[1]
    out = np.zeros((H, W, 4), np.uint8)
    info = ctx.render(cam, W, H, ds.intrinsics, max_steps=128, stop=1e-4, dst=out)
    rgba, spp = oc.render(cam, W, H, ds.intrinsics, 128, 1e-4)
    want = rgba.view(np.uint8).reshape(H, W, 4)
    diff = np.abs(out.astype(int) - want.astype(int))
    assert diff.max() <= 2 and diff.mean() < 0.1, (diff.max(), diff.mean())
    assert (out[..., 3] == 255).all()
    assert info.rays == W * H
    assert abs(int(info.samples) - int(spp.sum())) <= 0.001 * spp.sum() + 8
    # tiles: union over ranks equals the full render
    full = np.zeros_like(out)
    for r in range(3):
        part = np.zeros_like(out)
        ctx.render(cam, W, H, ds.intrinsics, max_steps=128, stop=1e-4, tile=16, rank=r, world=3, dst=part)
        mask = np.zeros((H, W), bool)
        for t in range(r, 9, 3):
            ty, tx = divmod(t, 3)
            mask[ty * 16:(ty + 1) * 16, tx * 16:(tx + 1) * 16] = True
        full[mask] = part[mask]
    assert np.array_equal(full, out)
    ctx.close()


def _psnr(img_rgba8, gt_rgba8):
    gt = gt_rgba8.astype(np.float64) / 255.0
    ref = gt[..., :3] * gt[..., 3:4] + (1.0 - gt[..., 3:4])
    mse = np.mean((img_rgba8[..., :3].astype(np.float64) / 255.0 - ref) ** 2)
    return 10.0 * np.log10(1.0 / mse)


def test_heldout_psnr_matches_oracle(cuda):
    """Train the GPU context and the oracle independently from the same
    initialisation for 60 steps, render held-out views with each, and compare
    PSNR against the exact renders: within 0.1 dB."""
    ds, ctx, oc, _ = make_pair(warmup=4, interval=4, n_views=8, size=48)
    for _ in range(60):
        ctx.train_step()
        oc.step()
    held = nerf_b200.make_scene(kind=0, seed=0, n_views=4, width=48, height=48, fov=0.69, radius=3.0, view_offset=8)
    g_psnr, o_psnr = [], []
    out = np.zeros((48, 48, 4), np.uint8)
    for v in range(4):
        ctx.render(held.cameras[v], 48, 48, held.intrinsics, max_steps=STEPS, stop=1e-4, dst=out)
        rgba, _ = oc.render(held.cameras[v], 48, 48, held.intrinsics, STEPS, 1e-4)
        g_psnr.append(_psnr(out, held.images[v]))
        o_psnr.append(_psnr(rgba.view(np.uint8).reshape(48, 48, 4), held.images[v]))
    g, o = float(np.mean(g_psnr)), float(np.mean(o_psnr))
    assert g > 12.0, g  # it learned something
    assert abs(g - o) < 0.1, (g, o)
    ctx.close()


def test_inference_abi(cuda):
    ds, ctx, oc, _ = make_pair(warmup=2, interval=1)
    for _ in range(3):
        ctx.train_step()
    img = ctx.inference(camera_idx=2, samples_per_ray=64)
    assert img.shape == (ds.height, ds.width, 4) and (img[..., 3] == 255).all()
    sync_oracle(ctx, oc)
    rgba, _ = oc.render(ds.cameras[2], ds.width, ds.height, ds.intrinsics, 64, nerf_b200.default_options().render_stop_transmittance)
    assert np.abs(img.astype(int) - rgba.view(np.uint8).reshape(img.shape).astype(int)).max() <= 2
    ctx.close()


def test_checkpoint_roundtrip_and_reset(cuda):
    _, ctx, _, _ = make_pair()
    for _ in range(2):
        ctx.train_step()
    master = ctx.params()[0]
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "w.nerf")
        ctx.save(path)
        ctx.set_params(np.zeros_like(master))
        ctx.load(path)
        m2, p16, am, av = ctx.params()
        assert np.array_equal(m2, master)
        assert np.array_equal(p16, master.astype(np.float16).view(np.uint16))
        assert not am.any() and not av.any()  # load resets the optimiser (reference behaviour)
        assert ctx.counters().frame_index == 0
        with pytest.raises(abi.NerfError) as e:
            ctx.load(os.path.join(td, "missing.nerf"))
        assert e.value.status == abi.NERF_STATUS_IO_ERROR
        with open(path, "r+b") as f:
            f.write(b"\xff" * 8)
        with pytest.raises(abi.NerfError) as e:
            ctx.load(path)
        assert e.value.status == abi.NERF_STATUS_IO_ERROR
    ctx.close()


def _snapshot(ctx):
    master, p16, m, v = ctx.params()
    d, b = ctx.occupancy()
    c = ctx.counters()
    return master, p16, m, v, d, b, (c.frame_index, c.next_rays, c.total_samples, c.total_rays, c.samples)


def test_training_state_resume(cuda):
    """Exact resume: a fresh context that loads the training state holds the saved masters, fp16 mirror, Adam moments,
    occupancy and step state bit for bit, and its next steps sample exactly the rays of the uninterrupted run (the
    sampler, the occupancy refresh and the step counters are deterministic); parameters after the resumed steps agree
    within the run-to-run spread of the fp16 gradient reductions."""
    # refresh at frames 4 and 8: the saved state holds a refreshed grid, and the three resumed steps (frames 5-7)
    # sample from it alone
    _, ctx, _, _ = make_pair(warmup=2, interval=4, target=3000, max_samples=8192)
    for _ in range(5):
        ctx.train_step()
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "state.nerf")
        ctx.save_state(path)
        saved = _snapshot(ctx)
        batches = []
        for _ in range(3):
            ctx.train_step()
            batches.append(ctx.batch())
        after = ctx.params()[0]
        _, ctx2, _, _ = make_pair(warmup=2, interval=4, target=3000, max_samples=8192)
        ctx2.load_state(path)
        restored = _snapshot(ctx2)
        for a, b in zip(saved[:6], restored[:6]):
            assert np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8))
        assert saved[6] == restored[6]
        for want in batches:
            ctx2.train_step()
            got = ctx2.batch()
            for k in ("counts", "index", "begin", "count"):
                assert np.array_equal(got[k], want[k]), k
            assert np.array_equal(got["pos_dt"].view(np.uint32), want["pos_dt"].view(np.uint32))
        after2 = ctx2.params()[0]
        assert np.linalg.norm(after2 - after) <= 1e-3 * np.linalg.norm(after)
        # a state for another hash-grid size is refused; so are missing and unconfigured cases
        ds = nerf_b200.make_scene(kind=0, seed=0, n_views=2, width=16, height=16)
        other = nerf_b200.Context(ds, grid_res=RES, max_sample_steps=RAYS * STEPS, max_batch_rays=4 * RAYS,
                                  options=nerf_b200.default_options(log2_hashmap_size=14, max_resolution=512))
        with pytest.raises(abi.NerfError) as e:
            other.load_state(path)
        assert e.value.status == abi.NERF_STATUS_STATE_ERROR
        other.configure(nerf_b200.training_config(rays=RAYS, steps=STEPS))
        with pytest.raises(abi.NerfError) as e:
            other.load_state(path)
        assert e.value.status == abi.NERF_STATUS_IO_ERROR
        with pytest.raises(abi.NerfError) as e:
            ctx2.load_state(os.path.join(td, "missing.nerf"))
        assert e.value.status == abi.NERF_STATUS_IO_ERROR
        other.close()
        ctx2.close()
    ctx.close()


def test_error_codes(cuda):
    ds = nerf_b200.make_scene(n_views=4, width=16, height=16)
    ctx = nerf_b200.Context(ds, grid_res=16, max_sample_steps=1 << 16, max_batch_rays=256)
    with pytest.raises(abi.NerfError) as e:
        ctx.train_step()
    assert e.value.status == abi.NERF_STATUS_STATE_ERROR
    with pytest.raises(abi.NerfError) as e:
        ctx.stats()
    assert e.value.status == abi.NERF_STATUS_STATE_ERROR
    for bad in [dict(rays=0), dict(steps=0), dict(steps=5000), dict(rays=512), dict(rays=256, steps=512),
                dict(update_interval=0)]:
        with pytest.raises(abi.NerfError) as e:
            ctx.configure(nerf_b200.training_config(**{**dict(rays=128, steps=64), **bad}))
        assert e.value.status == abi.NERF_STATUS_INVALID_USAGE, bad
    ctx.configure(nerf_b200.training_config(rays=128, steps=64))
    with pytest.raises(abi.NerfError) as e:
        ctx.inference(camera_idx=4)
    assert e.value.status == abi.NERF_STATUS_INVALID_USAGE
    ctx.train_step()
    assert ctx.stats().completed_steps == 1
    ctx.close()
