"""Golden fixtures from the reference backend's own kernels.

Run on a machine with a GPU after `make -C oracle/ref REF=<reference checkout>`:

    python tests/golden/make_ref_goldens.py

It loads oracle/_ref/libref_{stock,parity}.so (the reference's backend-cuda.cu
compiled with the launcher in oracle/ref/ref_harness.cu), runs the
reference's kernels on seeded inputs and writes tests/golden/ref_<variant>.npz.
tests/test_ref_goldens.py compares the CPU oracle with these files.

Cases (all seeded, sizes small enough for the oracle to finish in seconds):
  hash     hash_u32 (both copies) and rand01 on 0..4095, edge values and
           random words                              backend-cuda.cu:321-332, 1439-1446
  step     camera index and occupancy mode of frames 0..299 for 100
           cameras, warmup 32 / interval 1 and warmup 256 / interval 16
                                                     backend-cuda.cu:1479-1488
  sampler  512 training rays of frames 3 and 7 of the 8-view 64x64 smoke
           scene over a 30% random 32^3 bitfield, 128 steps per ray; kept
           rays reordered to ray index (the reference appends them in atomic
           order)                                    backend-cuda.cu:422-533
  loss     k_ray_march_mse_grad on 300 rays of 0..80 samples with sigma
           given as softplus^-1 of known densities    backend-cuda.cu:1095-1182
  adam     k_prepare_adam_step_scalars + k_adam_step_half on 1024 params
           for plain, clipped, guarded and decayed steps
                                                     backend-cuda.cu:1513-1554
  occ      one occupancy update of a 16^3 grid for refresh / warm-up init /
           no-op modes, 1000 queried cells            backend-cuda.cu:1555-1634
"""
import ctypes as C
import os
import pathlib
import sys

import numpy as np
import torch

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import nerf_b200  # noqa: E402

U32, F32, P = C.c_uint32, C.c_float, C.c_void_p
SCENE = dict(kind=0, seed=0, n_views=8, width=64, height=64, fov=0.69, radius=3.0)
AABB = np.array([-1, -1, -1, 1, 1, 1], np.float32)
GRID, RAYS, MAX_STEPS = 32, 512, 128
OCC_GRID, OCC_UPDATE = 16, 1000


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def empty(nbytes):
    return torch.zeros(max(1, int(nbytes)), dtype=torch.uint8, device="cuda")


def load(variant):
    lib = C.CDLL(str(ROOT / "oracle" / "_ref" / f"libref_{variant}.so"))
    lib.ref_struct_sizes.argtypes = [P]
    lib.ref_hash.argtypes = [P, P, P, P, U32]
    lib.ref_begin_step.argtypes = [U32, U32, U32, U32, P, P]
    lib.ref_sample_rays.argtypes = [U32, U32, P, P, P, U32, U32, F32, F32, F32, F32, U32, U32, P, P, U32, P, P, P]
    lib.ref_ray_march_mse_grad.argtypes = [P, P, P, P, P, U32, P, P, P, P]
    lib.ref_adam.argtypes = [P, P, P, P, P, U32, F32, F32, F32, U32, F32, U32, F32, U32, F32, F32, F32, P, P, P]
    lib.ref_occupancy.argtypes = [U32, U32, P, P, P, U32, U32, P, F32, F32, P, P]
    return lib


def check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what}: status {rc}")


def hash_case(lib, rng, out):
    x = np.concatenate([np.arange(4096), [0xFFFFFFFF, 0x80000000, 0x7FFFFFFF, 0xA511E9B3, 0x63D83595],
                        rng.integers(0, 2 ** 32, 4096)]).astype(np.uint32)
    n = len(x)
    xd, hs, hr, r = dev(x), empty(4 * n), empty(4 * n), empty(4 * n)
    check(lib.ref_hash(xd.data_ptr(), hs.data_ptr(), hr.data_ptr(), r.data_ptr(), n), "hash")
    out["hash_in"] = x
    out["hash_sampler"] = hs.cpu().numpy().view(np.uint32)
    out["hash_runtime"] = hr.cpu().numpy().view(np.uint32)
    out["rand01"] = r.cpu().numpy().view(np.float32)


def step_case(lib, state, out):
    rows = []
    for warmup, interval in ((32, 1), (256, 16)):
        for f in range(300):
            o = (U32 * 2)()
            check(lib.ref_begin_step(f, 100, warmup, interval, state.data_ptr(), o), "begin_step")
            rows.append((warmup, interval, f, o[0], o[1]))
    out["step"] = np.array(rows, np.uint32)


def sampler_case(lib, rng, sizes, state, out):
    ds = nerf_b200.make_scene(**SCENE)
    imgs, cams = dev(ds.images), dev(np.ascontiguousarray(ds.cameras, np.float32).reshape(-1))
    bits = np.packbits(rng.random(GRID ** 3) < 0.3, bitorder="little").view(np.uint32)
    bd = dev(bits)
    fx, fy, cx, cy = ds.intrinsics
    out["sampler_images_sum"] = np.array([int(ds.images.astype(np.uint64).sum())], np.uint64)
    out["sampler_bits"] = bits
    ray_size, step_size = sizes[0], sizes[1]
    for frame in (3, 7):
        camera = nerf_b200_camera(frame, ds.n)
        rays_d, steps_d, batch_d = empty(RAYS * ray_size), empty(RAYS * MAX_STEPS * step_size), empty(8)
        check(lib.ref_sample_rays(frame, camera, state.data_ptr(), cams.data_ptr(), imgs.data_ptr(), ds.width, ds.height,
                                  fx, fy, cx, cy, RAYS, MAX_STEPS, AABB.ctypes.data, bd.data_ptr(), GRID,
                                  rays_d.data_ptr(), steps_d.data_ptr(), batch_d.data_ptr()), "sample_rays")
        active, total = batch_d.cpu().numpy().view(np.uint32)[:2]
        rec = rays_d.cpu().numpy()[: active * ray_size].view(np.float32).reshape(active, ray_size // 4)
        stp = steps_d.cpu().numpy()[: total * step_size].view(np.float32).reshape(total, step_size // 4)
        # ray index from the pixel position (px, py) = rand01(seed ^ salt) * (W, H), with the reference's rand01
        seeds = (np.uint32(frame) * np.uint32(1315423911) ^ np.arange(RAYS, dtype=np.uint32) * np.uint32(9781)).astype(np.uint32)
        pix = []
        for salt, extent in ((0xA511E9B3, ds.width), (0x63D83595, ds.height)):
            rin = dev(seeds ^ np.uint32(salt))
            hs, hr, r01 = empty(4 * RAYS), empty(4 * RAYS), empty(4 * RAYS)
            check(lib.ref_hash(rin.data_ptr(), hs.data_ptr(), hr.data_ptr(), r01.data_ptr(), RAYS), "hash")
            pix.append((r01.cpu().numpy().view(np.float32) * np.float32(extent)).astype(np.float32).view(np.uint32))
        lookup = {}
        for i in range(RAYS):
            lookup.setdefault((int(pix[0][i]), int(pix[1][i])), []).append(i)
        index = np.zeros(active, np.uint32)
        for k in range(active):
            key = (int(rec[k, 9:10].view(np.uint32)[0]), int(rec[k, 10:11].view(np.uint32)[0]))
            cands = lookup[key]
            assert len(cands) == 1, "pixel position does not identify the ray"
            index[k] = cands[0]
        order = np.argsort(index)
        u = rec.view(np.uint32)
        begin, count = u[order, 15], u[order, 16]
        samples = np.concatenate([stp[b:b + c, :4] for b, c in zip(begin, count)]) if active else np.zeros((0, 4), np.float32)
        out[f"sampler_f{frame}_index"] = index[order]
        out[f"sampler_f{frame}_count"] = count
        out[f"sampler_f{frame}_ray"] = rec[order, :15]  # origin, dir, t_near, t_far, cone, px, py, gt rgba
        out[f"sampler_f{frame}_samples"] = samples
        out[f"sampler_f{frame}_camera"] = np.array([camera], np.uint32)


def nerf_b200_camera(frame, n):
    x = (frame * 747796405 + 2891336453) & 0xFFFFFFFF
    x ^= x >> 16
    x = (x * 0x7FEB352D) & 0xFFFFFFFF
    x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF
    x ^= x >> 16
    return x % n


def loss_case(lib, rng, sizes, out):
    n_rays = 300
    count = rng.integers(0, 81, n_rays).astype(np.uint32)
    count[:4] = [0, 1, 2, 80]
    begin = np.concatenate([[0], np.cumsum(count)[:-1]]).astype(np.uint32)
    S = int(count.sum())
    sigma = np.exp(rng.normal(0.5, 1.5, S)).clip(1e-3, 60.0).astype(np.float32)
    raw_sigma_ref = np.log(np.expm1(sigma.astype(np.float64))).astype(np.float32)
    raw_rgb = rng.normal(0.0, 1.5, (S, 3)).astype(np.float32)
    dt = rng.uniform(1e-3, 6e-2, S).astype(np.float32)
    gt = rng.random((n_rays, 4)).astype(np.float32)
    ray_size, step_size = sizes[0], sizes[1]
    rec = np.zeros((n_rays, ray_size // 4), np.float32)
    rec[:, 11:15] = gt
    rec.view(np.uint32)[:, 15] = begin
    rec.view(np.uint32)[:, 16] = count
    stp = np.zeros((max(S, 1), step_size // 4), np.float32)
    stp[:S, 3] = dt
    batch = np.array([n_rays, S], np.uint32)
    d_rgb, d_sig, trans, loss = empty(12 * S), empty(4 * S), empty(4 * S), empty(4)
    ins = [dev(raw_rgb), dev(raw_sigma_ref), dev(stp), dev(rec), dev(batch)]
    check(lib.ref_ray_march_mse_grad(ins[0].data_ptr(), ins[1].data_ptr(), ins[2].data_ptr(), ins[3].data_ptr(),
                                     ins[4].data_ptr(), n_rays, d_rgb.data_ptr(), d_sig.data_ptr(), trans.data_ptr(),
                                     loss.data_ptr()), "ray_march")
    out.update(loss_count=count, loss_begin=begin, loss_sigma=sigma, loss_raw_sigma_ref=raw_sigma_ref, loss_raw_rgb=raw_rgb,
               loss_dt=dt, loss_gt=gt, loss_sum=loss.cpu().numpy().view(np.float32),
               loss_d_rgb=d_rgb.cpu().numpy()[: 12 * S].view(np.float32).reshape(S, 3),
               loss_d_sigma_ref=d_sig.cpu().numpy()[: 4 * S].view(np.float32),
               loss_trans=trans.cpu().numpy()[: 4 * S].view(np.float32))


def adam_case(lib, rng, state, out):
    n = 1024
    scal = empty(64)
    cases = [  # step, grad_norm, nonfinite, lr, decay_ksteps, clip, guard
        (1, 0.5, 0, 1e-2, 0, 1.0, 100.0),
        (10, 5.0, 0, 1e-2, 0, 1.0, 100.0),
        (11, 500.0, 0, 1e-2, 0, 1.0, 100.0),
        (2500, 0.3, 0, 5e-3, 1, 1.0, 100.0),
        (3, 0.3, 1, 1e-2, 0, 1.0, 100.0),
    ]
    rows, results = [], []
    for i, (step, gn, nf, lr, dk, clip, guard) in enumerate(cases):
        p32 = rng.normal(0, 0.1, n).astype(np.float32)
        g16 = (rng.normal(0, 1, n) * 64).astype(np.float16)
        m = rng.normal(0, 0.01, n).astype(np.float32)
        v = rng.random(n).astype(np.float32) * 1e-3
        d = [dev(p32), dev(np.zeros(n, np.float16).view(np.uint16)), dev(g16.view(np.uint16)), dev(m), dev(v)]
        so = (F32 * 6)()
        check(lib.ref_adam(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), d[4].data_ptr(), n, 0.9,
                           0.999, 1e-8, step, gn, nf, lr, dk, clip, guard, 128.0, state.data_ptr(), scal.data_ptr(), so),
              "adam")
        rows.append((step, gn, nf, lr, dk, clip, guard))
        out[f"adam{i}_in"] = np.stack([p32, g16.astype(np.float32), m, v])
        out[f"adam{i}_out"] = np.stack([d[0].cpu().numpy(), d[1].cpu().numpy().view(np.float16).astype(np.float32),
                                        d[3].cpu().numpy(), d[4].cpu().numpy()])
        results.append(list(so))
    out["adam_cases"] = np.array(rows, np.float64)
    out["adam_scalars"] = np.array(results, np.float32)


def occ_case(lib, rng, state, out):
    cells, update = OCC_GRID ** 3, OCC_UPDATE
    for mode, frame in ((2, 37), (1, 0), (0, 5)):
        density = rng.uniform(0.0, 0.05, cells).astype(np.float32)
        density[np.abs(density * np.float32(0.97) - np.float32(0.01)) < 1e-4] = 0.03  # keep clear of the threshold
        bits = rng.integers(0, 2 ** 32, (cells + 31) // 32, dtype=np.uint64).astype(np.uint32)
        sigma = rng.uniform(0.0, 0.05, update).astype(np.float32)
        sigma[np.abs(sigma - np.float32(0.01)) < 1e-4] = 0.02
        raw = np.log(np.expm1(sigma.astype(np.float64))).astype(np.float32)
        d = [dev(density), dev(bits), dev(raw), torch.zeros(update * 7, dtype=torch.float32, device="cuda")]
        check(lib.ref_occupancy(frame, mode, state.data_ptr(), d[0].data_ptr(), d[1].data_ptr(), OCC_GRID, update,
                                AABB.ctypes.data, 0.97, 0.01, d[2].data_ptr(), d[3].data_ptr()), "occupancy")
        out[f"occ_m{mode}_frame"] = np.array([frame], np.uint32)
        out[f"occ_m{mode}_density_in"] = density
        out[f"occ_m{mode}_bits_in"] = bits
        out[f"occ_m{mode}_sigma"] = sigma
        out[f"occ_m{mode}_density_out"] = d[0].cpu().numpy()
        out[f"occ_m{mode}_bits_out"] = d[1].cpu().numpy()
        out[f"occ_m{mode}_inputs"] = d[3].cpu().numpy().reshape(update, 7)


def main():
    torch.cuda.set_device(0)
    for variant in ("stock", "parity"):
        lib = load(variant)
        sizes = (U32 * 5)()
        lib.ref_struct_sizes(sizes)
        sizes = list(sizes)
        assert sizes[:2] == [68, 28], sizes
        state = empty(sizes[3])
        rng = np.random.default_rng(2024)
        out = {"struct_sizes": np.array(sizes, np.uint32)}
        hash_case(lib, rng, out)
        step_case(lib, state, out)
        sampler_case(lib, rng, sizes, state, out)
        loss_case(lib, rng, sizes, out)
        adam_case(lib, rng, state, out)
        occ_case(lib, rng, state, out)
        path = ROOT / "tests" / "golden" / f"ref_{variant}.npz"
        np.savez_compressed(path, **out)
        print(variant, path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
