"""GPU parity of the individual kernels against the CPU oracle, through the C-ABI.

Bit-exact: hash-grid corner indices/weights and forward features, Adam, the
occupancy update.  Floating point with stated tolerances: fused field
forward (1e-2 abs on raw outputs, the contract for per-sample RGB/sigma at
fp16), field backward and hash scatter (relative L2), compositing.
"""
import ctypes as C

import numpy as np
import pytest

import nerf_b200
from nerf_b200 import abi
from nerf_b200.abi import check
from oracle import oracle
from gpu_util import dev, host, zeros

pytestmark = pytest.mark.gpu


def _unit_dirs(rng, n):
    d = rng.standard_normal((n, 3)).astype(np.float32)
    return (d / np.linalg.norm(d, axis=1, keepdims=True)).astype(np.float32)


def _edge_points(pos):
    pos[:8] = [[0, 0, 0], [1, 1, 1], [0.5, 0.5, 0.5], [1, 0, 1], [0.999999, 1e-7, 0.25],
               [1 / 3, 2 / 3, 1], [0.0625, 0.125, 0.9375], [1e-30, 1 - 1e-7, 0.5]]
    return pos


def _mlp_params(rng):
    sizes = [(64, 32), (16, 64), (64, 32), (64, 64), (16, 64)]
    out = []
    for o, i in sizes:
        s = np.sqrt(6.0 / (i + o))
        out.append(rng.uniform(-s, s, o * i))
    return np.concatenate(out).astype(np.float32)


@pytest.mark.parametrize("L,log2T,maxres", [(16, 14, 512), (16, 19, 2048), (16, 22, 8192), (8, 15, 256), (16, 24, 4096)])
def test_grid_forward_bit_exact(cuda, L, log2T, maxres):
    torch = cuda
    lib = abi.load()
    g = nerf_b200.grid_layout(L, log2T, 16, maxres)
    og = oracle.grid_layout(L, log2T, 16, maxres)
    rng = np.random.default_rng(7)
    n = 5000
    params = rng.uniform(-1, 1, 2 * g.offset[L]).astype(np.float16).view(np.uint16)
    pos = _edge_points(rng.random((n, 3)).astype(np.float32))
    pos_d, par_d, feat_d = dev(torch, pos), dev(torch, params), zeros(torch, (n, 2 * L), np.uint16)
    check("grid_forward", lib.nerf_b200_grid_forward(C.byref(g), pos_d.data_ptr(), n, par_d.data_ptr(), feat_d.data_ptr(), None))
    torch.cuda.synchronize()
    assert np.array_equal(host(feat_d, np.uint16), oracle.grid_forward(og, params, pos))


def test_grid_forward_empty_input(cuda):
    lib = abi.load()
    g = nerf_b200.grid_layout(16, 14, 16, 512)
    check("grid_forward", lib.nerf_b200_grid_forward(C.byref(g), None, 0, None, None, None))
    assert lib.nerf_b200_grid_forward(C.byref(g), None, 5, None, None, None) == abi.NERF_STATUS_INVALID_USAGE


@pytest.mark.parametrize("log2T", [14, 19])
def test_grid_backward_matches_oracle(cuda, log2T):
    torch = cuda
    lib = abi.load()
    L = 16
    g = nerf_b200.grid_layout(L, log2T, 16, 2048)
    og = oracle.grid_layout(L, log2T, 16, 2048)
    rng = np.random.default_rng(11)
    n = 2000
    pos = _edge_points(rng.random((n, 3)).astype(np.float32))
    dfeat = rng.standard_normal((n, 2 * L)).astype(np.float16)
    grad_d = zeros(torch, 2 * g.offset[L], np.uint16)
    pos_d, dfeat_d = dev(torch, pos), dev(torch, dfeat.view(np.uint16))  # keep the buffers alive across the launch
    check("grid_backward", lib.nerf_b200_grid_backward(C.byref(g), pos_d.data_ptr(), n, dfeat_d.data_ptr(),
                                                       grad_d.data_ptr(), None))
    torch.cuda.synchronize()
    got = host(grad_d, np.uint16).view(np.float16).astype(np.float64)
    want = oracle.grid_backward(og, pos, dfeat.astype(np.float32))
    # fp16 reductions round at every add: |err| stays within a few fp16 ulps of the largest sums
    assert np.abs(got - want).max() < 2e-2
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 5e-3
    assert np.array_equal(got != 0, want != 0) or np.mean((got != 0) != (want != 0)) < 1e-4


def _field_setup(rng, L=16, log2T=15, maxres=512, n=3000, grid_scale=0.5):
    g = nerf_b200.grid_layout(L, log2T, 16, maxres)
    og = oracle.grid_layout(L, log2T, 16, maxres)
    grid = rng.uniform(-grid_scale, grid_scale, 2 * g.offset[L]).astype(np.float32)
    params = np.concatenate([grid, _mlp_params(rng)]).astype(np.float16).view(np.uint16)
    pos = _edge_points(rng.random((n, 3)).astype(np.float32))
    dirs = _unit_dirs(rng, n)
    return g, og, params, pos, dirs


@pytest.mark.parametrize("n", [1, 63, 64, 3000])
def test_field_forward_matches_oracle(cuda, n):
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(3)
    g, og, params, pos, dirs = _field_setup(rng, n=max(n, 8))
    pos, dirs = pos[:n], dirs[:n]
    feat_d, raw_d = zeros(torch, (n, 32), np.uint16), zeros(torch, (n, 4), np.float32)
    par_d, pos_d, dir_d = dev(torch, params), dev(torch, pos), dev(torch, dirs)
    check("field_forward", lib.nerf_b200_field_forward(C.byref(g), par_d.data_ptr(), pos_d.data_ptr(), dir_d.data_ptr(), n,
                                                       feat_d.data_ptr(), raw_d.data_ptr(), None))
    torch.cuda.synchronize()
    feat = host(feat_d, np.uint16)
    assert np.array_equal(feat, oracle.grid_forward(og, params[: 2 * g.offset[16]], pos))
    want = oracle.mlp_forward(params[2 * g.offset[16]:], feat, dirs)
    got = host(raw_d)
    err = np.abs(got - want)
    assert err.max() < 1e-2, err.max()          # per-sample RGB/sigma contract at fp16
    assert np.median(err) < 1e-3


def test_field_backward_matches_oracle(cuda):
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(5)
    n = 3000
    g, og, params, pos, dirs = _field_setup(rng, n=n)
    n_grid = 2 * g.offset[16]
    feat = oracle.grid_forward(og, params[:n_grid], pos)
    dout = (rng.standard_normal((n, 4)) * 0.5).astype(np.float32)
    gg_d = zeros(torch, n_grid, np.uint16)
    part_d = zeros(torch, int(lib.nerf_b200_field_backward_partial_floats()), np.float32)
    mg_d = zeros(torch, 10240, np.float32)
    ins = [dev(torch, x) for x in (params, pos, dirs, feat, dout)]
    check("field_backward", lib.nerf_b200_field_backward(
        C.byref(g), ins[0].data_ptr(), ins[1].data_ptr(), ins[2].data_ptr(), n, ins[3].data_ptr(), ins[4].data_ptr(),
        gg_d.data_ptr(), part_d.data_ptr(), mg_d.data_ptr(), None))
    torch.cuda.synchronize()
    dfeat, wg = oracle.mlp_backward(params[n_grid:], feat, dirs, dout)
    got_w = host(mg_d).astype(np.float64)
    assert np.linalg.norm(got_w - wg) / np.linalg.norm(wg) < 1e-2
    for name, (a, b) in {"d0": (0, 2048), "d1": (2048, 3072), "c0": (3072, 5120), "c1": (5120, 9216), "c2": (9216, 9408)}.items():
        assert np.linalg.norm(got_w[a:b] - wg[a:b]) / (np.linalg.norm(wg[a:b]) + 1e-30) < 2e-2, name
    assert np.all(got_w[9408:] == 0)  # colour output rows 3..15 receive no gradient
    want_g = oracle.grid_backward(og, pos, dfeat)
    got_g = host(gg_d, np.uint16).view(np.float16).astype(np.float64)
    assert np.linalg.norm(got_g - want_g) / np.linalg.norm(want_g) < 2e-2


def test_mlp_only_matches_fused_field(cuda):
    """The MLP-only entry points on the hash features of the fused field give the fused field's raw outputs and
    weight gradients bit for bit (same tiles, same fragments, same fixed-order reduction), and feature gradients
    that scattered by the standalone grid backward match the fused scatter within fp16 reduction order."""
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(9)
    n = 3001
    g, og, params, pos, dirs = _field_setup(rng, n=n)
    n_grid = 2 * g.offset[16]
    par_d, pos_d, dir_d = dev(torch, params), dev(torch, pos), dev(torch, dirs)
    mlp_ptr = par_d.data_ptr() + 2 * n_grid
    feat_d, raw_d, raw2_d = zeros(torch, (n, 32), np.uint16), zeros(torch, (n, 4), np.float32), zeros(torch, (n, 4), np.float32)
    check("field_forward", lib.nerf_b200_field_forward(C.byref(g), par_d.data_ptr(), pos_d.data_ptr(), dir_d.data_ptr(), n,
                                                       feat_d.data_ptr(), raw_d.data_ptr(), None))
    check("mlp_forward", lib.nerf_b200_mlp_forward(mlp_ptr, feat_d.data_ptr(), dir_d.data_ptr(), n, raw2_d.data_ptr(), None))
    torch.cuda.synchronize()
    assert np.array_equal(host(raw_d).view(np.uint32), host(raw2_d).view(np.uint32))

    dout_d = dev(torch, (rng.standard_normal((n, 4)) * 0.5).astype(np.float32))
    parts = int(lib.nerf_b200_field_backward_partial_floats())
    gg_d, part_d, mg_d = zeros(torch, n_grid, np.uint16), zeros(torch, parts, np.float32), zeros(torch, 10240, np.float32)
    check("field_backward", lib.nerf_b200_field_backward(
        C.byref(g), par_d.data_ptr(), pos_d.data_ptr(), dir_d.data_ptr(), n, feat_d.data_ptr(), dout_d.data_ptr(),
        gg_d.data_ptr(), part_d.data_ptr(), mg_d.data_ptr(), None))
    dfeat_d, part2_d, mg2_d = zeros(torch, (n, 32), np.uint16), zeros(torch, parts, np.float32), zeros(torch, 10240, np.float32)
    check("mlp_backward", lib.nerf_b200_mlp_backward(mlp_ptr, feat_d.data_ptr(), dir_d.data_ptr(), n, dout_d.data_ptr(),
                                                     dfeat_d.data_ptr(), part2_d.data_ptr(), mg2_d.data_ptr(), None))
    gg2_d = zeros(torch, n_grid, np.uint16)
    check("grid_backward", lib.nerf_b200_grid_backward(C.byref(g), pos_d.data_ptr(), n, dfeat_d.data_ptr(), gg2_d.data_ptr(),
                                                       None))
    torch.cuda.synchronize()
    assert np.array_equal(host(mg_d).view(np.uint32), host(mg2_d).view(np.uint32))
    a = host(gg_d, np.uint16).view(np.float16).astype(np.float64)
    b = host(gg2_d, np.uint16).view(np.float16).astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(a) < 5e-3
    # invalid use: missing feature-gradient output
    assert lib.nerf_b200_mlp_backward(mlp_ptr, feat_d.data_ptr(), dir_d.data_ptr(), n, dout_d.data_ptr(), None,
                                      part2_d.data_ptr(), mg2_d.data_ptr(), None) == abi.NERF_STATUS_INVALID_USAGE


@pytest.mark.parametrize("n", [1, 127, 128, 3001])
def test_mlp_forward_tc_matches_mma_sync(cuda, n):
    """The tcgen05 MLP forward (128-row tiles, tensor-memory accumulators) against the mma.sync forward on the same
    fp16 features and directions: the operands are rounded at the same points, only the fp32 accumulation order
    differs, so raw outputs agree to well within the 1e-2 per-sample contract."""
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(21)
    mlp = _mlp_params(rng).astype(np.float16).view(np.uint16)
    feat = rng.standard_normal((n, 32)).astype(np.float16).view(np.uint16)
    dirs = _unit_dirs(rng, n)
    mlp_d, feat_d, dir_d = dev(torch, mlp), dev(torch, feat), dev(torch, dirs)
    raw_d, raw_tc_d = zeros(torch, (n, 4), np.float32), zeros(torch, (n, 4), np.float32)
    err_d = zeros(torch, 1, np.uint32)
    check("mlp_forward", lib.nerf_b200_mlp_forward(mlp_d.data_ptr(), feat_d.data_ptr(), dir_d.data_ptr(), n, raw_d.data_ptr(), None))
    check("mlp_forward_tc", lib.nerf_b200_mlp_forward_tc(mlp_d.data_ptr(), feat_d.data_ptr(), dir_d.data_ptr(), n,
                                                         raw_tc_d.data_ptr(), err_d.data_ptr(), None))
    torch.cuda.synchronize()
    assert int(host(err_d)[0]) == 0
    a, b = host(raw_d), host(raw_tc_d)
    err = np.abs(a - b)
    assert err.max() < 1e-2, err.max()
    assert np.median(err) < 1e-3
    want = oracle.mlp_forward(mlp, feat, dirs)
    assert np.abs(b - want).max() < 1e-2


@pytest.mark.parametrize("n", [1, 200, 3001])
def test_mlp_backward_tc_matches_mma_sync(cuda, n):
    """The tcgen05 MLP backward against the mma.sync backward on the same inputs: feature gradients within fp16
    rounding of each other, weight gradients within 1e-2 relative L2 (fp32 accumulation in a different order),
    and both against the CPU oracle."""
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(23)
    mlp = _mlp_params(rng).astype(np.float16).view(np.uint16)
    feat = rng.standard_normal((n, 32)).astype(np.float16).view(np.uint16)
    dirs = _unit_dirs(rng, n)
    dout = (rng.standard_normal((n, 4)) * 0.5).astype(np.float32)
    mlp_d, feat_d, dir_d, dout_d = dev(torch, mlp), dev(torch, feat), dev(torch, dirs), dev(torch, dout)
    parts = int(lib.nerf_b200_field_backward_partial_floats())
    outs = []
    for tc in (False, True):
        dx_d, part_d, mg_d = zeros(torch, (n, 32), np.uint16), zeros(torch, parts, np.float32), zeros(torch, 10240, np.float32)
        err_d = zeros(torch, 1, np.uint32)
        if tc:
            check("mlp_backward_tc", lib.nerf_b200_mlp_backward_tc(
                mlp_d.data_ptr(), feat_d.data_ptr(), dir_d.data_ptr(), n, dout_d.data_ptr(), dx_d.data_ptr(),
                part_d.data_ptr(), mg_d.data_ptr(), err_d.data_ptr(), None))
        else:
            check("mlp_backward", lib.nerf_b200_mlp_backward(
                mlp_d.data_ptr(), feat_d.data_ptr(), dir_d.data_ptr(), n, dout_d.data_ptr(), dx_d.data_ptr(),
                part_d.data_ptr(), mg_d.data_ptr(), None))
        torch.cuda.synchronize()
        assert int(host(err_d)[0]) == 0
        outs.append((host(dx_d, np.uint16).view(np.float16).astype(np.float64), host(mg_d).astype(np.float64)))
    (dx_ref, wg_ref), (dx_tc, wg_tc) = outs
    assert np.abs(dx_tc - dx_ref).max() <= 5e-3 * max(1.0, np.abs(dx_ref).max())
    assert np.linalg.norm(wg_tc - wg_ref) / np.linalg.norm(wg_ref) < 1e-2
    for name, (a, b) in {"d0": (0, 2048), "d1": (2048, 3072), "c0": (3072, 5120), "c1": (5120, 9216), "c2": (9216, 9408)}.items():
        assert np.linalg.norm(wg_tc[a:b] - wg_ref[a:b]) / (np.linalg.norm(wg_ref[a:b]) + 1e-30) < 1e-2, name
    assert np.all(wg_tc[9408:] == 0)
    dfeat_o, wg_o = oracle.mlp_backward(mlp, feat, dirs, dout)
    assert np.linalg.norm(wg_tc - wg_o) / np.linalg.norm(wg_o) < 1e-2
    assert np.linalg.norm(dx_tc - dfeat_o) / np.linalg.norm(dfeat_o) < 1e-2


def _records(begin, count, gt, bg, dirs):
    n = len(begin)
    rec = np.zeros((n, 12), np.float32)
    rec[:, 0:3] = dirs
    rec.view(np.uint32)[:, 3] = begin
    rec[:, 4:8] = gt
    rec[:, 8:11] = bg
    rec.view(np.uint32)[:, 11] = count
    return rec


@pytest.mark.parametrize("stop", [0.0, 1e-4])
def test_composite_matches_oracle(cuda, stop):
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(9)
    n_rays = 700
    count = rng.integers(0, 90, n_rays).astype(np.uint32)
    count[:5] = [0, 1, 2, 700, 1024]
    begin = np.concatenate([[0], np.cumsum(count)[:-1]]).astype(np.uint32)
    S = int(count.sum())
    raw = np.zeros((S, 4), np.float32)
    raw[:, 0] = rng.normal(0.0, 2.5, S)
    raw[:, 1:] = rng.normal(0.0, 1.5, (S, 3))
    dt = rng.uniform(1e-3, 6e-2, S).astype(np.float32)
    pos_dt = np.zeros((S, 4), np.float32)
    pos_dt[:, 3] = dt
    gt = rng.random((n_rays, 4)).astype(np.float32)
    bg = rng.random((n_rays, 3)).astype(np.float32)
    rec = _records(begin, count, gt, bg, _unit_dirs(rng, n_rays))
    inv_norm, ls = 1.0 / n_rays, 128.0
    dout_d, loss_d = zeros(torch, (S, 4), np.float32), zeros(torch, n_rays, np.float32)
    used_d, lsum_d = zeros(torch, n_rays, np.uint32), zeros(torch, 1, np.float32)
    rec_d, raw_d, pos_d = dev(torch, rec), dev(torch, raw), dev(torch, pos_dt)
    check("composite", lib.nerf_b200_composite(rec_d.data_ptr(), n_rays, raw_d.data_ptr(),
                                               pos_d.data_ptr(), inv_norm, ls, stop, dout_d.data_ptr(),
                                               loss_d.data_ptr(), used_d.data_ptr(), lsum_d.data_ptr(), None))
    torch.cuda.synchronize()
    dout, loss, used, _ = oracle.composite(raw, dt, begin, count, gt, bg, inv_norm, ls, stop)
    assert np.array_equal(host(used_d, np.uint32), used)
    assert np.allclose(host(loss_d), loss, rtol=1e-5, atol=1e-7)
    assert np.allclose(host(lsum_d)[0], loss.sum() * inv_norm, rtol=1e-4)
    got = host(dout_d)
    scale = np.abs(dout).max(axis=0)
    assert (np.abs(got - dout) <= 1e-4 * scale + 1e-9).all()


def test_adam_bit_exact(cuda):
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(13)
    n_grid, n_mlp = 16 * 257, 10240
    n = n_grid + n_mlp
    master = rng.normal(0, 0.1, n).astype(np.float32)
    p16 = master.astype(np.float16).view(np.uint16)
    gg = (rng.normal(0, 1, n_grid) * 4).astype(np.float16)
    gg[::97] = 0
    mg = rng.normal(0, 3, n_mlp).astype(np.float32)
    m = rng.normal(0, 1e-3, n).astype(np.float32)
    v = np.abs(rng.normal(0, 1e-5, n)).astype(np.float32)
    hp = abi.NerfHyperParams(1e-2, 0.9, 0.99, 1e-15, 1.0, 1e4, 128.0, 20)
    s = oracle.adam_scalars(3.5, 0, 7, hp)
    scal = np.array([s.learning_rate, s.grad_scale, s.inv_bias_correction1, s.inv_bias_correction2, s.inv_loss_scale], np.float32)
    d = {k: dev(torch, x) for k, x in dict(master=master, p16=p16, gg=gg.view(np.uint16), mg=mg, m=m, v=v).items()}
    check("adam", lib.nerf_b200_adam(d["master"].data_ptr(), d["p16"].data_ptr(), d["gg"].data_ptr(), d["mg"].data_ptr(),
                                     d["m"].data_ptr(), d["v"].data_ptr(), n_grid, n, scal.ctypes.data, 0, 0.9, 0.99, 1e-15, None))
    torch.cuda.synchronize()
    grad = np.concatenate([gg.astype(np.float32), mg])
    om, op, omm, ov = master.copy(), p16.copy(), m.copy(), v.copy()
    oracle.adam(om, op, grad, omm, ov, 0.9, 0.99, 1e-15, s)
    assert np.array_equal(host(d["master"]), om)
    assert np.array_equal(host(d["m"]), omm)
    assert np.array_equal(host(d["v"]), ov)
    assert np.array_equal(host(d["p16"], np.uint16), op)
    assert not host(d["gg"], np.uint16).any()  # grid gradients cleared for the next step


@pytest.mark.parametrize("res", [33, 64])
def test_occupancy_update_bit_exact(cuda, res):
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(17)
    cells = res ** 3
    words = (cells + 31) // 32
    density = rng.exponential(0.02, cells).astype(np.float32)
    bits = rng.integers(0, 2 ** 32, words, dtype=np.uint64).astype(np.uint32)
    for mode, upd, frame in [(1, 100, 0), (0, 100, 3), (2, 5000, 7), (2, cells, 3), (2, 777, 123456)]:
        sigma = rng.exponential(0.02, upd).astype(np.float32)
        d_d, b_d, s_d = dev(torch, density), dev(torch, bits), dev(torch, sigma)
        check("occupancy", lib.nerf_b200_occupancy_update(d_d.data_ptr(), b_d.data_ptr(), s_d.data_ptr(), cells,
                                                          upd, frame, mode, 0.95, 0.01, None))
        torch.cuda.synchronize()
        od, ob = density.copy(), bits.copy()
        oracle.occupancy_update(od, ob, sigma, cells, upd, frame, mode, 0.95, 0.01)
        assert np.array_equal(host(d_d), od), mode
        assert np.array_equal(host(b_d, np.uint32), ob), mode
        density, bits = od, ob
