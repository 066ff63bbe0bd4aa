"""Known-answer tests of the north-star model half of the oracle (CPU only).

The reference has no hash grid, SH encoding, 64-wide MLPs or trunc_exp, so
the oracle (oracle/oracle_core.cpp) is their definition, and the GPU kernels
are checked bit for bit against it.  These tests pin that definition against
an independent restatement written here in numpy from the published method
(Mueller et al., "Instant Neural Graphics Primitives with a Multiresolution
Hash Encoding", SIGGRAPH 2022, section 3; real spherical harmonics from
scipy's complex ones; plain backpropagation), so that a misreading shared by
the oracle and the kernels -- level scale, the half-cell offset, corner
order, the hash primes, the SH sign convention, the wiring of the two MLPs,
the trunc_exp gradient clamp -- fails here.

Conventions the implementation fixes where the paper leaves a choice (each
asserted below):
  * b = exp((ln N_max - ln N_min) / (L - 1)); the paper's level resolution is
    N_l = floor(N_min * b^l).  The grid uses the unfloored s_l = N_min * b^l - 1
    (rounded once to fp32) as the scale of level l, so that vertex spacing is
    1 / s_l, and a point x in [0,1] (clamped) maps to u = x * s_l + 0.5 (one
    rounding: a fused multiply-add); floor(s_l) + 1 = N_l except where the
    paper's float64 floor lands one below an integer (N_max 8192, levels 5,
    10, 15: floor(16 * b^15) = 8191 in float64 while s_15 rounds to 8191.0f).
  * R_l = ceil(s_l) + 2 vertices per axis; the cell corner is
    clamp(floor(u), 0, R_l - 2); a level is dense (1:1, index
    x + R_l (y + R_l z)) when R_l^3 <= T, else hashed with the paper's
    h(x) = (x * 1 xor y * 2654435761 xor z * 805459861) mod T.
  * Level l's entries start at the sum of the earlier levels' sizes: dense
    R_l^3 rounded up to a multiple of 8, hashed T.
  * Corner c: bit 0 = x, bit 1 = y, bit 2 = z (upper vertex when set); weight
    ((w_x * w_y) * w_z) in fp32 with w = f for the upper, 1 - f for the lower
    vertex, f = u - floor(u).
  * A level's two features: the fp32 fused-multiply-add chain over corners
    0..7 from zero, rounded once to fp16.
"""
import math

import numpy as np
import pytest
import scipy.special

from oracle import oracle

PRIMES = (1, 2654435761, 805459861)


# ------------------------------------------------------------- hash grid
def paper_levels(n_min, n_max, L):
    """(b, paper N_l, scale s_l as fp32) per level, from the paper's formula."""
    b = math.exp((math.log(n_max) - math.log(n_min)) / (L - 1))
    n_paper = [math.floor(n_min * b ** l) for l in range(L)]
    scale = [np.float32(n_min * b ** l - 1.0) for l in range(L)]
    return b, n_paper, scale


def layout(n_min, n_max, L, log2T):
    T = 1 << log2T
    _, _, scale = paper_levels(n_min, n_max, L)
    res, dense, off = [], [], [0]
    for s in scale:
        R = int(math.ceil(float(s))) + 2
        d = R ** 3 <= T
        res.append(R)
        dense.append(d)
        off.append(off[-1] + (((R ** 3 + 7) // 8) * 8 if d else T))
    return scale, res, dense, off


def fma32(a, b, c):
    """fp32 fused multiply-add: the float64 sum of an exact fp32 product and an fp32 addend, rounded once to fp32
    (exact here: both terms fit well inside float64's 53 bits for the magnitudes these tests use)."""
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def corners(p, scale, R, dense, off, log2T):
    """Entry indices and fp32 weights of the 8 corners of point p on one level."""
    T = 1 << log2T
    i, f = [], []
    for d in range(3):
        u = fma32(np.float32(min(1.0, max(0.0, float(p[d])))), scale, np.float32(0.5))
        fl = np.float32(math.floor(float(u)))
        f.append(np.float32(u - fl))
        i.append(min(max(int(fl), 0), R - 2))
    idx, w = [], []
    for c in range(8):
        v = [i[0] + (c & 1), i[1] + ((c >> 1) & 1), i[2] + ((c >> 2) & 1)]
        if dense:
            e = v[0] + R * (v[1] + R * v[2])
        else:
            e = 0
            for k in range(3):
                e ^= (v[k] * PRIMES[k]) & 0xFFFFFFFF
            e %= T
        idx.append(off + e)
        ws = [f[k] if (c >> k) & 1 else np.float32(1.0) - f[k] for k in range(3)]
        w.append(np.float32(np.float32(ws[0] * ws[1]) * ws[2]))
    return idx, w


def kat_points():
    rng = np.random.default_rng(2022)
    pts = [[0.0, 0.0, 0.0], [1.0, 1.0, 1.0], [0.5, 0.5, 0.5], [1.0, 0.0, 0.25], [-0.2, 1.3, 0.5],
           [0.999999, 1e-7, 0.123456], [0.25, 0.75, 0.0625]]
    pts += rng.random((13, 3)).tolist()
    return np.array(pts, np.float32)


@pytest.mark.parametrize("n_max", [2048, 8192])
def test_level_scales_and_paper_resolution(n_max):
    b, n_paper, scale = paper_levels(16, n_max, 16)
    assert b == pytest.approx(2 ** ((math.log2(n_max) - 4) / 15), rel=1e-15)
    g = oracle.grid_layout(16, 19, 16, n_max)
    for l in range(16):
        assert np.float32(g.scale[l]) == scale[l], l
        assert int(g.resolution[l]) == int(math.ceil(float(scale[l]))) + 2, l
    if n_max == 2048:
        assert n_paper == [16, 22, 30, 42, 58, 80, 111, 153, 212, 294, 406, 561, 776, 1072, 1482, 2048]
        assert [math.floor(float(s)) + 1 for s in scale] == n_paper
    else:
        assert n_paper == [16, 24, 36, 55, 84, 127, 194, 294, 445, 675, 1023, 1552, 2352, 3565, 5404, 8191]
        # float64 puts 16 * b^l just below 128, 1024 and 8192 at levels 5, 10 and 15 (b^3 = 2^(9/5)): the paper's
        # floor gives 127, 1023 and 8191, while the fp32 scales round to exactly 127, 1023 and 8191
        for l, n in ((5, 128), (10, 1024), (15, 8192)):
            assert n - 1e-9 < 16 * b ** l < n and n_paper[l] == n - 1
            assert scale[l] == np.float32(n - 1)
            assert math.floor(float(scale[l])) + 1 == n
        assert all(math.floor(float(s)) + 1 == n for l, (s, n) in enumerate(zip(scale, n_paper)) if l not in (5, 10, 15))


@pytest.mark.parametrize("log2T,n_max", [(15, 512), (15, 2048), (19, 2048), (22, 8192)])
def test_dense_hashed_switch_and_offsets(log2T, n_max):
    scale, res, dense, off = layout(16, n_max, 16, log2T)
    g = oracle.grid_layout(16, log2T, 16, n_max)
    assert [bool(g.dense[l]) for l in range(16)] == dense
    assert [int(g.offset[l]) for l in range(17)] == off
    if (log2T, n_max) == (19, 2048):
        # the bounded-training configuration: levels 0-4 dense with 17, 24, 32, 44, 60 vertices per axis,
        # levels 5-15 hashed: 6,119,864 entries, 12.24 M fp16 parameters
        assert dense == [True] * 5 + [False] * 11
        assert res[:5] == [17, 24, 32, 44, 60]
        assert off[16] == 4920 + 13824 + 32768 + 85184 + 216000 + 11 * (1 << 19) == 6119864


@pytest.mark.parametrize("log2T,n_max", [(15, 512), (19, 2048)])
def test_corner_indices_and_weights(log2T, n_max):
    scale, res, dense, off = layout(16, n_max, 16, log2T)
    g = oracle.grid_layout(16, log2T, 16, n_max)
    pts = kat_points()
    idx, w = oracle.grid_corners(g, pts)
    for n, p in enumerate(pts):
        for l in range(16):
            ei, ew = corners(p, scale[l], res[l], dense[l], off[l], log2T)
            assert list(idx[n, l]) == ei, (n, l)
            assert np.array_equal(w[n, l].view(np.uint32), np.array(ew, np.float32).view(np.uint32)), (n, l)
            assert abs(float(np.sum(np.array(ew, np.float64))) - 1.0) < 1e-6


def test_hash_function_values():
    """The spatial hash on fixed vertices (T = 2^19), written out."""
    T = 1 << 19
    for v, want in [((0, 0, 0), 0), ((1, 0, 0), 1), ((0, 1, 0), 2654435761 % T), ((0, 0, 1), 805459861 % T),
                    ((3, 5, 7), (3 ^ ((5 * 2654435761) & 0xFFFFFFFF) ^ ((7 * 805459861) & 0xFFFFFFFF)) % T)]:
        e = 0
        for k in range(3):
            e ^= (v[k] * PRIMES[k]) & 0xFFFFFFFF
        assert e % T == want


def test_forward_features_bit_exact():
    log2T, n_max = 15, 512
    scale, res, dense, off = layout(16, n_max, 16, log2T)
    g = oracle.grid_layout(16, log2T, 16, n_max)
    rng = np.random.default_rng(7)
    params = rng.uniform(-1.0, 1.0, 2 * off[16]).astype(np.float16)
    pts = kat_points()
    feat = oracle.grid_forward(g, params.view(np.uint16), pts).view(np.float16)
    for n, p in enumerate(pts):
        for l in range(16):
            ei, ew = corners(p, scale[l], res[l], dense[l], off[l], log2T)
            for ch in range(2):
                acc = np.float32(0.0)
                for c in range(8):
                    acc = fma32(ew[c], np.float32(params[2 * ei[c] + ch]), acc)
                assert np.float16(acc).view(np.uint16) == feat[n, 2 * l + ch].view(np.uint16), (n, l, ch)


# ------------------------------------------------------- spherical harmonics
def real_sh(d, lmax=3):
    """Real orthonormal SH from scipy's complex ones (which carry the Condon-Shortley phase): m > 0:
    sqrt(2) Re Y_l^m, m < 0: sqrt(2) Im Y_l^|m|, m = 0: Y_l^0; index l^2 + l + m."""
    x, y, z = (float(v) for v in d)
    theta = math.acos(max(-1.0, min(1.0, z)))
    phi = math.atan2(y, x)
    out = []
    for l in range(lmax + 1):
        for m in range(-l, l + 1):
            Y = complex(scipy.special.sph_harm_y(l, abs(m), theta, phi))
            out.append(Y.real if m == 0 else math.sqrt(2.0) * (Y.real if m > 0 else Y.imag))
    return np.array(out)


def sh_dirs():
    s2, s3 = 1 / math.sqrt(2), 1 / math.sqrt(3)
    return np.array([[1, 0, 0], [-1, 0, 0], [0, 1, 0], [0, -1, 0], [0, 0, 1], [0, 0, -1], [s3, s3, s3],
                     [s2, -s2, 0]], np.float32)


def test_sh_against_scipy_at_axes_and_diagonals():
    dirs = sh_dirs()
    got = oracle.sh4(dirs)
    for d, g in zip(dirs, got):
        want = real_sh(d)
        assert np.allclose(g, want, rtol=1e-6, atol=2e-7), (d, g, want)


def test_sh_closed_form_on_z_axis():
    """At +z only m = 0 survives: Y_l^0 = sqrt((2l+1)/(4 pi)) for l = 0..3."""
    got = oracle.sh4(np.array([[0, 0, 1]], np.float32))[0]
    want = np.zeros(16)
    for l in range(4):
        want[l * l + l] = math.sqrt((2 * l + 1) / (4 * math.pi))
    assert np.allclose(got, want, atol=2e-7)


# -------------------------------------------------------------------- MLPs
SHAPES = [(64, 32), (16, 64), (64, 32), (64, 64), (16, 64)]  # (out, in): density W0, W1, colour W0, W1, W2


def split_weights(flat):
    ws, o = [], 0
    for r, c in SHAPES:
        ws.append(flat[o:o + r * c].reshape(r, c).astype(np.float64))
        o += r * c
    assert o == 10240
    return ws


def f16(x):
    return np.asarray(x).astype(np.float16).astype(np.float64)


def mlp_numpy(flat16, feat16, dirs):
    """Forward of the field's two MLPs: density 32 -> 64 -> 16 (ReLU), colour (16 density outputs + 16 SH) -> 64
    -> 64 -> 3 (ReLU, ReLU, linear); matrix operands fp16 (the tensor-core contract), sums in float64 here.  Raw
    outputs: density channel 0 and the three colour logits."""
    Wd0, Wd1, Wc0, Wc1, Wc2 = split_weights(flat16.view(np.float16).astype(np.float64))
    x = feat16.view(np.float16).astype(np.float64)
    hd = f16(np.maximum(x @ Wd0.T, 0.0))
    yd = hd @ Wd1.T
    sh = np.stack([real_sh(d) for d in dirs])
    xc = np.concatenate([f16(yd), f16(sh)], axis=1)
    h1 = f16(np.maximum(xc @ Wc0.T, 0.0))
    h2 = f16(np.maximum(h1 @ Wc1.T, 0.0))
    yc = h2 @ Wc2[:3].T
    return np.concatenate([yd[:, :1], yc], axis=1), (x, hd, yd, xc, h1, h2)


def mlp_numpy_backward(flat16, trace, dout):
    Wd0, Wd1, Wc0, Wc1, Wc2 = split_weights(flat16.view(np.float16).astype(np.float64))
    x, hd, yd, xc, h1, h2 = trace
    dyc = dout[:, 1:4]
    dh2 = (dyc @ Wc2[:3]) * (h2 > 0)
    dh1 = (dh2 @ Wc1) * (h1 > 0)
    dxc = dh1 @ Wc0
    dyd = dxc[:, :16].copy()
    dyd[:, 0] += dout[:, 0]  # density output 0 is the raw density and the colour network's first input
    dhd = (dyd @ Wd1) * (hd > 0)
    dfeat = dhd @ Wd0
    gW = [dhd.T @ x, dyd.T @ hd, dh1.T @ xc, dh2.T @ h1, np.vstack([dyc.T @ h2, np.zeros((13, 64))])]
    return dfeat, np.concatenate([g.ravel() for g in gW])


def mlp_case(n=300, seed=11):
    rng = np.random.default_rng(seed)
    flat = np.concatenate([rng.uniform(-math.sqrt(6 / (i + o)), math.sqrt(6 / (i + o)), o * i) for o, i in SHAPES])
    flat16 = flat.astype(np.float16).view(np.uint16)
    feat16 = rng.uniform(-1, 1, (n, 32)).astype(np.float16).view(np.uint16)
    dirs = rng.standard_normal((n, 3)).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    return flat16, feat16, dirs


def test_mlp_forward_against_numpy():
    flat16, feat16, dirs = mlp_case()
    want, _ = mlp_numpy(flat16, feat16, dirs)
    got = oracle.mlp_forward(flat16, feat16, dirs)
    err = np.abs(got - want)
    # fp32 sums in the oracle vs float64 here; an fp16 rounding of an activation may flip by one ulp
    assert np.median(err) < 1e-5 and err.max() < 5e-3, (np.median(err), err.max())


def test_mlp_backward_against_numpy():
    flat16, feat16, dirs = mlp_case(seed=12)
    rng = np.random.default_rng(13)
    dout = rng.standard_normal((feat16.shape[0], 4)).astype(np.float32)
    _, trace = mlp_numpy(flat16, feat16, dirs)
    want_dfeat, want_w = mlp_numpy_backward(flat16, trace, dout.astype(np.float64))
    got_dfeat, got_w = oracle.mlp_backward(flat16, feat16, dirs, dout)
    # the oracle rounds each layer's gradient operand to fp16 (the tensor-core contract); none is rounded here
    assert np.linalg.norm(got_dfeat - want_dfeat) / np.linalg.norm(want_dfeat) < 2e-3
    assert np.linalg.norm(got_w - want_w) / np.linalg.norm(want_w) < 2e-3
    for k, (r, c) in enumerate(SHAPES):
        a = sum(o * i for o, i in SHAPES[:k])
        seg = slice(a, a + r * c)
        assert np.linalg.norm(got_w[seg] - want_w[seg]) / (np.linalg.norm(want_w[seg]) + 1e-30) < 5e-3, k
    assert not got_w[9216 + 3 * 64:].any()  # colour output rows 3..15 are unused


# -------------------------------------------------------------- trunc_exp
@pytest.mark.parametrize("x", [-20.0, -3.0, 2.0, 14.5, 20.0])
def test_trunc_exp_gradient_clamp(x):
    """One ray with one sample: sigma = exp(x) (unclamped) and d sigma / dx = exp(clamp(x, -15, 15)).  The loss is
    the alpha-weighted squared error of the composite on white; dt puts sigma * dt near 0.5 for every x."""
    dt = np.float32(0.5 / math.exp(x))
    raw = np.array([[x, 0.3, -0.7, 1.1]], np.float32)
    gt = np.array([[0.2, 0.6, 0.1, 0.8]], np.float32)
    bg = np.ones((1, 3), np.float32)
    dout, loss, used, rgb = oracle.composite(raw, np.array([dt]), np.array([0]), np.array([1]), gt, bg, 1.0, 1.0, 0.0)
    sigma = math.exp(x)
    e = math.exp(-sigma * float(dt))
    a = 1.0 - e
    c = 1.0 / (1.0 + np.exp(-raw[0, 1:].astype(np.float64)))
    pred = a * c + (1.0 - a) * 1.0
    wr = 0.1 + 0.9 * 0.8
    g = 2.0 * wr * (pred - gt[0, :3])
    assert loss[0] == pytest.approx(wr * np.sum((pred - gt[0, :3]) ** 2), rel=1e-5)
    d_alpha = float(np.sum(g * (c - 1.0)))
    want_sigma = d_alpha * float(dt) * e * math.exp(min(15.0, max(-15.0, x)))
    assert dout[0, 0] == pytest.approx(want_sigma, rel=1e-4), (dout[0, 0], want_sigma)
    assert np.allclose(dout[0, 1:], a * g * c * (1 - c), rtol=1e-5)


# ------------------------------------------- the GPU against the restatement
@pytest.mark.gpu
@pytest.mark.parametrize("log2T,n_max", [(15, 512), (19, 2048)])
def test_gpu_grid_forward_matches_restatement(cuda, log2T, n_max):
    """The CUDA hash-grid forward (nerf_b200_grid_forward through the C ABI) on the KAT points equals this file's
    restatement bit for bit, with no oracle in between."""
    import ctypes as C

    import nerf_b200
    from nerf_b200 import abi
    from gpu_util import dev, host, zeros
    torch = cuda
    lib = abi.load()
    scale, res, dense, off = layout(16, n_max, 16, log2T)
    g = nerf_b200.grid_layout(16, log2T, 16, n_max)
    assert [int(g.offset[l]) for l in range(17)] == off
    rng = np.random.default_rng(8)
    params = rng.uniform(-1.0, 1.0, 2 * off[16]).astype(np.float16)
    pts = kat_points()
    n = pts.shape[0]
    pos_d, par_d, feat_d = dev(torch, pts), dev(torch, params.view(np.uint16)), zeros(torch, (n, 32), np.uint16)
    abi.check("grid_forward", lib.nerf_b200_grid_forward(C.byref(g), pos_d.data_ptr(), n, par_d.data_ptr(),
                                                         feat_d.data_ptr(), None))
    torch.cuda.synchronize()
    got = host(feat_d, np.uint16)
    for k, p in enumerate(pts):
        for l in range(16):
            ei, ew = corners(p, scale[l], res[l], dense[l], off[l], log2T)
            for ch in range(2):
                acc = np.float32(0.0)
                for c in range(8):
                    acc = fma32(ew[c], np.float32(params[2 * ei[c] + ch]), acc)
                assert np.float16(acc).view(np.uint16) == got[k, 2 * l + ch], (k, l, ch)
