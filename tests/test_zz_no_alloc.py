"""The allocation-free field backward (nerf_b200_field_backward_noalloc).

Some callers cannot allocate device memory, for example a plugin running
inside a host application that owns the device memory budget, or code in
which a cudaMalloc would synchronise the device at a bad moment.  For them
the library offers a variant of nerf_b200_field_backward whose weight-gradient
scratch lives in a static device array instead of a caller-allocated buffer.
This test calls that variant several times in a row through the C ABI, with
different upstream gradients and then fewer rows (2500, 2500, 37, 0), and
checks each call against nerf_b200_field_backward with its own scratch on
the same inputs: the MLP weight gradients must be identical (same kernel,
same CTA count, same reduction order), so rows of the shared array left over
from a larger earlier call never leak into a smaller later one, and the
hash-table gradients, summed with fp16 reductions in nondeterministic order,
must agree within the relative L2 tolerance used by the other backward tests.
The first call's gradients are also compared with the CPU oracle's field
backward within the tolerances of the other field-backward tests.
The file name sorts last so that a run stopping at the first failure has
already run every other test.
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


def test_field_backward_noalloc_matches_allocating_entry_point(cuda):
    torch = cuda
    lib = abi.load()
    rng = np.random.default_rng(29)
    n = 2500
    g = nerf_b200.grid_layout(16, 15, 16, 512)
    og = oracle.grid_layout(16, 15, 16, 512)
    n_grid = 2 * g.offset[16]
    sizes = [(64, 32), (16, 64), (64, 32), (64, 64), (16, 64)]
    mlp = np.concatenate([rng.uniform(-np.sqrt(6 / (i + o)), np.sqrt(6 / (i + o)), o * i) for o, i in sizes])
    params = np.concatenate([rng.uniform(-0.5, 0.5, n_grid), mlp]).astype(np.float16).view(np.uint16)
    pos = rng.random((n, 3)).astype(np.float32)
    dirs = rng.standard_normal((n, 3)).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    feat = oracle.grid_forward(og, params[:n_grid], pos)
    assert lib.nerf_b200_field_backward_noalloc_max_rows() >= lib.nerf_b200_field_backward_partial_floats() // 10240
    par_d, pos_d, dir_d, feat_d = dev(torch, params), dev(torch, pos), dev(torch, dirs), dev(torch, feat)
    for call, rows in enumerate((n, n, 37, 0)):
        dout = np.zeros((n, 4), np.float32)
        dout[:rows] = rng.standard_normal((rows, 4)) * (0.5 + call)
        dout_d = dev(torch, dout)
        gg_ref, mg_ref = zeros(torch, n_grid, np.uint16), zeros(torch, 10240, np.float32)
        part = zeros(torch, int(lib.nerf_b200_field_backward_partial_floats()), np.float32)
        check("field_backward", lib.nerf_b200_field_backward(
            C.byref(g), par_d.data_ptr(), pos_d.data_ptr(), dir_d.data_ptr(), rows, feat_d.data_ptr(), dout_d.data_ptr(),
            gg_ref.data_ptr(), part.data_ptr(), mg_ref.data_ptr(), None))
        gg, mg = zeros(torch, n_grid, np.uint16), zeros(torch, 10240, np.float32)
        check("field_backward_noalloc", lib.nerf_b200_field_backward_noalloc(
            C.byref(g), par_d.data_ptr(), pos_d.data_ptr(), dir_d.data_ptr(), rows, feat_d.data_ptr(), dout_d.data_ptr(),
            gg.data_ptr(), mg.data_ptr(), None))
        torch.cuda.synchronize()
        assert np.array_equal(host(mg), host(mg_ref)), call
        a = host(gg, np.uint16).view(np.float16).astype(np.float64)
        b = host(gg_ref, np.uint16).view(np.float16).astype(np.float64)
        if rows == 0:
            assert not host(mg).any() and not a.any() and not b.any()
            continue
        assert np.linalg.norm(a - b) / np.linalg.norm(b) < 2e-2, call
        if call == 0:
            dfeat, wg = oracle.mlp_backward(params[n_grid:], feat[:rows], dirs[:rows], dout[:rows])
            got_w = host(mg).astype(np.float64)
            assert np.linalg.norm(got_w - wg) / np.linalg.norm(wg) < 1e-2
            want_g = oracle.grid_backward(og, pos[:rows], dfeat)
            assert np.linalg.norm(a - want_g) / np.linalg.norm(want_g) < 2e-2
    bad = lib.nerf_b200_field_backward_noalloc(C.byref(g), par_d.data_ptr(), pos_d.data_ptr(), dir_d.data_ptr(), 1 << 31,
                                               feat_d.data_ptr(), dout_d.data_ptr(), gg.data_ptr(), mg.data_ptr(), None)
    assert bad == abi.NERF_STATUS_INVALID_USAGE
