"""The allocation-free convolution entry point, spinn_cuda_conv2d_noalloc.

Some callers cannot allocate device memory while they run: SPINN is built for systems that
plan every byte ahead of time (a static arena, ennf2c programs with no run-time allocation),
and a host whose GPU memory belongs to another allocator is in the same position.  For them
spinn_cuda_conv2d_noalloc keeps all its temporaries in one fixed device array of the library.
These tests call it through the C ABI and compare it with the regular spinn_cuda_conv2d on
two consecutive calls of different shapes (the second must not see the first's leftovers),
and check that a problem larger than the fixed scratch is refused.  This file is collected
last so a failure here cannot hide any other test.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the per-layer tolerance used by every convolution test


def _noalloc(L, x, w, b, r, y, n, c, h, wd, oc, k, s, p, act):
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    return L.spinn_cuda_conv2d_noalloc(ptr(x), ptr(w), ptr(b), ptr(r), ptr(y), n, c, h, wd, oc, k, k, s, s, p, p,
                                       act, None)


CASES = [
    # n, c, h, w, oc, k, s, p, act (5 = +residual then ReLU)
    (2, 64, 28, 28, 128, 3, 1, 1, 5),
    (1, 3, 33, 31, 26, 7, 2, 3, 1),
]


def test_noalloc_matches_conv2d_on_two_calls(cuda_lib):
    import torch
    from spinn_b200 import lib, runtime
    L = lib.lib()
    rng = np.random.default_rng(2024)
    for (n, c, h, wd, oc, k, s, p, act) in CASES:
        oh, ow = (h + 2 * p - k) // s + 1, (wd + 2 * p - k) // s + 1
        x = rng.uniform(-1, 1, (n, c, h, wd)).astype(np.float32)
        w = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (oc, c, k, k)).astype(np.float32)
        b = rng.normal(0, 0.1, oc).astype(np.float32)
        r = rng.uniform(-1, 1, (n, oc, oh, ow)).astype(np.float32) if act in (4, 5) else None
        xd, wd_, bd = (torch.from_numpy(a).cuda() for a in (x, w, b))
        rd = torch.from_numpy(r).cuda() if r is not None else None
        y = torch.full((n, oc, oh, ow), float("nan"), device="cuda")
        rc = _noalloc(L, xd, wd_, bd, rd, y, n, c, h, wd, oc, k, s, p, act)
        assert rc == 0, lib.last_error()
        expect = torch.zeros((n, oc, oh, ow), device="cuda")
        runtime.conv2d(xd, w, expect, b, rd, runtime.conv_params((k, k), (s, s), (p, p, p, p), (1, 1), 1, 0, act))
        runtime.sync()
        got, want = y.cpu().numpy(), expect.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, want) <= TOL, rel_l2(got, want)


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_lib):
    import torch
    from spinn_b200 import lib
    L = lib.lib()
    t = torch.zeros(16, device="cuda")
    # 8 x 256 x 64 x 64 input alone is 32 MiB: more than the fixed scratch holds
    rc = _noalloc(L, t, t, None, None, t, 8, 256, 64, 64, 256, 3, 1, 1, 0)
    assert rc == lib.EINVAL
    assert "32 MiB" in lib.last_error()
