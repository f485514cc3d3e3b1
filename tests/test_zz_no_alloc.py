"""The allocation-free convolution entry point, spinn_cuda_conv2d_noalloc.

Some callers cannot allocate device memory while they run: SPINN is built for systems that
plan every byte ahead of time (a static arena, ennf2c programs with no run-time allocation),
and a host whose GPU memory belongs to another allocator is in the same position.  For them
spinn_cuda_conv2d_noalloc keeps all its temporaries in one fixed device array of the library.
These tests call it through the C ABI on two consecutive calls of different shapes (the second
must not see the first's leftovers) and compare each result with the C oracle's convolution
(oracle/spinn_oracle.c, the restatement of op_conv2d) and with the regular spinn_cuda_conv2d;
they check that repeated calls leave the device's free memory unchanged, and that problems
the entry point cannot take are refused.  This file is collected last so a failure here cannot
hide any other test.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the per-layer tolerance used by every convolution test


def _noalloc(L, x, w, b, r, y, n, c, h, wd, oc, k, s, p, act, stream=None):
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    return L.spinn_cuda_conv2d_noalloc(ptr(x), ptr(w), ptr(b), ptr(r), ptr(y), n, c, h, wd, oc, k, k, s, s, p, p,
                                       act, stream)


CASES = [
    # n, c, h, w, oc, k, s, p, act (5 = +residual then ReLU)
    (2, 64, 28, 28, 128, 3, 1, 1, 5),
    (1, 3, 33, 31, 26, 7, 2, 3, 1),
]


def _case(rng, n, c, h, wd, oc, k, s, p, act):
    import torch
    oh, ow = (h + 2 * p - k) // s + 1, (wd + 2 * p - k) // s + 1
    x = rng.uniform(-1, 1, (n, c, h, wd)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (oc, c, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, oc).astype(np.float32)
    r = rng.uniform(-1, 1, (n, oc, oh, ow)).astype(np.float32) if act in (4, 5) else None
    dev = {name: (torch.from_numpy(a).cuda() if a is not None else None)
           for name, a in (("x", x), ("w", w), ("b", b), ("r", r))}
    dev["y"] = torch.full((n, oc, oh, ow), float("nan"), device="cuda")
    return (x, w, b, r), dev


def _free_bytes():
    import torch
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]


def test_noalloc_matches_oracle_and_conv2d_on_two_calls(cuda_lib, port_oracle):
    import torch
    from spinn_b200 import lib, runtime
    L = lib.lib()
    rng = np.random.default_rng(2024)
    cases = [(_case(rng, *c), c) for c in CASES]
    for _round in range(2):  # the second round reuses the array the first round left behind
        for (host, dev), (n, c, h, wd, oc, k, s, p, act) in cases:
            x, w, b, r = host
            dev["y"].fill_(float("nan"))
            rc = _noalloc(L, dev["x"], dev["w"], dev["b"], dev["r"], dev["y"], n, c, h, wd, oc, k, s, p, act)
            assert rc == 0, lib.last_error()
            got = dev["y"].cpu().numpy()
            assert np.isfinite(got).all()
            ref = port_oracle.conv2d(x, w, b, r, (s, s), (p, p), (1, 1), 1, act)
            assert rel_l2(got, ref) <= TOL, rel_l2(got, ref)
            expect = torch.zeros_like(dev["y"])
            runtime.conv2d(dev["x"], w, expect, b, dev["r"],
                           runtime.conv_params((k, k), (s, s), (p, p, p, p), (1, 1), 1, 0, act))
            runtime.sync()
            assert rel_l2(got, expect.cpu().numpy()) <= TOL


def test_noalloc_leaves_free_device_memory_unchanged(cuda_lib):
    """After one call of each shape has resolved the array and loaded the kernels, further
    calls change the device's free memory by nothing at all."""
    from spinn_b200 import lib
    L = lib.lib()
    rng = np.random.default_rng(7)
    cases = [(_case(rng, *c)[1], c) for c in CASES]

    def call_all():
        for dev, (n, c, h, wd, oc, k, s, p, act) in cases:
            rc = _noalloc(L, dev["x"], dev["w"], dev["b"], dev["r"], dev["y"], n, c, h, wd, oc, k, s, p, act)
            assert rc == 0, lib.last_error()

    call_all()  # set-up: array address resolved, kernel code loaded
    before = _free_bytes()
    call_all()
    call_all()
    assert _free_bytes() == before


def test_noalloc_refuses_unsupported_problems_before_any_work(cuda_lib):
    import torch
    from spinn_b200 import lib
    L = lib.lib()
    t = torch.zeros(16, device="cuda")
    # 8 x 256 x 64 x 64 input alone is 32 MiB: more than the fixed scratch holds
    assert _noalloc(L, t, t, None, None, t, 8, 256, 64, 64, 256, 3, 1, 1, 0) == lib.EINVAL
    assert "32 MiB" in lib.last_error()
    # stride 9: beyond the tensor-core kernel's im2col range
    assert _noalloc(L, t, t, None, None, t, 1, 4, 40, 40, 8, 9, 9, 0, 0) == lib.EINVAL
    assert "stride" in lib.last_error()
    # more than 65535 images (tiny ones, so that the scratch would fit)
    assert _noalloc(L, t, t, None, None, t, 70000, 1, 1, 1, 1, 1, 1, 0, 0) == lib.EINVAL
    assert "65535" in lib.last_error()
    # nothing was queued: y is untouched
    assert (t == 0).all()
