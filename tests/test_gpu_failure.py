"""Failure detection without a GPU fault: a bounded mbarrier wait that nothing satisfies (the
wait primitive every tcgen05 kernel uses), and the bounded wait on a stream-K handoff flag,
expire, raise the device error flag, are reported as SPINN_CUDA_ETIMEOUT and cleared, and the
context keeps working."""
import time

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

ETIMEOUT, EINVAL = -5, -1


def test_bounded_wait_expiry_is_reported_and_recovered(cuda_lib, port_oracle):
    from spinn_b200 import lib, runtime
    L = lib.lib()
    t0 = time.time()
    assert L.spinn_cuda_selftest_wait_expiry(50_000_000) == ETIMEOUT  # 50 ms limit
    assert time.time() - t0 < 10.0
    assert L.spinn_cuda_sync() == 0  # the flag was cleared when reported
    # the context still runs work correctly
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (1, 32, 12, 12)).astype(np.float32)
    w = rng.normal(0, 0.1, (48, 32, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.1, 48).astype(np.float32)
    y = np.zeros((1, 48, 12, 12), np.float32)
    runtime.conv2d(x, w, y, b, None, runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 1))
    ref = port_oracle.conv2d(x, w, b, None, (1, 1), (1, 1), (1, 1), 1, 1, (12, 12))
    assert rel_l2(y, ref) <= 2e-3
    assert L.spinn_cuda_sync() == 0
    # limits outside (0, 1 s] are refused before anything is launched
    assert L.spinn_cuda_selftest_wait_expiry(0) == EINVAL
    assert L.spinn_cuda_selftest_wait_expiry(2_000_000_000) == EINVAL


def test_streamk_flag_wait_expiry_is_reported_and_recovered(cuda_lib, port_oracle):
    """The stream-K handoff wait (a head CTA waiting for a later CTA's partial sums) is bounded
    the same way: a flag nothing raises times out, is reported and cleared, and a stream-K
    launch afterwards runs correctly."""
    from spinn_b200 import lib, runtime
    L = lib.lib()
    t0 = time.time()
    assert L.spinn_cuda_selftest_flag_wait_expiry(50_000_000) == ETIMEOUT
    assert time.time() - t0 < 10.0
    assert L.spinn_cuda_sync() == 0
    assert L.spinn_cuda_selftest_flag_wait_expiry(0) == EINVAL
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, (256, 512, 7, 7)).astype(np.float32)
    w = rng.normal(0, 0.02, (512, 512, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.1, 512).astype(np.float32)
    y = np.zeros((256, 512, 7, 7), np.float32)
    before = L.spinn_cuda_stat_streamk_launches()
    runtime.conv2d(x, w, y, b, None, runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 1))
    assert L.spinn_cuda_stat_streamk_launches() > before
    ref = port_oracle.conv2d(x[-2:], w, b, None, (1, 1), (1, 1), (1, 1), 1, 1, (7, 7))
    assert rel_l2(y[-2:], ref) <= 2e-3
    assert L.spinn_cuda_sync() == 0
