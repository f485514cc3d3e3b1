"""The tcgen05 instruction-rate diagnostic (spinn_cuda_diag_mma_rate): per-SM cycles of one
kind::tf32 MMA with resident operands.  The tile planner's cost model assumes what these
checks pin: a 128 x N x 8 MMA costs about N/2 cycles from N = 128 up, narrower ones pay a
floor of roughly 46 cycles, M = 64 costs the same cycles as M = 128 for half the work, and
the shared-memory layout does not change the cost."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu

EINVAL = -1


def _rate(L, m, n, layout, iters=2048):
    c = ctypes.c_double(0.0)
    rc = L.spinn_cuda_diag_mma_rate(m, n, layout, iters, ctypes.byref(c))
    assert rc == 0
    assert c.value > 0
    return c.value


def test_mma_rate_shapes(cuda_lib):
    L = cuda_lib
    _rate(L, 128, 256, 3)  # warm-up
    c256 = _rate(L, 128, 256, 3)
    c128 = _rate(L, 128, 128, 3)
    c64 = _rate(L, 128, 64, 3)
    c32 = _rate(L, 128, 32, 3)
    m64 = _rate(L, 64, 256, 3)
    assert 0.8 * 128 <= c256 <= 1.25 * 128
    assert 1.7 <= c256 / c128 <= 2.3
    # the narrow-MMA floor: halving N from 64 to 32 saves almost nothing
    assert c32 >= 0.8 * c64
    assert c64 >= 0.6 * c128
    # M = 64 runs at half the MAC rate of M = 128
    assert 0.8 <= m64 / c256 <= 1.25


def test_mma_rate_layout_independent(cuda_lib):
    L = cuda_lib
    costs = [_rate(L, 128, 128, layout) for layout in range(4)]
    assert max(costs) <= 1.15 * min(costs)


def test_mma_rate_rejects_bad_arguments(cuda_lib):
    L = cuda_lib
    c = ctypes.c_double(0.0)
    assert L.spinn_cuda_diag_mma_rate(96, 128, 3, 16, ctypes.byref(c)) == EINVAL
    assert L.spinn_cuda_diag_mma_rate(128, 264, 3, 16, ctypes.byref(c)) == EINVAL
    assert L.spinn_cuda_diag_mma_rate(128, 40, 3, 16, ctypes.byref(c)) == EINVAL
    assert L.spinn_cuda_diag_mma_rate(128, 128, 4, 16, ctypes.byref(c)) == EINVAL
    assert L.spinn_cuda_diag_mma_rate(128, 128, 3, 0, ctypes.byref(c)) == EINVAL
    assert L.spinn_cuda_diag_mma_rate(128, 128, 3, 16, None) == EINVAL
    assert L.spinn_cuda_sync() == 0
