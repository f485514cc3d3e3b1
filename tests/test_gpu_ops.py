"""Operator-level parity on the GPU: spinn_cuda_conv2d / _gemm / _matmul through the C ABI
against the reference operators (oracle/_ref, O-fix) or the C port on identical inputs.

Tolerance: per-layer relative L2 <= 2e-3 (tf32 operands, fp32 accumulation).
"""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _conv_case(rng, n, c, h, w, oc, k, s, p, group=1, act=0, bias=True, res=False):
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c // group * k * k)), (oc, c // group, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, oc).astype(np.float32) if bias else None
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    r = rng.uniform(-1, 1, (n, oc, oh, ow)).astype(np.float32) if res else None
    return x, wt, b, r, (n, oc, oh, ow)


CONV_CASES = [
    # n, c, h, w, oc, k, s, p, group, act, bias, res
    (1, 64, 56, 56, 64, 3, 1, 1, 1, 1, True, False),     # benchmark configuration 0
    (2, 32, 9, 11, 48, 3, 1, 1, 1, 0, True, False),      # ragged M tile, OC not a multiple of 32
    (1, 64, 14, 14, 256, 1, 1, 0, 1, 5, True, True),     # 1x1 + residual + ReLU
    (2, 64, 20, 20, 512, 1, 1, 0, 1, 5, True, True),     # 1x1 + residual, several M and N tiles
    (2, 128, 15, 15, 128, 3, 2, 1, 1, 1, True, False),   # stride 2, odd spatial size
    (1, 3, 32, 32, 64, 7, 2, 3, 1, 1, True, False),      # stem: C=3 (padded to 4), 7x7/s2
    (1, 16, 20, 20, 32, 3, 1, 1, 1, 3, True, False),     # C=16 (64-B swizzle), SiLU
    (1, 8, 12, 12, 24, 3, 1, 1, 1, 4, False, True),      # C=8 (32-B swizzle), +residual, no bias
    (2, 256, 7, 7, 512, 1, 2, 0, 1, 0, True, False),     # 1x1 stride 2 downsample shape
    (1, 1024, 14, 14, 256, 1, 1, 0, 1, 1, True, False),  # deep K
    (1, 256, 7, 7, 256, 3, 1, 1, 1, 5, True, True),      # split-K (2 tiles, 72 K blocks) + residual in the finish
    (3, 512, 7, 7, 2048, 1, 1, 0, 1, 3, True, False),    # split-K, SiLU applied after the reduction
    (1, 32, 40, 40, 32, 3, 1, 1, 32, 3, True, False),    # depthwise (shared-memory spatial tiles)
    (2, 36, 17, 23, 36, 3, 2, 1, 36, 1, True, False),    # depthwise, stride 2, a partial 32-channel group
    (1, 64, 31, 29, 64, 5, 1, 2, 64, 3, True, False),    # depthwise 5x5, ragged tiles, SiLU
    (2, 96, 20, 20, 96, 3, 1, 1, 96, 5, True, True),     # depthwise + residual + ReLU
    (1, 128, 9, 40, 128, 3, 2, 1, 128, 0, False, False),  # depthwise, stride 2, no bias
    (4, 128, 80, 80, 128, 3, 2, 1, 128, 3, True, False),  # depthwise, YOLO-shaped downsampling
    (1, 32, 10, 10, 64, 3, 1, 1, 4, 1, True, False),     # grouped (CUDA cores)
    (2, 16, 20, 20, 64, 3, 1, 1, 1, 1, True, False),     # C=16, N=64, K=144: resident-weight shapes fit
    (2, 64, 9, 11, 40, 1, 1, 0, 1, 3, True, False),      # 1x1, N=40 < 64, K=64, ragged everything
]


@pytest.mark.parametrize("case", CONV_CASES, ids=lambda c: "x".join(map(str, c[:9])) + f"-a{c[9]}")
def test_conv2d_vs_reference(cuda_lib, port_oracle, case):
    from spinn_b200 import runtime
    n, c, h, w, oc, k, s, p, g, act, bias, res = case
    rng = np.random.default_rng(hash(case) & 0xFFFF)
    x, wt, b, r, yshape = _conv_case(rng, n, c, h, w, oc, k, s, p, g, act, bias, res)
    params = runtime.conv_params((k, k), (s, s), (p, p, p, p), (1, 1), g, 0, act)
    y = np.zeros(yshape, np.float32)
    runtime.conv2d(x, wt, y, b, r, params)
    ref = port_oracle.conv2d(x, wt, b, r, (s, s), (p, p), (1, 1), g, act, yshape[2:])
    assert np.isfinite(y).all()
    assert rel_l2(y, ref) <= TOL, rel_l2(y, ref)


def test_conv2d_device_tensors(cuda_lib, ref_oracle):
    """Same conv with device (torch) tensors in and out, against the reference op_conv2d."""
    import torch
    from spinn_b200 import runtime
    rng = np.random.default_rng(7)
    x, wt, b, _, yshape = _conv_case(rng, 2, 64, 28, 28, 128, 3, 1, 1)
    params = runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 1)
    ref = ref_oracle.conv2d(x, wt, b, None, params, yshape)
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros(yshape, device="cuda")
    runtime.conv2d(xd, wt, yd, b, None, params)
    runtime.sync()
    assert rel_l2(yd.cpu().numpy(), ref) <= TOL


GEMM_CASES = [
    # m, n, k, transA, transB, alpha, beta, c
    (256, 1000, 2048, 0, 1, 1.0, 1.0, "vector"),   # ResNet FC
    (256, 1000, 2048, 0, 0, 1.0, 1.0, "vector"),
    (256, 256, 256, 0, 0, 1.0, 1.0, "full"),
    (1024, 256, 4096, 1, 0, 1.0, 1.0, None),
    (130, 70, 50, 0, 0, 1.0, 1.0, "vector"),        # ragged everything, K % 4 != 0 -> re-pitch
    (1, 1000, 2048, 0, 1, 0.5, 2.0, "vector"),      # M == 1, alpha/beta
]


@pytest.mark.parametrize("case", GEMM_CASES, ids=lambda c: "x".join(map(str, c[:5])))
def test_gemm_vs_reference(cuda_lib, port_oracle, case):
    from spinn_b200 import runtime
    m, n, k, ta, tb, alpha, beta, cmode = case
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a = rng.uniform(-1, 1, (k, m) if ta else (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (n, k) if tb else (k, n)).astype(np.float32)
    c = None
    if cmode == "vector":
        c = rng.uniform(-1, 1, n).astype(np.float32)
    elif cmode == "full":
        c = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    y = np.zeros((m, n), np.float32)
    runtime.gemm(a, b, y, c, runtime.gemm_params(alpha, beta, ta, tb))
    ref = port_oracle.gemm(a, b, c, m, n, k, ta, tb, alpha, beta)
    assert rel_l2(y, ref) <= TOL, rel_l2(y, ref)


@pytest.mark.parametrize("shape", [((64, 96), (96, 80)), ((3, 50, 64), (3, 64, 40)), ((4, 33, 20), (20, 12))])
def test_matmul(cuda_lib, port_oracle, shape):
    from spinn_b200 import runtime
    rng = np.random.default_rng(11)
    a = rng.uniform(-1, 1, shape[0]).astype(np.float32)
    b = rng.uniform(-1, 1, shape[1]).astype(np.float32)
    y = np.zeros(np.broadcast_shapes(a.shape[:-2], b.shape[:-2]) + (a.shape[-2], b.shape[-1]), np.float32)
    runtime.matmul(a, b, y)
    ref = port_oracle.matmul(a, b)
    assert rel_l2(y, ref) <= TOL


def test_weight_cache_follows_content_at_a_reused_address(cuda_lib, port_oracle):
    """Cached device weights are keyed by host pointer; rewriting the same buffer with new
    weights (as when a freed model's memory is reused) must not serve the stale copy."""
    from spinn_b200 import runtime
    rng = np.random.default_rng(21)
    a = rng.uniform(-1, 1, (64, 96)).astype(np.float32)
    b = rng.uniform(-1, 1, (80, 96)).astype(np.float32)
    y = np.zeros((64, 80), np.float32)
    runtime.gemm(a, b, y, None, runtime.gemm_params(1.0, 1.0, 0, 1))
    assert rel_l2(y, port_oracle.gemm(a, b, None, 64, 80, 96, 0, 1)) <= TOL
    b[...] = rng.uniform(-1, 1, b.shape)          # same address, new contents
    runtime.gemm(a, b, y, None, runtime.gemm_params(1.0, 1.0, 0, 1))
    assert rel_l2(y, port_oracle.gemm(a, b, None, 64, 80, 96, 0, 1)) <= TOL
    x = rng.uniform(-1, 1, (1, 16, 8, 8)).astype(np.float32)
    w = rng.normal(0, 0.3, (16, 16, 3, 3)).astype(np.float32)
    yc = np.zeros((1, 16, 8, 8), np.float32)
    params = runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 0)
    runtime.conv2d(x, w, yc, None, None, params)
    w[...] = rng.normal(0, 0.3, w.shape)
    runtime.conv2d(x, w, yc, None, None, params)
    assert rel_l2(yc, port_oracle.conv2d(x, w, None, None, (1, 1), (1, 1))) <= TOL


def test_split_k_is_deterministic(cuda_lib):
    """A split-K launch (one tile, many K slices) reduces its partial sums in a fixed order:
    repeated runs are bit-identical."""
    from spinn_b200 import runtime
    rng = np.random.default_rng(5)
    x, wt, b, _, yshape = _conv_case(rng, 1, 512, 7, 7, 128, 3, 1, 1)
    params = runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 1)
    outs = []
    for _ in range(3):
        y = np.zeros(yshape, np.float32)
        runtime.conv2d(x, wt, y, b, None, params)
        outs.append(y)
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


# bn,ksplit,pair[,bk,ms[,wr]]: CTA pairs (cta_group::2), single CTAs with two 128-row M sub-tiles
# and the same with resident weights (wr=1; where infeasible the planner falls back), each with
# and without split-K
PAIR_SHAPES = ["256,1,2", "128,1,2", "256,3,2", "128,2,2",
               "64,1,1,32,2", "128,1,1,64,2", "64,2,1,64,2", "128,3,1,32,2",
               "64,1,1,32,2,1", "64,1,1,64,2,1", "64,2,1,32,2,1"]
TC_CASES = [c for c in CONV_CASES if c[8] == 1]


@pytest.mark.parametrize("tiles", PAIR_SHAPES)
@pytest.mark.parametrize("case", TC_CASES, ids=lambda c: "x".join(map(str, c[:9])) + f"-a{c[9]}")
def test_conv2d_cta_pair_tiles(cuda_lib, port_oracle, monkeypatch, case, tiles):
    """The 256-row tiles -- 2-SM (cta_group::2) pairs and single CTAs with two M sub-tiles --
    with and without split-K, forced on every conv shape; a tile whose second half lies past
    the last row must store nothing there."""
    from spinn_b200 import runtime
    monkeypatch.setenv("SPINN_TC_TILES", tiles)
    n, c, h, w, oc, k, s, p, g, act, bias, res = case
    rng = np.random.default_rng(hash(case) & 0xFFFF)
    x, wt, b, r, yshape = _conv_case(rng, n, c, h, w, oc, k, s, p, g, act, bias, res)
    params = runtime.conv_params((k, k), (s, s), (p, p, p, p), (1, 1), g, 0, act)
    y = np.full(yshape, np.nan, np.float32)
    runtime.conv2d(x, wt, y, b, r, params)
    ref = port_oracle.conv2d(x, wt, b, r, (s, s), (p, p), (1, 1), g, act, yshape[2:])
    assert np.isfinite(y).all()
    assert rel_l2(y, ref) <= TOL, rel_l2(y, ref)


@pytest.mark.parametrize("tiles", PAIR_SHAPES)
@pytest.mark.parametrize("case", GEMM_CASES, ids=lambda c: "x".join(map(str, c[:5])))
def test_gemm_cta_pair_tiles(cuda_lib, port_oracle, monkeypatch, case, tiles):
    from spinn_b200 import runtime
    monkeypatch.setenv("SPINN_TC_TILES", tiles)
    m, n, k, ta, tb, alpha, beta, cmode = case
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a = rng.uniform(-1, 1, (k, m) if ta else (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (n, k) if tb else (k, n)).astype(np.float32)
    c = None
    if cmode == "vector":
        c = rng.uniform(-1, 1, n).astype(np.float32)
    elif cmode == "full":
        c = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    y = np.zeros((m, n), np.float32)
    runtime.gemm(a, b, y, c, runtime.gemm_params(alpha, beta, ta, tb))
    ref = port_oracle.gemm(a, b, c, m, n, k, ta, tb, alpha, beta)
    assert rel_l2(y, ref) <= TOL, rel_l2(y, ref)


# bn,ksplit,pair,bk,ms,wr,sk: stream-K forced with CTA pairs, 256/128-wide single CTAs and two
# M sub-tiles
SK_SHAPES = ["256,1,2,64,1,0,1", "128,1,2,64,1,0,1", "256,1,1,32,1,0,1", "128,1,1,64,1,0,1",
             "64,1,1,32,2,0,1", "128,1,1,64,2,0,1"]
SK_CONV_CASES = [
    # n, c, h, w, oc, k, s, p, group, act, bias, res -- each has at least two k-blocks per
    # worker for every SK shape, and tiles split over two or more workers
    (2, 256, 28, 28, 200, 3, 1, 1, 1, 1, True, False),   # 3x3; last 256-row tile 32 rows; N ragged
    (8, 256, 14, 14, 256, 3, 1, 1, 1, 3, True, False),   # ResNet 14x14 3x3 shape, SiLU
    (16, 1024, 14, 14, 256, 1, 1, 0, 1, 0, False, False),  # 1x1, deep K, no bias
    (8, 16, 64, 64, 64, 3, 1, 1, 1, 1, True, False),     # C=16 (64-B swizzle), 3-5 k-blocks a tile
]


def _sk_launches():
    from spinn_b200 import lib
    return lib.lib().spinn_cuda_stat_streamk_launches()


@pytest.mark.parametrize("tiles", SK_SHAPES)
@pytest.mark.parametrize("case", SK_CONV_CASES, ids=lambda c: "x".join(map(str, c[:9])))
def test_conv2d_stream_k(cuda_lib, port_oracle, monkeypatch, case, tiles):
    """Stream-K: every worker an equal share of the k-blocks across tile boundaries; a tile
    split between workers is finished by the one holding its first k-blocks, which adds the
    others' partial sums after a flag handoff.  Results match the oracle, the schedule really
    ran, and repeated runs are bit-identical (partials added in worker order)."""
    from spinn_b200 import runtime
    monkeypatch.setenv("SPINN_TC_TILES", tiles)
    n, c, h, w, oc, k, s, p, g, act, bias, res = case
    rng = np.random.default_rng(hash(case) & 0xFFFF)
    x, wt, b, r, yshape = _conv_case(rng, n, c, h, w, oc, k, s, p, g, act, bias, res)
    params = runtime.conv_params((k, k), (s, s), (p, p, p, p), (1, 1), g, 0, act)
    ref = port_oracle.conv2d(x, wt, b, r, (s, s), (p, p), (1, 1), g, act, yshape[2:])
    outs = []
    for _ in range(2):
        before = _sk_launches()
        y = np.full(yshape, np.nan, np.float32)
        runtime.conv2d(x, wt, y, b, r, params)
        assert _sk_launches() > before, "stream-K schedule not taken"
        assert np.isfinite(y).all()
        assert rel_l2(y, ref) <= TOL, rel_l2(y, ref)
        outs.append(y)
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("tiles", SK_SHAPES)
def test_gemm_stream_k(cuda_lib, port_oracle, monkeypatch, tiles):
    from spinn_b200 import runtime
    monkeypatch.setenv("SPINN_TC_TILES", tiles)
    rng = np.random.default_rng(17)
    m, n, k = 1100, 300, 4000
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = rng.uniform(-1, 1, n).astype(np.float32)
    y = np.zeros((m, n), np.float32)
    before = _sk_launches()
    runtime.gemm(a, b, y, c, runtime.gemm_params(0.5, 1.0, 0, 0))
    assert _sk_launches() > before, "stream-K schedule not taken"
    ref = port_oracle.gemm(a, b, c, m, n, k, 0, 0, 0.5, 1.0)
    assert rel_l2(y, ref) <= TOL, rel_l2(y, ref)


def test_stream_k_chosen_for_short_last_wave(cuda_lib, port_oracle):
    """The planner takes stream-K by itself where whole tiles would leave a short last wave
    behind a long reduction (ResNet's 7x7 512-channel 3x3 layer at 256 images: 98 pair tiles
    of 72 k-blocks on 74 pair slots)."""
    from spinn_b200 import runtime
    rng = np.random.default_rng(23)
    x, wt, b, r, yshape = _conv_case(rng, 256, 512, 7, 7, 512, 3, 1, 1, 1, 1, True, False)
    params = runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 1)
    before = _sk_launches()
    y = np.zeros(yshape, np.float32)
    runtime.conv2d(x, wt, y, b, r, params)
    assert _sk_launches() > before
    for sl in (slice(0, 2), slice(254, 256)):  # first and last rows of the problem
        ref = port_oracle.conv2d(x[sl], wt, b, None, (1, 1), (1, 1), (1, 1), 1, 1, yshape[2:])
        assert rel_l2(y[sl], ref) <= TOL, rel_l2(y[sl], ref)


@pytest.mark.parametrize("tiles", [None, "256,1,2", "128,1,1", "64,1,1,64,2"])
def test_matmul_batched_one_launch(cuda_lib, port_oracle, monkeypatch, tiles):
    """Batched MatMul runs as one launch over [batch][M][K] planes (3-D tensor maps, the batch
    index in the work unit), with single CTAs, CTA pairs and two M sub-tiles, shared and
    per-batch B."""
    from spinn_b200 import runtime
    if tiles:
        monkeypatch.setenv("SPINN_TC_TILES", tiles)
    rng = np.random.default_rng(13)
    for sa, sb in (((6, 300, 64), (6, 64, 200)), ((5, 129, 36), (36, 70))):
        a = rng.uniform(-1, 1, sa).astype(np.float32)
        b = rng.uniform(-1, 1, sb).astype(np.float32)
        y = np.zeros(np.broadcast_shapes(a.shape[:-2], b.shape[:-2]) + (a.shape[-2], b.shape[-1]), np.float32)
        runtime.matmul(a, b, y)
        assert rel_l2(y, port_oracle.matmul(a, b)) <= TOL
