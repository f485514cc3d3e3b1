"""CPU checks of the oracle itself: the C port against the reference's golden vectors
(tests/golden/spinn_ref_vectors.npz, made by tests/golden/make_golden.py from the reference
operators) and against the reference library on random shapes, plus the reference
behaviours the design depends on (dropped group==1 epilogue, Gemm alpha quirk, MatMul
broadcast)."""
import os

import numpy as np
import pytest

from conftest import ROOT, rel_l2

GOLDEN = os.path.join(ROOT, "tests", "golden", "spinn_ref_vectors.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_golden_winograd_kats_pass_reference_criterion(golden):
    # SPINN/run_time/test_winograd.c:175 -- pass if max |diff| < 0.1
    assert np.abs(golden["kat1_conv"] - golden["kat1_wino"]).max() < 0.1
    assert np.abs(golden["kat2_conv"] - golden["kat2_wino"]).max() < 0.1
    # identity-diagonal kernel: y = x[i-1][j-1] + x[i][j] + x[i+1][j+1]
    x = golden["kat2_x"][0, 0]
    xp = np.pad(x, 1)
    expect = xp[:-2, :-2] + xp[1:-1, 1:-1] + xp[2:, 2:]
    assert np.array_equal(golden["kat2_conv"][0, 0], expect)


def test_port_reproduces_golden_convs(port_oracle, golden):
    g = golden
    y = port_oracle.conv2d(g["kat1_x"], g["kat1_w"], g["kat1_b"], pads=(1, 1))
    assert rel_l2(y, g["kat1_conv"]) < 1e-6
    y = port_oracle.conv2d(g["conv_res_x"], g["conv_res_w"], g["conv_res_b"], g["conv_res_r"], pads=(1, 1), act=5)
    assert rel_l2(y, g["conv_res_y"]) < 1e-6
    y = port_oracle.conv2d(g["conv_s2_x"], g["conv_s2_w"], g["conv_s2_b"], stride=(2, 2), pads=(1, 1), act=1)
    assert rel_l2(y, g["conv_s2_y"]) < 1e-6


def test_port_reproduces_golden_winograd_f23(port_oracle, golden):
    g = golden
    y = port_oracle.winograd_f23(g["kat1_x"], g["kat1_w"], g["kat1_b"], 1, 1, 4, 4, 0)
    assert np.abs(y - g["kat1_wino"]).max() < 1e-5
    y = port_oracle.winograd_f23(g["kat2_x"], g["kat2_w"], np.zeros(1, np.float32), 1, 1, 4, 4, 0)
    assert np.array_equal(y, g["kat2_wino"])


def test_port_reproduces_golden_gemm_matmul(port_oracle, golden):
    g = golden
    y = port_oracle.gemm(g["gemm_a"], g["gemm_b"], g["gemm_c"], 5, 7, 9, 0, 1, 1.0, 1.0)
    assert rel_l2(y, g["gemm_y"]) < 1e-6
    # the reference scales beta*C by alpha as well when M > 1 (gemm.c:62-69 + gemm_kernel.c:298-301)
    quirk = port_oracle.gemm(g["gemm_a"], g["gemm_b"], g["gemm_c"], 5, 7, 9, 0, 1, 0.5, 2.0, ref_quirk=1)
    assert rel_l2(quirk, g["gemm_alpha_y"]) < 1e-6
    onnx = port_oracle.gemm(g["gemm_a"], g["gemm_b"], g["gemm_c"], 5, 7, 9, 0, 1, 0.5, 2.0)
    assert rel_l2(onnx, g["gemm_alpha_y"]) > 1e-2
    y = port_oracle.matmul(g["matmul_a"], g["matmul_b"])
    assert rel_l2(y, g["matmul_y"]) < 1e-6


def test_reference_reproduces_golden(ref_oracle, golden):
    """The built reference is deterministic: it regenerates the committed vectors."""
    from spinn_b200 import runtime
    g = golden
    p5 = runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 5)
    y = ref_oracle.conv2d(g["conv_res_x"], g["conv_res_w"], g["conv_res_b"], g["conv_res_r"], p5, (2, 12, 10, 10))
    assert np.array_equal(y, g["conv_res_y"])


CONV_SHAPES = [
    # n, c, h, w, oc, k, s, p, group, act
    (1, 16, 12, 12, 24, 3, 1, 1, 1, 1),
    (2, 8, 11, 9, 8, 1, 1, 0, 1, 0),
    (1, 12, 13, 13, 16, 3, 2, 1, 1, 3),
    (1, 3, 20, 20, 16, 7, 2, 3, 1, 1),
    (1, 16, 10, 10, 16, 3, 1, 1, 16, 1),   # depthwise: reference takes sgemm_nn per group
    (1, 16, 8, 8, 32, 3, 1, 1, 4, 0),
    (2, 8, 7, 7, 8, 3, 1, 1, 1, 5),
]


@pytest.mark.parametrize("case", CONV_SHAPES)
def test_port_vs_reference_conv(ref_oracle, port_oracle, case):
    from spinn_b200 import runtime
    n, c, h, w, oc, k, s, p, g, act = case
    rng = np.random.default_rng(sum(case))
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, 0.2, (oc, c // g, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, oc).astype(np.float32)
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    r = rng.uniform(-1, 1, (n, oc, oh, ow)).astype(np.float32) if act in (4, 5) else None
    params = runtime.conv_params((k, k), (s, s), (p, p, p, p), (1, 1), g, 0, act)
    ref = ref_oracle.conv2d(x, wt, b, r, params, (n, oc, oh, ow))
    port = port_oracle.conv2d(x, wt, b, r, (s, s), (p, p), (1, 1), g, act, (oh, ow))
    assert rel_l2(port, ref) < 1e-5


def test_shipped_reference_drops_group1_epilogue(ref_oracle, port_oracle):
    """O-ship: op_conv2d's group==1 path returns the bare convolution (gemm_kernel.c:497-590)."""
    from spinn_b200 import runtime
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (1, 8, 6, 6)).astype(np.float32)
    w = rng.normal(0, 0.3, (8, 8, 3, 3)).astype(np.float32)
    b = rng.normal(0, 1.0, 8).astype(np.float32)
    params = runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 1)
    try:
        ref_oracle.set_fix(False)
        shipped = ref_oracle.conv2d(x, w, b, None, params, (1, 8, 6, 6))
    finally:
        ref_oracle.set_fix(True)
    bare = port_oracle.conv2d(x, w, None, None, (1, 1), (1, 1), (1, 1), 1, 0)
    fixed = port_oracle.conv2d(x, w, b, None, (1, 1), (1, 1), (1, 1), 1, 1)
    assert rel_l2(shipped, bare) < 1e-6
    assert (shipped < 0).any() and rel_l2(shipped, fixed) > 0.1


@pytest.mark.parametrize("ta,tb,cmode,alpha,beta", [(0, 0, "vec", 1.0, 1.0), (0, 1, "full", 1.0, 1.0),
                                                    (1, 0, None, 1.0, 1.0), (1, 1, "vec", 1.0, 0.5)])
def test_port_vs_reference_gemm(ref_oracle, port_oracle, ta, tb, cmode, alpha, beta):
    from spinn_b200 import runtime
    m, n, k = 17, 23, 29
    rng = np.random.default_rng(ta * 2 + tb)
    a = rng.uniform(-1, 1, (k, m) if ta else (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (n, k) if tb else (k, n)).astype(np.float32)
    c = None if cmode is None else rng.uniform(-1, 1, (n,) if cmode == "vec" else (m, n)).astype(np.float32)
    ref = ref_oracle.gemm(a, b, c, runtime.gemm_params(alpha, beta, ta, tb), (m, n))
    port = port_oracle.gemm(a, b, c, m, n, k, ta, tb, alpha, beta)
    assert rel_l2(port, ref) < 1e-5


def test_reference_matmul_broadcast_branch_is_unreachable(ref_oracle, port_oracle):
    """op_matmul returns -1 for batched A with a 2-D B (matmul.c:32-44 cannot be reached);
    the port (and spinn_cuda_matmul) broadcast B as ONNX specifies."""
    rng = np.random.default_rng(9)
    a = rng.uniform(-1, 1, (3, 4, 5)).astype(np.float32)
    b = rng.uniform(-1, 1, (5, 6)).astype(np.float32)
    with pytest.raises(RuntimeError):
        ref_oracle.matmul(a, b, (3, 4, 6))
    y = port_oracle.matmul(a, b)
    assert rel_l2(y, np.einsum("bmk,kn->bmn", a.astype(np.float64), b.astype(np.float64))) < 1e-6


def test_winograd_f43_matches_direct(port_oracle):
    rng = np.random.default_rng(4)
    for (n, c, hw, oc) in [(1, 8, 8, 8), (2, 5, 11, 7), (1, 16, 14, 16)]:
        x = rng.uniform(-1, 1, (n, c, hw, hw)).astype(np.float32)
        w = rng.normal(0, 0.3, (oc, c, 3, 3)).astype(np.float32)
        b = rng.normal(0, 0.1, oc).astype(np.float32)
        direct = port_oracle.conv2d(x, w, b, None, (1, 1), (1, 1), (1, 1), 1, 1)
        wino = port_oracle.winograd_f43(x, w, b, act=1)
        assert rel_l2(wino, direct) < 1e-5


def _topk_graph(shape, k):
    from spinn_b200 import netdef
    g = netdef.Graph("topk")
    b = netdef._Builder(g, np.random.default_rng(0))
    x = g.add_input("x", shape)
    v, i = b.topk(x, k)
    g.mark_output(v)
    g.mark_output(i)
    return g


@pytest.mark.parametrize("shape,k", [((2, 1000), 50), ((1, 8400), 300), ((4, 37), 100)])
def test_topk_reference_matches_port_with_ties(ref_oracle, port_oracle, tmp_path, shape, k):
    """op_topk (topk.c) on inputs with many equal values and signed zeros: values descending,
    ties in ascending index order (glibc qsort is a stable merge sort), k clamped to the axis."""
    from spinn_b200 import ennf
    rng = np.random.default_rng(sum(shape) + k)
    x = (rng.integers(-6, 7, shape) * 0.25).astype(np.float32)
    x[x == 0] = np.where(rng.random(int((x == 0).sum())) < 0.5, np.float32(-0.0), np.float32(0.0))
    img = ennf.convert(_topk_graph(shape, k))
    path = tmp_path / "topk.ennf"
    path.write_bytes(img)
    m = ennf.read(img)
    vid, iid = m.outputs
    ref = ref_oracle.run_model(str(path), x)
    port = port_oracle.run_model(img, x)
    assert np.array_equal(ref[vid], port[vid])
    assert np.array_equal(ref[iid].view(np.int64), port[iid])
