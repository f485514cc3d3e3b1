"""The benchmark configurations other than ResNet-101 (which tests/test_gpu_parity.py covers),
at the sizes the benchmark statement names and config_bench times, through the device runtime
against the reference's own CPU runtime (oracle/_ref, O-fix) on identical seeded inputs.

* configuration 1: the Gemm sweep Y = A B + C, (M, N, K) in {256, 1024, 4096}^3 and the ResNet
  FC shape (M=256, K=2048, N=1000, transB 0 and 1), against op_gemm
  (SPINN/run_time/ops/mm/gemm.c:7-78; alpha = beta = 1, where the reference is exact);
* configuration 2: ResNet-50 at batch 1 and 64;
* configuration 4: the YOLOv10n-shaped detector at batch 32 (640x640);
* the standalone BatchNormalization and unfused Relu device steps the converter leaves in a
  graph when no convolution precedes them (SPINN/run_time/ops/norm/batch_norm.c:17-76,
  ops/activation/relu.c:4-18).
"""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

SIZES = (256, 1024, 4096)
CFG1 = [(m, n, k, 0) for m in SIZES for n in SIZES for k in SIZES] + [(256, 1000, 2048, 0), (256, 1000, 2048, 1)]


def _ref(ref_oracle, tmp_path, img, x):
    p = tmp_path / "m.ennf"
    p.write_bytes(img)
    return list(ref_oracle.run_model(str(p), x).values())[0]


@pytest.mark.parametrize("m,n,k,tb", CFG1, ids=lambda v: str(v))
def test_cfg1_gemm_sweep(cuda_lib, ref_oracle, tmp_path, m, n, k, tb):
    from spinn_b200 import ennf, netdef, runtime
    g, a = netdef.gemm_case(m, n, k, trans_b=tb)
    img = ennf.convert(g)
    ref = _ref(ref_oracle, tmp_path, img, a).reshape(m, n)
    model = runtime.Model(img)
    y = model.run(a).reshape(m, n)
    model.close()
    assert np.isfinite(y).all()
    assert rel_l2(y, ref) <= 2e-3, rel_l2(y, ref)


@pytest.mark.parametrize("batch", [1, 64])
def test_cfg2_resnet50(cuda_lib, ref_oracle, tmp_path, batch):
    from spinn_b200 import ennf, netdef, runtime
    g = netdef.resnet(50, batch=batch, seed=2)
    x = netdef.resnet_input(batch, seed=2)
    img = ennf.convert(g)
    ref = _ref(ref_oracle, tmp_path, img, x).reshape(batch, -1)
    model = runtime.Model(img)
    y = model.run(x).reshape(batch, -1)
    model.close()
    scale = float(np.abs(ref).max())
    assert rel_l2(y, ref) <= 2e-3, rel_l2(y, ref)
    assert float(np.abs(y - ref).max()) <= 1e-2 * scale
    assert (y.argmax(1) == ref.argmax(1)).all()


def test_cfg4_yolo_shaped_batch32(cuda_lib, ref_oracle, tmp_path):
    from spinn_b200 import ennf, netdef, runtime
    g = netdef.yolo_shaped(batch=32, image=640)
    x = netdef.yolo_input(32, 640)
    img = ennf.convert(g)
    ref = _ref(ref_oracle, tmp_path, img, x)
    model = runtime.Model(img)
    y = model.run(x).ravel()
    model.close()
    assert rel_l2(y, ref) <= 2e-3, rel_l2(y, ref)
    assert float(np.abs(y - ref).max()) <= 1e-2          # absolute, as the benchmark states
    cls_y = y.reshape(32, 144, -1)[:, 64:]
    cls_r = ref.reshape(32, 144, -1)[:, 64:]
    top2 = np.sort(cls_r, axis=1)[:, -2:]
    robust = (top2[:, 1] - top2[:, 0]) > 1e-2
    assert (cls_y.argmax(1) == cls_r.argmax(1))[robust].all()


def _bn_relu_graph(batch, c, hw, relu: bool, bn: bool, seed=5):
    from spinn_b200 import netdef
    rng = np.random.default_rng(seed)
    g = netdef.Graph("bn_relu")
    b = netdef._Builder(g, rng)
    x = g.add_input("input", (batch, c, hw, hw))
    y = b.bn(x) if bn else x
    if relu:
        y = b.unary("Relu", y)
    g.mark_output(y)
    return g, rng.standard_normal((batch, c, hw, hw)).astype(np.float32)


@pytest.mark.parametrize("bn,relu,shape", [(True, False, (2, 64, 28)), (True, True, (3, 30, 17)),
                                           (False, True, (2, 6, 33))],
                         ids=["batchnorm", "batchnorm+relu", "relu"])
def test_standalone_batchnorm_and_relu(cuda_lib, ref_oracle, tmp_path, bn, relu, shape):
    """BatchNormalization that follows no convolution (not folded) and Relu that follows no
    convolution (not fused) run as their own device steps."""
    from spinn_b200 import ennf, lib, runtime
    g, x = _bn_relu_graph(*shape, relu=relu, bn=bn)
    img = ennf.convert(g)
    em = ennf.read(img)
    ops = [ennf.OP_NAME[nd.op_type] for nd in em.nodes]
    assert ops == (["BatchNormalization"] if bn else []) + (["Relu"] if relu else [])
    ref = _ref(ref_oracle, tmp_path, img, x)
    # the default plan rounds the graph input to tf32 when it converts it to NHWC (it feeds
    # tensor-core convolutions elsewhere); NO_ROUND keeps fp32 end to end
    for flags, tol in ((0, 2e-3), (lib.PLAN_NO_ROUND, 1e-6)):
        model = runtime.Model(img, flags=flags)
        y = model.run(x).ravel()
        model.close()
        assert rel_l2(y, ref) <= tol, (flags, rel_l2(y, ref))
        if relu:
            assert (y >= 0).all()
