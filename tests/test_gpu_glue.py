"""Device glue operators of the YOLO-shaped graphs (Split, Concat, Resize, Reshape, Transpose,
MatMul, Softmax, scalar Mul, Sigmoid, unfused Add) on small graphs, against the reference
runtime (oracle/_ref) on identical inputs."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def _run_both(ref_oracle, tmp_path, g, x):
    from spinn_b200 import ennf, runtime
    img = ennf.convert(g)
    p = tmp_path / "m.ennf"
    p.write_bytes(img)
    ref = list(ref_oracle.run_model(str(p), x).values())[0]
    y = runtime.Model(img).run(x).ravel()
    return y, ref


def _builder(shape, seed=0):
    from spinn_b200 import netdef
    g = netdef.Graph("glue")
    b = netdef._Builder(g, np.random.default_rng(seed))
    x = g.add_input("x", shape)
    xv = np.random.default_rng(seed + 1).uniform(-1, 1, shape).astype(np.float32)
    return g, b, x, xv


def test_split_concat_nhwc(cuda_lib, ref_oracle, tmp_path):
    g, b, x, xv = _builder((2, 8, 10, 10))
    y = b.conv_bn(x, 24, 3, 1)
    a, c = b.split2(y)
    y = b.concat([b.conv_bn(a, 12, 3, 1), c, b.conv_bn(c, 6, 1, 1)])   # 30 channels: pad lane zeroed
    y = b.conv_bn(y, 16, 3, 1)
    g.mark_output(y)
    out, ref = _run_both(ref_oracle, tmp_path, g, xv)
    assert rel_l2(out, ref) <= 2e-3, rel_l2(out, ref)


def test_resize_and_unfused_add(cuda_lib, ref_oracle, tmp_path):
    g, b, x, xv = _builder((1, 16, 7, 9))
    y = b.conv_bn(x, 16, 3, 1)
    y = b.upsample2(y)
    z = b.conv_bn(y, 16, 3, 1)
    y = b.add(z, y)                      # conv output has two consumers: Add stays a node
    y = b.conv_bn(y, 8, 1, 1, act="Relu")
    g.mark_output(y)
    out, ref = _run_both(ref_oracle, tmp_path, g, xv)
    assert rel_l2(out, ref) <= 2e-3, rel_l2(out, ref)


def test_attention_reshape_transpose_matmul_softmax(cuda_lib, ref_oracle, tmp_path):
    g, b, x, xv = _builder((2, 16, 6, 5))
    n, c, h, w = 2, 16, 6, 5
    qkv = b.conv_bn(x, 48, 1, 1, act=None)
    from spinn_b200.netdef import _split3
    q, k, v = (b.reshape(t, (n, 2, 8, h * w)) for t in _split3(b, qkv))
    att = b.softmax(b.scale(b.matmul(b.transpose(q, (0, 1, 3, 2)), k), 8 ** -0.5))
    o = b.reshape(b.matmul(v, b.transpose(att, (0, 1, 3, 2))), (n, 16, h, w))
    y = b.conv_bn(o, 16, 1, 1)
    g.mark_output(y)
    out, ref = _run_both(ref_oracle, tmp_path, g, xv)
    assert rel_l2(out, ref) <= 2e-3, rel_l2(out, ref)


def test_row_concat_and_sigmoid(cuda_lib, ref_oracle, tmp_path):
    g, b, x, xv = _builder((2, 8, 4, 4))
    y1 = b.reshape(b.conv_bn(x, 12, 3, 1), (2, 12, 16))
    y2 = b.reshape(b.conv_bn(x, 12, 1, 1), (2, 12, 16))
    y = b.unary("Sigmoid", b.concat([y1, y2], axis=2))
    g.mark_output(y)
    out, ref = _run_both(ref_oracle, tmp_path, g, xv)
    assert rel_l2(out, ref) <= 2e-3, rel_l2(out, ref)


@pytest.mark.parametrize("shape,k", [((2, 1000), 50), ((2, 8400), 300), ((4, 37), 100), ((3, 16384), 5)])
def test_topk_matches_reference(cuda_lib, ref_oracle, tmp_path, shape, k):
    """Device TopK against the reference op_topk: values and int64 indices identical,
    including ties and signed zeros."""
    from spinn_b200 import ennf, netdef, runtime
    g = netdef.Graph("topk")
    b = netdef._Builder(g, np.random.default_rng(0))
    x = g.add_input("x", shape)
    v, i = b.topk(x, k)
    g.mark_output(v)
    g.mark_output(i)
    rng = np.random.default_rng(sum(shape) + k)
    xv = rng.normal(0, 1, shape).astype(np.float32)
    xv[:, ::7] = np.round(xv[:, ::7], 1)       # ties
    xv[:, ::11] = np.float32(-0.0)
    img = ennf.convert(g)
    p = tmp_path / "topk.ennf"
    p.write_bytes(img)
    m = ennf.read(img)
    ref = ref_oracle.run_model(str(p), xv)
    model = runtime.Model(img)
    model.run(xv)
    assert np.array_equal(model.output(0).ravel(), ref[m.outputs[0]])
    assert np.array_equal(model.output(1).ravel(), ref[m.outputs[1]].view(np.int64))


@pytest.mark.parametrize("shape", [(2, 64, 23, 29), (1, 12, 9, 9), (3, 16, 112, 112), (1, 80, 15, 14)],
                         ids=lambda s: "x".join(map(str, s)))
def test_maxpool_3x3_s2(cuda_lib, ref_oracle, tmp_path, shape):
    """The ResNet stem pool (3x3, stride 2, pad 1): tiled kernel for <= 64 channels (ragged
    tiles, padded channel lanes), the generic kernel above; identical values to op_maxpool."""
    g, b, x, xv = _builder(shape)
    y = b.maxpool(b.conv_bn(x, shape[1], 3, 1), 3, 2, 1)
    g.mark_output(y)
    out, ref = _run_both(ref_oracle, tmp_path, g, xv)
    assert rel_l2(out, ref) <= 2e-3, rel_l2(out, ref)


def test_concat_aligned_parts_one_launch(cuda_lib, ref_oracle, tmp_path):
    """NHWC channel concat whose parts are all multiples of 4 channels (the one-launch path),
    five parts, the destination's channel count padded to a multiple of 4 by nothing."""
    g, b, x, xv = _builder((2, 8, 9, 7))
    parts = [b.conv_bn(x, c, 1, 1) for c in (8, 16, 4, 12, 8)]
    y = b.conv_bn(b.concat(parts), 12, 3, 1)
    g.mark_output(y)
    out, ref = _run_both(ref_oracle, tmp_path, g, xv)
    assert rel_l2(out, ref) <= 2e-3, rel_l2(out, ref)


def test_concat_read_in_parts_matches_materialised(cuda_lib):
    """A channel Concat whose only reader is a tensor-core convolution is not materialised: the
    convolution fetches each channel block from the Concat's inputs.  Same instructions per
    element as the copied Concat (plan flag NO_FUSE), so the outputs are bit-identical."""
    from spinn_b200 import ennf, lib, netdef, runtime
    img = ennf.convert(netdef.yolo_shaped(batch=2, image=320))
    x = netdef.yolo_input(2, 320)
    em = ennf.read(img)
    n_cat = sum(1 for nd in em.nodes if ennf.OP_NAME.get(nd.op_type) == "Concat")
    outs, cats = [], []
    for flags in (0, lib.PLAN_NO_FUSE):
        m = runtime.Model(img, flags=flags | lib.PLAN_PROFILE)
        outs.append(m.run(x))
        m.run_profiled()
        cats.append(sum(1 for op, ms, fl in m.profile() if ennf.OP_NAME.get(op) == "Concat"))
        m.close()
    assert np.array_equal(outs[0], outs[1])
    assert cats[1] == n_cat and cats[0] < n_cat - 10, cats


def test_head_concat_gathered_from_nhwc_parts(cuda_lib, ref_oracle, tmp_path):
    """Detection-head pattern: per level a channel Concat of two convolution outputs, a Reshape
    [N, C, H, W] -> [N, C, H*W] and one last-axis Concat of the levels as the graph output.  The
    last Concat gathers straight from the NHWC convolution outputs (no NCHW copies, no channel
    Concat, no output staging copy); one level's view has a second reader and is materialised
    the ordinary way.  Against the reference, and bit-identical to the unfused plan."""
    from spinn_b200 import ennf, lib, runtime
    g, b, x, xv = _builder((2, 8, 12, 10))
    levels = []
    y = x
    for i, width in enumerate((8, 16, 24)):
        y = b.conv_bn(y, width, 3, 2 if i else 1)
        n, c, h, w = g.shape(y)
        box = b.conv(y, 5, 1, 1, 0, bias=True)      # odd channel counts: pad lanes in NHWC
        cls = b.conv(y, 7, 3, 1, 1, bias=True)
        levels.append(b.reshape(b.concat([box, cls]), (n, 12, h * w)))
    extra = b.unary("Sigmoid", levels[1])           # a second reader: that view is materialised
    g.mark_output(b.concat(levels, axis=2))
    g.mark_output(extra)
    img = ennf.convert(g)
    p = tmp_path / "m.ennf"
    p.write_bytes(img)
    refs = list(ref_oracle.run_model(str(p), xv).values())
    outs, steps = [], []
    for flags in (0, lib.PLAN_NO_FUSE):
        m = runtime.Model(img, flags=flags)
        m.run(xv)
        outs.append([m.output(0).ravel().copy(), m.output(1).ravel().copy()])
        steps.append(m.plan_info()["steps"])
        m.close()
    for got, ref in zip(outs[0], refs):
        assert rel_l2(got, ref) <= 2e-3, rel_l2(got, ref)
    for a, c in zip(outs[0], outs[1]):
        assert np.array_equal(a, c)
    assert steps[0] < steps[1], steps


@pytest.mark.parametrize("shape,perm", [((3, 5, 37, 70), (0, 1, 3, 2)), ((33, 65), (1, 0)), ((2, 4, 3, 6), (0, 2, 1, 3))])
def test_transpose_matches_reference(cuda_lib, ref_oracle, tmp_path, shape, perm):
    """Transpose as a graph node: a swap of the last two axes runs as tiled matrix transposes,
    other permutations through the general kernel; both exact."""
    g, b, x, xv = _builder(shape)
    g.mark_output(b.transpose(x, perm))
    out, ref = _run_both(ref_oracle, tmp_path, g, xv)
    assert np.array_equal(out, ref)
