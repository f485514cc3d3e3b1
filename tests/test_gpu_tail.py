"""The bottleneck-tail kernel (tail.cu): a 1x1 expand with a fused residual (+ReLU) and the 1x1
reduce of its output in one launch, y kept on chip for the reduce.  The planner uses it when a
1x1 Conv with a fused Add (graph_opt.c's Conv+Add(+ReLU), SPINN/graph_opt.c:304-421) is followed
by a 1x1 Conv of its output and there are rows for two waves of 128-row tiles.

Checked here: the fused plan against the same model planned with NO_FUSE (every convolution
its own launch) and against the reference runtime (oracle/_ref, O-fix), on graphs built for
the purpose (ragged row counts, every reduce width the kernel takes, with and without the
reduce's ReLU) and on a ResNet-50 whose 56x56 stage fuses.
"""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _whole_tiles(monkeypatch):
    """The fused tail is compared bit for bit (1e-6) with the separate launches, which must
    then run as whole tiles: a stream-K launch sums a split tile's parts in another order."""
    monkeypatch.setenv("SPINN_NO_SK", "1")


def _tail_graph(batch, hw, n1, k1, n2, relu_reduce=True, seed=11):
    from spinn_b200 import netdef
    return netdef.bottleneck_tail(batch, hw, n1, k1, n2, relu_reduce, seed)


def _run(img, x, flags):
    from spinn_b200 import runtime
    m = runtime.Model(img, flags=flags)
    kinds = m.step_kinds()
    y = m.run(x)
    m.close()
    return y, kinds


# rows = batch * hw^2 must reach eight waves of 128-row tiles on 148 SMs (151,552)
TAIL_CASES = [
    # batch, hw, n1, k1, n2, relu on the reduce (the planner fuses expands of <= 128 input channels)
    (4, 199, 256, 64, 64, True),     # 158,404 rows: a partial last tile; the ResNet 56x56-stage widths
    (4, 200, 512, 128, 128, True),   # 160,000 rows, the ResNet 28x28-stage widths
    (3, 225, 1024, 64, 256, True),   # 151,875 rows, the widest reduce the kernel takes
    (5, 175, 256, 32, 96, False),    # 153,125 rows, K1 = 32, no ReLU after the reduce
]


@pytest.mark.parametrize("case", TAIL_CASES, ids=lambda c: "x".join(map(str, c[:5])) + ("-relu" if c[5] else ""))
def test_tail_fused_matches_unfused_and_reference(cuda_lib, ref_oracle, tmp_path, case):
    from spinn_b200 import ennf, lib
    batch, hw, n1, k1, n2, relu = case
    g, x = _tail_graph(batch, hw, n1, k1, n2, relu)
    img = ennf.convert(g)
    fused, kinds = _run(img, x, 0)
    assert 9 in kinds, kinds  # the tail kernel ran
    plain, kinds2 = _run(img, x, lib.PLAN_NO_FUSE)
    assert 9 not in kinds2
    assert np.isfinite(fused).all()
    # same accumulation order and epilogue as the separate launches
    assert rel_l2(fused, plain) <= 1e-6, rel_l2(fused, plain)
    p = tmp_path / "tail.ennf"
    p.write_bytes(img)
    ref = list(ref_oracle.run_model(str(p), x).values())[0].reshape(fused.shape)
    assert rel_l2(fused, ref) <= 2e-3, rel_l2(fused, ref)


def test_tail_fused_resnet50_stage1(cuda_lib, ref_oracle, tmp_path):
    """ResNet-50 at batch 64: the 56x56 stage has 200,704 rows, so its three block ends fuse
    (the first one is the stride-1 projection that carries the residual)."""
    from spinn_b200 import ennf, lib, netdef
    g = netdef.resnet(50, batch=64, seed=2)
    x = netdef.resnet_input(64, seed=2)
    img = ennf.convert(g)
    fused, kinds = _run(img, x, 0)
    assert kinds.count(9) == 3, kinds
    plain, _ = _run(img, x, lib.PLAN_NO_FUSE)
    fused, plain = fused.reshape(64, -1), plain.reshape(64, -1)
    assert rel_l2(fused, plain) <= 1e-6, rel_l2(fused, plain)
    p = tmp_path / "r50.ennf"
    p.write_bytes(img)
    ref = list(ref_oracle.run_model(str(p), x).values())[0].reshape(64, -1)
    assert rel_l2(fused, ref) <= 2e-3, rel_l2(fused, ref)
    assert float(np.abs(fused - ref).max()) <= 1e-2 * float(np.abs(ref).max())
    assert (fused.argmax(1) == ref.argmax(1)).all()
