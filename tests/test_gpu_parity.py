"""Parity of the benchmarked path itself: ResNet-101 (benchmark configuration 3) planned exactly
as bench.py plans it, at the global batch of 256 and at every per-GPU shard the 2/4/8-GPU runs
use (128 / 64 / 32 images, which select other tile shapes, split-K and CTA pairs), against the
reference's own CPU runtime (oracle/_ref, O-fix: SPINN/run_time/spinn_runtime.c:298-355) on the
same images.  Images are independent, so sampled images of a large GPU batch are checked
against a small CPU batch of exactly those images (the reference planner cannot plan batch 256:
its arena is clamped to INT_MAX bytes, SPINN/run_time/spinn_memory_planner.c:251).

Per-layer checks use the plan flag KEEP (every intermediate keeps its own arena range; the
kernels and their tile plans are those of the normal plan) and feed each convolution's own GPU
input through the reference operator (op_conv2d, SPINN/run_time/ops/conv/conv2d.c:92-232), so
that every layer is judged on its own error rather than the accumulated one.

Tolerances (the benchmark statement): per layer relative L2 <= 2e-3; end to end relative L2
<= 2e-3, identical argmax, max |error| <= 1e-2 of max |reference| (random He-init ResNet-101
logits reach ~1e8, where the absolute 1e-2 is far below fp32 resolution; see test_gpu_models).
"""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

DEPTH, SEED, IMAGE = 101, 3, 224


def _bench_model_image(batch: int):
    """The .ennf image bench.py builds (bench.build_model_image)."""
    import bench
    img, _ = bench.build_model_image(batch, DEPTH)
    return img


def _ref_logits(ref_oracle, tmp_path, images: np.ndarray) -> np.ndarray:
    p = tmp_path / f"r101_b{images.shape[0]}.ennf"
    p.write_bytes(_bench_model_image(images.shape[0]))
    return list(ref_oracle.run_model(str(p), images).values())[0].reshape(images.shape[0], -1)


def _check_logits(y, ref):
    scale = float(np.abs(ref).max())
    err = float(np.abs(y - ref).max())
    assert rel_l2(y, ref) <= 2e-3, rel_l2(y, ref)
    assert err <= 1e-2 * scale, (err, scale)
    assert (y.argmax(1) == ref.argmax(1)).all()


@pytest.mark.parametrize("shard,start", [(256, 0), (128, 128), (64, 192), (32, 224)],
                         ids=["1gpu-b256", "2gpu-rank1-b128", "4gpu-rank3-b64", "8gpu-rank7-b32"])
def test_resnet101_bench_plan_sampled_images(cuda_lib, ref_oracle, tmp_path, shard, start):
    """bench.py's model (plan flag PROFILE, the same graph it times) on rank `start // shard`'s
    shard of the global batch; the first four and last four images against the reference."""
    from spinn_b200 import lib, netdef, runtime
    m = runtime.Model(_bench_model_image(shard), flags=lib.PLAN_PROFILE)
    x = netdef.image_batch(start, shard, IMAGE, seed=SEED)
    y = m.run(x).reshape(shard, -1)
    m.close()
    idx = [0, 1, 2, 3, shard - 4, shard - 3, shard - 2, shard - 1]
    ref = _ref_logits(ref_oracle, tmp_path, x[idx])
    _check_logits(y[idx], ref)


def _per_layer(ref_oracle, model, em, images, max_rel=2e-3):
    """Every Conv (and MatMul) node of `em`: its GPU output for `images` against the reference
    operator applied to the GPU's own inputs of that node.  Returns the worst relative L2."""
    from spinn_b200 import ennf

    def dev(tid, i):
        return model.tensor(tid, em.tensors[tid].dims, i, 1)

    worst = 0.0
    checked = 0
    for k, nd in enumerate(em.nodes):
        op = ennf.OP_NAME.get(nd.op_type)
        if op not in ("Conv", "MatMul"):
            continue
        for i in images:
            y = dev(nd.outputs[0], i)
            if op == "Conv":
                p = ennf.ConvParams.unpack(nd.params)
                has_res = p.fused_act in (4, 5)
                n_real = len(nd.inputs) - (1 if has_res else 0)
                x = dev(nd.inputs[0], i)
                w = np.ascontiguousarray(em.weights[nd.inputs[1]])
                b = np.ascontiguousarray(em.weights[nd.inputs[2]]) if n_real > 2 else None
                r = dev(nd.inputs[-1], i) if has_res else None
                ref = ref_oracle.conv2d(x, w, b, r, nd.params, y.shape)
            else:
                a = dev(nd.inputs[0], i)
                bt = nd.inputs[1]
                bm = np.ascontiguousarray(em.weights[bt]) if bt in em.weights else dev(bt, i)
                ref = ref_oracle.matmul(a, bm, y.shape)
            e = rel_l2(y, ref)
            assert np.isfinite(y).all(), (k, op)
            assert e <= max_rel, (k, op, i, e)
            worst = max(worst, e)
            checked += 1
    return worst, checked


def test_resnet101_per_layer_b256(cuda_lib, ref_oracle):
    """All 104 convolutions of ResNet-101 at batch 256 (the tile plans bench.py times), images 0
    and 255, each layer against op_conv2d on the GPU's own input of that layer."""
    from spinn_b200 import ennf, lib, netdef, runtime
    img = _bench_model_image(256)
    em = ennf.read(img)
    m = runtime.Model(img, flags=lib.PLAN_KEEP)
    m.run(netdef.image_batch(0, 256, IMAGE, seed=SEED))
    worst, checked = _per_layer(ref_oracle, m, em, [0, 255])
    m.close()
    assert checked == 2 * 104
    print(f"ResNet-101 b256 per-layer worst relative L2 {worst:.2e}")


def test_resnet101_per_layer_b32(cuda_lib, ref_oracle):
    """The same at the 8-GPU shard size (32 images: split-K and other tile shapes)."""
    from spinn_b200 import ennf, lib, netdef, runtime
    img = _bench_model_image(32)
    em = ennf.read(img)
    m = runtime.Model(img, flags=lib.PLAN_KEEP)
    m.run(netdef.image_batch(224, 32, IMAGE, seed=SEED))
    worst, checked = _per_layer(ref_oracle, m, em, [31])
    m.close()
    assert checked == 104


def test_yolo_shaped_per_layer_b32(cuda_lib, ref_oracle):
    """Benchmark configuration 4 at batch 32: every Conv (tcgen05, depthwise and grouped) and
    every attention MatMul, image 0, against the reference operators on the GPU's own inputs."""
    from spinn_b200 import ennf, lib, netdef, runtime
    g = netdef.yolo_shaped(batch=32, image=640)
    img = ennf.convert(g)
    em = ennf.read(img)
    m = runtime.Model(img, flags=lib.PLAN_KEEP)
    m.run(netdef.yolo_input(32, 640))
    worst, checked = _per_layer(ref_oracle, m, em, [0])
    m.close()
    n_conv = sum(1 for nd in em.nodes if ennf.OP_NAME.get(nd.op_type) in ("Conv", "MatMul"))
    assert checked == n_conv


def test_copy_tensor_needs_keep_for_intermediates(cuda_lib):
    """Without KEEP only graph outputs may be read (an intermediate's arena range is reused)."""
    from spinn_b200 import ennf, lib, netdef, runtime
    g = netdef.resnet(50, batch=2, image=64, width=16, seed=9)
    img = ennf.convert(g)
    em = ennf.read(img)
    m = runtime.Model(img)
    x = netdef.resnet_input(2, image=64, seed=9)
    y = m.run(x)
    out = em.outputs[0]
    assert np.array_equal(m.tensor(out, em.tensors[out].dims), y.reshape(em.tensors[out].dims))
    conv_out = next(nd.outputs[0] for nd in em.nodes if ennf.OP_NAME.get(nd.op_type) == "Conv")
    with pytest.raises(lib.SpinnCudaError) as e:
        m.tensor(conv_out, em.tensors[conv_out].dims)
    assert e.value.code == lib.ESTATE
    m.close()
    k = runtime.Model(img, flags=lib.PLAN_KEEP)
    assert np.array_equal(k.run(x), y)  # same kernels, same numbers
    t = k.tensor(conv_out, em.tensors[conv_out].dims, 1, 1)
    assert t.shape == (1,) + tuple(em.tensors[conv_out].dims[1:]) and np.isfinite(t).all()
    with pytest.raises(lib.SpinnCudaError):
        k.tensor(conv_out, em.tensors[conv_out].dims, 2, 1)  # past the batch
    k.close()
