"""Device timings for the benchmark configurations other than ResNet-101 batch 256 (which
``bench.py`` measures): one JSON line per case.

    python -m spinn_b200.config_bench [--only cfg0,cfg1,cfg2,cfg4] [--iters 20]

* cfg0 -- Conv3x3(pad 1)+BN+ReLU, C=OC=64, 56x56, batch 1 and 256, im2col (tcgen05 implicit
  GEMM) and Winograd F(4x4,3x3) plans.
* cfg1 -- Gemm Y = A B + C, (M, N, K) in {256, 1024, 4096}^3 and the ResNet FC shape
  (M=256, K=2048, N=1000, transB 0/1).
* cfg2 -- ResNet-50, batch 1 and 64.
* cfg4 -- the YOLOv10n-shaped network (``netdef.yolo_shaped``), 640x640, batch 1 and 32.

Every case is planned once (weights uploaded, graph captured), its input staged on the device,
and the captured step list replayed: ``ms`` is the mean device time per run from CUDA events on
the launching stream after warm-up.  ``tflops`` uses algorithmic FLOPs (direct-convolution
FLOPs also for Winograd plans).  Synthetic data (seeded) stands in for the reference's models
and datasets.
"""
from __future__ import annotations

import argparse
import json


def _time(model, iters: int, warmup: int) -> float:
    import torch
    stream = torch.cuda.Stream()
    for _ in range(warmup):
        model.run_device(stream.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        model.run_device(stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def _case(name, graph, x, iters, warmup, flags=0, per_item=None, **extra):
    from spinn_b200 import ennf, runtime
    model = runtime.Model(ennf.convert(graph), flags=flags)
    model.run(x)  # stages the input on the device and validates the plan
    ms = _time(model, iters, warmup)
    flops = float(graph.flops())
    line = {"case": name, "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1), **extra}
    if per_item:
        line["items_per_s"] = round(per_item / ms * 1e3, 1)
    info = model.plan_info()
    line["steps"], line["kernels"] = info["steps"], info["kernels"]
    model.close()
    print(json.dumps(line), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="cfg0,cfg1,cfg2,cfg4")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    which = set(a.only.split(","))

    from spinn_b200 import lib, netdef

    if "cfg0" in which:
        for batch in (1, 256):
            g, x = netdef.conv_bn_relu(batch=batch)
            for plan, flags in (("im2col", 0), ("winograd", lib.PLAN_WINOGRAD)):
                _case(f"cfg0 conv3x3 64->64 56x56 batch {batch} {plan}", g, x, a.iters, a.warmup, flags,
                      per_item=batch)
    if "cfg1" in which:
        sizes = (256, 1024, 4096)
        for m in sizes:
            for n in sizes:
                for k in sizes:
                    g, x = netdef.gemm_case(m, n, k)
                    _case(f"cfg1 gemm M={m} N={n} K={k}", g, x, a.iters, a.warmup)
        for tb in (0, 1):
            g, x = netdef.gemm_case(256, 1000, 2048, trans_b=tb)
            _case(f"cfg1 gemm FC M=256 N=1000 K=2048 transB={tb}", g, x, a.iters, a.warmup)
    if "cfg2" in which:
        for batch in (1, 64):
            g = netdef.resnet(50, batch=batch, seed=2)
            _case(f"cfg2 resnet50 batch {batch}", g, netdef.resnet_input(batch, seed=2), a.iters, a.warmup,
                  per_item=batch)
    if "cfg4" in which:
        for batch in (1, 32):
            g = netdef.yolo_shaped(batch=batch, image=640)
            _case(f"cfg4 yolo-shaped 640 batch {batch}", g, netdef.yolo_input(batch, 640), a.iters, a.warmup,
                  per_item=batch)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
