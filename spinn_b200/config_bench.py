"""Device timings for the benchmark configurations other than ResNet-101 batch 256 (which
``bench.py`` measures): one JSON line per case.

    python -m spinn_b200.config_bench [--only cfg0,cfg1,cfg2,cfg4] [--iters 20]

* cfg0 -- Conv3x3(pad 1)+BN+ReLU, C=OC=64, 56x56, batch 1 and 256, im2col (tcgen05 implicit
  GEMM) and Winograd F(4x4,3x3) plans.
* cfg1 -- Gemm Y = A B + C, (M, N, K) in {256, 1024, 4096}^3 and the ResNet FC shape
  (M=256, K=2048, N=1000, transB 0/1).
* cfg2 -- ResNet-50, batch 1 and 64.
* cfg4 -- the YOLOv10n-shaped network (``netdef.yolo_shaped``), 640x640, batch 1 and 32.
* layer -- one fused convolution (Conv+BN+ReLU, optionally +residual or a projection shortcut)
  of a chosen shape, the unit the single-kernel ncu summaries capture; --tail times the
  bottleneck-tail pair fused and as separate launches:

    python -m spinn_b200.config_bench --layer --batch 128 --c 256 --hw 14 --oc 1024 --k 1 --projection
    python -m spinn_b200.config_bench --layer --tail --batch 4 --hw 199 --c 64 --oc 256 --tail-n2 64

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


def layer(a) -> int:
    """Times one fused convolution layer through the device runtime: device ms per run (CUDA
    events around the planned step list, inputs resident), algorithmic TFLOP/s and algorithmic
    GB/s (input + output [+ residual] + weights, each touched once)."""
    from spinn_b200 import lib, netdef

    pad = a.k // 2
    if a.tail:
        return tail(a)
    if a.projection:
        g, x = netdef.conv_bn_proj_add_relu(batch=a.batch, c=a.c, hw=a.hw, oc=a.oc, k=a.k)
    elif a.residual:
        g, x = netdef.conv_bn_add_relu(batch=a.batch, c=a.c, hw=a.hw)
    else:
        g, x = netdef.conv_bn_relu(batch=a.batch, c=a.c, hw=a.hw, oc=a.oc, k=a.k, stride=a.stride, pad=pad,
                                   group=a.group)
    from spinn_b200 import ennf, runtime
    model = runtime.Model(ennf.convert(g), flags=(lib.PLAN_WINOGRAD if a.winograd else 0) | lib.PLAN_PROFILE)
    model.run(x)  # stages the input on the device
    ms = _time(model, a.iters, a.warmup)
    # the convolution steps alone (the model also converts layouts at its input and output):
    # each step's minimum over profiled replays
    import torch
    stream = torch.cuda.Stream()
    prof = None
    for _ in range(max(3, a.warmup)):
        model.run_profiled(stream.cuda_stream)
        cur = model.profile()
        prof = cur if prof is None else [(o, min(t, pt), f) for (o, t, f), (_, pt, _) in zip(cur, prof)]
    conv_steps = [t for (o, t, f), k in zip(prof, model.step_kinds()) if o == ennf.OP["Conv"]]
    conv_ms = sum(conv_steps)
    oc = a.c if a.residual else a.oc
    oh = a.hw if a.projection else (a.hw + 2 * pad - a.k) // a.stride + 1
    cin = a.c // a.group
    # --projection: both convolutions (the shortcut 1x1 and the fused-residual one)
    flops = 2.0 * a.batch * oc * oh * oh * cin * (a.k * a.k + (1 if a.projection else 0))
    cpad = (a.c + 3) // 4 * 4
    res = a.residual or a.projection
    byts = 4.0 * (a.batch * a.hw * a.hw * cpad * (2 if a.projection else 1)
                  + a.batch * oh * oh * oc * ((3 if a.projection else 2) if res else 1)
                  + oc * cin * (a.k * a.k + (1 if a.projection else 0)))
    print(json.dumps({"layer": {k: v for k, v in vars(a).items() if k != "only"}, "ms_per_run": ms,
                      "conv_ms": conv_ms, "conv_steps_ms": conv_steps,
                      "tflops": flops / conv_ms / 1e9, "gbs": byts / conv_ms / 1e6,
                      "algorithmic_mb": byts / 1e6, "steps": model.plan_info()["steps"],
                      "kinds": model.step_kinds()}), flush=True)
    model.close()
    return 0


def tail(a) -> int:
    """Times the bottleneck-tail pair (1x1 c -> oc with a fused residual, then 1x1 oc -> tail_n2)
    planned fused and planned as separate launches (NO_FUSE): the two convolutions' device
    time each way, and the fused kernel's algorithmic GB/s (t2 + x read, y + t written, once)."""
    import torch
    from spinn_b200 import ennf, lib, netdef, runtime
    g, x = netdef.bottleneck_tail(a.batch, a.hw, a.oc, a.c, a.tail_n2)
    img = ennf.convert(g)
    out = {"layer": {k: v for k, v in vars(a).items() if k != "only"}}
    for name, flags in (("fused", 0), ("separate", lib.PLAN_NO_FUSE)):
        model = runtime.Model(img, flags=flags | lib.PLAN_PROFILE)
        model.run(x)
        _time(model, a.iters, a.warmup)
        stream = torch.cuda.Stream()
        prof = None
        for _ in range(max(3, a.warmup)):
            model.run_profiled(stream.cuda_stream)
            cur = model.profile()
            prof = cur if prof is None else [(o, min(t, pt), f) for (o, t, f), (_, pt, _) in zip(cur, prof)]
        kinds = model.step_kinds()
        # the first convolution (x -> t2) is not part of the pair
        conv = [t for (o, t, f), k in zip(prof, kinds) if k in (1, 9)]
        out[name + "_ms"] = sum(conv[1:])
        out[name + "_kinds"] = kinds
        model.close()
    rows = a.batch * a.hw * a.hw
    byts = 4.0 * rows * (a.c + a.oc + a.oc + a.tail_n2)
    out["algorithmic_mb"] = byts / 1e6
    out["fused_gbs"] = byts / out["fused_ms"] / 1e6
    print(json.dumps(out), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="cfg0,cfg1,cfg2,cfg4")
    ap.add_argument("--cfg4-batches", default="1,32", help="batches of the cfg4 cases")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layer", action="store_true", help="time one convolution layer (shape below)")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--c", type=int, default=256)
    ap.add_argument("--hw", type=int, default=14)
    ap.add_argument("--oc", type=int, default=256)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--group", type=int, default=1)
    ap.add_argument("--residual", action="store_true", help="conv+BN+Add+ReLU (needs c == oc, stride 1)")
    ap.add_argument("--projection", action="store_true",
                    help="bottleneck end with a projection shortcut: ReLU(BN(conv(x)) + BN(conv1x1(x))); "
                         "the second conv (c -> oc) carries the fused residual")
    ap.add_argument("--winograd", action="store_true", help="plan with Winograd F(4x4,3x3)")
    ap.add_argument("--tail", action="store_true",
                    help="the bottleneck-tail pair: 1x1 c -> oc with a residual, then 1x1 oc -> --tail-n2")
    ap.add_argument("--tail-n2", type=int, default=64)
    a = ap.parse_args(argv)
    if a.layer:
        return layer(a)
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
        for batch in [int(b) for b in a.cfg4_batches.split(",")]:
            g = netdef.yolo_shaped(batch=batch, image=640)
            _case(f"cfg4 yolo-shaped 640 batch {batch}", g, netdef.yolo_input(batch, 640), a.iters, a.warmup,
                  per_item=batch)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
