"""Times one fused convolution layer (Conv+BN+ReLU, optionally +residual) through the device
runtime -- a unit for tuning and for profiling a single kernel.

    python -m spinn_b200.layer_bench --batch 512 --c 256 --hw 14 --oc 256 --k 3 [--residual]
    python -m spinn_b200.layer_bench --batch 128 --c 256 --hw 14 --oc 1024 --k 1 --projection
    python -m spinn_b200.layer_bench --mma-rate

Prints one JSON line: device ms per run (CUDA events around the planned step list, inputs
resident), algorithmic TFLOP/s of the layer and algorithmic GB/s (input + output
[+ residual] + weights, each touched once).  --mma-rate instead prints one line per tf32 MMA
shape and shared-memory layout with its per-SM cost in cycles (spinn_cuda_diag_mma_rate).
"""
from __future__ import annotations

import argparse
import json


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--c", type=int, default=256)
    ap.add_argument("--hw", type=int, default=14)
    ap.add_argument("--oc", type=int, default=256)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--residual", action="store_true", help="conv+BN+Add+ReLU (needs c == oc, stride 1)")
    ap.add_argument("--projection", action="store_true",
                    help="bottleneck end with a projection shortcut: ReLU(BN(conv(x)) + BN(conv1x1(x))); "
                         "the second conv (c -> oc) carries the fused residual")
    ap.add_argument("--winograd", action="store_true", help="plan with Winograd F(4x4,3x3)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--mma-rate", action="store_true",
                    help="print the per-SM cycles of one tcgen05 tf32 MMA per shape and layout")
    a = ap.parse_args(argv)
    if a.mma_rate:
        return mma_rate()

    import numpy as np
    import torch

    from spinn_b200 import ennf, netdef, runtime

    pad = a.k // 2
    if a.projection:
        g, x = netdef.conv_bn_proj_add_relu(batch=a.batch, c=a.c, hw=a.hw, oc=a.oc, k=a.k)
    elif a.residual:
        g, x = netdef.conv_bn_add_relu(batch=a.batch, c=a.c, hw=a.hw)
    else:
        g, x = netdef.conv_bn_relu(batch=a.batch, c=a.c, hw=a.hw, oc=a.oc, k=a.k, stride=a.stride, pad=pad)
    from spinn_b200 import lib
    model = runtime.Model(ennf.convert(g), flags=lib.PLAN_WINOGRAD if a.winograd else 0)
    model.run(x)  # stages the input on the device
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    for _ in range(a.warmup):
        model.run_device(stream.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.iters):
        model.run_device(stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    oc = a.c if a.residual else a.oc
    oh = a.hw if a.projection else (a.hw + 2 * pad - a.k) // a.stride + 1
    # --projection: both convolutions (the shortcut 1x1 and the fused-residual one)
    flops = 2.0 * a.batch * oc * oh * oh * a.c * (a.k * a.k + (1 if a.projection else 0))
    cpad = (a.c + 3) // 4 * 4
    res = a.residual or a.projection
    byts = 4.0 * (a.batch * a.hw * a.hw * cpad * (2 if a.projection else 1)
                  + a.batch * oh * oh * oc * ((3 if a.projection else 2) if res else 1)
                  + oc * a.c * (a.k * a.k + (1 if a.projection else 0)))
    print(json.dumps({"layer": vars(a), "ms_per_run": ms, "tflops": flops / ms / 1e9, "gbs": byts / ms / 1e6,
                      "steps": model.plan_info()["steps"]}))
    model.close()
    return 0


MMA_SHAPES = ((128, 32), (128, 64), (128, 128), (128, 256), (64, 64), (64, 128), (64, 256))
LAYOUTS = ("none", "sw32", "sw64", "sw128")


def mma_rate(iters: int = 4096) -> int:
    """Cycles per kind::tf32 MMA by shape and layout; MAC/cycle relative to the 2048 MAC/cycle
    that a 128 x 256 x 8 instruction every 128 cycles delivers."""
    import ctypes

    from spinn_b200 import lib

    L = lib.lib()
    for layout, name in enumerate(LAYOUTS):
        for m, n in MMA_SHAPES:
            cyc = ctypes.c_double(0.0)
            L.spinn_cuda_diag_mma_rate(m, n, layout, iters, ctypes.byref(cyc))  # warm-up
            lib.check(L.spinn_cuda_diag_mma_rate(m, n, layout, iters, ctypes.byref(cyc)), "spinn_cuda_diag_mma_rate")
            mac = m * n * 8 / cyc.value if cyc.value > 0 else None
            print(json.dumps({"m": m, "n": n, "k": 8, "layout": name, "cycles_per_mma": cyc.value,
                              "mac_per_cycle": mac}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
